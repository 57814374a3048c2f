// Row-wise HBM-bound operators of joyomni_ops, sm_100a:
//
//   jo_fused_norm_scale_shift   LayerNorm/RMSNorm + adaLN modulate
//                               (reference: fused_norm_scale_shift.cu:69-143)
//   jo_rmsnorm                  plain RMSNorm (reference: rmsnorm.cu:38-61)
//   jo_per_token_quant_fp8      dynamic per-token e4m3 quantisation
//                               (reference: per_token_quant_fp8.cu:43-83)
//   jo_norm_modulate_quant_fp8  new fused entry: norm -> modulate -> round to the
//                               activation dtype -> per-token e4m3 quantisation
//
// Design (B200): every row is read from HBM exactly once with 16-byte
// coalesced, L1-bypassing loads into registers, reduced by a "team" of TEAM
// threads (warp shuffles; shared memory only when a team spans warps), then
// written once with streaming stores.  Small per-column tables (gamma, beta,
// weight, broadcast shift/scale) go through the read-only L1 path and are shared
// by all rows an SM processes.  The team size is chosen per row length so that
// each thread holds up to VPL 16-byte vectors in flight; for the headline
// shape (N = 5120 bf16) that is 2 warps per row, 10 vectors per thread.
//
// Numerics follow the reference kernels operation for operation (fp32 math,
// IEEE division for mean and scale, rsqrtf, the same product grouping, RNE
// output rounding, satfinite e4m3 conversion), so per-token FP8 codes and
// scales are bit-identical to the reference for identical input.
#include "jo_common.cuh"

namespace jo {
namespace {

enum RowOp : int { OP_NORM_MOD = 0, OP_RMSNORM = 1, OP_QUANT = 2, OP_NORM_MOD_QUANT = 3 };

struct RowArgs {
  const void* x;
  int64_t x_stride;  // elements between rows of x
  void* y;           // dense [M, N] output of OP_NORM_MOD / OP_RMSNORM
  const void* gamma; // [N] or null (OP_RMSNORM: the weight)
  const void* beta;  // [N] or null
  const void* scale; // modulation rows (see jo_fused_norm_scale_shift)
  const void* shift;
  int64_t mod_stride;
  int64_t mod_group;
  uint8_t* q;        // e4m3 [M, N]
  float* s;          // fp32 [M]
  int64_t M;
  int N;
  float eps;
};

// Sum (or max) over the TEAM threads that own one row.  Teams are aligned to
// TEAM-thread boundaries; for TEAM > 32 partial results meet in shared memory.
template <int TEAM, bool MAX>
__device__ __forceinline__ float team_reduce(float v, float* red) {
  constexpr int W = TEAM < 32 ? TEAM : 32;
#pragma unroll
  for (int o = W / 2; o > 0; o >>= 1) {
    float t = __shfl_xor_sync(0xffffffffu, v, o, 32);
    v = MAX ? fmaxf(v, t) : v + t;
  }
  if constexpr (TEAM > 32) {
    const int warp = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) red[warp] = v;
    __syncthreads();
    const int first = (threadIdx.x / TEAM) * (TEAM / 32);
    v = red[first];
#pragma unroll
    for (int w = 1; w < TEAM / 32; ++w) v = MAX ? fmaxf(v, red[first + w]) : v + red[first + w];
  }
  return v;
}

__device__ __forceinline__ float quant_inv(float s) { return s == 0.f ? 0.f : __frcp_rn(s); }

__device__ __forceinline__ float quant_val(float x, float inv) {
  float v = __fmul_rn(x, inv);
  return fmaxf(fminf(v, kFp8Max), -kFp8Max);
}

template <typename T, int OP, int NORM, int TEAM, int VPL>
__global__ void __launch_bounds__(TEAM > 256 ? TEAM : 256)
    row_kernel(const RowArgs a) {
  constexpr int CTA = TEAM > 256 ? TEAM : 256;
  constexpr int ROWS = CTA / TEAM;
  constexpr int VEC = 16 / sizeof(T);
  __shared__ float red[3][CTA / 32];

  const int tid = threadIdx.x;
  const int tl = tid % TEAM;
  const int64_t row = (int64_t)blockIdx.x * ROWS + tid / TEAM;
  const bool valid = row < a.M;
  const int N = a.N;
  const int nvec = N / VEC;

  Vec16<T> v[VPL];
  {
    const char* xr = static_cast<const char*>(a.x) + (valid ? row : 0) * a.x_stride * (int64_t)sizeof(T);
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int idx = i * TEAM + tl;
      v[i].raw = (valid && idx < nvec) ? ld_stream(xr + (int64_t)idx * 16) : make_uint4(0, 0, 0, 0);
    }
  }

  if constexpr (OP == OP_QUANT) {
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i)
#pragma unroll
      for (int j = 0; j < VEC; ++j) amax = fmaxf(amax, fabsf(v[i].get(j)));
    amax = team_reduce<TEAM, true>(amax, red[0]);
    const float s = amax / kFp8Max;
    if (valid && tl == 0) a.s[row] = s;
    const float inv = quant_inv(s);
    uint8_t* qr = a.q + (valid ? row : 0) * (int64_t)N;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int idx = i * TEAM + tl;
      if (valid && idx < nvec) {
        uint32_t w[VEC / 4];
#pragma unroll
        for (int j = 0; j < VEC; j += 4) {
          uint32_t lo = pack_e4m3x2(quant_val(v[i].get(j), inv), quant_val(v[i].get(j + 1), inv));
          uint32_t hi = pack_e4m3x2(quant_val(v[i].get(j + 2), inv), quant_val(v[i].get(j + 3), inv));
          w[j / 4] = lo | (hi << 16);
        }
        if constexpr (VEC == 8) {
          asm volatile("st.global.cs.v2.u32 [%0], {%1,%2};" ::"l"(qr + (int64_t)idx * 8), "r"(w[0]), "r"(w[1])
                       : "memory");
        } else {
          asm volatile("st.global.cs.u32 [%0], %1;" ::"l"(qr + (int64_t)idx * 4), "r"(w[0]) : "memory");
        }
      }
    }
    return;
  } else {
    // ---- statistics -----------------------------------------------------
    float mean = 0.f, r;
    if constexpr (NORM == JO_NORM_LAYER) {
      float sum = 0.f;
#pragma unroll
      for (int i = 0; i < VPL; ++i)
#pragma unroll
        for (int j = 0; j < VEC; ++j) sum += v[i].get(j);
      sum = team_reduce<TEAM, false>(sum, red[0]);
      mean = sum / (float)N;
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < VPL; ++i) {
        if (i * TEAM + tl < nvec) {
#pragma unroll
          for (int j = 0; j < VEC; ++j) {
            const float d = v[i].get(j) - mean;
            ss = fmaf(d, d, ss);
          }
        }
      }
      ss = team_reduce<TEAM, false>(ss, red[1]);
      r = rsqrtf(ss / (float)N + a.eps);
    } else {
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < VPL; ++i)
#pragma unroll
        for (int j = 0; j < VEC; ++j) ss = fmaf(v[i].get(j), v[i].get(j), ss);
      ss = team_reduce<TEAM, false>(ss, red[0]);
      r = rsqrtf(ss / (float)N + a.eps);
    }

    // ---- elementwise ----------------------------------------------------
    const char* g = static_cast<const char*>(a.gamma);
    const char* b = static_cast<const char*>(a.beta);
    const char* scr = nullptr;
    const char* shr = nullptr;
    bool mod_stream = false;
    if constexpr (OP != OP_RMSNORM) {
      const int64_t mrow = (valid ? row : 0) / a.mod_group;
      scr = static_cast<const char*>(a.scale) + mrow * a.mod_stride * (int64_t)sizeof(T);
      shr = static_cast<const char*>(a.shift) + mrow * a.mod_stride * (int64_t)sizeof(T);
      mod_stream = (a.mod_group == 1 && a.mod_stride != 0);
    }
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int idx = i * TEAM + tl;
      if (!(valid && idx < nvec)) continue;
      const int64_t off = (int64_t)idx * 16;
      if constexpr (OP == OP_RMSNORM) {
        Vec16<T> w;
        w.raw = ld_cached(g + off);
#pragma unroll
        for (int j = 0; j < VEC; ++j) v[i].set(j, v[i].get(j) * r * w.get(j));
      } else {
        Vec16<T> gv, bv, sc, sh;
        if (g) gv.raw = ld_cached(g + off);
        if (NORM == JO_NORM_LAYER && g && b) bv.raw = ld_cached(b + off);
        sc.raw = mod_stream ? ld_stream(scr + off) : ld_cached(scr + off);
        sh.raw = mod_stream ? ld_stream(shr + off) : ld_cached(shr + off);
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
          float t;
          if constexpr (NORM == JO_NORM_LAYER) {
            const float gj = g ? gv.get(j) : 1.f;
            const float bj = (g && b) ? bv.get(j) : 0.f;
            t = ((v[i].get(j) - mean) * r * gj + bj) * (1.f + sc.get(j)) + sh.get(j);
          } else {
            const float gj = g ? gv.get(j) : 1.f;
            t = (v[i].get(j) * r * gj) * (1.f + sc.get(j)) + sh.get(j);
          }
          v[i].set(j, t);  // rounds to T (RNE), as the reference's T(float) store
        }
      }
    }

    if constexpr (OP == OP_NORM_MOD || OP == OP_RMSNORM) {
      char* yr = static_cast<char*>(a.y) + (valid ? row : 0) * (int64_t)N * (int64_t)sizeof(T);
#pragma unroll
      for (int i = 0; i < VPL; ++i) {
        const int idx = i * TEAM + tl;
        if (valid && idx < nvec) st_stream(yr + (int64_t)idx * 16, v[i].raw);
      }
    } else {
      // OP_NORM_MOD_QUANT: quantise the rounded y row exactly as the reference
      // per-token kernel would quantise the bf16/fp16 tensor written by
      // fused_norm_scale_shift.
      float amax = 0.f;
#pragma unroll
      for (int i = 0; i < VPL; ++i) {
        if (i * TEAM + tl < nvec) {
#pragma unroll
          for (int j = 0; j < VEC; ++j) amax = fmaxf(amax, fabsf(v[i].get(j)));
        }
      }
      amax = team_reduce<TEAM, true>(amax, red[2]);
      const float s = amax / kFp8Max;
      if (valid && tl == 0) a.s[row] = s;
      const float inv = quant_inv(s);
      uint8_t* qr = a.q + (valid ? row : 0) * (int64_t)N;
#pragma unroll
      for (int i = 0; i < VPL; ++i) {
        const int idx = i * TEAM + tl;
        if (valid && idx < nvec) {
          uint32_t w[2];
#pragma unroll
          for (int j = 0; j < 8; j += 4) {
            uint32_t lo = pack_e4m3x2(quant_val(v[i].get(j), inv), quant_val(v[i].get(j + 1), inv));
            uint32_t hi = pack_e4m3x2(quant_val(v[i].get(j + 2), inv), quant_val(v[i].get(j + 3), inv));
            w[j / 4] = lo | (hi << 16);
          }
          asm volatile("st.global.cs.v2.u32 [%0], {%1,%2};" ::"l"(qr + (int64_t)idx * 8), "r"(w[0]), "r"(w[1])
                       : "memory");
        }
      }
    }
  }
}

// Fallback for rows that are not 16-byte aligned (N % 8 != 0 for 2-byte types,
// unaligned base pointers): one 256-thread CTA per row, scalar accesses, the
// row re-read from L2 per pass.  Same arithmetic as row_kernel.
template <typename T, int OP, int NORM>
__global__ void __launch_bounds__(256) row_kernel_scalar(const RowArgs a) {
  __shared__ float red[3][8];
  const int64_t row = blockIdx.x;
  const int N = a.N;
  const T* xr = static_cast<const T*>(a.x) + row * a.x_stride;
  auto block_reduce = [&](float v, float* rd, bool is_max) {
    for (int o = 16; o > 0; o >>= 1) {
      float t = __shfl_xor_sync(0xffffffffu, v, o, 32);
      v = is_max ? fmaxf(v, t) : v + t;
    }
    if ((threadIdx.x & 31) == 0) rd[threadIdx.x >> 5] = v;
    __syncthreads();
    v = rd[0];
    for (int w = 1; w < 8; ++w) v = is_max ? fmaxf(v, rd[w]) : v + rd[w];
    return v;
  };
  if constexpr (OP == OP_QUANT) {
    float amax = 0.f;
    for (int i = threadIdx.x; i < N; i += 256) amax = fmaxf(amax, fabsf(to_f32(xr[i])));
    amax = block_reduce(amax, red[0], true);
    const float s = amax / kFp8Max;
    if (threadIdx.x == 0) a.s[row] = s;
    const float inv = quant_inv(s);
    for (int i = threadIdx.x; i < N; i += 256) {
      __nv_fp8_storage_t c = __nv_cvt_float_to_fp8(quant_val(to_f32(xr[i]), inv), __NV_SATFINITE, __NV_E4M3);
      a.q[row * N + i] = c;
    }
    return;
  } else {
    float mean = 0.f, r;
    if constexpr (NORM == JO_NORM_LAYER) {
      float sum = 0.f;
      for (int i = threadIdx.x; i < N; i += 256) sum += to_f32(xr[i]);
      sum = block_reduce(sum, red[0], false);
      mean = sum / (float)N;
      float ss = 0.f;
      for (int i = threadIdx.x; i < N; i += 256) {
        const float d = to_f32(xr[i]) - mean;
        ss = fmaf(d, d, ss);
      }
      ss = block_reduce(ss, red[1], false);
      r = rsqrtf(ss / (float)N + a.eps);
    } else {
      float ss = 0.f;
      for (int i = threadIdx.x; i < N; i += 256) {
        const float xv = to_f32(xr[i]);
        ss = fmaf(xv, xv, ss);
      }
      ss = block_reduce(ss, red[0], false);
      r = rsqrtf(ss / (float)N + a.eps);
    }
    const T* g = static_cast<const T*>(a.gamma);
    const T* b = static_cast<const T*>(a.beta);
    const T* sc = nullptr;
    const T* sh = nullptr;
    if constexpr (OP != OP_RMSNORM) {
      sc = static_cast<const T*>(a.scale) + (row / a.mod_group) * a.mod_stride;
      sh = static_cast<const T*>(a.shift) + (row / a.mod_group) * a.mod_stride;
    }
    auto y_at = [&](int i) -> T {
      const float xv = to_f32(xr[i]);
      float t;
      if constexpr (OP == OP_RMSNORM) {
        t = xv * r * to_f32(g[i]);
      } else if constexpr (NORM == JO_NORM_LAYER) {
        const float gj = g ? to_f32(g[i]) : 1.f;
        const float bj = (g && b) ? to_f32(b[i]) : 0.f;
        t = ((xv - mean) * r * gj + bj) * (1.f + to_f32(sc[i])) + to_f32(sh[i]);
      } else {
        const float gj = g ? to_f32(g[i]) : 1.f;
        t = (xv * r * gj) * (1.f + to_f32(sc[i])) + to_f32(sh[i]);
      }
      return from_f32<T>(t);
    };
    if constexpr (OP == OP_NORM_MOD || OP == OP_RMSNORM) {
      T* yr = static_cast<T*>(a.y) + row * N;
      for (int i = threadIdx.x; i < N; i += 256) yr[i] = y_at(i);
    } else {
      float amax = 0.f;
      for (int i = threadIdx.x; i < N; i += 256) amax = fmaxf(amax, fabsf(to_f32(y_at(i))));
      amax = block_reduce(amax, red[2], true);
      const float s = amax / kFp8Max;
      if (threadIdx.x == 0) a.s[row] = s;
      const float inv = quant_inv(s);
      for (int i = threadIdx.x; i < N; i += 256) {
        a.q[row * N + i] = __nv_cvt_float_to_fp8(quant_val(to_f32(y_at(i)), inv), __NV_SATFINITE, __NV_E4M3);
      }
    }
  }
}

inline int pow2ceil(int v) {
  int p = 1;
  while (p < v) p <<= 1;
  return p;
}

template <typename T, int OP, int NORM, int TEAM, int VPL>
void launch_team(const RowArgs& a, cudaStream_t st) {
  constexpr int CTA = TEAM > 256 ? TEAM : 256;
  constexpr int ROWS = CTA / TEAM;
  const int64_t grid = (a.M + ROWS - 1) / ROWS;
  row_kernel<T, OP, NORM, TEAM, VPL><<<(unsigned)grid, CTA, 0, st>>>(a);
}

// Picks the team geometry for a row of nvec 16-byte vectors.
template <typename T, int OP, int NORM>
int dispatch(const RowArgs& a, bool vec_ok, cudaStream_t st, const char* what) {
  if (a.M == 0) return JO_OK;
  constexpr int VEC = 16 / sizeof(T);
  const int nvec = a.N / VEC;
  if (!vec_ok || nvec > 16 * 1024) {
    row_kernel_scalar<T, OP, NORM><<<(unsigned)a.M, 256, 0, st>>>(a);
    return check_launch(what);
  }
  if (nvec <= 64) {
    const int team = pow2ceil((nvec + 3) / 4);
    if (team <= 4) launch_team<T, OP, NORM, 4, 4>(a, st);
    else if (team <= 8) launch_team<T, OP, NORM, 8, 4>(a, st);
    else launch_team<T, OP, NORM, 16, 4>(a, st);
  } else {
    int team = pow2ceil((nvec + 15) / 16);
    if (team < 8) team = 8;
    switch (team) {
      case 8: launch_team<T, OP, NORM, 8, 16>(a, st); break;
      case 16: launch_team<T, OP, NORM, 16, 16>(a, st); break;
      case 32: launch_team<T, OP, NORM, 32, 16>(a, st); break;
      case 64: launch_team<T, OP, NORM, 64, 16>(a, st); break;
      case 128: launch_team<T, OP, NORM, 128, 16>(a, st); break;
      case 256: launch_team<T, OP, NORM, 256, 16>(a, st); break;
      case 512: launch_team<T, OP, NORM, 512, 16>(a, st); break;
      default: launch_team<T, OP, NORM, 1024, 16>(a, st); break;
    }
  }
  return check_launch(what);
}

template <int OP, int NORM>
int dispatch_dtype(int dtype, const RowArgs& a, bool vec_ok, cudaStream_t st, const char* what) {
  switch (dtype) {
    case JO_DTYPE_BF16: return dispatch<__nv_bfloat16, OP, NORM>(a, vec_ok, st, what);
    case JO_DTYPE_F16: return dispatch<__half, OP, NORM>(a, vec_ok, st, what);
    case JO_DTYPE_F32:
      if constexpr (OP == OP_NORM_MOD || OP == OP_RMSNORM) return dispatch<float, OP, NORM>(a, vec_ok, st, what);
      [[fallthrough]];
    default:
      set_error("%s: unsupported dtype tag %d", what, dtype);
      return JO_ERR_DTYPE;
  }
}

inline int elem_size(int dtype) {
  return dtype == JO_DTYPE_F32 ? 4 : (dtype == JO_DTYPE_F16 || dtype == JO_DTYPE_BF16) ? 2 : 0;
}

}  // namespace
}  // namespace jo

using namespace jo;

extern "C" {

int jo_fused_norm_scale_shift(void* y, const void* x, const void* gamma, const void* beta,
                              const void* scale, const void* shift, int64_t M, int64_t N,
                              int64_t x_stride, int64_t mod_stride, int64_t mod_group,
                              int norm_type, float eps, int dtype, void* stream) {
  const char* what = "fused_norm_scale_shift";
  JO_REQUIRE(norm_type == JO_NORM_LAYER || norm_type == JO_NORM_RMS, JO_ERR_INVALID,
             "norm_type must be 0 (layer) or 1 (rms)");
  JO_REQUIRE(M >= 0 && N >= 0 && N <= (1 << 30), JO_ERR_INVALID, "%s: invalid shape [%lld, %lld]", what,
             (long long)M, (long long)N);
  JO_REQUIRE((N % 4) == 0, JO_ERR_INVALID, "N must be divisible by 4");
  const int es = elem_size(dtype);
  JO_REQUIRE(es > 0, JO_ERR_DTYPE, "Unsupported dtype; use float32/float16/bfloat16");
  JO_REQUIRE(mod_group >= 1 && mod_stride >= 0 && x_stride >= N, JO_ERR_INVALID,
             "%s: invalid strides (x_stride %lld, mod_stride %lld, mod_group %lld)", what, (long long)x_stride,
             (long long)mod_stride, (long long)mod_group);
  JO_REQUIRE(M == 0 || N == 0 || (x && y && scale && shift), JO_ERR_INVALID, "%s: null tensor pointer", what);
  int st = require_sm100();
  if (st != JO_OK) return st;
  if (M == 0 || N == 0) return JO_OK;
  RowArgs a{x, x_stride, y, gamma, beta, scale, shift, mod_stride, mod_group, nullptr, nullptr, M, (int)N, eps};
  const bool vec_ok = aligned16(x) && aligned16(y) && aligned16(scale) && aligned16(shift) &&
                      (!gamma || aligned16(gamma)) && (!beta || aligned16(beta)) && ((N * es) % 16 == 0) &&
                      ((x_stride * es) % 16 == 0) && ((mod_stride * es) % 16 == 0);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return norm_type == JO_NORM_LAYER ? dispatch_dtype<OP_NORM_MOD, JO_NORM_LAYER>(dtype, a, vec_ok, s, what)
                                    : dispatch_dtype<OP_NORM_MOD, JO_NORM_RMS>(dtype, a, vec_ok, s, what);
}

int jo_rmsnorm(void* out, const void* x, const void* weight, int64_t M, int64_t N, int64_t x_stride, float eps,
               int dtype, void* stream) {
  const char* what = "rmsnorm";
  JO_REQUIRE(M >= 0 && N >= 0 && N <= (1 << 30), JO_ERR_INVALID, "%s: invalid shape", what);
  const int es = elem_size(dtype);
  JO_REQUIRE(es > 0, JO_ERR_DTYPE, "Unsupported dtype; use float32/float16/bfloat16");
  JO_REQUIRE(x_stride >= N, JO_ERR_INVALID, "%s: x_stride %lld < N", what, (long long)x_stride);
  JO_REQUIRE(M == 0 || N == 0 || (x && out && weight), JO_ERR_INVALID, "%s: null tensor pointer", what);
  int st = require_sm100();
  if (st != JO_OK) return st;
  if (M == 0 || N == 0) return JO_OK;
  RowArgs a{x, x_stride, out, weight, nullptr, nullptr, nullptr, 0, 1, nullptr, nullptr, M, (int)N, eps};
  const bool vec_ok = aligned16(x) && aligned16(out) && aligned16(weight) && ((N * es) % 16 == 0) &&
                      ((x_stride * es) % 16 == 0);
  return dispatch_dtype<OP_RMSNORM, JO_NORM_RMS>(dtype, a, vec_ok, static_cast<cudaStream_t>(stream), what);
}

int jo_per_token_quant_fp8(const void* input, int in_dtype, void* out_q, float* out_s, int64_t M, int64_t K,
                           void* stream) {
  const char* what = "per_token_quant_fp8";
  JO_REQUIRE(in_dtype == JO_DTYPE_BF16 || in_dtype == JO_DTYPE_F16, JO_ERR_DTYPE,
             "per_token_quant_fp8: input must be bf16 or fp16");
  JO_REQUIRE(M >= 0 && K >= 0 && K <= (1 << 30), JO_ERR_INVALID, "%s: invalid shape", what);
  JO_REQUIRE((K % 4) == 0, JO_ERR_INVALID, "hidden_dim must be divisible by 4, got %lld", (long long)K);
  JO_REQUIRE(M == 0 || (input && out_q && out_s), JO_ERR_INVALID, "%s: null tensor pointer", what);
  int st = require_sm100();
  if (st != JO_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (M == 0) return JO_OK;
  if (K == 0) {
    // An empty row has amax 0, so its scale is 0 (per_token_quant_fp8.cu:63).
    if (cudaMemsetAsync(out_s, 0, (size_t)M * sizeof(float), s) != cudaSuccess) return check_launch(what);
    return JO_OK;
  }
  RowArgs a{input, K, nullptr, nullptr, nullptr, nullptr, nullptr, 0, 1,
            static_cast<uint8_t*>(out_q), out_s, M, (int)K, 0.f};
  const bool vec_ok = aligned16(input) && aligned8(out_q) && (K % 8) == 0;
  return dispatch_dtype<OP_QUANT, JO_NORM_RMS>(in_dtype, a, vec_ok, s, what);
}

int jo_norm_modulate_quant_fp8(const void* x, const void* gamma, const void* beta, const void* scale,
                               const void* shift, int64_t M, int64_t N, int64_t mod_stride, int64_t mod_group,
                               int norm_type, float eps, int dtype, void* out_q, float* out_s, void* stream) {
  const char* what = "norm_modulate_quant_fp8";
  JO_REQUIRE(norm_type == JO_NORM_LAYER || norm_type == JO_NORM_RMS, JO_ERR_INVALID,
             "norm_type must be 0 (layer) or 1 (rms)");
  JO_REQUIRE(dtype == JO_DTYPE_BF16 || dtype == JO_DTYPE_F16, JO_ERR_DTYPE,
             "%s: x must be bf16 or fp16", what);
  JO_REQUIRE(M >= 0 && N >= 0 && N <= (1 << 30), JO_ERR_INVALID, "%s: invalid shape", what);
  JO_REQUIRE((N % 4) == 0, JO_ERR_INVALID, "N must be divisible by 4");
  JO_REQUIRE(mod_group >= 1 && mod_stride >= 0, JO_ERR_INVALID, "%s: invalid modulation strides", what);
  JO_REQUIRE(M == 0 || N == 0 || (x && scale && shift && out_q && out_s), JO_ERR_INVALID,
             "%s: null tensor pointer", what);
  int st = require_sm100();
  if (st != JO_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (M == 0) return JO_OK;
  if (N == 0) {
    if (cudaMemsetAsync(out_s, 0, (size_t)M * sizeof(float), s) != cudaSuccess) return check_launch(what);
    return JO_OK;
  }
  RowArgs a{x, N, nullptr, gamma, beta, scale, shift, mod_stride, mod_group,
            static_cast<uint8_t*>(out_q), out_s, M, (int)N, eps};
  const bool vec_ok = aligned16(x) && aligned8(out_q) && aligned16(scale) && aligned16(shift) &&
                      (!gamma || aligned16(gamma)) && (!beta || aligned16(beta)) && (N % 8) == 0 &&
                      ((mod_stride * 2) % 16 == 0);
  return norm_type == JO_NORM_LAYER ? dispatch_dtype<OP_NORM_MOD_QUANT, JO_NORM_LAYER>(dtype, a, vec_ok, s, what)
                                    : dispatch_dtype<OP_NORM_MOD_QUANT, JO_NORM_RMS>(dtype, a, vec_ok, s, what);
}

}  // extern "C"
