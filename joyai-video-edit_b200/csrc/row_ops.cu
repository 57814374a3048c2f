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
// coalesced, L1-bypassing loads into registers, reduced by a "team" of
// threads (warp shuffles; shared memory only when a team spans warps), then
// written once with streaming stores.  The grid is persistent and each thread
// keeps the same columns for every row it handles, so per-column tables sit
// in shared memory once per CTA and the next row is prefetched while the
// current one is processed.  The broadcast-modulation and quantisation paths
// at N >= 1024 use the deeper cp.async-staged kernel in row_staged.cu.
//
// Numerics follow the reference kernels operation for operation (fp32 math,
// IEEE division for mean and scale, rsqrtf, the same product grouping, RNE
// output rounding, satfinite e4m3 conversion), so per-token FP8 codes and
// scales are bit-identical to the reference for identical input.
#include "jo_common.cuh"

namespace jo {
int staged_rows_launch(int op, int norm, int dtype, const void* x, void* y, const void* gamma, const void* beta,
                       const void* scale, const void* shift, int64_t mod_stride, int64_t mod_group, uint8_t* q,
                       float* s, int64_t M, int N, float eps, cudaStream_t st);
namespace {

enum RowOp : int { OP_NORM_MOD = 0, OP_RMSNORM = 1, OP_QUANT = 2, OP_NORM_MOD_QUANT = 3 };
constexpr int STAGED_NORM_MODROW = 4;        // staged kernel: per-row scale / shift rows
constexpr int STAGED_NORM_MODROW_QUANT = 5;  // the same, quantised

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

// Reduction over the `team` threads that own one row.  Sub-warp teams
// (team < 32, a power of two, aligned inside a warp) use xor shuffles only;
// larger teams are whole warps of one CTA (one row per CTA) and meet in shared
// memory.  `red` must be a slot not reused before the next __syncthreads of the
// following reduction (callers alternate slot sets by row parity).
template <bool MAX>
__device__ __forceinline__ float team_reduce(float v, int team, float* red) {
  const int width = team < 32 ? team : 32;
  for (int o = width >> 1; o > 0; o >>= 1) {
    const float t = __shfl_xor_sync(0xffffffffu, v, o, 32);
    v = MAX ? fmaxf(v, t) : v + t;
  }
  if (team > 32) {
    const int warp = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) red[warp] = v;
    __syncthreads();
    v = red[0];
    for (int w = 1; w < (team >> 5); ++w) v = MAX ? fmaxf(v, red[w]) : v + red[w];
  }
  return v;
}

__device__ __forceinline__ float quant_inv(float s) { return s == 0.f ? 0.f : __frcp_rn(s); }

__device__ __forceinline__ float quant_val(float x, float inv) {
  float v = __fmul_rn(x, inv);
  return fmaxf(fminf(v, kFp8Max), -kFp8Max);
}

template <typename T, int VPL>
__device__ __forceinline__ void load_vecs(Vec16<T> (&v)[VPL], const char* base, int tl, int team, int nvec,
                                          bool ok, bool stream) {
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int idx = i * team + tl;
    if (ok && idx < nvec)
      v[i].raw = stream ? ld_stream(base + (int64_t)idx * 16) : ld_cached(base + (int64_t)idx * 16);
    else
      v[i].raw = make_uint4(0, 0, 0, 0);
  }
}

template <typename T, int VPL>
__device__ __forceinline__ void store_codes(const Vec16<T> (&v)[VPL], uint8_t* qr, int tl, int team, int nvec,
                                            float inv) {
  constexpr int VEC = Vec16<T>::N;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int idx = i * team + tl;
    if (idx < nvec) {
      uint32_t w[VEC / 4];
#pragma unroll
      for (int j = 0; j < VEC; j += 4) {
        const uint32_t lo = pack_e4m3x2(quant_val(v[i].get(j), inv), quant_val(v[i].get(j + 1), inv));
        const uint32_t hi = pack_e4m3x2(quant_val(v[i].get(j + 2), inv), quant_val(v[i].get(j + 3), inv));
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
}

__device__ __forceinline__ uint4 lds16(const uint4* p) {
  uint4 r;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "r"((unsigned)__cvta_generic_to_shared(p)));
  return r;
}

// Persistent, column-stationary row kernel.  A team of `team` threads owns a
// row; thread tl of the team always handles the 16-byte vectors tl, tl+team,
// ... of every row it processes.  Per-column tables (gamma, beta, rmsnorm
// weight and, for a broadcast modulation vector, shift and scale) are staged
// once per CTA in shared memory.  Per-row or grouped modulation rows are
// loaded alongside x.  The next row (x and its modulation rows) is prefetched
// into a second register set while the current row is reduced and written.
template <typename T, int OP, int NORM, int VPL, bool MODROW>
__global__ void __launch_bounds__(256, 2) row_kernel(const RowArgs a, const int team, const int rows_per_cta) {
  constexpr int VEC = Vec16<T>::N;
  constexpr bool HAS_MOD = (OP == OP_NORM_MOD || OP == OP_NORM_MOD_QUANT);
  constexpr bool MOD_SMEM = HAS_MOD && !MODROW;
  __shared__ float red[2][3][8];
  extern __shared__ uint4 tab[];

  const int tid = threadIdx.x;
  const int tl = tid % team;
  const int tsub = tid / team;
  const int N = a.N;
  const int nvec = N / VEC;
  const int64_t M = a.M;
  const int64_t stride = (int64_t)gridDim.x * rows_per_cta;
  const int64_t xrow_bytes = a.x_stride * (int64_t)sizeof(T);
  const int64_t mrow_bytes = a.mod_stride * (int64_t)sizeof(T);
  const char* xb = static_cast<const char*>(a.x);
  const bool mod_stream = a.mod_group == 1;

  // ---- shared-memory tables: [gamma][beta][scale][shift], nvec vectors each --
  const bool has_g = (OP != OP_QUANT) && a.gamma != nullptr;
  const bool has_b = (NORM == JO_NORM_LAYER && HAS_MOD) && has_g && a.beta != nullptr;
  const uint4* tg = tab;
  const uint4* tb = tab + nvec;
  const uint4* tsc = tab + 2 * nvec;
  const uint4* tsh = tab + 3 * nvec;
  if constexpr (OP != OP_QUANT) {
    for (int i = tid; i < nvec; i += blockDim.x) {
      uint4* t = tab;
      if (has_g) t[i] = ld_cached(static_cast<const char*>(a.gamma) + (int64_t)i * 16);
      if (has_b) t[nvec + i] = ld_cached(static_cast<const char*>(a.beta) + (int64_t)i * 16);
      if constexpr (MOD_SMEM) {
        t[2 * nvec + i] = ld_cached(static_cast<const char*>(a.scale) + (int64_t)i * 16);
        t[3 * nvec + i] = ld_cached(static_cast<const char*>(a.shift) + (int64_t)i * 16);
      }
    }
    __syncthreads();
  }

  Vec16<T> SC[MODROW ? VPL : 1], SH[MODROW ? VPL : 1];
  Vec16<T> SCn[MODROW ? VPL : 1], SHn[MODROW ? VPL : 1];
  auto mod_base = [&](const void* p, int64_t row) {
    return static_cast<const char*>(p) + (row / a.mod_group) * mrow_bytes;
  };

  // ---- prologue: first row ------------------------------------------------
  int64_t base = (int64_t)blockIdx.x * rows_per_cta;
  Vec16<T> X[VPL], XN[VPL];
  {
    const int64_t row = base + tsub;
    const bool ok = row < M;
    load_vecs<T, VPL>(X, xb + (ok ? row : 0) * xrow_bytes, tl, team, nvec, ok, true);
    if constexpr (MODROW) {
      load_vecs<T, VPL>(SC, mod_base(a.scale, ok ? row : 0), tl, team, nvec, ok, mod_stream);
      load_vecs<T, VPL>(SH, mod_base(a.shift, ok ? row : 0), tl, team, nvec, ok, mod_stream);
    }
  }

  int parity = 0;
  for (; base < M; base += stride, parity ^= 1) {
    const int64_t row = base + tsub;
    const bool valid = row < M;
    {  // prefetch the next row of this team
      const int64_t nrow = row + stride;
      const bool nok = nrow < M;
      load_vecs<T, VPL>(XN, xb + (nok ? nrow : 0) * xrow_bytes, tl, team, nvec, nok, true);
      if constexpr (MODROW) {
        load_vecs<T, VPL>(SCn, mod_base(a.scale, nok ? nrow : 0), tl, team, nvec, nok, mod_stream);
        load_vecs<T, VPL>(SHn, mod_base(a.shift, nok ? nrow : 0), tl, team, nvec, nok, mod_stream);
      }
    }
    float* rs = red[parity][0];

    if constexpr (OP == OP_QUANT) {
      float amax = 0.f;
#pragma unroll
      for (int i = 0; i < VPL; ++i)
#pragma unroll
        for (int j = 0; j < VEC; ++j) amax = fmaxf(amax, fabsf(X[i].get(j)));
      amax = team_reduce<true>(amax, team, rs);
      const float s = amax / kFp8Max;
      if (valid) {
        if (tl == 0) a.s[row] = s;
        store_codes<T, VPL>(X, a.q + row * (int64_t)N, tl, team, nvec, quant_inv(s));
      }
    } else {
      // ---- statistics -----------------------------------------------------
      float mean = 0.f, r;
      // Two fp32 chains per thread (even / odd element of each pair), added
      // before the team reduction -- the same order as the staged kernel.
      if constexpr (NORM == JO_NORM_LAYER) {
        float2 s2 = make_float2(0.f, 0.f);
#pragma unroll
        for (int i = 0; i < VPL; ++i)
#pragma unroll
          for (int j = 0; j < VEC; j += 2) s2 = add2(s2, make_float2(X[i].get(j), X[i].get(j + 1)));
        float sum = team_reduce<false>(s2.x + s2.y, team, rs);
        mean = sum / (float)N;
        float2 q2 = make_float2(0.f, 0.f);
        const float2 nm = make_float2(-mean, -mean);
#pragma unroll
        for (int i = 0; i < VPL; ++i) {
          if (i * team + tl < nvec) {
#pragma unroll
            for (int j = 0; j < VEC; j += 2) {
              const float2 d = add2(make_float2(X[i].get(j), X[i].get(j + 1)), nm);
              q2 = fma2(d, d, q2);
            }
          }
        }
        const float ss = team_reduce<false>(q2.x + q2.y, team, red[parity][1]);
        r = rsqrtf(ss / (float)N + a.eps);
      } else {
        float2 q2 = make_float2(0.f, 0.f);
#pragma unroll
        for (int i = 0; i < VPL; ++i)
#pragma unroll
          for (int j = 0; j < VEC; j += 2) {
            const float2 f = make_float2(X[i].get(j), X[i].get(j + 1));
            q2 = fma2(f, f, q2);
          }
        const float ss = team_reduce<false>(q2.x + q2.y, team, rs);
        r = rsqrtf(ss / (float)N + a.eps);
      }
      // ---- elementwise (in place in X, rounded to T) ----------------------
#pragma unroll
      for (int i = 0; i < VPL; ++i) {
        const int idx = i * team + tl;
        if (idx >= nvec) continue;
        Vec16<T> g, b, sc, sh;
        if (has_g) g.raw = lds16(tg + idx);
        if constexpr (OP == OP_RMSNORM) {
#pragma unroll
          for (int j = 0; j < VEC; ++j) X[i].set(j, X[i].get(j) * r * g.get(j));
        } else {
          if (has_b) b.raw = lds16(tb + idx);
          if constexpr (MOD_SMEM) {
            sc.raw = lds16(tsc + idx);
            sh.raw = lds16(tsh + idx);
          } else {
            sc = SC[i];
            sh = SH[i];
          }
#pragma unroll
          for (int j = 0; j < VEC; ++j) {
            float t;
            const float gj = has_g ? g.get(j) : 1.f;
            if constexpr (NORM == JO_NORM_LAYER) {
              const float bj = has_b ? b.get(j) : 0.f;
              t = ((X[i].get(j) - mean) * r * gj + bj) * (1.f + sc.get(j)) + sh.get(j);
            } else {
              t = (X[i].get(j) * r * gj) * (1.f + sc.get(j)) + sh.get(j);
            }
            X[i].set(j, t);  // RNE to T, as the reference's T(float) store
          }
        }
      }
      if constexpr (OP == OP_NORM_MOD || OP == OP_RMSNORM) {
        if (valid) {
          char* yr = static_cast<char*>(a.y) + row * (int64_t)N * (int64_t)sizeof(T);
#pragma unroll
          for (int i = 0; i < VPL; ++i) {
            const int idx = i * team + tl;
            if (idx < nvec) st_stream(yr + (int64_t)idx * 16, X[i].raw);
          }
        }
      } else {
        // OP_NORM_MOD_QUANT: quantise the rounded row exactly as the reference
        // per-token kernel quantises the tensor fused_norm_scale_shift wrote.
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < VPL; ++i) {
          if (i * team + tl < nvec) {
#pragma unroll
            for (int j = 0; j < VEC; ++j) amax = fmaxf(amax, fabsf(X[i].get(j)));
          }
        }
        amax = team_reduce<true>(amax, team, red[parity][2]);
        const float s = amax / kFp8Max;
        if (valid) {
          if (tl == 0) a.s[row] = s;
          store_codes<T, VPL>(X, a.q + row * (int64_t)N, tl, team, nvec, quant_inv(s));
        }
      }
    }
    // rotate the prefetched row into place
#pragma unroll
    for (int i = 0; i < VPL; ++i) X[i] = XN[i];
    if constexpr (MODROW) {
#pragma unroll
      for (int i = 0; i < VPL; ++i) {
        SC[i] = SCn[i];
        SH[i] = SHn[i];
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

// Persistent grid: as many CTAs as fit on the device (occupancy API, cached per
// kernel instance, CTA size and shared-memory size), capped by the work.
template <typename T, int OP, int NORM, int VPL, bool MODROW>
void launch_rows(const RowArgs& a, int team, cudaStream_t st) {
  const int cta = team >= 32 ? team : 256;
  const int rows_per_cta = cta / team;
  const int nvec = a.N / (16 / (int)sizeof(T));
  const int ntab = OP == OP_QUANT ? 0 : (MODROW || OP == OP_RMSNORM) ? 2 : 4;
  const size_t smem = (size_t)ntab * nvec * 16;
  struct Cache {
    bool attr_set;
    int cta, blocks;
    size_t smem;
  };
  static Cache cache[kMaxDevices] = {};
  Cache& c = cache[device_slot()];
  if (!c.attr_set) {
    cudaFuncSetAttribute(row_kernel<T, OP, NORM, VPL, MODROW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         16 * 2048 * 4);
    c.attr_set = true;
    c.cta = -1;
  }
  if (c.cta != cta || c.smem != smem) {
    int per_sm = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, row_kernel<T, OP, NORM, VPL, MODROW>, cta, smem);
    c.blocks = (per_sm > 0 ? per_sm : 1) * sm_count();
    c.cta = cta;
    c.smem = smem;
  }
  const int64_t need = (a.M + rows_per_cta - 1) / rows_per_cta;
  const int64_t grid = need < c.blocks ? need : c.blocks;
  row_kernel<T, OP, NORM, VPL, MODROW><<<(unsigned)grid, cta, smem, st>>>(a, team, rows_per_cta);
}

// Team geometry for a row of nvec 16-byte vectors: VPL vectors per thread
// (4 preferred), team = whole warps spanning the row (at most 256 threads), or
// a power-of-two sub-warp team for short rows.  Longer rows take the scalar path.
inline bool pick_team(int nvec, int& vpl, int& team) {
  if (nvec <= 8) {
    vpl = 2;
    team = pow2ceil((nvec + 1) / 2);
    return true;
  }
  for (int v : {4, 8}) {
    int t = (nvec + v - 1) / v;
    t = t <= 16 ? pow2ceil(t) : (t + 31) / 32 * 32;
    if (t <= 256) {
      vpl = v;
      team = t;
      return true;
    }
  }
  return false;
}

template <typename T, int OP, int NORM>
int dispatch(const RowArgs& a, bool vec_ok, cudaStream_t st, const char* what) {
  if (a.M == 0) return JO_OK;
  constexpr int VEC = 16 / sizeof(T);
  const int nvec = a.N / VEC;
  int vpl = 0, team = 0;
  if (!vec_ok || !pick_team(nvec, vpl, team)) {
    row_kernel_scalar<T, OP, NORM><<<(unsigned)a.M, 256, 0, st>>>(a);
    return check_launch(what);
  }
  // Modulation rows that change along M are loaded with x; a single broadcast
  // vector is staged in shared memory.
  const bool modrow = (OP == OP_NORM_MOD || OP == OP_NORM_MOD_QUANT) && a.mod_stride != 0 && a.mod_group < a.M;
  if (modrow) {
    if constexpr (OP == OP_NORM_MOD || OP == OP_NORM_MOD_QUANT) {
      if (vpl == 2) launch_rows<T, OP, NORM, 2, true>(a, team, st);
      else if (vpl == 4) launch_rows<T, OP, NORM, 4, true>(a, team, st);
      else launch_rows<T, OP, NORM, 8, true>(a, team, st);
    }
  } else {
    if (vpl == 2) launch_rows<T, OP, NORM, 2, false>(a, team, st);
    else if (vpl == 4) launch_rows<T, OP, NORM, 4, false>(a, team, st);
    else launch_rows<T, OP, NORM, 8, false>(a, team, st);
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
  const bool broadcast = (mod_stride == 0 || mod_group >= M) && x_stride == N;
  if (vec_ok && broadcast &&
      staged_rows_launch(OP_NORM_MOD, norm_type, dtype, x, y, gamma, beta, scale, shift, 0, 1, nullptr, nullptr, M,
                         (int)N, eps, s) == JO_OK)
    return check_launch(what);
  // Per-row (or per-group) modulation rows: the staged kernel streams x,
  // scale and shift rows together through its cp.async ring.
  if (vec_ok && x_stride == N &&
      staged_rows_launch(STAGED_NORM_MODROW, norm_type, dtype, x, y, gamma, beta, scale, shift, mod_stride,
                         mod_group, nullptr, nullptr, M, (int)N, eps, s) == JO_OK)
    return check_launch(what);
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
  if (vec_ok && staged_rows_launch(OP_QUANT, JO_NORM_RMS, in_dtype, input, nullptr, nullptr, nullptr, nullptr,
                                   nullptr, 0, 1, static_cast<uint8_t*>(out_q), out_s, M, (int)K, 0.f, s) == JO_OK)
    return check_launch(what);
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
  const bool broadcast = mod_stride == 0 || mod_group >= M;
  if (vec_ok && broadcast &&
      staged_rows_launch(OP_NORM_MOD_QUANT, norm_type, dtype, x, nullptr, gamma, beta, scale, shift, 0, 1,
                         static_cast<uint8_t*>(out_q), out_s, M, (int)N, eps, s) == JO_OK)
    return check_launch(what);
  if (vec_ok && !broadcast &&
      staged_rows_launch(STAGED_NORM_MODROW_QUANT, norm_type, dtype, x, nullptr, gamma, beta, scale, shift,
                         mod_stride, mod_group, static_cast<uint8_t*>(out_q), out_s, M, (int)N, eps, s) == JO_OK)
    return check_launch(what);
  return norm_type == JO_NORM_LAYER ? dispatch_dtype<OP_NORM_MOD_QUANT, JO_NORM_LAYER>(dtype, a, vec_ok, s, what)
                                    : dispatch_dtype<OP_NORM_MOD_QUANT, JO_NORM_RMS>(dtype, a, vec_ok, s, what);
}

}  // extern "C"
