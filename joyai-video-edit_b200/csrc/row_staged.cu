// Staged (deep-pipelined) row kernel for the bandwidth-critical broadcast-
// modulation paths: the fused norm -> modulate -> per-token FP8 entry, the
// broadcast norm -> modulate, and plain per-token quantisation (N >= 1024).
//
// Why a second kernel: with a register-resident row the number of rows in
// flight per SM is bounded by registers (about 3 rows of 10 KB at N = 5120),
// which leaves HBM latency exposed.  Here every thread streams its own 16-byte
// pieces of the next rows of its team into shared memory with cp.async
// (L1-bypassing), so rows are in flight without register cost and without a
// CTA barrier: a thread only ever reads back the pieces it copied itself
// (visible after cp.async.wait_group).  A team processes R rows per iteration
// so that the per-row fixed work (reductions, divisions, address set-up) and
// the column-table reads are shared by R rows, and warps carry R independent
// dependency chains.
//
// Layout in shared memory (dynamic):
//   float tables[ntab][N]           gamma, (beta), 1 + scale, shift in fp32, staged once
//   uint4 ring[TEAMS][S][R][nvec]   per-team ring of S stages of R rows
// Teams are `team` threads (whole warps); a CTA holds TEAMS teams that
// synchronise among themselves with named barriers (id 1 + team index).
//
// Numerics equal row_ops.cu (and the reference kernels): (1 + scale) is formed
// in fp32 exactly as the reference does per element, only earlier.  The per-
// row absmax runs on the 16-bit bit patterns (exact for non-NaN values, and it
// flags NaN/Inf rows); rows whose codes could involve NaN or Inf take the
// reference's explicit-clamp form, all others rely on the identical satfinite
// saturation of the e4m3 conversion.
#include "jo_common.cuh"

#include <stdlib.h>
#include <type_traits>

namespace jo {
namespace staged {

// OP_NORM_MODROW: norm -> modulate with per-row [M, N] scale / shift rows,
// staged through the ring beside x (three rows per ring slot).
// OP_NORM_MODROW_QUANT: the same followed by per-token e4m3 quantisation.
// Modulation row of token `row`: row / mod_group, mod_stride elements apart.
enum : int { OP_NORM_MOD = 0, OP_QUANT = 2, OP_NORM_MOD_QUANT = 3, OP_NORM_MODROW = 4, OP_NORM_MODROW_QUANT = 5 };
constexpr bool is_modrow(int op) { return op == OP_NORM_MODROW || op == OP_NORM_MODROW_QUANT; }
constexpr int kMaxTeams = 15;  // teams per CTA (named barriers 1..15)

struct Args {
  const void* x;
  void* y;            // OP_NORM_MOD output [M, N]
  const void* gamma;  // [N] or null
  const void* beta;   // [N] or null (layer norm, with gamma)
  const void* scale;  // [N] broadcast
  const void* shift;  // [N] broadcast
  uint8_t* q;
  float* s;
  int64_t mod_stride;  // per-row modulation (OP_NORM_MODROW*): elements between rows
  int64_t mod_group;   // tokens sharing one modulation row
  int64_t M;
  int N;
  float eps;
};

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((unsigned)__cvta_generic_to_shared(smem)),
               "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void team_bar(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
__device__ __forceinline__ uint4 lds16(const void* p) {
  uint4 r;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "r"((unsigned)__cvta_generic_to_shared(p)));
  return r;
}
__device__ __forceinline__ float4 lds16f(const float* p) {
  float4 r;
  asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "r"((unsigned)__cvta_generic_to_shared(p)));
  return r;
}

// Unpack two bf16/fp16 from a word.  The bf16 form is an opaque (volatile)
// asm so each use recomputes it: keeping fp32 copies of a whole row alive
// across the row reduction would cost 2 registers per element.
template <typename T> __device__ __forceinline__ float2 unpack2_r(uint32_t w) { return unpack2<T>(w); }
template <> __device__ __forceinline__ float2 unpack2_r<__nv_bfloat16>(uint32_t w) {
  uint32_t lo, hi;
  asm volatile("shl.b32 %0, %2, 16;\n\tand.b32 %1, %2, 0xffff0000;" : "=r"(lo), "=r"(hi) : "r"(w));
  return make_float2(__uint_as_float(lo), __uint_as_float(hi));
}

// Team-wide reductions of R independent values (one per row).  Warp shuffles
// first; teams spanning several warps meet in shared memory behind a named
// barrier and every thread adds the warp partials in the same order.  `red`
// slots must not be reused before the next barrier of the following reduction
// (callers alternate slot sets by iteration parity).  `team` folds to a
// constant in the fixed-geometry kernels, which unrolls the partial loop.
template <int R, typename V, typename F>
__device__ __forceinline__ void team_reduce(V (&v)[R], int team, int bar_id, V* red, F op) {
  const int nw = team >> 5;
  if (nw > 1) {
    const int w = (threadIdx.x % team) >> 5;
    if ((threadIdx.x & 31) == 0)
#pragma unroll
      for (int r = 0; r < R; ++r) red[r * 16 + w] = v[r];
    team_bar(bar_id, team);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      V t = red[r * 16];
#pragma unroll
      for (int i = 1; i < nw; ++i) t = op(t, red[r * 16 + i]);
      v[r] = t;
    }
  }
}
template <int R>
__device__ __forceinline__ void team_sum(float (&v)[R], int team, int bar_id, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int r = 0; r < R; ++r) v[r] += __shfl_xor_sync(0xffffffffu, v[r], o, 32);
  team_reduce<R>(v, team, bar_id, red, [](float x, float y) { return x + y; });
}
template <int R>
__device__ __forceinline__ void team_umax(uint32_t (&v)[R], int team, int bar_id, float* red) {
#pragma unroll
  for (int r = 0; r < R; ++r) v[r] = __reduce_max_sync(0xffffffffu, v[r]);
  team_reduce<R>(v, team, bar_id, reinterpret_cast<uint32_t*>(red),
                 [](uint32_t x, uint32_t y) { return max(x, y); });
}

// Row statistics on the tensor cores, m16n8k16 with fp32 accumulation, on
// the registers as loaded: the squares of the words that sit in A rows g land
// on the diagonal D[g][g], those in rows g + 8 on D[g+8][g] (the other
// products are unused cross terms), so the two forms accumulate in separate
// registers; with B = ones every D[g][n] gains the plain sum of rows g.  The
// products are exact in fp32 (16-bit inputs); only the accumulation order
// differs from a scalar loop.
template <typename T> struct MmaType;
template <> struct MmaType<__nv_bfloat16> { static constexpr uint32_t kOnes = 0x3f803f80u; };
template <> struct MmaType<__half> { static constexpr uint32_t kOnes = 0x3c003c00u; };
// m16n8k16: A fragment {a0, a1, a2, a3} = (row g, k 0-1), (row g + 8, k 0-1),
// (row g, k 8-9), (row g + 8, k 8-9) of this thread's group; B {b0, b1} =
// (k 0-1, column g), (k 8-9, column g).  With A = {x, y, z, w} (the four words
// of one loaded vector, no moves) and B = {x, z}, D[g][g] gains x.x + z.z over
// the group; with B = {y, w}, D[g + 8][g] gains y.y + w.w.
template <typename T>
__device__ __forceinline__ void mma_k16(float (&c)[4], const uint4& a, uint32_t b0, uint32_t b1) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value)
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1));
  else
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1));
}
// Sum of squares of one 16-byte vector: words x, z into the top diagonal of
// cu, words y, w into the bottom diagonal of cv (two instructions per vector).
template <typename T>
__device__ __forceinline__ void mma_sumsq(float (&cu)[4], float (&cv)[4], const uint4& v) {
  mma_k16<T>(cu, v, v.x, v.z);
  mma_k16<T>(cv, v, v.y, v.w);
}
// Plain sum of one 16-byte vector into c (column 0 of rows g and g + 8).
template <typename T>
__device__ __forceinline__ void mma_sum(float (&c)[4], const uint4& v) {
  mma_k16<T>(c, v, MmaType<T>::kOnes, MmaType<T>::kOnes);
}
// This lane's share of the squares: D[g][g] of cu plus D[g+8][g] of cv; of
// the plain sums: D[g][0] + D[g+8][0]; zero on the other lanes.
__device__ __forceinline__ float mma_diag(const float (&cu)[4], const float (&cv)[4]) {
  const int lane = threadIdx.x & 31, g = lane >> 2;
  return (lane & 3) == (g >> 1) ? ((g & 1) ? cu[1] + cv[3] : cu[0] + cv[2]) : 0.f;
}
__device__ __forceinline__ float mma_col0(const float (&c)[4]) { return (threadIdx.x & 3) == 0 ? c[0] + c[2] : 0.f; }

// Codes of one 16-byte vector (8 elements in 4 words) -> 8 bytes:
// e4m3(x * inv) with round-to-nearest-even and satfinite saturation.  For a
// non-NaN product that equals the reference's explicit clamp to +-448 followed
// by the conversion (an infinite product saturates to +-448 either way).
template <typename T>
__device__ __forceinline__ uint2 codes8(const uint4& v, float inv) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  float2 f[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) f[k] = mul2(unpack2<T>(w[k]), make_float2(inv, inv));
  return make_uint2(pack_e4m3x4(f[0].x, f[0].y, f[1].x, f[1].y), pack_e4m3x4(f[2].x, f[2].y, f[3].x, f[3].y));
}
// A NaN product converts to a NaN code (0x7f / 0xff), where the reference's
// fminf/fmaxf clamp turns it into +448 (0x7e).  Rewrites those bytes.
__device__ __forceinline__ uint32_t fix_nan_codes(uint32_t c) {
  const uint32_t m = __vcmpeq4(c & 0x7f7f7f7fu, 0x7f7f7f7fu);  // 0xff in NaN bytes
  return (c & ~m) | (0x7e7e7e7eu & m);
}

__device__ __forceinline__ void st_cs8(void* p, uint2 v) {
  asm volatile("st.global.cs.v2.u32 [%0], {%1,%2};" ::"l"(p), "r"(v.x), "r"(v.y) : "memory");
}

// Quantise R rows held in X (16-bit elements; bits[r] = team max of |x| as a
// 16-bit pattern, NaN-flagging) and write codes + scales.  EXACT: the team
// covers the row exactly (no index checks).
template <typename T, int VPL, int R, bool EXACT>
__device__ __forceinline__ void quant_rows(const Vec16<T> (&X)[R][VPL], const uint32_t (&bits)[R],
                                           const int64_t row0, const bool (&ok)[R], uint8_t* q, float* sout,
                                           int N, int team, int tl, int bar_id, float* red_slow) {
  const int nvec = N / 8;
  float amax[R];
  bool any_slow = false;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    amax[r] = from_bits16<T>(bits[r]);
    any_slow |= !(bits[r] < Bits16<T>::kInf);
  }
  if (any_slow) {  // team-uniform: NaN or Inf in a row; reference amax ignores NaN (fmaxf)
    uint32_t b2[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      uint32_t acc = 0;  // never NaN: a NaN operand yields the other one
#pragma unroll
      for (int i = 0; i < VPL; ++i) {
        acc = absmax_h2_nonan<T>(acc, X[r][i].raw.x);
        acc = absmax_h2_nonan<T>(acc, X[r][i].raw.y);
        acc = absmax_h2_nonan<T>(acc, X[r][i].raw.z);
        acc = absmax_h2_nonan<T>(acc, X[r][i].raw.w);
      }
      b2[r] = absmax_h2_fold(acc);
    }
    team_umax<R>(b2, team, bar_id, red_slow);
#pragma unroll
    for (int r = 0; r < R; ++r) amax[r] = from_bits16<T>(b2[r]);
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const float s = div448_h(amax[r]);  // == amax / 448 (amax is a 16-bit value)
    if (ok[r] && tl == 0) sout[row0 + r] = s;
    const float inv = s == 0.f ? 0.f : __frcp_rn(s);
    const bool fast = (bits[r] < Bits16<T>::kInf) && inv < __int_as_float(0x7f800000);
    if (!ok[r]) continue;
    uint8_t* qr = q + (row0 + r) * (int64_t)N + tl * 8;
#pragma unroll
    for (int i = 0; i < VPL; ++i)
      if (EXACT || i * team + tl < nvec) {
        uint2 c = codes8<T>(X[r][i].raw, inv);
        if (!fast) c = make_uint2(fix_nan_codes(c.x), fix_nan_codes(c.y));
        st_cs8(qr + i * team * 8, c);
      }
  }
}

constexpr int staged_max_threads(int vpl, int r) { return vpl * r >= 10 ? 256 : vpl * r == 8 ? 640 : 512; }
// Fixed geometries: N = VPL * NW * 256 is known at compile time, so the
// number of teams per CTA is too: as many as the shared memory holds (fp32
// tables + S * R rows of ring + reduction scratch per team), at most 1024
// threads and kMaxTeams teams.
constexpr int fixed_teams(int op, int norm, int vpl, int s, int r, int nw) {
  const int n = vpl * nw * 256;
  const int tab = (op == OP_QUANT || is_modrow(op)) ? 0 : 2 * n * 4;
  const int per_team = s * r * n * 2 * (is_modrow(op) ? 3 : 1) + 2 * 4 * r * 16 * 4;
  int t = (224 * 1024 - tab) / per_team;
  if (t * nw * 32 > 1024) t = 1024 / (nw * 32);
  return t > kMaxTeams ? kMaxTeams : t;
}
constexpr int staged_threads(int op, int norm, int vpl, int s, int r, int nw) {
  return nw == 0 ? staged_max_threads(vpl, r) : fixed_teams(op, norm, vpl, s, r, nw) * nw * 32;
}

// NW > 0: the team is NW warps and covers a row exactly (N = VPL * NW * 256,
// checked by the host), so every index check folds away and every address
// offset within a row is an immediate.  NW == 0: run-time team size.
template <typename T, int OP, int NORM, int VPL, int S, int R, int NW>
__global__ void __launch_bounds__(staged_threads(OP, NORM, VPL, S, R, NW), 1)
    staged_rows(const Args a, const int team_rt, const int teams) {
  constexpr bool HAS_NORM = (OP != OP_QUANT);
  constexpr bool MODROW = is_modrow(OP);
  constexpr bool QOUT = (OP == OP_NORM_MOD_QUANT || OP == OP_NORM_MODROW_QUANT);  // codes + scales out
  constexpr int NST = MODROW ? 3 : 1;  // rows per ring slot: x (+ scale, shift)
  constexpr bool EXACT = NW > 0;
  extern __shared__ __align__(16) unsigned char smem_raw[];

  const int team = EXACT ? NW * 32 : team_rt;
  const int nvec = EXACT ? VPL * NW * 32 : a.N / 8;
  const int N = nvec * 8;
  const int tid = threadIdx.x;
  const int tm = tid / team;       // team in CTA
  const int tl = tid - tm * team;  // thread in team
  const int bar_id = 1 + tm;
  // 1/N once: the row statistics scale by it (within 1 ulp of a division; the
  // tensor-core sums already differ from a scalar loop in summation order).
  const float inv_n = 1.f / (float)N;

  // ---- fp32 column tables (broadcast modulation) -------------------------
  // The per-column constants are folded once per CTA:
  //   rms:   y = (x * r) * A + B,             A = g * (1 + sc), B = sh
  //   layer: y = ((x - mean) * r) * A + B,    A = g * (1 + sc), B = b * (1 + sc) + sh
  // (1 + sc) is formed in fp32 as the reference does; the products and sums
  // are regrouped, which moves an output by at most one bf16 ulp where the
  // unrounded value sits at a rounding boundary (the row statistics already
  // differ from the reference in summation order).
  constexpr int NTAB = (HAS_NORM && !MODROW) ? 2 : 0;
  float* tA = reinterpret_cast<float*>(smem_raw);
  float* tB = tA + N;
  uint4* ring = reinterpret_cast<uint4*>(smem_raw + (size_t)NTAB * N * sizeof(float)) +
                (size_t)tm * S * R * NST * nvec;
  // per-team reduction scratch [2 parities][4 slots][R * 16] after all rings
  typedef float RedT[4][R * 16];
  RedT* red = reinterpret_cast<RedT*>(reinterpret_cast<float*>(
                  reinterpret_cast<uint4*>(smem_raw + (size_t)NTAB * N * sizeof(float)) + (size_t)teams * S * R * NST * nvec)) +
              (size_t)tm * 2;
  if constexpr (HAS_NORM && !MODROW) {
    const bool has_g = a.gamma != nullptr;
    const bool has_b = NORM == JO_NORM_LAYER && has_g && a.beta != nullptr;
    const T* g = static_cast<const T*>(a.gamma);
    const T* b = static_cast<const T*>(a.beta);
    const T* sc = static_cast<const T*>(a.scale);
    const T* sh = static_cast<const T*>(a.shift);
    // Bank-conflict-free layout: element c = 8*v + 4*h + e of a table is
    // stored at h*(N/2) + 4*v + e, so the 16-byte reads of consecutive threads
    // (consecutive v, same h) are contiguous.
    for (int i = tid; i < N; i += blockDim.x) {
      const int v = i >> 3, h = (i >> 2) & 1, e = i & 3;
      const int d = h * (N >> 1) + 4 * v + e;
      const float g1 = has_g ? to_f32(g[i]) : 1.f;
      const float c1 = 1.f + to_f32(sc[i]);
      tA[d] = __fmul_rn(g1, c1);
      tB[d] = NORM == JO_NORM_LAYER ? __fmaf_rn(has_b ? to_f32(b[i]) : 0.f, c1, to_f32(sh[i])) : to_f32(sh[i]);
    }
    __syncthreads();
  }

  const int64_t M = a.M;
  const int64_t ngroups = (M + R - 1) / R;
  const int64_t gteam = (int64_t)blockIdx.x * teams + tm;
  const int64_t tstride = (int64_t)gridDim.x * teams;
  const char* xb = static_cast<const char*>(a.x) + tl * 16;
  const int64_t rowb = (int64_t)N * sizeof(T);
  uint4* ring_t = ring + tl;

  auto issue = [&](int64_t grp, int stage) {
    if (grp < ngroups) {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int64_t row = grp * R + r;
        if (row < M) {
          const char* src = xb + row * rowb;
          uint4* dst = ring_t + (size_t)((stage * R + r) * NST) * nvec;
#pragma unroll
          for (int i = 0; i < VPL; ++i)
            if (EXACT || i * team + tl < nvec) cp_async16(dst + i * team, src + i * team * 16);
          if constexpr (MODROW) {
            const int64_t mrow = a.mod_group == 1 ? row : row / a.mod_group;
            const int64_t moff = tl * 16 + mrow * a.mod_stride * (int64_t)sizeof(T);
            const char* scr = static_cast<const char*>(a.scale) + moff;
            const char* shr = static_cast<const char*>(a.shift) + moff;
#pragma unroll
            for (int i = 0; i < VPL; ++i)
              if (EXACT || i * team + tl < nvec) {
                cp_async16(dst + nvec + i * team, scr + i * team * 16);
                cp_async16(dst + 2 * nvec + i * team, shr + i * team * 16);
              }
          }
        }
      }
    }
    cp_commit();
  };

#pragma unroll
  for (int s = 0; s < S - 1; ++s) issue(gteam + s * tstride, s);

  int stage = 0;
  int parity = 0;
  for (int64_t grp = gteam; grp < ngroups; grp += tstride, parity ^= 1) {
    issue(grp + (int64_t)(S - 1) * tstride, (stage + S - 1) % S);
    cp_wait<S - 1>();
    Vec16<T> X[R][VPL];
    const int64_t row0 = grp * R;
    bool ok[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      ok[r] = row0 + r < M;
      const uint4* src = ring_t + (size_t)((stage * R + r) * NST) * nvec;
#pragma unroll
      for (int i = 0; i < VPL; ++i)
        // EXACT: rows past M read stale ring data; nothing of them is stored.
        X[r][i].raw = EXACT ? lds16(src + i * team)
                            : (ok[r] && i * team + tl < nvec) ? lds16(src + i * team) : make_uint4(0, 0, 0, 0);
    }
    const int cur = stage;  // ring slot of this group (modulation rows)
    (void)cur;
    stage = (stage + 1 == S) ? 0 : stage + 1;

    if constexpr (OP == OP_QUANT) {
      uint32_t bits[R];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        uint32_t acc = 0;
#pragma unroll
        for (int i = 0; i < VPL; ++i) {
          acc = absmax_h2<T>(acc, X[r][i].raw.x);
          acc = absmax_h2<T>(acc, X[r][i].raw.y);
          acc = absmax_h2<T>(acc, X[r][i].raw.z);
          acc = absmax_h2<T>(acc, X[r][i].raw.w);
        }
        bits[r] = absmax_h2_fold(acc);
      }
      team_umax<R>(bits, team, bar_id, red[parity][0]);
      quant_rows<T, VPL, R, EXACT>(X, bits, row0, ok, a.q, a.s, N, team, tl, bar_id, red[parity][1]);
    } else {
      // Row statistics on the tensor cores (two accumulator chains per row),
      // then the team reduction.  Zero-filled tail vectors add nothing.
      float mean[R], rr[R];
      if constexpr (NORM == JO_NORM_LAYER) {
        float sum[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
          float ca[4] = {0.f, 0.f, 0.f, 0.f}, cb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int i = 0; i < VPL; ++i) mma_sum<T>((i & 1) ? cb : ca, X[r][i].raw);
          sum[r] = mma_col0(ca) + mma_col0(cb);
        }
        team_sum<R>(sum, team, bar_id, red[parity][0]);
        float ss[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
          mean[r] = sum[r] * inv_n;
          const float2 nm = make_float2(-mean[r], -mean[r]);
          float2 q2 = make_float2(0.f, 0.f);
#pragma unroll
          for (int i = 0; i < VPL; ++i)
            if (EXACT || i * team + tl < nvec) {
              const uint32_t w[4] = {X[r][i].raw.x, X[r][i].raw.y, X[r][i].raw.z, X[r][i].raw.w};
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const float2 d = add2(unpack2_r<T>(w[k]), nm);
                q2 = fma2(d, d, q2);
              }
            }
          ss[r] = q2.x + q2.y;
        }
        team_sum<R>(ss, team, bar_id, red[parity][1]);
#pragma unroll
        for (int r = 0; r < R; ++r) rr[r] = rsqrtf(ss[r] * inv_n + a.eps);
      } else {
        float ss[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
          mean[r] = 0.f;
          float ca[4] = {0.f, 0.f, 0.f, 0.f}, cb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int i = 0; i < VPL; ++i) mma_sumsq<T>(ca, cb, X[r][i].raw);
          ss[r] = mma_diag(ca, cb);
        }
        team_sum<R>(ss, team, bar_id, red[parity][0]);
#pragma unroll
        for (int r = 0; r < R; ++r) rr[r] = rsqrtf(ss[r] * inv_n + a.eps);
      }
      // y = ((x - mean) * r * g + b) * (1 + sc) + sh  (layer)
      // y = (x * r * g) * (1 + sc) + sh                (rms)
      // in the reference's grouping, two lanes per instruction.
      uint32_t acc[R];
#pragma unroll
      for (int r = 0; r < R; ++r) acc[r] = 0;
      if constexpr (MODROW) {
        // Per-row scale / shift from the ring; gamma / beta (16-bit, [N]) from
        // the L1-cached global copy.  Same expression and grouping as below.
        const bool has_g = a.gamma != nullptr;
        const bool has_b = NORM == JO_NORM_LAYER && has_g && a.beta != nullptr;
#pragma unroll
        for (int i = 0; i < VPL; ++i) {
          if (!(EXACT || i * team + tl < nvec)) continue;
          const int idx = i * team + tl;
          const uint4 gv = has_g ? ld_cached(static_cast<const char*>(a.gamma) + idx * 16)
                                 : make_uint4(MmaType<T>::kOnes, MmaType<T>::kOnes, MmaType<T>::kOnes, MmaType<T>::kOnes);
          const uint4 bv = has_b ? ld_cached(static_cast<const char*>(a.beta) + idx * 16) : make_uint4(0, 0, 0, 0);
          const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w}, bw[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
          for (int r = 0; r < R; ++r) {
            const uint4* slot = ring_t + (size_t)((cur * R + r) * NST) * nvec + i * team;
            const uint4 scv = lds16(slot + nvec), shv = lds16(slot + 2 * nvec);
            const uint32_t cw[4] = {scv.x, scv.y, scv.z, scv.w}, sw[4] = {shv.x, shv.y, shv.z, shv.w};
            uint32_t* wr = reinterpret_cast<uint32_t*>(&X[r][i].raw);
            const float2 rv = make_float2(rr[r], rr[r]);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              float2 f = unpack2_r<T>(wr[k]);
              const float2 g2 = unpack2<T>(gw[k]);
              const float2 c2 = add2(make_float2(1.f, 1.f), unpack2<T>(cw[k]));
              const float2 s2 = unpack2<T>(sw[k]);
              if constexpr (NORM == JO_NORM_LAYER) {
                const float2 nm = make_float2(-mean[r], -mean[r]);
                f = fma2(fma2(mul2(add2(f, nm), rv), g2, unpack2<T>(bw[k])), c2, s2);
              } else {
                f = fma2(mul2(mul2(f, rv), g2), c2, s2);
              }
              wr[k] = pack2<T>(f.x, f.y);
              if constexpr (QOUT) acc[r] = absmax_h2<T>(acc[r], wr[k]);
            }
          }
        }
      } else
#pragma unroll
      for (int i = 0; i < VPL; ++i) {
        if (!(EXACT || i * team + tl < nvec)) continue;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int c = h * (N >> 1) + 4 * (i * team + tl);
          const float4 A = lds16f(tA + c);
          const float4 B = lds16f(tB + c);
          const float2 a01 = make_float2(A.x, A.y), a23 = make_float2(A.z, A.w);
          const float2 b01 = make_float2(B.x, B.y), b23 = make_float2(B.z, B.w);
#pragma unroll
          for (int r = 0; r < R; ++r) {
            uint32_t* wr = reinterpret_cast<uint32_t*>(&X[r][i].raw);
            const float2 rv = make_float2(rr[r], rr[r]);
            float2 f0 = unpack2_r<T>(wr[2 * h]);
            float2 f1 = unpack2_r<T>(wr[2 * h + 1]);
            if constexpr (NORM == JO_NORM_LAYER) {
              const float2 nm = make_float2(-mean[r], -mean[r]);
              f0 = fma2(mul2(add2(f0, nm), rv), a01, b01);
              f1 = fma2(mul2(add2(f1, nm), rv), a23, b23);
            } else {
              f0 = fma2(mul2(f0, rv), a01, b01);
              f1 = fma2(mul2(f1, rv), a23, b23);
            }
            wr[2 * h] = pack2<T>(f0.x, f0.y);      // RNE to T
            wr[2 * h + 1] = pack2<T>(f1.x, f1.y);
            if constexpr (QOUT) {
              acc[r] = absmax_h2<T>(acc[r], wr[2 * h]);
              acc[r] = absmax_h2<T>(acc[r], wr[2 * h + 1]);
            }
          }
        }
      }
      if constexpr (!QOUT) {
#pragma unroll
        for (int r = 0; r < R; ++r) {
          if (!ok[r]) continue;
          char* yr = static_cast<char*>(a.y) + (row0 + r) * rowb + tl * 16;
#pragma unroll
          for (int i = 0; i < VPL; ++i)
            if (EXACT || i * team + tl < nvec) st_stream(yr + i * team * 16, X[r][i].raw);
        }
      } else {
        uint32_t bits[R];
#pragma unroll
        for (int r = 0; r < R; ++r) bits[r] = absmax_h2_fold(acc[r]);
        team_umax<R>(bits, team, bar_id, red[parity][2]);
        quant_rows<T, VPL, R, EXACT>(X, bits, row0, ok, a.q, a.s, N, team, tl, bar_id, red[parity][3]);
      }
    }
  }
  cp_wait<0>();
}

template <typename T, int OP, int NORM, int VPL, int S, int R, int NW>
int launch(const Args& a, int team, cudaStream_t st) {
  const int nvec = a.N / 8;
  if (NW > 0 && (team != NW * 32 || nvec != VPL * NW * 32)) return JO_ERR_INVALID;
  constexpr int NST = is_modrow(OP) ? 3 : 1;
  const size_t tab = (OP != OP_QUANT && !is_modrow(OP)) ? (size_t)2 * a.N * sizeof(float) : 0;
  const size_t per_team = (size_t)S * R * NST * nvec * 16 + (size_t)2 * 4 * R * 16 * sizeof(float);
  // Up to 640 threads and ~224 KB of shared memory per CTA, one CTA per SM.
  int teams = NW > 0 ? fixed_teams(OP, NORM, VPL, S, R, NW) : staged_max_threads(VPL, R) / team;
  if (teams > kMaxTeams) teams = kMaxTeams;
  if (teams < 1) return JO_ERR_INVALID;  // team wider than the CTA budget: caller falls back
  while (teams > 1 && tab + teams * per_team > 224 * 1024) --teams;
  const size_t smem = tab + teams * per_team;
  if (smem > 224 * 1024) return JO_ERR_INVALID;
  static size_t attr[kMaxDevices] = {};
  size_t& opted = attr[device_slot()];
  if (opted < smem) {
    cudaFuncSetAttribute(staged_rows<T, OP, NORM, VPL, S, R, NW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
    opted = smem;
  }
  const int64_t need = ((a.M + R - 1) / R + teams - 1) / teams;
  const int64_t grid = need < sm_count() ? need : sm_count();
  staged_rows<T, OP, NORM, VPL, S, R, NW><<<(unsigned)grid, team * teams, smem, st>>>(a, team, teams);
  return JO_OK;
}

}  // namespace staged

// Geometry of the staged kernel: vectors per thread, rows per team
// iteration, ring stages.  The team spans the row (ceil32(nvec / vpl) threads).
struct StagedGeom {
  int vpl, r, s;
};

static StagedGeom pick_geom(int nvec, int op, int norm) {
  // JO_STAGED_GEOM="vpl,r,s" overrides the choice (used to compare geometries).
  static int ov = -1;
  static StagedGeom g_ov{4, 2, 2};
  if (ov < 0) {
    ov = 0;
    if (const char* e = getenv("JO_STAGED_GEOM")) {
      int v, r, st;
      if (sscanf(e, "%d,%d,%d", &v, &r, &st) == 3) {
        g_ov = StagedGeom{v, r, st};
        ov = 1;
      }
    }
  }
  if (ov == 1) return g_ov;
  // N = 5120: fixed-geometry instantiations, the measured best (B200,
  // M = 10530).  The broadcast norm -> modulate and its fused quantising form
  // share one geometry per norm type, so their row statistics are summed in
  // the same order and the fused codes equal quantising the bf16 output:
  // rms 2-warp teams of 10 vectors per thread, layer 4-warp teams of 5 (also
  // quantisation alone); per-row modulation 4-warp teams of 5, two rows.
  if (nvec == 640) {
    if ((op == staged::OP_NORM_MOD_QUANT || op == staged::OP_NORM_MOD) && norm == JO_NORM_RMS)
      return StagedGeom{10, 1, 2};
    if (staged::is_modrow(op)) return StagedGeom{5, 2, 2};
    return StagedGeom{5, 1, 2};
  }
  // N = 4096, the shipped model's hidden size (deploy/xvideo/config.py:22):
  // 4-warp teams of 4 vectors for every norm type (measured on B200 at
  // M = 10530, fused rms: 24.8 us against 31.0 us for 2-warp teams of 8).
  if (nvec == 512) {
    if (staged::is_modrow(op)) return StagedGeom{4, 2, 2};
    return StagedGeom{4, 1, 2};
  }
  return StagedGeom{4, 2, 2};
}

// JO_STAGED_FIXED=0 disables the fixed-geometry instantiations (comparison).
static bool fixed_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("JO_STAGED_FIXED");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

#define N_FIXED_OK(g, nvec) ((nvec) == 640 || (nvec) == 512)
template <typename T, int OP, int NORM>
static int launch_geom(const staged::Args& a, int nvec, StagedGeom g, cudaStream_t st) {
  using namespace staged;
  const int team = ((nvec + g.vpl - 1) / g.vpl + 31) / 32 * 32;
  if (team > 512) return JO_ERR_INVALID;
  if constexpr (is_modrow(OP)) {
    // One row of x, scale and shift per slot, two slots per team.
    if (fixed_enabled() && g.vpl == 5 && nvec == 640) return launch<T, OP, NORM, 5, 2, 1, 4>(a, team, st);
    if (fixed_enabled() && g.vpl == 4 && nvec == 640) return launch<T, OP, NORM, 4, 2, 1, 5>(a, team, st);
    if (fixed_enabled() && g.vpl == 4 && nvec == 512) return launch<T, OP, NORM, 4, 2, 1, 4>(a, team, st);
    return launch<T, OP, NORM, 4, 2, 1, 0>(a, ((nvec + 3) / 4 + 31) / 32 * 32, st);
  } else {
  // Fixed geometries for the model's widths: N = 5120 (hidden), 4096 and 3072.
  if (g.vpl == 4 && g.r == 2 && g.s == 2 && team * 4 == nvec && fixed_enabled()) {
    if (team == 160) return launch<T, OP, NORM, 4, 2, 2, 5>(a, team, st);
    if (team == 96) return launch<T, OP, NORM, 4, 2, 2, 3>(a, team, st);
    if (team == 128) return launch<T, OP, NORM, 4, 2, 2, 4>(a, team, st);
  }
  if (fixed_enabled() && N_FIXED_OK(g, nvec)) {
#define JO_F(V, R, S, W) \
  if (g.vpl == V && g.r == R && g.s == S && nvec == V * W * 32) return launch<T, OP, NORM, V, S, R, W>(a, team, st);
    JO_F(5, 1, 2, 4)
    JO_F(5, 2, 2, 4)
    JO_F(10, 1, 2, 2)
    JO_F(4, 1, 2, 4)
#undef JO_F
  }
#define JO_G(V, R, S) \
  if (g.vpl == V && g.r == R && g.s == S) return launch<T, OP, NORM, V, S, R, 0>(a, team, st);
  JO_G(4, 2, 2)
  JO_G(4, 1, 3)
  JO_G(10, 1, 2)
  JO_G(20, 1, 2)
#undef JO_G
  return launch<T, OP, NORM, 4, 2, 2, 0>(a, ((nvec + 3) / 4 + 31) / 32 * 32, st);
  }
}

// Entry used by row_ops.cu.  Returns JO_ERR_INVALID (no launch) when the shape
// is not covered, so the caller falls back to the register kernel.
int staged_rows_launch(int op, int norm, int dtype, const void* x, void* y, const void* gamma, const void* beta,
                       const void* scale, const void* shift, int64_t mod_stride, int64_t mod_group, uint8_t* q,
                       float* s, int64_t M, int N, float eps, cudaStream_t st) {
  using namespace staged;
  if (dtype != JO_DTYPE_BF16 && dtype != JO_DTYPE_F16) return JO_ERR_INVALID;
  const int nvec = N / 8;
  if (N % 8 != 0 || nvec < 128) return JO_ERR_INVALID;
  if (is_modrow(op) && (mod_group < 1 || mod_stride < N)) return JO_ERR_INVALID;
  Args a{x, y, gamma, beta, scale, shift, q, s, mod_stride, mod_group, M, N, eps};
  const StagedGeom g = pick_geom(nvec, op, norm);
#define JO_ST(T)                                                                                          \
  do {                                                                                                    \
    if (op == OP_QUANT) return launch_geom<T, OP_QUANT, JO_NORM_RMS>(a, nvec, g, st);                    \
    if (op == OP_NORM_MOD_QUANT)                                                                          \
      return norm == JO_NORM_RMS ? launch_geom<T, OP_NORM_MOD_QUANT, JO_NORM_RMS>(a, nvec, g, st)        \
                                 : launch_geom<T, OP_NORM_MOD_QUANT, JO_NORM_LAYER>(a, nvec, g, st);     \
    if (op == OP_NORM_MODROW_QUANT)                                                                       \
      return norm == JO_NORM_RMS ? launch_geom<T, OP_NORM_MODROW_QUANT, JO_NORM_RMS>(a, nvec, g, st)     \
                                 : launch_geom<T, OP_NORM_MODROW_QUANT, JO_NORM_LAYER>(a, nvec, g, st);  \
    if (op == OP_NORM_MODROW)                                                                             \
      return norm == JO_NORM_RMS ? launch_geom<T, OP_NORM_MODROW, JO_NORM_RMS>(a, nvec, g, st)           \
                                 : launch_geom<T, OP_NORM_MODROW, JO_NORM_LAYER>(a, nvec, g, st);        \
    if (op == OP_NORM_MOD)                                                                                \
      return norm == JO_NORM_RMS ? launch_geom<T, OP_NORM_MOD, JO_NORM_RMS>(a, nvec, g, st)              \
                                 : launch_geom<T, OP_NORM_MOD, JO_NORM_LAYER>(a, nvec, g, st);           \
  } while (0)
  if (dtype == JO_DTYPE_BF16) JO_ST(__nv_bfloat16);
  else JO_ST(__half);
#undef JO_ST
  return JO_ERR_INVALID;
}

}  // namespace jo
