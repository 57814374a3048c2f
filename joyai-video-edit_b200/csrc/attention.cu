// Non-causal, unmasked multi-head attention forward for sm_100a on the
// 5th-generation tensor cores: O = softmax(scale * Q K^T) V per (batch, head),
// bf16 in / bf16 out, fp32 scores and accumulators in tensor memory.
//
// Replaces the attention call of the reference block: _flash_attention4 /
// _sdpa_attention (deploy/xvideo/models/dit/dit.py:150-178) over queries
// [current image | text] and keys [cache | current] (dit.py:399-420), i.e. an
// external FA4 / cuDNN kernel.  Layout is the reference's NHD: q [B, Lq, H, D],
// k and v [B, Lk, H, D], out [B, Lq, H, D]; any token / head / batch strides
// that keep 16-byte rows (the head-sharded q buffer and K/V cache of the
// sequence-parallel stack are [tokens, heads_per_rank, 128] views).
//
// Kernel organisation (one CTA per SM, 320 threads; CTA = one (batch, head)
// and 256 queries as two 128-row tiles Q0, Q1):
//   warp 8      TMA producer: Q0, Q1 once, then K_j and V_j (128 keys x 128 dims,
//               128-byte swizzle) through two-slot rings (full/empty mbarriers)
//   warp 9      TMEM allocator + MMA issuer (one thread):
//                 S_t = Q_t K_j^T   tcgen05.mma kind::f16, A and B from shared memory
//                 O_t += P_t V_j    A = P_t from tensor memory, B = V_j (MN-major)
//               issued in the order QK0 QK1 | PV0 QK0' PV1 QK1' | ... so that the
//               softmax of one tile overlaps the MMAs of the other
//   warps 0-7   softmax, warpgroup t for tile t; thread = one query row:
//               tcgen05.ld the 128 scores, row max, p = 2^(s*c - m) (c = scale *
//               log2 e), row sum, P as bf16 written over the first 64 columns of
//               S_t (tcgen05.st), then signal the MMA warp.  The running max is
//               only raised (and O_t rescaled in tensor memory) when it grows by
//               more than 2^8, so most key tiles skip the O round trip.
//               At the end: O_t / l, bf16, stored to global memory.
// Tensor memory (512 columns): O0 [0,128) O1 [128,256) S0/P0 [256,384) S1/P1 [384,512).
// P_t aliases S_t: the MMA that overwrites S_t (next QK_t) is issued after the
// PV_t that reads P_t, and tcgen05.mma operations of one thread execute in
// issue order.
//
// Every mbarrier wait is bounded; on expiry the CTA raises an abort flag and
// records a code readable with jo_attention_last_fault(), drains its own
// in-flight copies and MMAs (bounded), frees its tensor memory and returns.
#include <cuda.h>
#include <math.h>
#include <stdlib.h>

#include "jo_common.cuh"

namespace jo {
namespace attn {

constexpr int D = 128;        // head dim
constexpr int BQ = 128;       // query rows per tile (two tiles per CTA)
constexpr int BK = 128;       // keys per tile
constexpr int THREADS = 320;
constexpr int HALF = BQ * 128;                    // 16 KB: 128 rows x 64 dims (128 B)
constexpr int TILE = 2 * HALF;                    // 32 KB: 128 rows x 128 dims
constexpr int SMEM_Q = 0;                         // Q0, Q1
constexpr int SMEM_K = 2 * TILE;                  // K ring, 2 slots
constexpr int SMEM_V = 4 * TILE;                  // V ring, 2 slots
constexpr int SMEM_BAR = 6 * TILE;                // 192 KB
constexpr int SMEM_BYTES = SMEM_BAR + 256 + 1024; // barriers + alignment slack
constexpr long long kTimeoutCycles = 4000000000LL;

__device__ int g_fault = 0;

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > kTimeoutCycles) {
      *abort_flag = 1;
      atomicCAS(&g_fault, 0, code);
      return false;
    }
  }
}
__device__ __forceinline__ void mbar_drain(uint32_t bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity) && clock64() - t0 < kTimeoutCycles) {
  }
}

// 4-D tiled TMA load (dims: dim, head, token, batch) completing on `bar`.
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, int x, int y, int z, int w,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(bar)
      : "memory");
}

// Shared-memory matrix descriptor, 128-byte swizzle.  K-major operands (Q, K):
// 8-row atoms of 1024 B (SBO), LBO unused.  MN-major operand (V): SBO = 1024 B
// between 8-key groups, LBO = 16 KB between the two 64-dim halves.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;  // sm_100 descriptor version
  d |= (uint64_t)2 << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::f16: A = B = BF16, D = F32, M x N; b_mn = B is MN-major.
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n, bool b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(
          d_tmem),
      "l"(a), "l"(b), "r"(id), "r"(acc));
}
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t id, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(
          d_tmem),
      "r"(a_tmem), "l"(b), "r"(id), "r"(acc));
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

#define JO_R8(i) "=r"(r[i]), "=r"(r[i + 1]), "=r"(r[i + 2]), "=r"(r[i + 3]), "=r"(r[i + 4]), "=r"(r[i + 5]), \
                 "=r"(r[i + 6]), "=r"(r[i + 7])
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : JO_R8(0), JO_R8(8), JO_R8(16), JO_R8(24)
      : "r"(taddr));
}
#undef JO_R8
#define JO_W8(i) "r"(r[i]), "r"(r[i + 1]), "r"(r[i + 2]), "r"(r[i + 3]), "r"(r[i + 4]), "r"(r[i + 5]), \
                 "r"(r[i + 6]), "r"(r[i + 7])
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      JO_W8(0), JO_W8(8), JO_W8(16), JO_W8(24)
      : "memory");
}
#undef JO_W8
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// max of three floats in one instruction (NaN operands are ignored).
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// S_t = Q_t K^T over the 8 k-steps of 16 dims (O_t at TMEM column 128 t,
// S_t / P_t at 256 + 128 t).
__device__ __forceinline__ void issue_qk(uint32_t tmem, uint32_t sq, uint32_t sk, int t, int ks) {
  constexpr uint32_t ID_QK = idesc_bf16(BQ, BK, false);
  const uint32_t a0 = sq + t * TILE, b0 = sk + ks * TILE;
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const uint32_t off = (kk >> 2) * HALF + (kk & 3) * 32;
    mma_ss(tmem + 256 + 128 * t, sdesc(a0 + off, 16), sdesc(b0 + off, 16), ID_QK, kk != 0);
  }
}
// O_t (+)= P_t V over the 8 k-steps of 16 keys; P_t read from tensor memory.
__device__ __forceinline__ void issue_pv(uint32_t tmem, uint32_t sv, int t, int vs, bool acc) {
  constexpr uint32_t ID_PV = idesc_bf16(BQ, D, true);
  const uint32_t b0 = sv + vs * TILE;
#pragma unroll
  for (int kk = 0; kk < BK / 16; ++kk)
    mma_ts(tmem + 128 * t, tmem + 256 + 128 * t + kk * 8, sdesc(b0 + kk * 2048, HALF), ID_PV,
           (acc || kk != 0) ? 1u : 0u);
}

constexpr int kMaxRanks = 8;  // destinations of the scattering epilogue

struct Params {
  __nv_bfloat16* o;
  int64_t o_bs, o_ts, o_hs;  // output strides (elements)
  int Lq, Lk, H;
  int n_kt;                  // key tiles
  float scale_log2;          // softmax scale * log2(e)
  // Scattering epilogue (nranks > 0, batch 1): query row r of the gathered
  // order belongs to rank k with seg[k] <= r < seg[k + 1] and is stored at
  // token r - seg[k], head head0 + h of that rank's [tokens, heads, 128]
  // buffer dst[k] (dst_ts elements between tokens).
  __nv_bfloat16* dst[kMaxRanks];
  int seg[kMaxRanks + 1];
  int nranks;
  int head0;
  int64_t dst_ts;
};

// barrier slots (8 bytes each) after the operand rings
enum : int { B_Q = 0, B_KF = 1, B_KE = 3, B_VF = 5, B_VE = 7, B_SF = 9, B_PF = 11, B_OF = 13, B_N = 14 };

__global__ void __launch_bounds__(THREADS, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                    const __grid_constant__ CUtensorMap tv, const Params p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SMEM_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + B_N);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const uint32_t bar0 = smem_u32(bars);
#define BAR(i) (bar0 + 8u * (uint32_t)(i))

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int n_kt = p.n_kt;

  if (threadIdx.x == 0) {
    mbar_init(BAR(B_Q), 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(BAR(B_KF + s), 1);
      mbar_init(BAR(B_KE + s), 1);
      mbar_init(BAR(B_VF + s), 1);
      mbar_init(BAR(B_VE + s), 1);
      mbar_init(BAR(B_SF + s), 1);
      mbar_init(BAR(B_PF + s), 4);  // one arrival per softmax warp
    }
    mbar_init(BAR(B_OF), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 9) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_slot))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sq = smem_u32(smem + SMEM_Q), sk = smem_u32(smem + SMEM_K), sv = smem_u32(smem + SMEM_V);

  if (warp == 8) {
    // ------------------------------------------------------------- producer --
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tq)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tk)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tv)) : "memory");
      mbar_expect_tx(BAR(B_Q), 2 * TILE);
      for (int t = 0; t < 2; ++t)
        for (int hf = 0; hf < 2; ++hf)
          tma_load_4d(sq + t * TILE + hf * HALF, &tq, hf * 64, h, qb * 2 * BQ + t * BQ, b, BAR(B_Q));
      int j = 0;
      for (; j < n_kt; ++j) {
        const int s = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(BAR(B_KE + s), ph ^ 1, abort_flag, 1)) break;
        mbar_expect_tx(BAR(B_KF + s), TILE);
        for (int hf = 0; hf < 2; ++hf) tma_load_4d(sk + s * TILE + hf * HALF, &tk, hf * 64, h, j * BK, b, BAR(B_KF + s));
        if (!mbar_wait(BAR(B_VE + s), ph ^ 1, abort_flag, 2)) {
          ++j;
          break;
        }
        mbar_expect_tx(BAR(B_VF + s), TILE);
        for (int hf = 0; hf < 2; ++hf) tma_load_4d(sv + s * TILE + hf * HALF, &tv, hf * 64, h, j * BK, b, BAR(B_VF + s));
      }
      // Drain: every copy issued must land before the CTA exits.
      mbar_drain(BAR(B_Q), 0);
      for (int i = (j > 2 ? j - 2 : 0); i < j; ++i) {
        mbar_drain(BAR(B_KF + (i & 1)), (i >> 1) & 1);
        mbar_drain(BAR(B_VF + (i & 1)), (i >> 1) & 1);
      }
    }
  } else if (warp == 9) {
    // ----------------------------------------------------------- MMA issuer --
    if (lane == 0) {
      bool ok = mbar_wait(BAR(B_Q), 0, abort_flag, 3) && mbar_wait(BAR(B_KF), 0, abort_flag, 4);
      if (ok) {
        fence_after();
        issue_qk(tmem, sq, sk, 0, 0);
        mma_commit(BAR(B_SF + 0));
        issue_qk(tmem, sq, sk, 1, 0);
        mma_commit(BAR(B_SF + 1));
        mma_commit(BAR(B_KE + 0));
      }
      for (int j = 0; j < n_kt && ok; ++j) {
        const int vs = j & 1;
        const uint32_t ph = j & 1;
        if (!mbar_wait(BAR(B_VF + vs), (j >> 1) & 1, abort_flag, 5) || !mbar_wait(BAR(B_PF + 0), ph, abort_flag, 6)) {
          ok = false;
          break;
        }
        fence_after();
        issue_pv(tmem, sv, 0, vs, j > 0);
        const bool more = j + 1 < n_kt;
        const int ks = (j + 1) & 1;
        if (more) {
          if (!mbar_wait(BAR(B_KF + ks), ((j + 1) >> 1) & 1, abort_flag, 7)) {
            ok = false;
            break;
          }
          fence_after();
          issue_qk(tmem, sq, sk, 0, ks);
          mma_commit(BAR(B_SF + 0));
        }
        if (!mbar_wait(BAR(B_PF + 1), ph, abort_flag, 8)) {
          ok = false;
          break;
        }
        fence_after();
        issue_pv(tmem, sv, 1, vs, j > 0);
        mma_commit(BAR(B_VE + vs));
        if (more) {
          issue_qk(tmem, sq, sk, 1, ks);
          mma_commit(BAR(B_SF + 1));
          mma_commit(BAR(B_KE + ks));
        }
      }
      mma_commit(BAR(B_OF));
      mbar_drain(BAR(B_OF), 0);  // every MMA of this CTA has completed
    }
  } else {
    // -------------------------------------------------------------- softmax --
    const int t = warp >> 2;                 // query tile of this warpgroup
    const int quarter = warp & 3;            // TMEM lane quarter
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tmem + 256 + t * 128 + lane_off;
    const uint32_t tO = tmem + t * 128 + lane_off;
    const float c = p.scale_log2;
    const int last_valid = p.Lk - (n_kt - 1) * BK;  // keys in the last tile
    float m = -INFINITY;                     // running max of s*c (may lag the true max by < 8)
    float l = 0.f;                           // running sum of p
    bool ok = true;
    for (int j = 0; j < n_kt; ++j) {
      if (!mbar_wait(BAR(B_SF + t), j & 1, abort_flag, 9)) {
        ok = false;
        break;
      }
      fence_after();
      float s[128];
      uint32_t* su = reinterpret_cast<uint32_t*>(s);
#pragma unroll
      for (int cch = 0; cch < 4; ++cch) tmem_ld32(tS + cch * 32, su + cch * 32);
      tmem_wait_ld();
      if (j == n_kt - 1 && last_valid < BK) {
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (i >= last_valid) s[i] = -INFINITY;
      }
      // Row max as four independent chains of three-input max (depth 17
      // instead of a 127-long dependent chain).
      float mq[4] = {s[0], s[1], s[2], s[3]};
#pragma unroll
      for (int i = 4; i < 124; i += 8)
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) mq[q4] = max3f(mq[q4], s[i + 2 * q4], s[i + 2 * q4 + 1]);
      mq[0] = max3f(mq[0], s[124], s[125]);
      mq[1] = max3f(mq[1], s[126], s[127]);
      const float mx = max3f(mq[0], mq[1], fmaxf(mq[2], mq[3]));
      const float mt = mx * c;
      // Raise the running max only when the tile's max exceeds it by 2^8 (or on
      // the first tile); otherwise p <= 2^8 stays well inside fp32 / bf16 range.
      const bool need = mt > m + 8.f;
      const bool any_need = __any_sync(0xffffffffu, need);
      const float m_new = need ? mt : m;
      const float alpha = ex2(m - m_new);  // 1 when the max is kept; 0 on the first tile
      m = m_new;
      const float mneg = -m;
      // p = 2^(s*c - m): the argument two lanes per instruction, the row sum
      // in four independent paired accumulators.
      const float2 c2 = make_float2(c, c), mn2 = make_float2(mneg, mneg);
      float2 ra[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      // P goes to tensor memory in four chunks of 32 keys as soon as each is
      // done, so the stores overlap the exponentials of the next chunk.
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 32 * ch; i < 32 * ch + 32; i += 2) {
          float2 e = fma2(make_float2(s[i], s[i + 1]), c2, mn2);
          e.x = ex2(e.x);
          e.y = ex2(e.y);
          pk[(i - 32 * ch) >> 1] = pack2<__nv_bfloat16>(e.x, e.y);
          ra[(i >> 1) & 3] = add2(ra[(i >> 1) & 3], e);
        }
        tmem_st16(tS + 16 * ch, pk);
      }
      const float2 r01 = add2(ra[0], ra[1]), r23 = add2(ra[2], ra[3]);
      const float rs = (r01.x + r01.y) + (r23.x + r23.y);
      l = __fmaf_rn(l, alpha, rs);
      // O_t *= alpha, in tensor memory (PV_t of the previous tile has completed:
      // it was issued before the QK_t whose completion released this S tile).
      if (any_need && j > 0) {
#pragma unroll 1
        for (int cch = 0; cch < 4; ++cch) {
          uint32_t o[32];
          tmem_ld32(tO + cch * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(tO + cch * 32, o);
        }
      }
      tmem_wait_st();
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR(B_PF + t));
    }
    // ---- epilogue: O / l -> bf16 -> global ----
    if (ok && mbar_wait(BAR(B_OF), 0, abort_flag, 10)) {
      fence_after();
      const int row = qb * 2 * BQ + t * BQ + quarter * 32 + lane;
      const float inv = 1.f / l;
      __nv_bfloat16* orow = p.o + (int64_t)b * p.o_bs + (int64_t)row * p.o_ts + (int64_t)h * p.o_hs;
      if (p.nranks > 0) {
        // owning rank of this query row (selects, no indexed parameter loads)
        __nv_bfloat16* base = p.dst[0];
        int s0 = 0;
#pragma unroll
        for (int i = 1; i < kMaxRanks; ++i)
          if (i < p.nranks && row >= p.seg[i]) {
            base = p.dst[i];
            s0 = p.seg[i];
          }
        orow = base + (int64_t)(row - s0) * p.dst_ts + (int64_t)(p.head0 + h) * D;
      }
#pragma unroll 1
      for (int cch = 0; cch < 4; ++cch) {
        uint32_t o[32];
        tmem_ld32(tO + cch * 32, o);
        tmem_wait_ld();
        if (row < p.Lq) {
          uint32_t w[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            w[i] = pack2<__nv_bfloat16>(__uint_as_float(o[2 * i]) * inv, __uint_as_float(o[2 * i + 1]) * inv);
          uint4* dst = reinterpret_cast<uint4*>(orow + cch * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i) dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
        }
      }
    }
  }

  fence_before();
  __syncthreads();
  fence_after();
  if (warp == 9) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
  }
#undef BAR
}

// ------------------------------------------------------------------- host --
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
    else
      cudaGetLastError();
  }
  return fn;
}

// 4-D map over a bf16 [B, L, H, 128] view (strides in elements), box 64 dims x
// 1 head x 128 tokens x 1 batch, 128-byte swizzle, zero fill out of bounds.
static bool make_map(CUtensorMap* map, const void* base, int64_t B, int64_t L, int64_t H, int64_t bs, int64_t ts,
                     int64_t hs) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)L, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)hs * 2, (cuuint64_t)ts * 2, (cuuint64_t)bs * 2};
  cuuint32_t box[4] = {64, 1, 128, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct ScatterSpec {
  void* const* dst;
  const int64_t* seg;
  int ranks;
  int64_t head0, dst_ts, dst_tokens;
};

static int launch(const char* what, const void* q, const void* k, const void* v, void* out, int64_t batch,
                  int64_t Lq, int64_t Lk, int64_t heads, int64_t head_dim, const int64_t* q_strides,
                  const int64_t* k_strides, const int64_t* v_strides, const int64_t* o_strides, float scale, int dtype,
                  const ScatterSpec* sc, void* stream) {
  JO_REQUIRE(dtype == JO_DTYPE_BF16, JO_ERR_DTYPE, "%s: only bf16 is supported", what);
  JO_REQUIRE(head_dim == D, JO_ERR_INVALID, "%s: head_dim must be 128 (got %lld)", what, (long long)head_dim);
  JO_REQUIRE(batch >= 0 && Lq >= 0 && Lk >= 0 && heads >= 0 && batch < 65536 && heads < 65536 && Lq < (1LL << 31) &&
                 Lk < (1LL << 31),
             JO_ERR_INVALID, "%s: invalid shape", what);
  JO_REQUIRE(q_strides && k_strides && v_strides && o_strides, JO_ERR_INVALID, "%s: null strides", what);
  if (batch == 0 || Lq == 0 || heads == 0) return JO_OK;
  JO_REQUIRE(Lk > 0, JO_ERR_INVALID, "%s: attention over zero keys", what);
  JO_REQUIRE(q && k && v && (out || sc), JO_ERR_INVALID, "%s: null tensor pointer", what);
  const int64_t* S[4] = {q_strides, k_strides, v_strides, o_strides};
  for (int i = 0; i < 4; ++i)
    for (int j = 0; j < 3; ++j)
      JO_REQUIRE(S[i][j] >= 0 && S[i][j] % 8 == 0, JO_ERR_ALIGN,
                 "%s: batch / token / head strides must be non-negative multiples of 8 elements", what);
  JO_REQUIRE(aligned16(q) && aligned16(k) && aligned16(v) && (sc || aligned16(out)), JO_ERR_ALIGN,
             "%s: tensors must be 16-byte aligned", what);
  Params p;
  p.o = static_cast<__nv_bfloat16*>(out);
  p.o_bs = o_strides[0];
  p.o_ts = o_strides[1];
  p.o_hs = o_strides[2];
  p.Lq = (int)Lq;
  p.Lk = (int)Lk;
  p.H = (int)heads;
  p.n_kt = (int)((Lk + BK - 1) / BK);
  p.scale_log2 = scale * 1.4426950408889634f;
  p.nranks = 0;
  p.head0 = 0;
  p.dst_ts = 0;
  for (int i = 0; i < kMaxRanks; ++i) p.dst[i] = nullptr;
  for (int i = 0; i <= kMaxRanks; ++i) p.seg[i] = (int)Lq;
  if (sc) {
    // Every store must land inside its destination: a destination may be
    // another GPU's memory.
    JO_REQUIRE(batch == 1, JO_ERR_INVALID, "%s: the scattering form takes one batch", what);
    JO_REQUIRE(sc->ranks >= 1 && sc->ranks <= kMaxRanks && sc->dst && sc->seg, JO_ERR_INVALID,
               "%s: 1..%d destinations with their segment table required", what, kMaxRanks);
    JO_REQUIRE(sc->head0 >= 0 && sc->dst_ts % 8 == 0 && sc->dst_ts >= (sc->head0 + heads) * D, JO_ERR_INVALID,
               "%s: destination token stride %lld too small for heads %lld..%lld of 128", what,
               (long long)sc->dst_ts, (long long)sc->head0, (long long)(sc->head0 + heads));
    JO_REQUIRE(sc->seg[0] == 0 && sc->seg[sc->ranks] == Lq, JO_ERR_INVALID,
               "%s: the segments must cover the %lld query rows", what, (long long)Lq);
    for (int r = 0; r < sc->ranks; ++r) {
      JO_REQUIRE(sc->seg[r + 1] >= sc->seg[r] && sc->seg[r + 1] - sc->seg[r] <= sc->dst_tokens, JO_ERR_INVALID,
                 "%s: segment %d (%lld rows) is negative or exceeds the destination's %lld token rows", what, r,
                 (long long)(sc->seg[r + 1] - sc->seg[r]), (long long)sc->dst_tokens);
      JO_REQUIRE(sc->dst[r] && aligned16(sc->dst[r]), JO_ERR_ALIGN,
                 "%s: destination %d is null or not 16-byte aligned", what, r);
      p.dst[r] = static_cast<__nv_bfloat16*>(sc->dst[r]);
      p.seg[r] = (int)sc->seg[r];
    }
    p.seg[sc->ranks] = (int)Lq;
    p.nranks = sc->ranks;
    p.head0 = (int)sc->head0;
    p.dst_ts = sc->dst_ts;
  }
  int st = require_sm100();
  if (st != JO_OK) return st;
  CUtensorMap tq, tk, tv;
  if (!make_map(&tq, q, batch, Lq, heads, q_strides[0], q_strides[1], q_strides[2]) ||
      !make_map(&tk, k, batch, Lk, heads, k_strides[0], k_strides[1], k_strides[2]) ||
      !make_map(&tv, v, batch, Lk, heads, v_strides[0], v_strides[1], v_strides[2])) {
    set_error("%s: cuTensorMapEncodeTiled failed", what);
    return JO_ERR_CUDA;
  }
  static bool attr[kMaxDevices] = {};
  const int dev = device_slot();
  if (!attr[dev]) {
    cudaFuncSetAttribute(attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    attr[dev] = true;
  }
  dim3 grid((unsigned)((Lq + 2 * BQ - 1) / (2 * BQ)), (unsigned)heads, (unsigned)batch);
  attn_fwd_kernel<<<grid, THREADS, SMEM_BYTES, static_cast<cudaStream_t>(stream)>>>(tq, tk, tv, p);
  return check_launch(what);
}

}  // namespace attn
}  // namespace jo

extern "C" {

int jo_attention_fwd(const void* q, const void* k, const void* v, void* out, int64_t batch, int64_t Lq, int64_t Lk,
                     int64_t heads, int64_t head_dim, const int64_t* q_strides, const int64_t* k_strides,
                     const int64_t* v_strides, const int64_t* o_strides, float scale, int dtype, void* stream) {
  return jo::attn::launch("attention_fwd", q, k, v, out, batch, Lq, Lk, heads, head_dim, q_strides, k_strides,
                          v_strides, o_strides, scale, dtype, nullptr, stream);
}

int jo_attention_fwd_scatter(const void* q, const void* k, const void* v, int64_t Lq, int64_t Lk, int64_t heads,
                             int64_t head_dim, const int64_t* q_strides, const int64_t* k_strides,
                             const int64_t* v_strides, void* const* dst, const int64_t* seg_start, int ranks,
                             int64_t head0, int64_t dst_token_stride, int64_t dst_tokens, float scale, int dtype,
                             void* stream) {
  const int64_t zero[3] = {0, 0, 0};
  const jo::attn::ScatterSpec sc{dst, seg_start, ranks, head0, dst_token_stride, dst_tokens};
  return jo::attn::launch("attention_fwd_scatter", q, k, v, nullptr, 1, Lq, Lk, heads, head_dim, q_strides,
                          k_strides, v_strides, zero, scale, dtype, &sc, stream);
}

// Fault code of the attention kernel's bounded waits (0 = none); reset != 0
// clears it.  One sticky value per device, shared by every launch.  Synchronous.
int jo_attention_last_fault(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, jo::attn::g_fault, sizeof(int)) != cudaSuccess) {
    cudaGetLastError();
    return JO_ERR_CUDA;
  }
  if (reset) {
    int z = 0;
    cudaMemcpyToSymbol(jo::attn::g_fault, &z, sizeof(int));
  }
  return v;
}

}  // extern "C"
