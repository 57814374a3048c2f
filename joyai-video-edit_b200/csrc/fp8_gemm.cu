// FP8 (e4m3 x e4m3 -> fp32) scaled GEMM for sm_100a on the 5th-generation
// tensor cores (tcgen05 + TMEM), with the per-token x per-channel scale, bias
// and optional GELU-tanh epilogue fused.
//
// Replaces joyomni_ops::fp8_scaled_mm (deploy/joyomni_ops/csrc/fp8_gemm.cu:1450-1548,
// Sm100 CUTLASS kernel :796-1170).  Epilogue arithmetic follows that kernel's
// visitor tree (:833-860): t = sb[n] * acc (fp32), D = out(fma(sa[m], t, bias[n]))
// or out(sa[m] * t) without bias.  The GELU variant applies
// 0.5*y*(1+tanh(sqrt(2/pi)*(y+0.044715*y^3))) to the rounded D, as the reference
// model applies F.gelu(approximate="tanh") after fp8_scaled_mm (dit.py:90-92).
//
// Layout: A [M, K] row-major (K contiguous); B given as the column-major [K, N]
// operand of the reference, i.e. N rows of K contiguous codes.  Both operands
// are therefore K-major, loaded by TMA with 128-byte swizzle into the canonical
// UMMA K-major SW128 layout.  No cluster multicast anywhere: every CTA loads its
// own tiles; operand reuse across CTAs comes from L2 via a grouped tile order.
//
// Kernel organisation (one persistent CTA per SM, 320 threads):
//   warp 0      TMA producer: K-blocks of 128 bytes for A (128 rows) and B (256 rows)
//               into a ring of STAGES shared-memory stages (full/empty mbarriers)
//   warp 1      TMEM allocator + MMA issuer: 4 x tcgen05.mma.kind::f8f6f4 (K = 32)
//               per stage into one of two 128 x 256 fp32 accumulators in TMEM
//               (512 columns), tcgen05.commit releases the stage / publishes the tile
//   warps 2..9  epilogue, two warps per TMEM lane quarter, each draining half of
//               the columns: tcgen05.ld 32 columns at a time (the next chunk's load
//               in flight), scales + bias (+ GELU), bf16/fp16 stores; the
//               accumulator is handed back so the MMA of the next tile overlaps
//               this epilogue.
// Every mbarrier wait is bounded by a clock-based timeout; on expiry the CTA sets
// an abort flag, records an error code readable with jo_gemm_last_fault(), waits
// (bounded) for its own in-flight copies, frees its TMEM and returns.
#include <cuda.h>
#include <stdlib.h>

#include "jo_common.cuh"

namespace jo {
namespace gemm {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 128;  // bytes = fp8 elements per K-block
constexpr int STAGES = 4;
constexpr int A_STAGE = BM * BK;              // 16 KB
constexpr int B_STAGE = BN * BK;              // 32 KB
constexpr int STAGE_BYTES = A_STAGE + B_STAGE;
constexpr int THREADS = 320;            // producer, MMA issuer, 8 epilogue warps
constexpr int EPI_WARPS = 8;
constexpr int TMEM_COLS = 512;
constexpr long long kTimeoutCycles = 4000000000LL;  // ~2 s at 1.9 GHz

// Sticky fault code of the bounded mbarrier waits, one per device and shared
// by every GEMM launch on it: the first wait that times out records its code
// (the output of that launch is then incomplete).  Read and cleared by
// jo_gemm_last_fault(); the stack harness checks it once per chunk.
__device__ int g_fault = 0;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
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
// Bounded wait.  Returns false (and raises the CTA abort flag) on timeout or
// when another role already aborted.
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

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// UMMA shared-memory descriptor: K-major, 128-byte swizzle, 8-row atoms of 1024 B.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);          // start address
  d |= (uint64_t)1 << 16;                           // leading byte offset (unused for SW128 K-major)
  d |= (uint64_t)(1024 >> 4) << 32;                 // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;                           // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                           // SWIZZLE_128B
  return d;
}

// Instruction descriptor: kind::f8f6f4, A = B = E4M3, D = F32, both K-major, M x N.
__host__ __device__ constexpr uint32_t idesc(int m, int n) {
  return (1u << 4)                      // D format F32
         | (0u << 7) | (0u << 10)       // A, B = E4M3
         | ((uint32_t)(n >> 3) << 17)   // N / 8
         | ((uint32_t)(m >> 4) << 24);  // M / 16
}

__device__ __forceinline__ void mma_f8(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t id, uint32_t accum) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n}\n" ::"r"(
          tmem_d),
      "l"(a), "l"(b), "r"(id), "r"(accum));
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// GELU, tanh form: 0.5 * y * (1 + tanh(u)) with u = sqrt(2/pi) * (y + 0.044715 y^3)
// (F.gelu(approximate="tanh") as the reference model applies it, dit.py:90-92),
// evaluated through the identity 0.5 * (1 + tanh(u)) = 1 / (1 + 2^(-2 u log2 e)):
// one SFU exponential and one SFU reciprocal, each accurate to about 2^-22
// relative, and no cancellation for negative y (where 1 + tanh(u) is small and
// an approximate tanh would lose most of its digits).
__device__ __forceinline__ float ex2_approx(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ float rcp_approx(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
// Two lanes at a time: the exponent -2 u log2(e) = y * (A + B y^2) with
// A = -2 log2(e) sqrt(2/pi) and B = A * 0.044715 (folded in double, rounded
// once), three paired fp32 instructions instead of five scalar ones per element.
__device__ __forceinline__ float2 gelu_tanh2(float2 y) {
  const float2 kA = make_float2(-2.3022082f, -2.3022082f);
  const float2 kB = make_float2(-0.10294324f, -0.10294324f);
  const float2 a = mul2(y, fma2(kB, mul2(y, y), kA));
  const float2 d = add2(make_float2(ex2_approx(a.x), ex2_approx(a.y)), make_float2(1.f, 1.f));
  return mul2(y, make_float2(rcp_approx(d.x), rcp_approx(d.y)));
}

struct Params {
  void* d;
  const float* sa;
  const float* sb;
  const void* bias;
  int M, N, K;
  int m_blocks, n_blocks, k_blocks;
  int epilogue;  // JO_EPI_*
  const void* resid;  // JO_EPI_RESID_GATE: residual [M, N] (may alias d)
  const void* gate;   // JO_EPI_RESID_GATE: gate [N]
  int group;          // 2-SM kernel: pair-tile rows per rasterisation group
  // Head-scatter output (jo_fp8_scaled_mm_scatter): output column n is part
  // n / sc_width (q, k, v) of head h = (n % sc_width) / sc_dh, owned by rank
  // h / sc_hpr; row m goes to token sc_tok0 + m of that rank's
  // [tokens, sc_hpr, sc_dh] buffer sc_dst[part * 8 + rank] (a peer's memory
  // for other ranks: plain 16-byte stores over NVLink).
  int scatter;
  int sc_width, sc_dh, sc_hpr;
  int64_t sc_tok0;
  void* sc_dst[24];
};

template <typename OutT>
__device__ __forceinline__ OutT* scatter_dst(const Params& p, int m, int n0) {
  const int part = n0 / p.sc_width;
  const int col = n0 - part * p.sc_width;
  const int h = col / p.sc_dh;
  const int d = h / p.sc_hpr;
  const int hl = h - d * p.sc_hpr;
  OutT* base = static_cast<OutT*>(p.sc_dst[part * 8 + d]);
  return base + ((p.sc_tok0 + m) * p.sc_hpr + hl) * (int64_t)p.sc_dh + (col - h * p.sc_dh);
}

// Epilogue of one 32-column chunk of one output row (one thread = one row):
//   o = out(fma(sa, sb[n] * acc, bias[n]))  or  out(sa * (sb[n] * acc))
//   GELU:        o = out(gelu_tanh(o))
//   RESID_GATE:  o = out(res[m, n] + gate[n] * o)
// (fp8_gemm.cu:833-860 of the reference for the first line; the GELU and
// gated-residual forms are the model's following eager ops, dit.py:90-92 and
// sgl_fused_ops.py:114-117, applied to the rounded GEMM output.)
template <typename OutT>
__device__ __forceinline__ void epilogue_chunk(const uint32_t (&r)[32], const Params& p, int m, float sa, int n0,
                                               OutT* dst) {
  const OutT* bias = static_cast<const OutT*>(p.bias);
  const bool full = n0 + 32 <= p.N;
  float y[32];
#pragma unroll
  for (int j = 0; j < 32; j += 4) {
    float sbv[4], bv[4] = {0.f, 0.f, 0.f, 0.f};
    if (full) {
      const float4 s4 = __ldg(reinterpret_cast<const float4*>(p.sb + n0 + j));
      sbv[0] = s4.x; sbv[1] = s4.y; sbv[2] = s4.z; sbv[3] = s4.w;
      if (bias) {
        const uint2 b2 = __ldg(reinterpret_cast<const uint2*>(bias + n0 + j));
        const OutT* bb = reinterpret_cast<const OutT*>(&b2);
#pragma unroll
        for (int e = 0; e < 4; ++e) bv[e] = to_f32(bb[e]);
      }
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int n = n0 + j + e;
        sbv[e] = n < p.N ? p.sb[n] : 0.f;
        if (bias) bv[e] = n < p.N ? to_f32(bias[n]) : 0.f;
      }
    }
    // Paired fp32 (each lane an IEEE round-to-nearest mul / fma, so the
    // result is that of the scalar expression).
    const float2 sa2 = make_float2(sa, sa);
#pragma unroll
    for (int e = 0; e < 4; e += 2) {
      const float2 acc = make_float2(__uint_as_float(r[j + e]), __uint_as_float(r[j + e + 1]));
      const float2 tt = mul2(make_float2(sbv[e], sbv[e + 1]), acc);
      float2 o = bias ? fma2(sa2, tt, make_float2(bv[e], bv[e + 1])) : mul2(sa2, tt);
      if (p.epilogue == JO_EPI_GELU_TANH) o = gelu_tanh2(unpack2<OutT>(pack2<OutT>(o.x, o.y)));
      y[j + e] = o.x;
      y[j + e + 1] = o.y;
    }
  }
  if (p.epilogue == JO_EPI_RESID_GATE) {
    const OutT* res = static_cast<const OutT*>(p.resid) + (size_t)m * p.N;
    const OutT* gate = static_cast<const OutT*>(p.gate);
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int n = n0 + j;
      if (full || n < p.N) y[j] = __fmaf_rn(to_f32(gate[n]), to_f32(from_f32<OutT>(y[j])), to_f32(res[n]));
    }
  }
  if (full) {
    uint32_t w[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) w[j] = pack2<OutT>(y[2 * j], y[2 * j + 1]);
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int j = 0; j < 4; ++j) d4[j] = make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (n0 + j < p.N) dst[j] = from_f32<OutT>(y[j]);
  }
}

// One epilogue warp's share of an accumulator tile: the 32 rows of its TMEM
// lane quarter, columns [128 half, 128 half + 128) of the BN columns, in four
// 32-column chunks; the TMEM load of the next chunk is in flight while the
// current one is converted and stored.  Eight warps (two per lane quarter)
// drain a tile in about half the time four would.
template <typename OutT>
__device__ __forceinline__ void drain_tile(const Params& p, uint32_t tbase, int m, bool mok, float sa, int nb,
                                           int half) {
  OutT* drow = static_cast<OutT*>(p.d) + (size_t)(mok ? m : 0) * p.N;
  constexpr int CH = BN / 2 / 32;
  const uint32_t t0 = tbase + half * (BN / 2);
  uint32_t r[2][32];
  __syncwarp();
  tmem_ld32(t0, r[0]);
#pragma unroll
  for (int i = 0; i < CH; ++i) {
    tmem_wait_ld();  // chunk i has landed (nothing else is outstanding)
    if (i + 1 < CH) tmem_ld32(t0 + (i + 1) * 32, r[(i + 1) & 1]);
    const int n0 = nb * BN + half * (BN / 2) + i * 32;
    if (mok && n0 < p.N)
      epilogue_chunk<OutT>(r[i & 1], p, m, sa, n0, p.scatter ? scatter_dst<OutT>(p, m, n0) : drow + n0);
  }
}

// Grouped rasterisation: GROUP m-blocks share the n sweep, keeping the live
// A and B panels of all 148 CTAs inside L2.
__device__ __forceinline__ void tile_coords(int t, const Params& p, int& mb, int& nb) {
  constexpr int GROUP = 16;
  const int per_group = GROUP * p.n_blocks;
  const int g = t / per_group;
  const int first = g * GROUP;
  const int rows = min(GROUP, p.m_blocks - first);
  const int r = t % per_group;
  mb = first + r % rows;
  nb = r / rows;
}

template <typename OutT>
__global__ void __launch_bounds__(THREADS, 1)
    fp8_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                    const Params p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  // bars: full[STAGES], empty[STAGES], tmem_full[2], tmem_empty[2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t full0 = smem_u32(bars);
  const uint32_t empty0 = smem_u32(bars + STAGES);
  const uint32_t tfull0 = smem_u32(bars + 2 * STAGES);
  const uint32_t tempty0 = smem_u32(bars + 2 * STAGES + 2);
  const int num_tiles = p.m_blocks * p.n_blocks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull0 + 8 * b, 1);
      mbar_init(tempty0 + 8 * b, EPI_WARPS);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer --
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_a)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_b)) : "memory");
      uint32_t it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int mb, nb;
        tile_coords(t, p, mb, nb);
        for (int kb = 0; kb < p.k_blocks; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(empty0 + 8 * s, ph ^ 1, abort_flag, 1)) { ok = false; break; }
          const uint32_t sa = smem_u32(smem + s * STAGE_BYTES);
          mbar_expect_tx(full0 + 8 * s, STAGE_BYTES);
          tma_load_2d(sa, &tmap_a, kb * BK, mb * BM, full0 + 8 * s);
          tma_load_2d(sa + A_STAGE, &tmap_b, kb * BK, nb * BN, full0 + 8 * s);
        }
      }
      // Drain: every copy this thread issued must have landed before the CTA exits.
      const uint32_t n = it < (uint32_t)STAGES ? it : (uint32_t)STAGES;
      for (uint32_t j = it - n; j < it; ++j) {
        const int s = j % STAGES;
        const long long t0 = clock64();
        while (!mbar_try_wait(full0 + 8 * s, (j / STAGES) & 1) && clock64() - t0 < kTimeoutCycles) {
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer --
    if (lane == 0) {
      constexpr uint32_t ID = idesc(BM, BN);
      uint32_t it = 0;
      int tc = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++tc) {
        const int buf = tc & 1;
        const uint32_t tph = (tc >> 1) & 1;
        if (!mbar_wait(tempty0 + 8 * buf, tph ^ 1, abort_flag, 2)) break;
        fence_after();
        const uint32_t dtm = tmem_base + buf * BN;
        for (int kb = 0; kb < p.k_blocks; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(full0 + 8 * s, ph, abort_flag, 3)) { ok = false; break; }
          fence_after();
          const uint32_t sa = smem_u32(smem + s * STAGE_BYTES);
          const uint32_t sb = sa + A_STAGE;
#pragma unroll
          for (int k = 0; k < BK / 32; ++k) {
            mma_f8(dtm, sdesc(sa + 32 * k), sdesc(sb + 32 * k), ID, (kb | k) != 0);
          }
          mma_commit(empty0 + 8 * s);   // stage free once these MMAs have read it
        }
        if (ok) mma_commit(tfull0 + 8 * buf);  // accumulator ready for the epilogue
      }
      // Drain outstanding MMAs before TMEM is released.
      if (it > 0) {
        const uint32_t j = it - 1;
        const long long t0 = clock64();
        while (!mbar_try_wait(empty0 + 8 * (j % STAGES), (j / STAGES) & 1) && clock64() - t0 < kTimeoutCycles) {
        }
      }
    }
  } else {
    // ------------------------------------------------------------- epilogue --
    const int quarter = warp & 3;          // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;      // column half of the tile
    const int row_in_tile = quarter * 32 + lane;
    int tc = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++tc) {
      int mb, nb;
      tile_coords(t, p, mb, nb);
      const int buf = tc & 1;
      const uint32_t tph = (tc >> 1) & 1;
      if (!mbar_wait(tfull0 + 8 * buf, tph, abort_flag, 4)) break;
      fence_after();
      const int m = mb * BM + row_in_tile;
      const bool mok = m < p.M;
      const float sa = mok ? __ldg(p.sa + m) : 0.f;
      drain_tile<OutT>(p, tmem_base + ((uint32_t)(quarter * 32) << 16) + buf * BN, m, mok, sa, nb, half);
      // hand the accumulator back to the MMA warp
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty0 + 8 * buf);
    }
    if (p.scatter) __threadfence_system();  // head-scatter: peer stores visible system-wide
  }

  fence_before();
  __syncthreads();
  fence_after();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                 : "memory");
  }
}

// ------------------------------------------------------- 2-SM variant --
// A CTA pair (cluster of 2) computes a 256 x 256 tile with tcgen05.mma
// cta_group::2: CTA r holds A rows [r*128, r*128+128) and B rows (N) of the same
// half in its own shared memory at identical offsets; the even CTA issues the
// MMAs, which read both CTAs' operands and write each CTA's 128 accumulator
// rows into that CTA's TMEM.  Per CTA and K-block only 32 KB cross L2 (16 KB of
// A + 16 KB of B) for 128 x 256 outputs, against 48 KB in the 1-SM kernel, and
// the ring is 6 stages deep.  Loads are plain per-CTA TMA loads (no multicast);
// their completion is counted on the even CTA's barrier (.cta_group::2).
constexpr int STAGES2 = 6;
constexpr int A2_STAGE = 128 * BK;   // 16 KB: this CTA's 128 rows of A
constexpr int B2_STAGE = 128 * BK;   // 16 KB: this CTA's 128 rows of B
constexpr int STAGE2_BYTES = A2_STAGE + B2_STAGE;

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t map_to_rank(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx_cluster(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_cluster(uint32_t bar, uint32_t parity, volatile int* abort_flag, int code) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > kTimeoutCycles) {
      *abort_flag = 1;
      atomicCAS(&g_fault, 0, code);
      return false;
    }
  }
}
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, int x, int y,
                                                 uint32_t leader_bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(leader_bar)
      : "memory");
}
__device__ __forceinline__ void mma_f8_pair(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t id, uint32_t accum) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n}\n" ::"r"(
          tmem_d),
      "l"(a), "l"(b), "r"(id), "r"(accum));
}
// Arrive (once all prior MMAs of this thread complete) on the barrier at the
// same shared-memory offset in both CTAs of the pair.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar) {
  asm volatile(
      "{\n .reg .b16 m;\n mov.b16 m, 3;\n"
      " tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n}\n" ::"r"(
          bar)
      : "memory");
}

__device__ __forceinline__ void tile_coords2(int t, int m_blocks, int n_blocks, int group, int& mb, int& nb) {
  const int GROUP = group;
  const int per_group = GROUP * n_blocks;
  const int g = t / per_group;
  const int first = g * GROUP;
  const int rows = min(GROUP, m_blocks - first);
  const int r = t % per_group;
  mb = first + r % rows;
  nb = r / rows;
}

template <typename OutT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    fp8_gemm_2sm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                        const Params p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES2 * STAGE2_BYTES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES2 + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const uint32_t full0 = smem_u32(bars);
  const uint32_t empty0 = smem_u32(bars + STAGES2);
  const uint32_t tfull0 = smem_u32(bars + 2 * STAGES2);
  const uint32_t tempty0 = smem_u32(bars + 2 * STAGES2 + 2);
  // p.m_blocks counts 256-row pair tiles here
  const int num_tiles = p.m_blocks * p.n_blocks;
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES2; ++s) {
      mbar_init(full0 + 8 * s, 1);    // leader only uses it: 1 expect_tx arrival + both CTAs' bytes
      mbar_init(empty0 + 8 * s, 1);   // one multicast commit per use
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull0 + 8 * b, 1);   // one multicast commit per tile
      mbar_init(tempty0 + 8 * b, 2 * EPI_WARPS);  // leader only: epilogue warps of both CTAs
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  fence_before();
  cluster_sync();
  fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer --
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_a)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_b)) : "memory");
      const uint32_t lfull0 = map_to_rank(full0, 0);
      uint32_t it = 0;
      bool ok = true;
      for (int t = pair; t < num_tiles && ok; t += npairs) {
        int mb, nb;
        tile_coords2(t, p.m_blocks, p.n_blocks, p.group, mb, nb);
        for (int kb = 0; kb < p.k_blocks; ++kb, ++it) {
          const int s = it % STAGES2;
          const uint32_t ph = (it / STAGES2) & 1;
          if (!mbar_wait(empty0 + 8 * s, ph ^ 1, abort_flag, 11)) { ok = false; break; }
          const uint32_t sa = smem_u32(smem + s * STAGE2_BYTES);
          if (leader) mbar_expect_tx_cluster(full0 + 8 * s, 2 * STAGE2_BYTES);
          tma_load_2d_pair(sa, &tmap_a, kb * BK, mb * 256 + rank * 128, lfull0 + 8 * s);
          tma_load_2d_pair(sa + A2_STAGE, &tmap_b, kb * BK, nb * BN + rank * 128, lfull0 + 8 * s);
        }
      }
      // Drain: the last use of each stage must be consumed (its empty phase completes)
      // before this CTA may exit, so no copy of ours is still in flight.
      const uint32_t n = it < (uint32_t)STAGES2 ? it : (uint32_t)STAGES2;
      for (uint32_t j = it - n; j < it; ++j) {
        const long long t0 = clock64();
        while (!mbar_try_wait(empty0 + 8 * (j % STAGES2), (j / STAGES2) & 1) && clock64() - t0 < kTimeoutCycles) {
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------- MMA issuer (even CTA) --
    if (leader && lane == 0) {
      constexpr uint32_t ID = idesc(256, BN);
      uint32_t it = 0;
      int tc = 0;
      bool ok = true;
      for (int t = pair; t < num_tiles && ok; t += npairs, ++tc) {
        const int buf = tc & 1;
        const uint32_t tph = (tc >> 1) & 1;
        if (!mbar_wait_cluster(tempty0 + 8 * buf, tph ^ 1, abort_flag, 12)) break;
        fence_after();
        const uint32_t dtm = tmem_base + buf * BN;
        for (int kb = 0; kb < p.k_blocks; ++kb, ++it) {
          const int s = it % STAGES2;
          const uint32_t ph = (it / STAGES2) & 1;
          if (!mbar_wait_cluster(full0 + 8 * s, ph, abort_flag, 13)) { ok = false; break; }
          fence_after();
          const uint32_t sa = smem_u32(smem + s * STAGE2_BYTES);
          const uint32_t sb = sa + A2_STAGE;
#pragma unroll
          for (int k = 0; k < BK / 32; ++k)
            mma_f8_pair(dtm, sdesc(sa + 32 * k), sdesc(sb + 32 * k), ID, (kb | k) != 0);
          mma_commit_pair(empty0 + 8 * s);
        }
        if (ok) mma_commit_pair(tfull0 + 8 * buf);
      }
      if (it > 0) {
        const uint32_t j = it - 1;
        const long long t0 = clock64();
        while (!mbar_try_wait(empty0 + 8 * (j % STAGES2), (j / STAGES2) & 1) && clock64() - t0 < kTimeoutCycles) {
        }
      }
    }
  } else {
    // ------------------------------------------------------------- epilogue --
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row_in_tile = quarter * 32 + lane;
    const uint32_t ltempty0 = map_to_rank(tempty0, 0);
    int tc = 0;
    for (int t = pair; t < num_tiles; t += npairs, ++tc) {
      int mb, nb;
      tile_coords2(t, p.m_blocks, p.n_blocks, p.group, mb, nb);
      const int buf = tc & 1;
      const uint32_t tph = (tc >> 1) & 1;
      if (!mbar_wait_cluster(tfull0 + 8 * buf, tph, abort_flag, 14)) break;
      fence_after();
      const int m = mb * 256 + (int)rank * 128 + row_in_tile;
      const bool mok = m < p.M;
      const float sa = mok ? __ldg(p.sa + m) : 0.f;
      drain_tile<OutT>(p, tmem_base + ((uint32_t)(quarter * 32) << 16) + buf * BN, m, mok, sa, nb, half);
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(ltempty0 + 8 * buf);
    }
    if (p.scatter) __threadfence_system();  // head-scatter: peer stores visible system-wide
  }

  fence_before();
  cluster_sync();
  fence_after();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                 : "memory");
  }
}

// ------------------------------------------------------------------- host --
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
    else
      cudaGetLastError();
  }
  return fn;
}

// 2-D K-major map over `rows` rows of `k` bytes with a box of box_rows x 128 B.
static bool make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t k, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)k};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// JOYOMNI_GEMM_2SM=0 selects the 1-SM kernel for every shape (A/B testing).
static bool use_2sm() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("JOYOMNI_GEMM_2SM");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

template <typename OutT>
int launch_2sm(const CUtensorMap& ta, const CUtensorMap& tb, Params p, cudaStream_t st) {
  const int smem = STAGES2 * STAGE2_BYTES + 1024 + 256;
  // The shared-memory opt-in and the occupancy query are per device: a
  // process may launch on several GPUs.
  const int dev = device_slot();
  static bool attr[kMaxDevices] = {};
  static int max_pairs_dev[kMaxDevices] = {};
  if (!attr[dev]) {
    cudaFuncSetAttribute(fp8_gemm_2sm_kernel<OutT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cudaLaunchConfig_t q = {};
    q.gridDim = dim3(2 * 74);
    q.blockDim = dim3(THREADS);
    q.dynamicSmemBytes = smem;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    q.attrs = at;
    q.numAttrs = 1;
    int nc = 0;
    if (cudaOccupancyMaxActiveClusters(&nc, fp8_gemm_2sm_kernel<OutT>, &q) != cudaSuccess || nc <= 0) {
      cudaGetLastError();
      nc = sm_count() / 2;
    }
    max_pairs_dev[dev] = nc;
    attr[dev] = true;
  }
  const int max_pairs = max_pairs_dev[dev];
  p.m_blocks = (p.M + 255) / 256;
  static int group_env = -1;
  if (group_env < 0) {
    const char* e = getenv("JOYOMNI_GEMM_GROUP");
    group_env = e ? atoi(e) : 0;
  }
  // Rasterisation: GROUP pair-tile rows (A panel of GROUP*256 rows) share each
  // sweep over N.  ~28 MB of A per group keeps both the A panel and the B
  // panels being swept resident in L2 (measured at M = 10530, K = 5120: group
  // 21 reads 219 MB from DRAM against 515 MB for group 8, and runs 4 % faster
  // under the power cap).
  p.group = group_env > 0 ? group_env : (int)((28LL << 20) / (256LL * p.K));
  if (p.group < 4) p.group = 4;
  if (p.group > p.m_blocks) p.group = p.m_blocks;
  const int tiles = p.m_blocks * p.n_blocks;
  const int pairs = tiles < max_pairs ? tiles : max_pairs;
  if (getenv("JOYOMNI_GEMM_DEBUG"))
    fprintf(stderr, "[jo gemm 2sm] max_pairs %d tiles %d grid %d smem %d\n", max_pairs, tiles, 2 * pairs, smem);
  fp8_gemm_2sm_kernel<OutT><<<2 * pairs, THREADS, smem, st>>>(ta, tb, p);
  return check_launch("fp8_scaled_mm");
}

struct ScatterSpec {
  int width, dh, hpr;
  int64_t tok0;
  void* dst[24];
};

template <typename OutT>
int launch(const void* A, const void* B, const float* sa, const float* sb, const void* bias, void* D, int64_t M,
           int64_t N, int64_t K, int epi, const void* resid, const void* gate, cudaStream_t st,
           const ScatterSpec* sc = nullptr) {
  CUtensorMap ta, tb;
  const bool pair = M > 128 && use_2sm();
  if (!make_map(&ta, A, M, K, BM) || !make_map(&tb, B, N, K, pair ? 128 : BN)) {
    set_error("fp8_scaled_mm: cuTensorMapEncodeTiled failed (pointer %p/%p, M %lld N %lld K %lld)", A, B,
              (long long)M, (long long)N, (long long)K);
    return JO_ERR_CUDA;
  }
  Params p;
  p.d = D;
  p.sa = sa;
  p.sb = sb;
  p.bias = bias;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.m_blocks = (int)((M + BM - 1) / BM);
  p.n_blocks = (int)((N + BN - 1) / BN);
  p.k_blocks = (int)((K + BK - 1) / BK);
  p.epilogue = epi;
  p.resid = resid;
  p.gate = gate;
  p.scatter = sc != nullptr;
  p.sc_width = sc ? sc->width : 0;
  p.sc_dh = sc ? sc->dh : 0;
  p.sc_hpr = sc ? sc->hpr : 0;
  p.sc_tok0 = sc ? sc->tok0 : 0;
  for (int i = 0; i < 24; ++i) p.sc_dst[i] = sc ? sc->dst[i] : nullptr;
  if (pair) return launch_2sm<OutT>(ta, tb, p, st);
  const int smem = STAGES * STAGE_BYTES + 1024 + 256;
  const int dev = device_slot();
  static bool attr[kMaxDevices] = {};
  if (!attr[dev]) {
    cudaFuncSetAttribute(fp8_gemm_kernel<OutT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    attr[dev] = true;
  }
  const int tiles = p.m_blocks * p.n_blocks;
  const int grid = tiles < sm_count() ? tiles : sm_count();
  fp8_gemm_kernel<OutT><<<grid, THREADS, smem, st>>>(ta, tb, p);
  return check_launch("fp8_scaled_mm");
}

}  // namespace gemm
}  // namespace jo

extern "C" {

int jo_fp8_scaled_mm_ex(const void* mat_a, const void* mat_b, const float* scales_a, const float* scales_b,
                        const void* bias, void* out, int64_t M, int64_t N, int64_t K, int out_dtype, int epilogue,
                        const void* residual, const void* gate, void* stream) {
  using namespace jo;
  const char* what = "fp8_scaled_mm";
  JO_REQUIRE(out_dtype == JO_DTYPE_BF16 || out_dtype == JO_DTYPE_F16, JO_ERR_DTYPE,
             "out_dtype must be Half or BFloat16");
  JO_REQUIRE(epilogue == JO_EPI_NONE || epilogue == JO_EPI_GELU_TANH || epilogue == JO_EPI_RESID_GATE,
             JO_ERR_INVALID, "%s: unknown epilogue %d", what, epilogue);
  JO_REQUIRE(epilogue != JO_EPI_RESID_GATE || (residual && gate), JO_ERR_INVALID,
             "%s: the gated-residual epilogue needs residual and gate", what);
  JO_REQUIRE(M >= 0 && N >= 0 && K >= 0 && M < (1LL << 31) && N < (1LL << 31) && K < (1LL << 31), JO_ERR_INVALID,
             "%s: invalid shape", what);
  JO_REQUIRE(K % 16 == 0, JO_ERR_INVALID, "mat_a must be multiple of 16 bytes for memory alignment");
  JO_REQUIRE((N * 2) % 16 == 0, JO_ERR_INVALID, "out must be multiple of 16 bytes for memory alignment");
  JO_REQUIRE(M == 0 || N == 0 || (mat_a && mat_b && scales_a && scales_b && out), JO_ERR_INVALID,
             "%s: null tensor pointer", what);
  JO_REQUIRE(aligned16(mat_a) && aligned16(mat_b) && aligned16(out) && aligned16(scales_b) &&
                 (!bias || aligned8(bias)),
             JO_ERR_ALIGN, "%s: operands must be 16-byte aligned (bias 8-byte)", what);
  int st = require_sm100();
  if (st != JO_OK) return st;
  if (M == 0 || N == 0) return JO_OK;
  JO_REQUIRE(K > 0, JO_ERR_INVALID, "%s: K must be positive", what);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return out_dtype == JO_DTYPE_BF16
             ? gemm::launch<__nv_bfloat16>(mat_a, mat_b, scales_a, scales_b, bias, out, M, N, K, epilogue, residual,
                                           gate, s)
             : gemm::launch<__half>(mat_a, mat_b, scales_a, scales_b, bias, out, M, N, K, epilogue, residual, gate,
                                    s);
}

int jo_fp8_scaled_mm(const void* mat_a, const void* mat_b, const float* scales_a, const float* scales_b,
                     const void* bias, void* out, int64_t M, int64_t N, int64_t K, int out_dtype, int epilogue,
                     void* stream) {
  if (epilogue == JO_EPI_RESID_GATE) {
    jo::set_error("fp8_scaled_mm: the gated-residual epilogue needs jo_fp8_scaled_mm_ex");
    return JO_ERR_INVALID;
  }
  return jo_fp8_scaled_mm_ex(mat_a, mat_b, scales_a, scales_b, bias, out, M, N, K, out_dtype, epilogue, nullptr,
                             nullptr, stream);
}

// FP8 GEMM whose epilogue scatters each (row, head) of the [M, parts*ranks*
// heads_per_rank*head_dim] result to the rank that owns the head (the
// sequence-parallel all-to-all fused into the GEMM).  dst[part * ranks + r] is
// rank r's [tokens, heads_per_rank, head_dim] buffer for part `part` (a peer
// pointer for r != this rank, opened with jo_ipc_open) of dst_tokens token
// rows; row m lands at token tok0 + m < dst_tokens.  Stores only (no TMA, no multicast); each epilogue thread ends
// with a system-scope fence, and the caller orders the consumers after a
// cross-rank synchronisation.
int jo_fp8_scaled_mm_scatter(const void* mat_a, const void* mat_b, const float* scales_a, const float* scales_b,
                             const void* bias, int64_t M, int64_t N, int64_t K, int out_dtype,
                             const void* const* dst, int parts, int ranks, int heads_per_rank, int head_dim,
                             int64_t tok0, int64_t dst_tokens, void* stream) {
  using namespace jo;
  const char* what = "fp8_scaled_mm_scatter";
  JO_REQUIRE(out_dtype == JO_DTYPE_BF16 || out_dtype == JO_DTYPE_F16, JO_ERR_DTYPE,
             "out_dtype must be Half or BFloat16");
  JO_REQUIRE(parts >= 1 && parts <= 3 && ranks >= 1 && ranks <= 8 && heads_per_rank >= 1 && head_dim >= 32 &&
                 head_dim % 32 == 0 && tok0 >= 0,
             JO_ERR_INVALID, "%s: parts 1..3, ranks 1..8, head_dim a multiple of 32, tok0 >= 0", what);
  JO_REQUIRE(N == (int64_t)parts * ranks * heads_per_rank * head_dim, JO_ERR_INVALID,
             "%s: N (%lld) must equal parts * ranks * heads_per_rank * head_dim", what, (long long)N);
  JO_REQUIRE(M >= 0 && K > 0 && M < (1LL << 31) && N < (1LL << 31) && K < (1LL << 31) && K % 16 == 0,
             JO_ERR_INVALID, "%s: invalid shape", what);
  JO_REQUIRE(M == 0 || (mat_a && mat_b && scales_a && scales_b && dst), JO_ERR_INVALID, "%s: null pointer", what);
  // Every destination holds dst_tokens token rows; rows tok0 .. tok0+M-1 must
  // fit, since a destination may be another GPU's memory.
  JO_REQUIRE(dst_tokens >= 0 && tok0 + M <= dst_tokens, JO_ERR_INVALID,
             "%s: rows %lld..%lld do not fit destinations of %lld tokens", what, (long long)tok0,
             (long long)(tok0 + M), (long long)dst_tokens);
  JO_REQUIRE(aligned16(mat_a) && aligned16(mat_b) && aligned16(scales_b) && (!bias || aligned8(bias)),
             JO_ERR_ALIGN, "%s: operands must be 16-byte aligned (bias 8-byte)", what);
  gemm::ScatterSpec sc;
  sc.width = ranks * heads_per_rank * head_dim;
  sc.dh = head_dim;
  sc.hpr = heads_per_rank;
  sc.tok0 = tok0;
  for (int i = 0; i < 24; ++i) sc.dst[i] = nullptr;
  for (int part = 0; part < parts; ++part)
    for (int r = 0; r < ranks; ++r) {
      void* d = const_cast<void*>(dst[part * ranks + r]);
      JO_REQUIRE(d && aligned16(d), JO_ERR_ALIGN, "%s: destination %d of part %d is null or not 16-byte aligned",
                 what, r, part);
      sc.dst[part * 8 + r] = d;
    }
  int st = require_sm100();
  if (st != JO_OK) return st;
  if (M == 0) return JO_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return out_dtype == JO_DTYPE_BF16
             ? gemm::launch<__nv_bfloat16>(mat_a, mat_b, scales_a, scales_b, bias, sc.dst[0], M, N, K, JO_EPI_NONE,
                                           nullptr, nullptr, s, &sc)
             : gemm::launch<__half>(mat_a, mat_b, scales_a, scales_b, bias, sc.dst[0], M, N, K, JO_EPI_NONE, nullptr,
                                    nullptr, s, &sc);
}

// Fault code of the GEMM kernel's bounded waits (0 = none) and reset.  Reads
// a device symbol synchronously; intended for tests and diagnostics only.
int jo_gemm_last_fault(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, jo::gemm::g_fault, sizeof(int)) != cudaSuccess) {
    cudaGetLastError();
    return JO_ERR_CUDA;
  }
  if (reset) {
    int z = 0;
    cudaMemcpyToSymbol(jo::gemm::g_fault, &z, sizeof(int));
  }
  return v;
}

}  // extern "C"
