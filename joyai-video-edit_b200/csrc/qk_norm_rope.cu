// Fused per-head RMSNorm + interleaved-pair 3D RoPE, in place on q and k (bf16).
// Reference: deploy/joyomni_ops/csrc/fused_qknorm_rope_3d_kernel.cu:56-143 (kernel),
//            :179-208 (host checks).
//
// Design (B200): one head vector (D bf16) is owned by D/8 lanes that each move
// one 16-byte vector, so a warp covers 32*8/D heads ("slot group") and every
// access is a full 16-byte coalesced load/store.  The same lanes process the q
// and the k vector of a (token, head) slot, so the per-lane norm weights live
// in registers and the token's cos/sin entries are fetched once for both.
// The default kernel is persistent (one wave): each warp walks a contiguous
// run of slot groups with an incremental (token, head) cursor while a per-
// thread cp.async ring in shared memory keeps the next groups in flight.
//
// Numerics: the sum of squares is accumulated and reduced in exactly the
// reference's order.  The reference gives each of 32 lanes D/32 consecutive
// elements, accumulates them with fused multiply-adds, then reduces with an xor
// butterfly over lane masks 16,8,4,2,1.  Here a lane holds P = 256/D reference
// partials; they are kept separate through the butterfly over the high lane bits
// and combined locally in the order of the low bits, which reproduces the
// reference sum bit for bit.  Scaling, weighting and rotation use the
// reference's expression forms (x * (r * w); x1*c - x2*s; x1*s + x2*c).
#include "jo_common.cuh"

#include <stdlib.h>

namespace jo {
namespace {

// q_ts / k_ts: elements between consecutive tokens (num_heads * D when dense);
// heads of a token are D elements apart.  ROPE = false normalises only.
template <int D, int U, bool ROPE>
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(
    __nv_bfloat16* __restrict__ q, __nv_bfloat16* __restrict__ k, int64_t slots, int seq_len, int num_heads,
    float eps, const __nv_bfloat16* __restrict__ qw, const __nv_bfloat16* __restrict__ kw,
    const __nv_bfloat16* __restrict__ cosp, const __nv_bfloat16* __restrict__ sinp, int64_t q_ts, int64_t k_ts) {
  constexpr int LPH = D / 8;        // lanes per head vector
  constexpr int HPW = 32 / LPH;     // head slots per warp per group
  constexpr int P = 256 / D;        // reference lanes folded into one lane
  constexpr int EP = 8 / P;         // elements per reference partial
  const int lane = threadIdx.x & 31;
  const int hl = lane % LPH;        // lane within the head
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;

  Vec16<__nv_bfloat16> wq, wk;
  wq.raw = ld_cached(qw + hl * 8);
  wk.raw = ld_cached(kw + hl * 8);

  Vec16<__nv_bfloat16> vq[U], vk[U];
  int64_t slot[U], qo[U], ko[U];
  uint32_t tokr[U];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    slot[u] = (warp * U + u) * HPW + lane / LPH;
    // (batch, token) row and head of the slot; the host guarantees
    // slots < 2^31, so 32-bit division suffices (64-bit division would cost
    // ~10 instructions per element here).
    const uint32_t s32 = (uint32_t)slot[u];
    const uint32_t tok = s32 / (uint32_t)num_heads;
    const uint32_t head = s32 - tok * (uint32_t)num_heads;
    tokr[u] = tok;
    qo[u] = (int64_t)tok * q_ts + head * D + hl * 8;
    ko[u] = (int64_t)tok * k_ts + head * D + hl * 8;
    if (slot[u] < slots) {
      vq[u].raw = ld_stream(q + qo[u]);
      vk[u].raw = ld_stream(k + ko[u]);
    }
  }

#pragma unroll
  for (int u = 0; u < U; ++u) {
    const bool ok = slot[u] < slots;
    const uint32_t tk = tokr[u];
    const int64_t token = !ok ? 0 : (tk < (uint32_t)seq_len ? tk : tk % (uint32_t)seq_len);
    // cos/sin entries for this lane's 4 pairs: indices hl*4 .. hl*4+3.
    uint2 c2 = make_uint2(0, 0), s2 = make_uint2(0, 0);
    if (ROPE) {
      c2 = __ldg(reinterpret_cast<const uint2*>(cosp + token * (D / 2) + hl * 4));
      s2 = __ldg(reinterpret_cast<const uint2*>(sinp + token * (D / 2) + hl * 4));
    }
    const __nv_bfloat16* cv = reinterpret_cast<const __nv_bfloat16*>(&c2);
    const __nv_bfloat16* sv = reinterpret_cast<const __nv_bfloat16*>(&s2);
#pragma unroll
    for (int which = 0; which < 2; ++which) {
      Vec16<__nv_bfloat16>& v = which ? vk[u] : vq[u];
      const Vec16<__nv_bfloat16>& w = which ? wk : wq;
      float e[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) e[j] = ok ? v.get(j) : 0.f;
      float part[P];
#pragma unroll
      for (int p = 0; p < P; ++p) {
        float acc = 0.f;
#pragma unroll
        for (int j = 0; j < EP; ++j) acc = __fmaf_rn(e[p * EP + j], e[p * EP + j], acc);
        part[p] = acc;
      }
      // Butterfly over the reference lane bits held in different lanes
      // (highest first), each partial separately.
#pragma unroll
      for (int m = LPH / 2; m > 0; m >>= 1)
#pragma unroll
        for (int p = 0; p < P; ++p) part[p] += __shfl_xor_sync(0xffffffffu, part[p], m, 32);
      // Remaining reference lane bits live inside this lane.
#pragma unroll
      for (int m = P / 2; m > 0; m >>= 1)
#pragma unroll
        for (int p = 0; p < m; ++p) part[p] = part[p] + part[p + m];
      const float rms_rcp = rsqrtf(part[0] / static_cast<float>(D) + eps);
#pragma unroll
      for (int j = 0; j < 8; ++j) e[j] *= rms_rcp * w.get(j);
      if (!ROPE) {
#pragma unroll
        for (int j = 0; j < 8; j += 2)
          reinterpret_cast<__nv_bfloat162*>(&v.raw)[j / 2] = __float22bfloat162_rn(make_float2(e[j], e[j + 1]));
        continue;
      }
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        const float c = __bfloat162float(cv[j / 2]);
        const float s = __bfloat162float(sv[j / 2]);
        const float x1 = e[j], x2 = e[j + 1];
        const float o0 = x1 * c - x2 * s;
        const float o1 = x1 * s + x2 * c;
        __nv_bfloat162 o = __float22bfloat162_rn(make_float2(o0, o1));
        reinterpret_cast<__nv_bfloat162*>(&v.raw)[j / 2] = o;
      }
    }
    if (ok) {
      st_stream(q + qo[u], vq[u].raw);
      st_stream(k + ko[u], vk[u].raw);
    }
  }
}

// One (token, head) slot's q or k vector of this lane: RMS over the head in
// the reference's summation order, weight, then the interleaved-pair rotation.
// The lane holds EL consecutive elements of the head (EL / 8 16-byte words),
// i.e. the partials of P = EL / (D / 32) consecutive lanes of the reference's
// 32-lane reduction; they are kept separate through the butterfly over the
// lane bits held by other lanes and combined locally in the order of the
// remaining bits, which reproduces the reference sum bit for bit (every lane
// of an xor butterfly ends with the same bits).  wf: this lane's EL weights;
// cf / sf: its EL / 2 cos / sin entries (shared by q and k of the slot).
template <int D, int EL, bool ROPE>
__device__ __forceinline__ void norm_rope_lane(uint4 (&v)[EL / 8], const float (&wf)[EL], const float (&cf)[EL / 2],
                                               const float (&sf)[EL / 2], float eps) {
  constexpr int LPH = D / EL;
  constexpr int EP = D / 32;
  constexpr int P = EL / EP;
  float e[EL];
#pragma unroll
  for (int j = 0; j < EL; j += 2) {
    const float2 f = unpack2<__nv_bfloat16>((&v[j / 8].x)[(j % 8) / 2]);
    e[j] = f.x;
    e[j + 1] = f.y;
  }
  float part[P];
#pragma unroll
  for (int p = 0; p < P; ++p) {
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < EP; ++j) acc = __fmaf_rn(e[p * EP + j], e[p * EP + j], acc);
    part[p] = acc;
  }
#pragma unroll
  for (int m = LPH / 2; m > 0; m >>= 1)
#pragma unroll
    for (int p = 0; p < P; ++p) part[p] += __shfl_xor_sync(0xffffffffu, part[p], m, 32);
#pragma unroll
  for (int m = P / 2; m > 0; m >>= 1)
#pragma unroll
    for (int p = 0; p < m; ++p) part[p] = part[p] + part[p + m];
  const float rms_rcp = rsqrtf(part[0] / static_cast<float>(D) + eps);
#pragma unroll
  for (int j = 0; j < EL; ++j) e[j] *= rms_rcp * wf[j];
#pragma unroll
  for (int j = 0; j < EL; j += 2) {
    float o0 = e[j], o1 = e[j + 1];
    if (ROPE) {
      const float c = cf[j / 2], s = sf[j / 2];
      const float x1 = e[j], x2 = e[j + 1];
      o0 = x1 * c - x2 * s;
      o1 = x1 * s + x2 * c;
    }
    (&v[j / 8].x)[(j % 8) / 2] = pack2<__nv_bfloat16>(o0, o1);
  }
}

__device__ __forceinline__ void cpa16(void* smem, const void* g) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((unsigned)__cvta_generic_to_shared(smem)), "l"(g)
               : "memory");
}
__device__ __forceinline__ void cpa8(void* smem, const void* g) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"((unsigned)__cvta_generic_to_shared(smem)), "l"(g)
               : "memory");
}
__device__ __forceinline__ void cpa_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cpa_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Ring form, persistent: the grid is one wave (blocks per SM x SMs) and every
// warp owns a contiguous run of slot groups (HPW slots each, so mostly heads
// of one token), balanced to within one group, which it walks with a cursor
// (token, head, position in the RoPE table) advanced by HPW heads per group --
// no division per group.  Each lane moves EL elements of a head.  The groups
// ahead are staged by each thread into its own shared-memory slots with
// cp.async (S - 1 groups in flight per thread at no register cost); a thread
// only reads back the slots it filled itself, after cp.async.wait_group, so no
// barrier is needed.  Slot layout [stage][word][thread] (dynamic shared
// memory): consecutive threads touch consecutive 16-byte words
// (conflict-free).  Every lane of a warp runs the same number of iterations
// (the head reduction shuffles need the full warp); slots past the end are
// masked.
template <int EL>
struct RingWords {
  static constexpr int V = EL / 8;            // 16-byte words of q (and of k)
  static constexpr int CS = EL == 8 ? 1 : 2;  // words of cos + sin
  static constexpr int N = 2 * V + CS;
};

template <int D, int EL, int S, bool ROPE>
__global__ void __launch_bounds__(256) qk_norm_rope_ring(
    __nv_bfloat16* __restrict__ q, __nv_bfloat16* __restrict__ k, int64_t slots, int seq_len, int num_heads,
    float eps, const __nv_bfloat16* __restrict__ qw, const __nv_bfloat16* __restrict__ kw,
    const __nv_bfloat16* __restrict__ cosp, const __nv_bfloat16* __restrict__ sinp, int64_t q_ts, int64_t k_ts) {
  constexpr int LPH = D / EL;
  constexpr int HPW = 32 / LPH;
  constexpr int V = RingWords<EL>::V;
  constexpr int NW = RingWords<EL>::N;
  extern __shared__ uint4 ring_raw[];
  auto slotw = [&](int stage, int w) -> uint4* { return ring_raw + ((size_t)stage * NW + w) * 256 + threadIdx.x; };
  const int lane = threadIdx.x & 31;
  const int hl = lane % LPH;
  const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const uint32_t nwarps = (gridDim.x * blockDim.x) >> 5;

  // this warp's groups [g0, g0 + ng): the first `rem` warps take one extra
  const uint32_t groups = (uint32_t)((slots + HPW - 1) / HPW);
  const uint32_t base = groups / nwarps, rem = groups % nwarps;
  const uint32_t g0 = warp * base + (warp < rem ? warp : rem);
  const int ng = (int)(base + (warp < rem ? 1 : 0));
  if (ng == 0) return;  // warp-uniform

  float wqf[EL], wkf[EL];
#pragma unroll
  for (int w = 0; w < V; ++w) {
    Vec16<__nv_bfloat16> a, b;
    a.raw = ld_cached(qw + hl * EL + w * 8);
    b.raw = ld_cached(kw + hl * EL + w * 8);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      wqf[w * 8 + j] = a.get(j);
      wkf[w * 8 + j] = b.get(j);
    }
  }

  struct Cursor {
    uint32_t slot, tok, head, tr;
  };
  Cursor ci;  // issue cursor (runs S - 1 groups ahead)
  ci.slot = g0 * HPW + lane / LPH;
  ci.tok = ci.slot / (uint32_t)num_heads;
  ci.head = ci.slot - ci.tok * (uint32_t)num_heads;
  ci.tr = ci.tok < (uint32_t)seq_len ? ci.tok : ci.tok % (uint32_t)seq_len;
  Cursor cc = ci;  // compute cursor
  auto advance = [&](Cursor& c) {
    c.slot += HPW;
    c.head += HPW;
    while (c.head >= (uint32_t)num_heads) {
      c.head -= (uint32_t)num_heads;
      ++c.tok;
      if (++c.tr == (uint32_t)seq_len) c.tr = 0;
    }
  };
  auto issue = [&](int stage) {
    if (ci.slot < (uint64_t)slots) {
      const __nv_bfloat16* qs = q + ((int64_t)ci.tok * q_ts + ci.head * D + hl * EL);
      const __nv_bfloat16* ks = k + ((int64_t)ci.tok * k_ts + ci.head * D + hl * EL);
#pragma unroll
      for (int w = 0; w < V; ++w) {
        cpa16(slotw(stage, w), qs + w * 8);
        cpa16(slotw(stage, V + w), ks + w * 8);
      }
      if (ROPE) {
        const __nv_bfloat16* cs = cosp + (int64_t)ci.tr * (D / 2) + hl * (EL / 2);
        const __nv_bfloat16* ss = sinp + (int64_t)ci.tr * (D / 2) + hl * (EL / 2);
        if constexpr (EL == 8) {
          uint2* d = reinterpret_cast<uint2*>(slotw(stage, 2 * V));
          cpa8(d, cs);
          cpa8(d + 1, ss);
        } else {
          cpa16(slotw(stage, 2 * V), cs);
          cpa16(slotw(stage, 2 * V + 1), ss);
        }
      }
    }
    cpa_commit();
    advance(ci);
  };

#pragma unroll
  for (int g = 0; g < S - 1; ++g) {
    if (g < ng) issue(g);
    else cpa_commit();  // keep the group count uniform for wait_group
  }
  int si = S - 1, sc = 0;  // ring stage of the next issue / of the next compute
  for (int g = 0; g < ng; ++g) {
    if (g + S - 1 < ng) issue(si);
    else cpa_commit();
    si = si + 1 == S ? 0 : si + 1;
    cpa_wait<S - 1>();
    const bool ok = cc.slot < (uint64_t)slots;
    uint4 vq[V], vk[V];
    float cf[EL / 2], sf[EL / 2];
#pragma unroll
    for (int w = 0; w < V; ++w) {
      vq[w] = ok ? *slotw(sc, w) : make_uint4(0, 0, 0, 0);
      vk[w] = ok ? *slotw(sc, V + w) : make_uint4(0, 0, 0, 0);
    }
    if (ROPE) {
      uint32_t cw[EL / 4], sw[EL / 4];
      if constexpr (EL == 8) {
        const uint4 cs = ok ? *slotw(sc, 2 * V) : make_uint4(0, 0, 0, 0);
        cw[0] = cs.x; cw[1] = cs.y; sw[0] = cs.z; sw[1] = cs.w;
      } else {
        const uint4 c4 = ok ? *slotw(sc, 2 * V) : make_uint4(0, 0, 0, 0);
        const uint4 s4 = ok ? *slotw(sc, 2 * V + 1) : make_uint4(0, 0, 0, 0);
        cw[0] = c4.x; cw[1] = c4.y; cw[2] = c4.z; cw[3] = c4.w;
        sw[0] = s4.x; sw[1] = s4.y; sw[2] = s4.z; sw[3] = s4.w;
      }
#pragma unroll
      for (int j = 0; j < EL / 4; ++j) {
        const float2 c = unpack2<__nv_bfloat16>(cw[j]), sn = unpack2<__nv_bfloat16>(sw[j]);
        cf[2 * j] = c.x; cf[2 * j + 1] = c.y;
        sf[2 * j] = sn.x; sf[2 * j + 1] = sn.y;
      }
    } else {
#pragma unroll
      for (int j = 0; j < EL / 2; ++j) cf[j] = sf[j] = 0.f;
    }
    sc = sc + 1 == S ? 0 : sc + 1;
    norm_rope_lane<D, EL, ROPE>(vq, wqf, cf, sf, eps);
    norm_rope_lane<D, EL, ROPE>(vk, wkf, cf, sf, eps);
    if (ok) {
      __nv_bfloat16* qd = q + ((int64_t)cc.tok * q_ts + cc.head * D + hl * EL);
      __nv_bfloat16* kd = k + ((int64_t)cc.tok * k_ts + cc.head * D + hl * EL);
#pragma unroll
      for (int w = 0; w < V; ++w) {
        st_stream(qd + w * 8, vq[w]);
        st_stream(kd + w * 8, vk[w]);
      }
    }
    advance(cc);
  }
  cpa_wait<0>();
}

template <int D, int EL, int S>
int launch_ring(void* q, void* k, int64_t slots, int seq_len, int num_heads, float eps, const void* qw,
                const void* kw, const void* c, const void* s, int64_t q_ts, int64_t k_ts, cudaStream_t st) {
  constexpr int HPW = 32 / (D / EL);
  auto* qp = static_cast<__nv_bfloat16*>(q);
  auto* kp = static_cast<__nv_bfloat16*>(k);
  auto* qwp = static_cast<const __nv_bfloat16*>(qw);
  auto* kwp = static_cast<const __nv_bfloat16*>(kw);
  auto* cp = static_cast<const __nv_bfloat16*>(c);
  auto* sp = static_cast<const __nv_bfloat16*>(s);
  auto kern = c ? qk_norm_rope_ring<D, EL, S, true> : qk_norm_rope_ring<D, EL, S, false>;
  const int smem = S * RingWords<EL>::N * 256 * 16;
  static int per_sm[kMaxDevices][2] = {};
  int& bps = per_sm[device_slot()][c ? 1 : 0];
  if (bps == 0) {
    cudaFuncSetAttribute(qk_norm_rope_ring<D, EL, S, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cudaFuncSetAttribute(qk_norm_rope_ring<D, EL, S, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&bps, kern, 256, smem) != cudaSuccess || bps < 1) {
      cudaGetLastError();
      bps = 1;
    }
  }
  const int64_t groups = (slots + HPW - 1) / HPW;
  const int64_t need = (groups + 7) / 8;  // one group per warp at least
  const int64_t wave = (int64_t)bps * sm_count();
  const int64_t blocks = need < wave ? need : wave;
  kern<<<(unsigned)blocks, 256, smem, st>>>(qp, kp, slots, seq_len, num_heads, eps, qwp, kwp, cp, sp, q_ts, k_ts);
  return check_launch("fused_qk_norm_rope_3d_paired");
}

template <int D, int U>
int launch_u(void* q, void* k, int64_t slots, int seq_len, int num_heads, float eps, const void* qw, const void* kw,
             const void* c, const void* s, int64_t q_ts, int64_t k_ts, cudaStream_t st) {
  constexpr int HPW = 32 / (D / 8);
  const int64_t warps = (slots + (int64_t)HPW * U - 1) / ((int64_t)HPW * U);
  const int64_t blocks = (warps + 7) / 8;
  auto* qp = static_cast<__nv_bfloat16*>(q);
  auto* kp = static_cast<__nv_bfloat16*>(k);
  auto* qwp = static_cast<const __nv_bfloat16*>(qw);
  auto* kwp = static_cast<const __nv_bfloat16*>(kw);
  auto* cp = static_cast<const __nv_bfloat16*>(c);
  auto* sp = static_cast<const __nv_bfloat16*>(s);
  if (c)
    qk_norm_rope_kernel<D, U, true><<<(unsigned)blocks, 256, 0, st>>>(qp, kp, slots, seq_len, num_heads, eps, qwp,
                                                                      kwp, cp, sp, q_ts, k_ts);
  else
    qk_norm_rope_kernel<D, U, false><<<(unsigned)blocks, 256, 0, st>>>(qp, kp, slots, seq_len, num_heads, eps, qwp,
                                                                       kwp, cp, sp, q_ts, k_ts);
  return check_launch("fused_qk_norm_rope_3d_paired");
}

// Kernel choice for measurements: JO_QKR_U=1/2 selects the one-shot kernel
// (one slot group per warp, U groups), JO_QKR_S=2/4 the ring depth of the
// persistent ring kernel (default, 3 stages); JO_QKR_EL=16 selects 16-element
// lanes (8 is the default), used only when cos/sin are 16-byte aligned.
static int env_int(const char* name, int dflt) {
  const char* e = getenv(name);
  return e ? atoi(e) : dflt;
}

template <int D>
int launch(void* q, void* k, int64_t slots, int seq_len, int num_heads, float eps, const void* qw, const void* kw,
           const void* c, const void* s, int64_t q_ts, int64_t k_ts, cudaStream_t st) {
  // 8 elements per lane (D / 8 lanes per head) by default; JO_QKR_EL=16 gives
  // each lane 16 (fewer shuffles and per-slot overhead per element, but 104
  // registers: measured 26.7 against 16.2 us on config 1).
  static const int u = env_int("JO_QKR_U", 0), ring = env_int("JO_QKR_S", 3), el = env_int("JO_QKR_EL", 8);
  if (u == 1) return launch_u<D, 1>(q, k, slots, seq_len, num_heads, eps, qw, kw, c, s, q_ts, k_ts, st);
  if (u == 2) return launch_u<D, 2>(q, k, slots, seq_len, num_heads, eps, qw, kw, c, s, q_ts, k_ts, st);
  // 16-element lanes stage cos / sin rows with 16-byte copies: tables that are
  // only 8-byte aligned take the 8-element form.
  if (el != 16 || (c && !(aligned16(c) && aligned16(s)))) {
    if (ring == 2) return launch_ring<D, 8, 2>(q, k, slots, seq_len, num_heads, eps, qw, kw, c, s, q_ts, k_ts, st);
    if (ring == 4) return launch_ring<D, 8, 4>(q, k, slots, seq_len, num_heads, eps, qw, kw, c, s, q_ts, k_ts, st);
    return launch_ring<D, 8, 3>(q, k, slots, seq_len, num_heads, eps, qw, kw, c, s, q_ts, k_ts, st);
  }
  if (ring == 2) return launch_ring<D, 16, 2>(q, k, slots, seq_len, num_heads, eps, qw, kw, c, s, q_ts, k_ts, st);
  if (ring == 4) return launch_ring<D, 16, 4>(q, k, slots, seq_len, num_heads, eps, qw, kw, c, s, q_ts, k_ts, st);
  return launch_ring<D, 16, 3>(q, k, slots, seq_len, num_heads, eps, qw, kw, c, s, q_ts, k_ts, st);
}

}  // namespace
}  // namespace jo

extern "C" int jo_fused_qk_norm_rope_3d_paired(void* q, void* k, int64_t batch, int64_t seq_len, int64_t num_heads,
                                               int64_t head_dim, float eps, const void* q_weight,
                                               const void* k_weight, const void* cos, const void* sin,
                                               void* stream) {
  using namespace jo;
  JO_REQUIRE(batch >= 0 && seq_len >= 0 && num_heads >= 0, JO_ERR_INVALID,
             "fused_qk_norm_rope_3d_paired: negative size");
  JO_REQUIRE(head_dim == 64 || head_dim == 128 || head_dim == 256, JO_ERR_INVALID,
             "Unsupported head_dim for fused_qk_norm_rope_3d_paired: %lld", (long long)head_dim);
  JO_REQUIRE(seq_len < (1LL << 31) && num_heads < (1LL << 31), JO_ERR_INVALID,
             "fused_qk_norm_rope_3d_paired: size too large");
  const int64_t slots = batch * seq_len * num_heads;
  JO_REQUIRE(slots < (1LL << 31), JO_ERR_INVALID, "fused_qk_norm_rope_3d_paired: too many (token, head) slots");
  JO_REQUIRE(slots == 0 || (q && k && q_weight && k_weight && cos && sin), JO_ERR_INVALID,
             "fused_qk_norm_rope_3d_paired: null tensor pointer");
  JO_REQUIRE(aligned16(q) && aligned16(k) && aligned16(q_weight) && aligned16(k_weight) && aligned8(cos) &&
                 aligned8(sin),
             JO_ERR_ALIGN, "fused_qk_norm_rope_3d_paired: q/k/weights must be 16-byte aligned, cos/sin 8-byte");
  int st = require_sm100();
  if (st != JO_OK) return st;
  if (slots == 0) return JO_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t ts = num_heads * head_dim;
  switch (head_dim) {
    case 64: return launch<64>(q, k, slots, (int)seq_len, (int)num_heads, eps, q_weight, k_weight, cos, sin, ts, ts, s);
    case 128:
      return launch<128>(q, k, slots, (int)seq_len, (int)num_heads, eps, q_weight, k_weight, cos, sin, ts, ts, s);
    default:
      return launch<256>(q, k, slots, (int)seq_len, (int)num_heads, eps, q_weight, k_weight, cos, sin, ts, ts, s);
  }
}

// Strided variant (no reference counterpart): q and k are [B*L, H, D] views
// whose tokens are q_token_stride / k_token_stride elements apart, e.g. the q
// and k thirds of a fused [B*L, 3, H, D] QKV GEMM output, normalised (and,
// when cos/sin are given, rotated) in place without the reference shim's
// .contiguous() copies (deploy/xvideo/models/dit/sgl_fused_ops.py:74-75).
// cos = sin = NULL: per-head RMSNorm only (the text stream's q/k norm,
// dit.py:384-385).
extern "C" int jo_qk_norm_rope_strided(void* q, void* k, int64_t batch, int64_t seq_len, int64_t num_heads,
                                       int64_t head_dim, int64_t q_token_stride, int64_t k_token_stride, float eps,
                                       const void* q_weight, const void* k_weight, const void* cos, const void* sin,
                                       void* stream) {
  using namespace jo;
  JO_REQUIRE(batch >= 0 && seq_len >= 0 && num_heads >= 0, JO_ERR_INVALID, "qk_norm_rope_strided: negative size");
  JO_REQUIRE(head_dim == 64 || head_dim == 128 || head_dim == 256, JO_ERR_INVALID,
             "Unsupported head_dim for qk_norm_rope_strided: %lld", (long long)head_dim);
  JO_REQUIRE(q_token_stride >= num_heads * head_dim && k_token_stride >= num_heads * head_dim &&
                 q_token_stride % 8 == 0 && k_token_stride % 8 == 0,
             JO_ERR_INVALID, "qk_norm_rope_strided: token strides must cover the heads and be multiples of 8");
  JO_REQUIRE((cos == nullptr) == (sin == nullptr), JO_ERR_INVALID, "qk_norm_rope_strided: give both cos and sin or neither");
  const int64_t slots = batch * seq_len * num_heads;
  JO_REQUIRE(slots < (1LL << 31), JO_ERR_INVALID, "qk_norm_rope_strided: too many (token, head) slots");
  JO_REQUIRE(slots == 0 || (q && k && q_weight && k_weight), JO_ERR_INVALID, "qk_norm_rope_strided: null pointer");
  JO_REQUIRE(aligned16(q) && aligned16(k) && aligned16(q_weight) && aligned16(k_weight) &&
                 (!cos || (aligned8(cos) && aligned8(sin))),
             JO_ERR_ALIGN, "qk_norm_rope_strided: q/k/weights must be 16-byte aligned, cos/sin 8-byte");
  int st = require_sm100();
  if (st != JO_OK) return st;
  if (slots == 0) return JO_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (head_dim) {
    case 64:
      return launch<64>(q, k, slots, (int)seq_len, (int)num_heads, eps, q_weight, k_weight, cos, sin, q_token_stride,
                        k_token_stride, s);
    case 128:
      return launch<128>(q, k, slots, (int)seq_len, (int)num_heads, eps, q_weight, k_weight, cos, sin, q_token_stride,
                         k_token_stride, s);
    default:
      return launch<256>(q, k, slots, (int)seq_len, (int)num_heads, eps, q_weight, k_weight, cos, sin, q_token_stride,
                         k_token_stride, s);
  }
}
