// Fused per-head RMSNorm + interleaved-pair 3D RoPE, in place on q and k (bf16).
// Reference: deploy/joyomni_ops/csrc/fused_qknorm_rope_3d_kernel.cu:56-143 (kernel),
//            :179-208 (host checks).
//
// Design (B200): one head vector (D bf16) is owned by D/8 lanes that each move
// one 16-byte vector, so a warp covers 32*8/D heads and every access is a full
// 16-byte coalesced load/store.  The same lanes process the q and the k vector
// of a (token, head) slot, so the per-lane norm weights live in registers and
// the token's cos/sin entries are fetched once (L1) for both.  Each warp
// handles U slot groups with all loads issued before any math.
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

// Slot groups per warp (loads in flight per lane = 2 * U).  U = 1 measured
// fastest on B200 (more CTAs in flight beat deeper per-warp batches);
// JO_QKR_U overrides for measurements.
static int qkr_u() {
  static int u = -1;
  if (u < 0) {
    const char* e = getenv("JO_QKR_U");
    u = e ? atoi(e) : 1;
    if (u != 1 && u != 2 && u != 4 && u != 8) u = 1;
  }
  return u;
}

template <int D>
int launch(void* q, void* k, int64_t slots, int seq_len, int num_heads, float eps, const void* qw, const void* kw,
           const void* c, const void* s, int64_t q_ts, int64_t k_ts, cudaStream_t st) {
  switch (qkr_u()) {
    case 1: return launch_u<D, 1>(q, k, slots, seq_len, num_heads, eps, qw, kw, c, s, q_ts, k_ts, st);
    case 4: return launch_u<D, 4>(q, k, slots, seq_len, num_heads, eps, qw, kw, c, s, q_ts, k_ts, st);
    case 8: return launch_u<D, 8>(q, k, slots, seq_len, num_heads, eps, qw, kw, c, s, q_ts, k_ts, st);
    case 2: return launch_u<D, 2>(q, k, slots, seq_len, num_heads, eps, qw, kw, c, s, q_ts, k_ts, st);
    default: return launch_u<D, 1>(q, k, slots, seq_len, num_heads, eps, qw, kw, c, s, q_ts, k_ts, st);
  }
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
