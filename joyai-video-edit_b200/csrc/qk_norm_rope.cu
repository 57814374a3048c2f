// Fused per-head RMSNorm + interleaved-pair 3D RoPE, in place on q and k (bf16).
// Reference: deploy/joyomni_ops/csrc/fused_qknorm_rope_3d_kernel.cu:56-143 (kernel),
//            :179-208 (host checks).
//
// Design (B200): one head vector (D bf16) is owned by D/8 lanes that each move
// one 16-byte vector, so a warp covers 32*8/D heads and every access is a full
// 16-byte coalesced load/store.  The same lanes process the q and the k vector
// of a (token, head) slot, so the per-lane norm weights live in registers for
// the whole kernel and the token's cos/sin entries are fetched once (L1) for
// both.  Each warp handles U slot groups with all loads issued before any math
// (2*U 16-byte loads in flight per lane) to keep HBM busy.
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

namespace jo {
namespace {

template <int D, int U>
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(
    __nv_bfloat16* __restrict__ q, __nv_bfloat16* __restrict__ k, int64_t slots, int seq_len, int num_heads,
    float eps, const __nv_bfloat16* __restrict__ qw, const __nv_bfloat16* __restrict__ kw,
    const __nv_bfloat16* __restrict__ cosp, const __nv_bfloat16* __restrict__ sinp) {
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
  int64_t slot[U];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    slot[u] = (warp * U + u) * HPW + lane / LPH;
    if (slot[u] < slots) {
      vq[u].raw = ld_stream(q + slot[u] * D + hl * 8);
      vk[u].raw = ld_stream(k + slot[u] * D + hl * 8);
    }
  }

#pragma unroll
  for (int u = 0; u < U; ++u) {
    const bool ok = slot[u] < slots;
    const int64_t token = ok ? (slot[u] / num_heads) % seq_len : 0;
    // cos/sin entries for this lane's 4 pairs: indices hl*4 .. hl*4+3.
    uint2 c2 = __ldg(reinterpret_cast<const uint2*>(cosp + token * (D / 2) + hl * 4));
    uint2 s2 = __ldg(reinterpret_cast<const uint2*>(sinp + token * (D / 2) + hl * 4));
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
      st_stream(q + slot[u] * D + hl * 8, vq[u].raw);
      st_stream(k + slot[u] * D + hl * 8, vk[u].raw);
    }
  }
}

template <int D>
int launch(void* q, void* k, int64_t slots, int seq_len, int num_heads, float eps, const void* qw, const void* kw,
           const void* c, const void* s, cudaStream_t st) {
  constexpr int U = 2;
  constexpr int HPW = 32 / (D / 8);
  const int64_t warps = (slots + (int64_t)HPW * U - 1) / ((int64_t)HPW * U);
  const int64_t blocks = (warps + 7) / 8;
  qk_norm_rope_kernel<D, U><<<(unsigned)blocks, 256, 0, st>>>(
      static_cast<__nv_bfloat16*>(q), static_cast<__nv_bfloat16*>(k), slots, seq_len, num_heads, eps,
      static_cast<const __nv_bfloat16*>(qw), static_cast<const __nv_bfloat16*>(kw),
      static_cast<const __nv_bfloat16*>(c), static_cast<const __nv_bfloat16*>(s));
  return check_launch("fused_qk_norm_rope_3d_paired");
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
  JO_REQUIRE(slots == 0 || (q && k && q_weight && k_weight && cos && sin), JO_ERR_INVALID,
             "fused_qk_norm_rope_3d_paired: null tensor pointer");
  JO_REQUIRE(aligned16(q) && aligned16(k) && aligned16(q_weight) && aligned16(k_weight) && aligned8(cos) &&
                 aligned8(sin),
             JO_ERR_ALIGN, "fused_qk_norm_rope_3d_paired: q/k/weights must be 16-byte aligned, cos/sin 8-byte");
  int st = require_sm100();
  if (st != JO_OK) return st;
  if (slots == 0) return JO_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (head_dim) {
    case 64: return launch<64>(q, k, slots, (int)seq_len, (int)num_heads, eps, q_weight, k_weight, cos, sin, s);
    case 128: return launch<128>(q, k, slots, (int)seq_len, (int)num_heads, eps, q_weight, k_weight, cos, sin, s);
    default: return launch<256>(q, k, slots, (int)seq_len, (int)num_heads, eps, q_weight, k_weight, cos, sin, s);
  }
}
