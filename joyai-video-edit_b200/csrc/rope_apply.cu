// Interleaved-pair RoPE of bf16 keys with fp32 tables: the pre-RoPE KV-cache
// path, where keys are stored after the per-head RMSNorm and rotated later at
// the (shifted, clamped) positions they take in the attention window.
//
// Replaces apply_rotary_emb on cached keys (deploy/xvideo/models/dit/rope.py:21-28,
// called by _concat_kv_entries at dit.py:211-217 and by the graph runner's
// commit at deploy/xvideo/serving/graph_runner.py:137-142).  Arithmetic of that
// torch expression, (x.float() * cos + rotate_half(x.float()) * sin).type_as(x),
// as separate fp32 operations (no contraction), per pair (x0, x1):
//   o0 = RN(RN(x0 * c) + RN(-x1 * s)),  o1 = RN(RN(x1 * c) + RN(x0 * s)),
// then bf16 round-to-nearest-even.
//
// Layout: x, out [L, H, D] bf16 views with token / head strides (elements,
// multiples of 8; the D elements of a row contiguous); cos, sin fp32 [L, D/2].
// One thread per 8 elements (16 bytes) of a (token, head) row; the table pieces
// of a token are read through L1 (reused by every head).  In place allowed.
#include "jo_common.cuh"

namespace jo {
namespace {

struct RopeArgs {
  __nv_bfloat16* out;
  const __nv_bfloat16* x;
  const float* cos;
  const float* sin;
  int64_t L, H;
  int64_t x_ts, x_hs, o_ts, o_hs;
};

template <int D>
__global__ void __launch_bounds__(256) rope_apply_kernel(const RopeArgs a) {
  constexpr int TPR = D / 8;  // threads per (token, head) row
  const int64_t rows = a.L * a.H;
  const int64_t total = rows * TPR;
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < total; g += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = g / TPR;
    const int part = (int)(g - row * TPR);
    const int64_t tok = row / a.H;
    const int64_t h = row - tok * a.H;
    // plain (coherent) load: out may alias x
    const uint4 xv = *reinterpret_cast<const uint4*>(a.x + tok * a.x_ts + h * a.x_hs + part * 8);
    const float4 c = __ldg(reinterpret_cast<const float4*>(a.cos + tok * (D / 2) + part * 4));
    const float4 s = __ldg(reinterpret_cast<const float4*>(a.sin + tok * (D / 2) + part * 4));
    const uint32_t w[4] = {xv.x, xv.y, xv.z, xv.w};
    const float cc[4] = {c.x, c.y, c.z, c.w}, sc[4] = {s.x, s.y, s.z, s.w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 e = unpack2<__nv_bfloat16>(w[k]);
      const float o0 = __fadd_rn(__fmul_rn(e.x, cc[k]), __fmul_rn(-e.y, sc[k]));
      const float o1 = __fadd_rn(__fmul_rn(e.y, cc[k]), __fmul_rn(e.x, sc[k]));
      o[k] = pack2<__nv_bfloat16>(o0, o1);
    }
    st_stream(a.out + tok * a.o_ts + h * a.o_hs + part * 8, make_uint4(o[0], o[1], o[2], o[3]));
  }
}

}  // namespace
}  // namespace jo

extern "C" int jo_rope_apply(void* out, const void* x, const float* cos, const float* sin, int64_t L, int64_t H,
                             int64_t D, int64_t x_token_stride, int64_t x_head_stride, int64_t out_token_stride,
                             int64_t out_head_stride, void* stream) {
  using namespace jo;
  const char* what = "rope_apply";
  JO_REQUIRE(D == 64 || D == 128 || D == 256, JO_ERR_INVALID, "%s: head_dim must be 64, 128 or 256", what);
  JO_REQUIRE(L >= 0 && H >= 0, JO_ERR_INVALID, "%s: invalid shape", what);
  if (L == 0 || H == 0) return JO_OK;
  JO_REQUIRE(out && x && cos && sin, JO_ERR_INVALID, "%s: null pointer", what);
  JO_REQUIRE(x_token_stride % 8 == 0 && x_head_stride % 8 == 0 && out_token_stride % 8 == 0 &&
                 out_head_stride % 8 == 0,
             JO_ERR_ALIGN, "%s: strides must be multiples of 8 elements", what);
  JO_REQUIRE(aligned16(out) && aligned16(x) && aligned16(cos) && aligned16(sin), JO_ERR_ALIGN,
             "%s: tensors must be 16-byte aligned", what);
  int st = require_sm100();
  if (st != JO_OK) return st;
  RopeArgs a{static_cast<__nv_bfloat16*>(out), static_cast<const __nv_bfloat16*>(x), cos, sin, L, H,
             x_token_stride, x_head_stride, out_token_stride, out_head_stride};
  const int64_t threads = L * H * (D / 8);
  const int64_t want = (threads + 255) / 256;
  const int64_t cap = (int64_t)sm_count() * 8;
  const unsigned grid = (unsigned)(want < cap ? want : cap);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (D == 64)
    rope_apply_kernel<64><<<grid, 256, 0, s>>>(a);
  else if (D == 128)
    rope_apply_kernel<128><<<grid, 256, 0, s>>>(a);
  else
    rope_apply_kernel<256><<<grid, 256, 0, s>>>(a);
  return check_launch(what);
}
