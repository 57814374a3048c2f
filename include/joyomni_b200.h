/*
 * joyomni_b200 — C ABI of the B200-native (sm_100a) joyomni_ops operator set.
 *
 * Every entry point takes raw device pointers, sizes and a cudaStream_t passed
 * as `void*` (NULL = legacy default stream), enqueues its kernels on that
 * stream, never synchronises the host and never allocates device memory, so
 * every call can be captured in a CUDA graph.  Each returns JO_OK (0) or a
 * negative JO_ERR_* status; the message is in jo_last_error() (thread-local).
 *
 * Reference interfaces replaced (paths inside jd-opensource/JoyAI-Video-Edit):
 *   deploy/joyomni_ops/csrc/pybind.cpp:33-58          TORCH_LIBRARY(joyomni_ops) schema
 *   deploy/joyomni_ops/joyomni_ops/__init__.py:31-58  Python wrappers
 */
#ifndef JOYOMNI_B200_H_
#define JOYOMNI_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------- */
#define JO_OK 0
#define JO_ERR_INVALID (-1)   /* bad shape / size / argument  -> RuntimeError        */
#define JO_ERR_DTYPE (-2)     /* unsupported dtype            -> RuntimeError        */
#define JO_ERR_ALIGN (-3)     /* misaligned pointer / stride  -> RuntimeError        */
#define JO_ERR_ARCH (-4)      /* device is not sm_100         -> NotImplementedError */
#define JO_ERR_CUDA (-5)      /* CUDA runtime / launch error  -> RuntimeError        */

/* ---- dtype tags ------------------------------------------------------ */
#define JO_DTYPE_F32 0
#define JO_DTYPE_F16 1
#define JO_DTYPE_BF16 2
#define JO_DTYPE_E4M3 3

/* ---- norm types (deploy/joyomni_ops/csrc/fused_norm_scale_shift.cu:25) - */
#define JO_NORM_LAYER 0
#define JO_NORM_RMS 1

/* ---- GEMM epilogues --------------------------------------------------- */
#define JO_EPI_NONE 0
#define JO_EPI_GELU_TANH 1
#define JO_EPI_RESID_GATE 2   /* out = residual + gate[n] * out (jo_fp8_scaled_mm_ex) */

/* Library version (major*10000 + minor*100 + patch). */
int jo_version(void);

/* Message of the last failed call on this host thread ("" if none). */
const char* jo_last_error(void);

/* Compute capability (major*10+minor) of `device`, or a negative status. */
int jo_device_arch(int device);

/*
 * Fused per-head RMSNorm + interleaved-pair 3D RoPE, in place on q and k.
 * Replaces joyomni_ops::fused_qk_norm_rope_3d_paired
 *   (deploy/joyomni_ops/csrc/fused_qknorm_rope_3d_kernel.cu:179-208).
 * q, k: bf16 [batch, seq_len*num_heads, head_dim], contiguous, 16-byte aligned.
 * q_weight, k_weight: bf16 [head_dim].  cos, sin: bf16 [seq_len, head_dim/2].
 * head_dim in {64, 128, 256}.
 */
int jo_fused_qk_norm_rope_3d_paired(void* q, void* k, int64_t batch, int64_t seq_len,
                                    int64_t num_heads, int64_t head_dim, float eps,
                                    const void* q_weight, const void* k_weight,
                                    const void* cos, const void* sin, void* stream);

/*
 * Strided form of jo_fused_qk_norm_rope_3d_paired (no reference counterpart):
 * q and k are [batch*seq_len, num_heads, head_dim] bf16 views whose tokens are
 * q_token_stride / k_token_stride elements apart (e.g. the q and k thirds of a
 * fused QKV GEMM output), processed in place with the same arithmetic.  With
 * cos = sin = NULL only the per-head RMSNorm is applied.  Strides % 8 == 0.
 */
int jo_qk_norm_rope_strided(void* q, void* k, int64_t batch, int64_t seq_len, int64_t num_heads,
                            int64_t head_dim, int64_t q_token_stride, int64_t k_token_stride, float eps,
                            const void* q_weight, const void* k_weight, const void* cos, const void* sin,
                            void* stream);

/*
 * y = Norm(x; gamma, beta) * (1 + scale) + shift, norm_type JO_NORM_LAYER/RMS.
 * Replaces joyomni_ops::fused_norm_scale_shift
 *   (deploy/joyomni_ops/csrc/fused_norm_scale_shift.cu:172-209).
 * x: [M, N] with row stride x_stride (elements); y: [M, N] dense.
 * gamma, beta: NULL or [N] of x's dtype (beta used only by LayerNorm, and only
 * when gamma is given, as in the reference).  scale, shift: rows of N elements
 * with row stride mod_stride; x-row m reads modulation row m / mod_group
 * (mod_group = 1 is the reference's per-row [M, N] layout; mod_group = L
 * broadcasts a [B, N] table over L tokens; mod_stride = 0 broadcasts one [N]
 * vector).  N % 4 == 0.  dtype: JO_DTYPE_F32/F16/BF16.
 */
int jo_fused_norm_scale_shift(void* y, const void* x, const void* gamma, const void* beta,
                              const void* scale, const void* shift, int64_t M, int64_t N,
                              int64_t x_stride, int64_t mod_stride, int64_t mod_group,
                              int norm_type, float eps, int dtype, void* stream);

/*
 * out = x * rsqrt(mean(x^2) + eps) * weight, per row.
 * Replaces joyomni_ops::rmsnorm (deploy/joyomni_ops/csrc/rmsnorm.cu:76-95).
 * x: [M, N] with row stride x_stride; out: [M, N] dense; weight [N] (x's dtype).
 */
int jo_rmsnorm(void* out, const void* x, const void* weight, int64_t M, int64_t N,
               int64_t x_stride, float eps, int dtype, void* stream);

/*
 * Dynamic per-token FP8 e4m3 quantisation:
 *   s[m] = max|x[m,:]| / 448 ; q = e4m3_satfinite_rn(clamp(x * (s ? 1/s : 0), +-448)).
 * Replaces joyomni_ops::sgl_per_token_quant_fp8
 *   (deploy/joyomni_ops/csrc/per_token_quant_fp8.cu:148-176).  Bit-exact.
 * input: bf16/fp16 [M, K] contiguous, K % 4 == 0.  out_q: e4m3 [M, K]; out_s: fp32 [M].
 */
int jo_per_token_quant_fp8(const void* input, int in_dtype, void* out_q, float* out_s,
                           int64_t M, int64_t K, void* stream);

/*
 * New fused entry (no reference counterpart; it composes
 * fused_norm_scale_shift.cu:69-143 with per_token_quant_fp8.cu:43-83 as the
 * reference model does in deploy/xvideo/models/dit/dit.py:351-357 ->
 * fp8_linear.py:143-167): y = Norm(x)*(1+scale)+shift rounded to x's dtype,
 * then per-token FP8 quantisation of y.  Arguments as jo_fused_norm_scale_shift
 * (x dense) plus out_q e4m3 [M, N] and out_s fp32 [M].  dtype: F16/BF16.
 */
int jo_norm_modulate_quant_fp8(const void* x, const void* gamma, const void* beta,
                               const void* scale, const void* shift, int64_t M, int64_t N,
                               int64_t mod_stride, int64_t mod_group, int norm_type, float eps,
                               int dtype, void* out_q, float* out_s, void* stream);

/*
 * D[m, n] = out(fma(sa[m], sb[n] * acc[m, n], bias[n])) (or out(sa[m] * (sb[n] * acc))
 * without bias), acc = sum_k A[m, k] * B[k, n] over e4m3 codes in fp32 on the
 * tcgen05 tensor cores; epilogue JO_EPI_GELU_TANH applies GELU-tanh to the
 * rounded result.  Replaces joyomni_ops::fp8_scaled_mm
 *   (deploy/joyomni_ops/csrc/fp8_gemm.cu:1450-1548; epilogue :833-860).
 * mat_a: e4m3 [M, K] row-major; mat_b: e4m3 column-major [K, N] (N rows of K
 * codes); scales_a fp32 [M]; scales_b fp32 [N]; bias NULL or [N] of out_dtype;
 * out [M, N] row-major, out_dtype JO_DTYPE_BF16/F16.  K % 16 == 0, N % 8 == 0,
 * operands 16-byte aligned.
 */
int jo_fp8_scaled_mm(const void* mat_a, const void* mat_b, const float* scales_a, const float* scales_b,
                     const void* bias, void* out, int64_t M, int64_t N, int64_t K, int out_dtype, int epilogue,
                     void* stream);

/*
 * Extended GEMM entry (no reference counterpart): jo_fp8_scaled_mm plus the
 * gated-residual epilogue JO_EPI_RESID_GATE, out = out_dtype(residual[m, n] +
 * gate[n] * out_dtype(GEMM result)) -- the model's torch.addcmul after the
 * projection GEMMs (deploy/xvideo/models/dit/sgl_fused_ops.py:114-117) folded
 * into the epilogue.  residual: [M, N] of out_dtype (may alias out); gate: [N].
 */
int jo_fp8_scaled_mm_ex(const void* mat_a, const void* mat_b, const float* scales_a, const float* scales_b,
                        const void* bias, void* out, int64_t M, int64_t N, int64_t K, int out_dtype, int epilogue,
                        const void* residual, const void* gate, void* stream);

/*
 * RoPE of bf16 keys with fp32 tables (the pre-RoPE KV-cache path: keys stored
 * after the per-head RMSNorm and rotated at the positions they take in the
 * attention window).  Replaces apply_rotary_emb on cached keys
 *   (deploy/xvideo/models/dit/rope.py:21-28; callers dit.py:211-217 and
 *    deploy/xvideo/serving/graph_runner.py:137-142), with that expression's
 * fp32 roundings: o0 = RN(RN(x0*c) + RN(-x1*s)), o1 = RN(RN(x1*c) + RN(x0*s))
 * per interleaved pair, then bf16.  x, out: [L, H, head_dim] bf16 with token /
 * head strides (elements, multiples of 8); cos, sin: fp32 [L, head_dim/2].
 * head_dim in {64, 128, 256}; out may alias x.
 */
int jo_rope_apply(void* out, const void* x, const float* cos, const float* sin, int64_t L, int64_t H,
                  int64_t head_dim, int64_t x_token_stride, int64_t x_head_stride, int64_t out_token_stride,
                  int64_t out_head_stride, void* stream);

/*
 * Multi-head attention forward, non-causal and unmasked, on the tcgen05
 * tensor cores: out = softmax(scale * q k^T) v per (batch, head), fp32 scores
 * and accumulators, bf16 in and out.  Replaces the reference block's external
 * attention call, _flash_attention4 / _sdpa_attention
 *   (deploy/xvideo/models/dit/dit.py:150-178, called at dit.py:419).
 * Layout NHD as there: q [batch, Lq, heads, head_dim], k and v [batch, Lk,
 * heads, head_dim], out [batch, Lq, heads, head_dim]; each *_strides array
 * holds the batch, token and head strides in elements (multiples of 8; the
 * head_dim elements of a row are contiguous).  head_dim == 128, dtype
 * JO_DTYPE_BF16, Lk >= 1, 16-byte aligned tensors.
 */
int jo_attention_fwd(const void* q, const void* k, const void* v, void* out, int64_t batch, int64_t Lq, int64_t Lk,
                     int64_t heads, int64_t head_dim, const int64_t* q_strides, const int64_t* k_strides,
                     const int64_t* v_strides, const int64_t* o_strides, float scale, int dtype, void* stream);

/*
 * Attention whose epilogue scatters its output to the ranks that own the
 * query tokens (sequence parallelism, new entry; no reference counterpart:
 * the reference runs attention on one GPU).  Computes jo_attention_fwd for
 * batch 1 over this rank's `heads` heads of all Lq tokens in the gathered
 * order, and stores query row r of head h into dst[k] at token r - seg_start[k],
 * head head0 + h of a [tokens, all heads, 128] buffer with dst_token_stride
 * elements between tokens, where seg_start[k] <= r < seg_start[k + 1]
 * (seg_start has ranks + 1 entries, 0 first, Lq last).  This is the
 * all-to-all that turns the head shard back into a token shard (replaces
 * torch.distributed.all_to_all_single after attention).  Every segment must
 * fit its destination's dst_tokens token rows and head0 + heads heads must
 * fit the stride (JO_ERR_INVALID otherwise): a destination may be another
 * GPU's memory (a peer pointer from jo_ipc_open).  1 <= ranks <= 8.  The
 * caller synchronises the ranks before any rank reads its buffer.
 */
int jo_attention_fwd_scatter(const void* q, const void* k, const void* v, int64_t Lq, int64_t Lk, int64_t heads,
                             int64_t head_dim, const int64_t* q_strides, const int64_t* k_strides,
                             const int64_t* v_strides, void* const* dst, const int64_t* seg_start, int ranks,
                             int64_t head0, int64_t dst_token_stride, int64_t dst_tokens, float scale, int dtype,
                             void* stream);

/* Diagnostic: fault code left by an attention wait that timed out (0 = none);
 * reset != 0 clears it.  Synchronous; for tests and end-of-chunk checks. */
int jo_attention_last_fault(int reset);

/* Diagnostic: fault code left by a GEMM wait that timed out (0 = none);
 * reset != 0 clears it.  Synchronous; for tests. */
int jo_gemm_last_fault(int reset);

/*
 * Sequence-parallel exchange fused into the FP8 GEMM (no reference
 * counterpart: the reference runs the denoiser on one GPU).  Computes the
 * jo_fp8_scaled_mm result [M, N] with N = parts * ranks * heads_per_rank *
 * head_dim (parts = q, k, v) and, instead of writing it row-major, stores
 * row m of head h of part p into dst[p * ranks + h / heads_per_rank] at token
 * tok0 + m, local head h % heads_per_rank of a [tokens, heads_per_rank,
 * head_dim] buffer: the all-to-all that turns a token shard into a head shard
 * (replaces torch.distributed.all_to_all_single after the QKV projection).
 * Every destination holds dst_tokens token rows and tok0 + M <= dst_tokens
 * is required (JO_ERR_INVALID otherwise): a destination may be another GPU's
 * memory.  Destinations of other ranks are peer pointers from jo_ipc_open.  The caller
 * synchronises the ranks (e.g. a one-element collective on the same stream)
 * before any rank reads its buffers.
 */
int jo_fp8_scaled_mm_scatter(const void* mat_a, const void* mat_b, const float* scales_a, const float* scales_b,
                             const void* bias, int64_t M, int64_t N, int64_t K, int out_dtype,
                             const void* const* dst, int parts, int ranks, int heads_per_rank, int head_dim,
                             int64_t tok0, int64_t dst_tokens, void* stream);

/*
 * Peer-memory plumbing (legacy CUDA IPC, no multicast objects) for the
 * exchange above.  jo_ipc_get_handle writes the 64-byte handle of the
 * allocation holding dev_ptr and the byte offset of dev_ptr in it;
 * jo_ipc_open maps another process's handle on the current device;
 * jo_ipc_close unmaps it.
 */
int jo_ipc_get_handle(const void* dev_ptr, void* handle_out, int64_t* offset_out);
int jo_ipc_open(const void* handle, void** base_out);
int jo_ipc_close(void* base);

#ifdef __cplusplus
}
#endif

#endif /* JOYOMNI_B200_H_ */
