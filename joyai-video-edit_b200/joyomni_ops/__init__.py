"""joyomni_ops — B200-native (sm_100a) drop-in for the reference joyomni_ops package.

Same module name, function names, argument meaning, in-place semantics and error
behaviour as the reference Python shim (deploy/joyomni_ops/joyomni_ops/__init__.py:31-58)
and its TORCH_LIBRARY schema (deploy/joyomni_ops/csrc/pybind.cpp:33-58), so
deploy/xvideo's ``sgl_fused_ops.py`` and ``fp8_linear.py`` import it unchanged.
Every op runs hand-written sm_100a kernels from ``libjoyomni_b200.so`` through
its C ABI; there is no CPU fallback.  Validation mirrors the reference's
TORCH_CHECKs and raises RuntimeError with the same messages (NotImplementedError
on a non-sm_100 device, as TORCH_CHECK_NOT_IMPLEMENTED does).

Extra entry points with no reference counterpart:
  * ``norm_modulate_quant_fp8`` — norm -> adaLN modulate -> per-token FP8 in one pass;
  * ``fp8_scaled_mm_gelu``      — FP8 GEMM with the GELU-tanh epilogue fused;
  * ``attention``               — tcgen05 attention forward over NHD bf16 tensors
  * ``attention_scatter``       — the same, output rows stored to the ranks owning them
    (the reference model's external FA4 / SDPA call, dit.py:150-178);
  * broadcast modulation in ``fused_norm_scale_shift``: scale/shift given as an
    expanded view (row stride 0) are read in place instead of being materialised.
"""
from __future__ import annotations

import ctypes
import math
from typing import Optional

import torch

from . import _lib
from ._lib import check as _check, lib as _L

__all__ = [
    "fused_qk_norm_rope_3d_paired",
    "fused_norm_scale_shift",
    "rmsnorm",
    "sgl_per_token_quant_fp8",
    "fp8_scaled_mm",
    "has_fp8",
    "norm_modulate_quant_fp8",
    "fp8_scaled_mm_gelu",
    "qk_norm_rope_strided",
    "fp8_scaled_mm_residual",
    "attention",
    "attention_scatter",
    "rope_apply",
]

_DT = {torch.float32: _lib.JO_DTYPE_F32, torch.float16: _lib.JO_DTYPE_F16, torch.bfloat16: _lib.JO_DTYPE_BF16}


def _fail(msg: str):
    raise RuntimeError(msg)


def _chk(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _check_cuda(t: torch.Tensor, name: str) -> None:
    _chk(t.is_cuda, f"{name} must be a CUDA tensor")


def _check_input(t: torch.Tensor, name: str, dt: torch.dtype) -> None:
    # JO_CHECK_INPUT (deploy/joyomni_ops/include/joyomni_ops.h:8-15)
    _check_cuda(t, name)
    _chk(t.is_contiguous(), f"{name} must be contiguous")
    _chk(t.dtype == dt, f"{name} dtype is {t.dtype}, expected {dt}")


class _Device:
    """CUDAGuard equivalent: make ``dev`` current for the call, return its stream."""

    __slots__ = ("dev", "prev")

    def __init__(self, t: torch.Tensor):
        self.dev = t.device.index
        self.prev = None

    def __enter__(self) -> int:
        cur = torch.cuda.current_device()
        if cur != self.dev:
            self.prev = cur
            torch.cuda.set_device(self.dev)
        return torch.cuda.current_stream(self.dev).cuda_stream

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)
        return False


# --------------------------------------------------------------------------
# fused_qk_norm_rope_3d_paired  (fused_qknorm_rope_3d_kernel.cu:179-208)
# --------------------------------------------------------------------------
def fused_qk_norm_rope_3d_paired(q, k, seq_len, num_heads, eps, q_weight, k_weight, cos, sin):
    """In-place fused RMSNorm(q,k) + 3D RoPE. q/k: [B, seq_len*num_heads, head_dim] bf16."""
    _chk(q.dim() == 3, "q must be 3D [batch, seq_len*num_heads, head_dim]")
    _chk(k.dim() == 3, "k must be 3D [batch, seq_len*num_heads, head_dim]")
    _chk(q.shape == k.shape, "q and k must have the same shape")
    _chk(q_weight.dim() == 1 and k_weight.dim() == 1, "weights must be 1D [head_dim]")
    _chk(cos.dim() == 2 and sin.dim() == 2, "cos/sin must be 2D [seq_len, head_dim/2]")
    for t, n in ((q, "q"), (k, "k"), (q_weight, "q_weight"), (k_weight, "k_weight"), (cos, "cos"), (sin, "sin")):
        _check_input(t, n, torch.bfloat16)
    B, _, D = q.shape
    _chk(q.size(1) == seq_len * num_heads, "q.size(1) must equal seq_len*num_heads")
    _chk(q_weight.size(0) == D and k_weight.size(0) == D, "weight size must match head_dim")
    _chk(cos.size(0) == seq_len and cos.size(1) == D // 2, "cos shape must be [seq_len, head_dim/2]")
    _chk(sin.size(0) == seq_len and sin.size(1) == D // 2, "sin shape must be [seq_len, head_dim/2]")
    with _Device(q) as st:
        _check(_L.jo_fused_qk_norm_rope_3d_paired(
            q.data_ptr(), k.data_ptr(), B, int(seq_len), int(num_heads), D, float(eps),
            q_weight.data_ptr(), k_weight.data_ptr(), cos.data_ptr(), sin.data_ptr(), st))


def qk_norm_rope_strided(q, k, eps, q_weight, k_weight, cos=None, sin=None):
    """In place on strided views q, k: [B, L, H, D] bf16 (last two dims dense,
    tokens uniformly strided), e.g. ``qkv.view(B, L, 3, H, D)[:, :, 0]``.
    Per-head RMSNorm with q/k weights, then interleaved-pair RoPE with
    cos/sin [L, D/2] when given (norm only when cos is None).  Same arithmetic
    as fused_qk_norm_rope_3d_paired, without copying q/k out of the QKV buffer."""
    _chk(q.dim() == 4 and k.shape == q.shape, "q/k must be [B, L, H, D] views of the same shape")
    B, L, H, D = q.shape
    for t, n in ((q, "q"), (k, "k")):
        _check_cuda(t, n)
        _chk(t.dtype == torch.bfloat16, f"{n} dtype is {t.dtype}, expected torch.bfloat16")
        _chk(t.stride(3) == 1 and t.stride(2) == D, f"{n}: heads must be dense [H, D]")
        _chk(B == 1 or t.stride(0) == L * t.stride(1), f"{n}: tokens must be uniformly strided")
    for t, n in ((q_weight, "q_weight"), (k_weight, "k_weight")):
        _check_input(t, n, torch.bfloat16)
    if cos is not None:
        _check_input(cos, "cos", torch.bfloat16)
        _check_input(sin, "sin", torch.bfloat16)
        _chk(cos.shape == (L, D // 2) and sin.shape == (L, D // 2), "cos shape must be [seq_len, head_dim/2]")
    with _Device(q) as st:
        _check(_L.jo_qk_norm_rope_strided(
            q.data_ptr(), k.data_ptr(), B, L, H, D, q.stride(1), k.stride(1), float(eps), q_weight.data_ptr(),
            k_weight.data_ptr(), cos.data_ptr() if cos is not None else None,
            sin.data_ptr() if sin is not None else None, st))


# --------------------------------------------------------------------------
# fused_norm_scale_shift  (fused_norm_scale_shift.cu:172-209)
# --------------------------------------------------------------------------
def _norm_type_code(norm_type) -> int:
    if isinstance(norm_type, str):
        return 0 if norm_type == "layer" else 1 if norm_type == "rms" else -1
    return int(norm_type)


def _mod_layout(scale: torch.Tensor, shift: torch.Tensor, M: int, N: int):
    """(scale, shift, row stride, rows per modulation row) for [M,N]/[G,N]/[N] tables."""
    if scale.dim() == 1:
        scale, shift = scale.view(1, N), shift.view(1, N)
    if scale.stride(-1) != 1:
        scale = scale.contiguous()
    if shift.stride(-1) != 1:
        shift = shift.contiguous()
    G = scale.size(0)
    if scale.stride(0) != shift.stride(0):
        scale, shift = scale.contiguous(), shift.contiguous()
    stride = scale.stride(0) if G > 1 else 0
    group = max(1, M // G) if G > 0 else 1
    return scale, shift, stride, group


def fused_norm_scale_shift(x, gamma, beta, scale, shift, norm_type, eps=1e-5):
    """Norm(x; gamma, beta) * (1 + scale) + shift. norm_type: 'layer' or 'rms'."""
    nt = _norm_type_code(norm_type)
    _check_cuda(x, "x")
    _check_cuda(scale, "scale")
    _check_cuda(shift, "shift")
    _chk(x.dim() == 2, "x must be 2D [M, N]")
    _chk(x.stride(-1) == 1 or x.numel() == 0, "x last dim must be contiguous")
    M, N = x.shape
    _chk(N % 4 == 0, "N must be divisible by 4")
    _chk(scale.dim() == 2 and shift.dim() == 2, "scale/shift must be 2D [M, N]")
    _chk(scale.size(0) == M and shift.size(0) == M, "scale/shift rows must equal M (per-row modulation)")
    _chk(scale.size(1) == N and shift.size(1) == N, "scale/shift last dim must be N")
    _chk(scale.stride(-1) == 1 and shift.stride(-1) == 1, "scale/shift last dim must be contiguous")
    _chk(x.dtype == scale.dtype and x.dtype == shift.dtype, "x/scale/shift dtype must match")
    _chk(nt in (0, 1), "norm_type must be 0 (layer) or 1 (rms)")
    if x.dtype not in _DT:
        _fail("Unsupported dtype; use float32/float16/bfloat16")
    has_gamma = gamma is not None
    has_beta = beta is not None
    if has_gamma:
        _chk(gamma.numel() == N, "gamma must be length N")
        gamma = gamma.contiguous()
    if has_beta:
        _chk(beta.numel() == N, "beta must be length N")
        beta = beta.contiguous()
    # An expanded [M, N] view (row stride 0) is honoured as a broadcast.
    if scale.stride(0) != shift.stride(0) or (scale.stride(0) not in (0, N)):
        scale, shift = scale.contiguous(), shift.contiguous()
    mod_stride = scale.stride(0)
    y = torch.empty((M, N), dtype=x.dtype, device=x.device)
    with _Device(x) as st:
        _check(_L.jo_fused_norm_scale_shift(
            y.data_ptr(), x.data_ptr(), gamma.data_ptr() if has_gamma else None,
            beta.data_ptr() if has_beta else None, scale.data_ptr(), shift.data_ptr(),
            M, N, x.stride(0) if M > 1 else N, mod_stride, 1, nt, float(eps), _DT[x.dtype], st))
    return y


# --------------------------------------------------------------------------
# rmsnorm  (rmsnorm.cu:76-95)
# --------------------------------------------------------------------------
def rmsnorm(x, weight, eps=1e-6, *, out=None):
    """(x / RMS(x)) * weight. x: [M, N], weight: [N].  `out` (keyword, an
    extension): a dense [M, N] destination, e.g. rows of a preallocated buffer."""
    _check_cuda(x, "x")
    _check_cuda(weight, "weight")
    _chk(x.dim() == 2, "x must be 2D [M, N]")
    _chk(x.stride(-1) == 1 or x.numel() == 0, "x last dim must be contiguous")
    _chk(weight.dim() == 1 and weight.numel() == x.size(1), "weight must be 1D [N]")
    _chk(x.dtype == weight.dtype, "x and weight dtype must match")
    if x.dtype not in _DT:
        _fail("Unsupported dtype; use float32/float16/bfloat16")
    M, N = x.shape
    weight = weight.contiguous()
    if out is None:
        out = torch.empty((M, N), dtype=x.dtype, device=x.device)
    else:
        _chk(out.shape == (M, N) and out.dtype == x.dtype and out.is_cuda and out.is_contiguous(),
             "out must be a dense [M, N] tensor of x's dtype")
    with _Device(x) as st:
        _check(_L.jo_rmsnorm(out.data_ptr(), x.data_ptr(), weight.data_ptr(), M, N,
                             x.stride(0) if M > 1 else N, float(eps), _DT[x.dtype], st))
    return out


def has_fp8() -> bool:
    return _lib.has("jo_fp8_scaled_mm")


# --------------------------------------------------------------------------
# sgl_per_token_quant_fp8  (per_token_quant_fp8.cu:148-176)
# --------------------------------------------------------------------------
def sgl_per_token_quant_fp8(input, output_q, output_s):
    _check_cuda(input, "input")
    _chk(input.is_contiguous(), "input must be contiguous")
    _check_cuda(output_q, "output_q")
    _check_cuda(output_s, "output_s")
    _chk(input.dim() == 2, "input must be 2D [num_tokens, hidden_dim]")
    M, K = input.shape
    _chk(K % 4 == 0, f"hidden_dim must be divisible by 4, got {K}")
    if input.dtype not in (torch.bfloat16, torch.float16):
        _fail("per_token_quant_fp8: input must be bf16 or fp16")
    # The reference trusts the caller on the outputs; a short buffer would be
    # overrun there, so refuse it here instead.
    _chk(output_q.numel() * output_q.element_size() >= M * K, "output_q is smaller than input")
    _chk(output_s.numel() * output_s.element_size() >= M * 4, "output_s must hold num_tokens float32 scales")
    with _Device(input) as st:
        _check(_L.jo_per_token_quant_fp8(input.data_ptr(), _DT[input.dtype], output_q.data_ptr(),
                                         output_s.data_ptr(), M, K, st))


# --------------------------------------------------------------------------
# norm_modulate_quant_fp8 (new fused entry: K2 + K4 in one pass)
# --------------------------------------------------------------------------
def norm_modulate_quant_fp8(x, gamma, beta, scale, shift, norm_type, eps, output_q, output_s):
    """output_q, output_s = per_token_quant_fp8(Norm(x; gamma, beta) * (1 + scale) + shift).

    x: [M, N] bf16/fp16 contiguous.  scale/shift: [N], [G, N] (each row shared by
    M/G consecutive rows of x) or [M, N], x's dtype.  gamma/beta: None or [N].
    The normalised row is rounded to x's dtype before quantisation, exactly as
    fused_norm_scale_shift followed by sgl_per_token_quant_fp8 would compute it.
    """
    nt = _norm_type_code(norm_type)
    _check_input(x, "x", x.dtype)
    _chk(x.dim() == 2, "x must be 2D [M, N]")
    M, N = x.shape
    _chk(x.dtype in (torch.bfloat16, torch.float16), "x must be bf16 or fp16")
    _chk(nt in (0, 1), "norm_type must be 0 (layer) or 1 (rms)")
    _chk(N % 4 == 0, "N must be divisible by 4")
    _check_cuda(scale, "scale")
    _check_cuda(shift, "shift")
    _chk(scale.shape == shift.shape, "scale/shift must have the same shape")
    _chk(scale.dtype == x.dtype and shift.dtype == x.dtype, "x/scale/shift dtype must match")
    _chk(scale.size(-1) == N and scale.dim() in (1, 2), "scale/shift must be [N], [G, N] or [M, N]")
    if scale.dim() == 2:
        _chk(scale.size(0) >= 1 and M % scale.size(0) == 0, "scale/shift rows must divide M")
    sc, sh, mstride, mgroup = _mod_layout(scale, shift, M, N)
    if gamma is not None:
        _chk(gamma.numel() == N and gamma.dtype == x.dtype, "gamma must be length N with x's dtype")
        gamma = gamma.contiguous()
    if beta is not None:
        _chk(beta.numel() == N and beta.dtype == x.dtype, "beta must be length N with x's dtype")
        beta = beta.contiguous()
    _check_cuda(output_q, "output_q")
    _check_cuda(output_s, "output_s")
    _chk(output_q.numel() * output_q.element_size() >= M * N, "output_q is smaller than x")
    _chk(output_s.numel() * output_s.element_size() >= M * 4, "output_s must hold M float32 scales")
    with _Device(x) as st:
        _check(_L.jo_norm_modulate_quant_fp8(
            x.data_ptr(), gamma.data_ptr() if gamma is not None else None,
            beta.data_ptr() if beta is not None else None, sc.data_ptr(), sh.data_ptr(),
            M, N, mstride, mgroup, nt, float(eps), _DT[x.dtype], output_q.data_ptr(), output_s.data_ptr(), st))


# --------------------------------------------------------------------------
# fp8_scaled_mm  (fp8_gemm.cu:1450-1548)
# --------------------------------------------------------------------------
def _fp8_mm_checks(mat_a, mat_b, scales_a, scales_b, out_dtype, bias):
    _chk(mat_a.is_cuda, "mat_a must be a CUDA tensor")
    _chk(mat_b.is_cuda, "mat_b must be a CUDA tensor")
    _chk(mat_a.dim() == 2, "mat_a must be a 2D tensor")
    _chk(mat_b.dim() == 2, "mat_b must be a 2D tensor")
    _chk(mat_a.stride(1) == 1, "mat_a must be a row major tensor")
    _chk(mat_b.stride(0) == 1, "mat_b must be a column major tensor")
    _chk(mat_a.size(1) == mat_b.size(0), "mat_a and mat_b shapes cannot be multiplied")
    _chk((mat_a.size(1) * mat_a.element_size()) % 16 == 0, "mat_a must be multiple of 16 bytes for memory alignment")
    _chk((mat_b.size(0) * mat_b.element_size()) % 16 == 0, "mat_b must be multiple of 16 bytes for memory alignment")
    _chk(mat_a.dtype == torch.float8_e4m3fn, "mat_a must be Float8_e4m3fn")
    _chk(mat_b.dtype == torch.float8_e4m3fn, "mat_b must be Float8_e4m3fn")
    _chk(out_dtype in (torch.float16, torch.bfloat16), "out_dtype must be Half or BFloat16")
    _chk(scales_a.numel() == mat_a.size(0), "size of scales_a is not matched")
    _chk(scales_b.numel() == mat_b.size(1), "size of scales_b is not matched")
    _chk(scales_a.is_contiguous(), "scales_a must be contiguous")
    _chk(scales_b.is_contiguous(), "scales_b msut be contiguous")
    _chk(scales_a.dtype == torch.float32, "scales_a must be Float32")
    _chk(scales_b.dtype == torch.float32, "scales_b must be Float32")
    if bias is not None:
        _chk(bias.numel() == mat_b.size(1), "size of bias is not matched")
        _chk(bias.is_contiguous(), "bias must be contiguous")
        _chk(bias.dtype == out_dtype, "bias dtype must match output dtype")
    M, N = mat_a.size(0), mat_b.size(1)
    _chk((N * torch.empty((), dtype=out_dtype).element_size()) % 16 == 0,
         "out must be multiple of 16 bytes for memory alignment")


def _fp8_mm(mat_a, mat_b, scales_a, scales_b, out_dtype, bias, epilogue, out=None, residual=None, gate=None):
    if not has_fp8():
        raise NotImplementedError("joyomni_b200 was built without the FP8 GEMM")
    _fp8_mm_checks(mat_a, mat_b, scales_a, scales_b, out_dtype, bias)
    M, K = mat_a.shape
    N = mat_b.size(1)
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=mat_a.device)
    else:
        _chk(out.shape == (M, N) and out.dtype == out_dtype and out.is_cuda, "out must be [M, N] of out_dtype")
        _chk(out.stride(1) == 1 and (M <= 1 or out.stride(0) == N), "out rows must be dense")
    if residual is not None:
        _chk(residual.shape == (M, N) and residual.dtype == out_dtype and residual.stride(1) == 1
             and (M <= 1 or residual.stride(0) == N), "residual must be a dense [M, N] tensor of out_dtype")
        _chk(gate is not None and gate.numel() == N and gate.dtype == out_dtype, "gate must be [N] of out_dtype")
        gate = gate.contiguous()
    lda = mat_a.stride(0) if M > 1 else K
    ldb = mat_b.stride(1) if N > 1 else K
    _chk(lda == K and ldb == K, "mat_a rows and mat_b columns must be densely packed")
    with _Device(mat_a) as st:
        _check(_L.jo_fp8_scaled_mm_ex(
            mat_a.data_ptr(), mat_b.data_ptr(), scales_a.data_ptr(), scales_b.data_ptr(),
            bias.data_ptr() if bias is not None else None, out.data_ptr(), M, N, K,
            _DT[out_dtype], epilogue, residual.data_ptr() if residual is not None else None,
            gate.data_ptr() if gate is not None else None, st))
    return out


def fp8_scaled_mm(mat_a, mat_b, scales_a, scales_b, out_dtype, bias: Optional[torch.Tensor] = None, *, out=None):
    """Reference signature; `out` (keyword, an extension) writes into a caller
    buffer, e.g. a row slice of a larger [L, N] tensor."""
    return _fp8_mm(mat_a, mat_b, scales_a, scales_b, out_dtype, bias, _lib.JO_EPI_NONE, out=out)


def fp8_scaled_mm_gelu(mat_a, mat_b, scales_a, scales_b, out_dtype, bias: Optional[torch.Tensor] = None, *,
                       out=None):
    """gelu_tanh(fp8_scaled_mm(...)): GELU applied to the rounded GEMM output, as the
    reference model applies F.gelu(approximate="tanh") after fp8_scaled_mm
    (deploy/xvideo/models/dit/dit.py:90-92)."""
    return _fp8_mm(mat_a, mat_b, scales_a, scales_b, out_dtype, bias, _lib.JO_EPI_GELU_TANH, out=out)


def fp8_scaled_mm_residual(mat_a, mat_b, scales_a, scales_b, out_dtype, bias, residual, gate, *, out=None):
    """residual + gate * fp8_scaled_mm(...) (rounded GEMM output, then the gated
    add of torch.addcmul(residual, y, gate), deploy/xvideo/models/dit/sgl_fused_ops.py:114-117)
    in the GEMM epilogue.  out may be the residual itself (in place)."""
    return _fp8_mm(mat_a, mat_b, scales_a, scales_b, out_dtype, bias, _lib.JO_EPI_RESID_GATE, out=out,
                   residual=residual, gate=gate)


def fp8_scaled_mm_scatter(mat_a, mat_b, scales_a, scales_b, out_dtype, bias, dst_ptrs, parts, ranks,
                          heads_per_rank, head_dim, tok0, dst_tokens):
    """fp8_scaled_mm whose epilogue scatters the [M, parts*ranks*heads_per_rank*
    head_dim] result by head: row m, head h of part p goes to token tok0 + m,
    local head h % heads_per_rank of the [tokens, heads_per_rank, head_dim]
    buffer at dst_ptrs[p * ranks + h // heads_per_rank] (device addresses; a
    peer rank's buffer through joyomni_stack.peer).  Every destination holds
    dst_tokens token rows; tok0 + M must not exceed it.  The sequence-parallel
    all-to-all after the QKV projection, fused into the GEMM (new entry)."""
    if not has_fp8():
        raise NotImplementedError("joyomni_b200 was built without the FP8 GEMM")
    _fp8_mm_checks(mat_a, mat_b, scales_a, scales_b, out_dtype, bias)
    M, K = mat_a.shape
    N = mat_b.size(1)
    _chk(len(dst_ptrs) == parts * ranks, "dst_ptrs must hold parts * ranks addresses")
    _chk(N == parts * ranks * heads_per_rank * head_dim, "N must equal parts * ranks * heads_per_rank * head_dim")
    _chk(0 <= tok0 and tok0 + M <= dst_tokens, "rows tok0 .. tok0 + M must fit the destinations' dst_tokens rows")
    lda = mat_a.stride(0) if M > 1 else K
    ldb = mat_b.stride(1) if N > 1 else K
    _chk(lda == K and ldb == K, "mat_a rows and mat_b columns must be densely packed")
    arr = (ctypes.c_void_p * len(dst_ptrs))(*[int(p) for p in dst_ptrs])
    with _Device(mat_a) as st:
        _check(_L.jo_fp8_scaled_mm_scatter(
            mat_a.data_ptr(), mat_b.data_ptr(), scales_a.data_ptr(), scales_b.data_ptr(),
            bias.data_ptr() if bias is not None else None, M, N, K, _DT[out_dtype], arr, parts, ranks,
            heads_per_rank, head_dim, tok0, dst_tokens, st))


def check_gemm_fault(device=None) -> None:
    """Raise RuntimeError if a GEMM or attention launch on `device` (default:
    the current one) gave up on a bounded wait since the last check, and clear
    the codes.  Each kernel family keeps one sticky code per device shared by
    all its launches, so a non-zero value means some launch since the last
    check returned incomplete output.  Synchronises the device; call it at a
    point that already synchronises (end of a chunk, end of a benchmark phase)."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        torch.cuda.synchronize(dev)
        codes = {"fp8_scaled_mm": _L.jo_gemm_last_fault(1) if has_fp8() else 0,
                 "attention": _L.jo_attention_last_fault(1)}
    for name, code in codes.items():
        if code < 0:
            _check(code)
        if code != 0:
            raise RuntimeError(f"{name}: a launch timed out waiting on its pipeline (fault code {code}); "
                               "its output is incomplete")


# --------------------------------------------------------------------------
# rope_apply  (replaces rope.py:21-28 apply_rotary_emb on pre-RoPE cached keys)
# --------------------------------------------------------------------------
def rope_apply(x, cos, sin, *, out=None):
    """RoPE of bf16 keys x [L, H, D] (token / head strides multiples of 8, last
    dim contiguous) with fp32 tables cos, sin [L, D/2]: the arithmetic of
    apply_rotary_emb (deploy/xvideo/models/dit/rope.py:21-28) as the pre-RoPE
    KV-cache path applies it to cached keys.  Returns a new [L, H, D] tensor or
    writes `out` (which may be x itself)."""
    _chk(x.is_cuda and cos.is_cuda and sin.is_cuda, "x, cos and sin must be CUDA tensors")
    _chk(x.dim() == 3 and x.dtype == torch.bfloat16 and x.stride(2) == 1, "x must be a [L, H, D] bf16 view")
    L, H, D = x.shape
    for t in (cos, sin):
        _chk(t.dtype == torch.float32 and t.shape == (L, D // 2) and t.is_contiguous(),
             "cos and sin must be contiguous fp32 [L, D/2]")
    if out is None:
        out = torch.empty((L, H, D), dtype=torch.bfloat16, device=x.device)
    _chk(out.shape == x.shape and out.dtype == torch.bfloat16 and out.stride(2) == 1, "out must match x")
    with _Device(x) as st:
        _check(_L.jo_rope_apply(out.data_ptr(), x.data_ptr(), cos.data_ptr(), sin.data_ptr(), L, H, D,
                                x.stride(0), x.stride(1), out.stride(0), out.stride(1), st))
    return out


# --------------------------------------------------------------------------
# attention  (replaces dit.py:150-178: FA4 / SDPA over NHD tensors)
# --------------------------------------------------------------------------
def attention(query, key, value, *, out=None, scale: Optional[float] = None):
    """softmax(scale * q k^T) v, non-causal, for bf16 NHD tensors q [B, Lq, H, 128],
    k and v [B, Lk, H, 128] (the layout of the reference's _flash_attention4,
    deploy/xvideo/models/dit/dit.py:161-178); returns [B, Lq, H, 128] bf16 (or
    writes `out`).  3-D [L, H, 128] views are taken as batch 1.  Any strides
    whose last dimension is contiguous and whose others are multiples of 8
    elements are read in place.  scale defaults to 1/sqrt(128)."""
    squeeze = query.dim() == 3
    q, k, v = (t.unsqueeze(0) if t.dim() == 3 else t for t in (query, key, value))
    for name, t in (("query", q), ("key", k), ("value", v)):
        _chk(t.is_cuda, f"{name} must be a CUDA tensor")
        _chk(t.dim() == 4, f"{name} must be [B, L, H, D]")
        _chk(t.dtype == torch.bfloat16, f"{name} must be BFloat16")
        _chk(t.size(3) == 128 and t.stride(3) == 1, f"{name} must have a contiguous head_dim of 128")
    B, Lq, H, Dh = q.shape
    _chk(k.shape[0] == B and v.shape[0] == B and k.shape[2] == H and v.shape[2] == H, "batch / heads mismatch")
    _chk(k.shape[1] == v.shape[1], "key and value lengths differ")
    if out is None:
        o = torch.empty((B, Lq, H, Dh), dtype=torch.bfloat16, device=q.device)
    else:
        o = out.unsqueeze(0) if out.dim() == 3 else out
        _chk(o.shape == (B, Lq, H, Dh) and o.dtype == torch.bfloat16 and o.stride(3) == 1,
             "out must be a [B, Lq, H, 128] bf16 tensor")
    sc = (1.0 / math.sqrt(Dh)) if scale is None else float(scale)

    def strides(t):
        return (ctypes.c_int64 * 3)(t.stride(0), t.stride(1), t.stride(2))
    with _Device(q) as st:
        _check(_L.jo_attention_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), B, Lq, k.shape[1], H, Dh,
                                   strides(q), strides(k), strides(v), strides(o), sc, _lib.JO_DTYPE_BF16, st))
    if out is not None:
        return out
    return o[0] if squeeze else o



def attention_scatter(query, key, value, dst_ptrs, seg_start, head0, total_heads, dst_tokens, *,
                      scale: Optional[float] = None):
    """attention() over this rank's heads of all tokens (q [Lq, h, 128], k and v
    [Lk, h, 128], bf16, batch 1) whose output rows go straight to the ranks that
    own them: query row r with seg_start[k] <= r < seg_start[k + 1] is stored at
    token r - seg_start[k], head head0 + j of the [dst_tokens, total_heads, 128]
    bf16 buffer at device address dst_ptrs[k] (a peer rank's buffer through
    joyomni_stack.peer).  The sequence-parallel all-to-all after attention,
    fused into the attention epilogue (new entry); the caller synchronises the
    ranks before they read their buffers."""
    q, k, v = query, key, value
    for name, t in (("query", q), ("key", k), ("value", v)):
        _chk(t.is_cuda, f"{name} must be a CUDA tensor")
        _chk(t.dim() == 3, f"{name} must be [L, H, D]")
        _chk(t.dtype == torch.bfloat16, f"{name} must be BFloat16")
        _chk(t.size(2) == 128 and t.stride(2) == 1, f"{name} must have a contiguous head_dim of 128")
    Lq, H, Dh = q.shape
    _chk(k.shape[1] == H and v.shape[1] == H and k.shape[0] == v.shape[0], "key / value shapes do not match")
    R = len(dst_ptrs)
    _chk(1 <= R <= 8 and len(seg_start) == R + 1, "1..8 destinations and ranks + 1 segment starts required")
    _chk(seg_start[0] == 0 and seg_start[R] == Lq, "the segments must cover the query rows")
    _chk(all(0 <= seg_start[i + 1] - seg_start[i] <= dst_tokens for i in range(R)),
         "every segment must fit the destinations' dst_tokens rows")
    _chk(0 <= head0 and head0 + H <= total_heads, "heads head0 .. head0 + H must fit total_heads")
    sc = (1.0 / math.sqrt(Dh)) if scale is None else float(scale)

    def strides(t):
        return (ctypes.c_int64 * 3)(0, t.stride(0), t.stride(1))
    arr = (ctypes.c_void_p * R)(*[int(p) for p in dst_ptrs])
    seg = (ctypes.c_int64 * (R + 1))(*[int(s) for s in seg_start])
    with _Device(q) as st:
        _check(_L.jo_attention_fwd_scatter(q.data_ptr(), k.data_ptr(), v.data_ptr(), Lq, k.shape[0], H, Dh,
                                           strides(q), strides(k), strides(v), arr, seg, R, head0,
                                           total_heads * Dh, dst_tokens, sc, _lib.JO_DTYPE_BF16, st))


from . import _torch_ops  # noqa: E402,F401  (registers torch.ops.joyomni_ops.*)
