"""CPU oracle for the joyomni_ops hot path — TEST INFRASTRUCTURE ONLY.

A plain-numpy restatement of the reference kernels' arithmetic, used by tests/,
``__graft_entry__.smoke()`` and bench.py's CPU baseline as the checker.  It is
never part of the product path (the product fails loudly without its CUDA
library).  Each function cites the reference file:line it follows
(paths inside jd-opensource/JoyAI-Video-Edit).

Tensor convention: 16-bit float tensors are carried as float32 arrays whose
values are exactly representable in the 16-bit type (``round_bf16`` /
``round_f16`` produce them); FP8 e4m3 tensors are uint8 code arrays.

Parity pinning: the reference ships no golden vectors (its tests print
max-abs only, deploy/joyomni_ops/tests/test_parity_light.py:19-22).  The oracle
is pinned against fixtures produced by the reference's own CUDA kernels
(``tests/golden/make_golden.py`` runs ``oracle/_ref`` on a B200) and its
e4m3/bf16 encoders against PyTorch's casts.
"""
from __future__ import annotations

import math

import numpy as np

F32 = np.float32
FP8_MAX = F32(448.0)

# ---------------------------------------------------------------------------
# number formats
# ---------------------------------------------------------------------------


def round_bf16(x) -> np.ndarray:
    """float32 -> nearest bf16 (round-to-nearest-even), returned as float32."""
    a = np.ascontiguousarray(np.asarray(x, dtype=F32))
    u = a.view(np.uint32).astype(np.uint64)
    nan = np.isnan(a)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    r = (r << 16).astype(np.uint32)
    out = r.view(F32).copy()
    out[nan] = np.nan
    return out.reshape(a.shape)


def bf16_bits(x) -> np.ndarray:
    """bf16-valued float32 array -> uint16 bit patterns."""
    a = np.ascontiguousarray(round_bf16(x))
    return (a.view(np.uint32) >> 16).astype(np.uint16)


def bf16_from_bits(b) -> np.ndarray:
    b = np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16
    return b.view(F32)


def round_f16(x) -> np.ndarray:
    return np.asarray(x, dtype=F32).astype(np.float16).astype(F32)


def round_to(x, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return round_bf16(x)
    if dtype == "f16":
        return round_f16(x)
    return np.asarray(x, dtype=F32)


def e4m3_encode(x) -> np.ndarray:
    """float32 -> e4m3fn codes, round-to-nearest-even, saturating to +-448 (satfinite);
    NaN -> 0x7F.  This is the conversion the reference performs with
    ``static_cast<__nv_fp8_e4m3>(float)`` (per_token_quant_fp8.cu:74)."""
    a = np.asarray(x, dtype=F32)
    sign = (np.signbit(a)).astype(np.uint8) << 7
    m = np.abs(a).astype(np.float64)
    out = np.zeros(a.shape, dtype=np.uint8)
    nan = np.isnan(a)
    sat = (m >= 448.0) & ~nan
    sub = (m < 2.0 ** -6) & ~nan
    nrm = ~(nan | sat | sub)
    # subnormals: multiples of 2^-9 (code 8 == 2^-6 continues into the normals)
    out[sub] = np.rint(m[sub] * 512.0).astype(np.uint8)
    mn = m[nrm]
    e = np.floor(np.log2(mn)).astype(np.int64)
    # guard log2 rounding at exact powers of two
    e = np.where(mn < np.ldexp(1.0, e), e - 1, e)
    e = np.where(mn >= np.ldexp(1.0, e + 1), e + 1, e)
    frac = mn / np.ldexp(1.0, e) - 1.0          # [0, 1)
    q = np.rint(frac * 8.0).astype(np.int64)   # RNE on the 3-bit mantissa
    e = np.where(q == 8, e + 1, e)
    q = np.where(q == 8, 0, q)
    code = ((e + 7) << 3) | q
    code = np.minimum(code, 0x7E)              # satfinite
    out[nrm] = code.astype(np.uint8)
    out[sat] = 0x7E
    out[nan] = 0x7F
    return out | sign


def _e4m3_table() -> np.ndarray:
    t = np.zeros(256, dtype=F32)
    for c in range(256):
        s = -1.0 if c & 0x80 else 1.0
        e = (c >> 3) & 0xF
        m = c & 7
        if e == 15 and m == 7:
            v = np.nan
        elif e == 0:
            v = s * m * 2.0 ** -9
        else:
            v = s * (1.0 + m / 8.0) * 2.0 ** (e - 7)
        t[c] = v
    return t


E4M3_TABLE = _e4m3_table()


def e4m3_decode(codes) -> np.ndarray:
    return E4M3_TABLE[np.asarray(codes, dtype=np.uint8)]


# ---------------------------------------------------------------------------
# K4 per-token FP8 quantisation   (per_token_quant_fp8.cu:43-83)
# ---------------------------------------------------------------------------


def per_token_quant_fp8(x):
    """x: [M, K] float32 holding bf16/fp16 values -> (codes uint8 [M, K], scales f32 [M]).

    amax = fmaxf-reduction of |x| starting at 0 (NaN ignored)  :55-62
    s    = amax / 448 (IEEE fp32 division)                     :63
    inv  = s == 0 ? 0 : 1/s                                    :65
    q    = e4m3(fmaxf(fminf(x*inv, 448), -448))                :71-74
    """
    x = np.asarray(x, dtype=F32)
    M, K = x.shape
    if K == 0:
        return np.zeros((M, 0), np.uint8), np.zeros(M, F32)
    amax = np.fmax.reduce(np.abs(x), axis=1, initial=F32(0)).astype(F32)
    s = (amax / FP8_MAX).astype(F32)
    with np.errstate(divide="ignore", over="ignore", invalid="ignore"):
        inv = np.where(s == 0, F32(0), (F32(1) / np.where(s == 0, F32(1), s))).astype(F32)
        v = (x * inv[:, None]).astype(F32)
    v = np.fmax(np.fmin(v, FP8_MAX), -FP8_MAX)
    return e4m3_encode(v), s


# ---------------------------------------------------------------------------
# K2 fused norm + adaLN modulate   (fused_norm_scale_shift.cu:69-143)
# ---------------------------------------------------------------------------


def _expand_mod(t, M, N):
    t = np.asarray(t, dtype=F32)
    if t.ndim == 1:
        return np.broadcast_to(t[None, :], (M, N))
    G = t.shape[0]
    return np.repeat(t, M // G, axis=0) if G != M else t


def fused_norm_scale_shift(x, gamma, beta, scale, shift, norm_type, eps, dtype="bf16"):
    """y = Norm(x; gamma, beta) * (1 + scale) + shift, rounded to ``dtype``.

    RMS   (norm_type 1): r = rsqrt(sum(x^2)/N + eps); y = ((x*r)*g)*(1+sc)+sh    :95-101,118,136-139
    Layer (norm_type 0): mu = sum(x)/N; r = rsqrt(sum((x-mu)^2)/N + eps);
                         y = ((x-mu)*r*g + b)*(1+sc)+sh                        :104-117,131-134
    g = 1, b = 0 when gamma is None; beta is used only together with gamma    :125,130
    Sums are accumulated in float64 and rounded once (the kernel's fp32 tree
    order is not specified by the interface).
    """
    x = np.asarray(x, dtype=F32)
    M, N = x.shape
    sc = _expand_mod(scale, M, N)
    sh = _expand_mod(shift, M, N)
    g = np.ones(N, F32) if gamma is None else np.asarray(gamma, dtype=F32)
    b = np.zeros(N, F32) if (gamma is None or beta is None) else np.asarray(beta, dtype=F32)
    eps = F32(eps)
    nf = F32(N)
    if norm_type in (1, "rms"):
        ss = (x.astype(np.float64) ** 2).sum(axis=1).astype(F32)
        r = (F32(1) / np.sqrt((ss / nf + eps).astype(F32))).astype(F32)
        t = ((x * r[:, None]).astype(F32) * g).astype(F32)
        y = (t * (F32(1) + sc).astype(F32)).astype(F32) + sh
    elif norm_type in (0, "layer"):
        mu = (x.astype(np.float64).sum(axis=1)).astype(F32) / nf
        d = (x - mu[:, None]).astype(F32)
        ss = (d.astype(np.float64) ** 2).sum(axis=1).astype(F32)
        r = (F32(1) / np.sqrt((ss / nf + eps).astype(F32))).astype(F32)
        t = (((d * r[:, None]).astype(F32) * g).astype(F32) + b).astype(F32)
        y = (t * (F32(1) + sc).astype(F32)).astype(F32) + sh
    else:
        raise ValueError("norm_type must be 0 (layer) or 1 (rms)")
    return round_to(y.astype(F32), dtype)


# ---------------------------------------------------------------------------
# K3 rmsnorm   (rmsnorm.cu:38-61)
# ---------------------------------------------------------------------------


def rmsnorm(x, w, eps, dtype="bf16"):
    """out = (x * rsqrt(sum(x^2)/N + eps)) * w, rounded to ``dtype``.   :51-60"""
    x = np.asarray(x, dtype=F32)
    N = x.shape[1]
    ss = (x.astype(np.float64) ** 2).sum(axis=1).astype(F32)
    r = (F32(1) / np.sqrt((ss / F32(N) + F32(eps)).astype(F32))).astype(F32)
    y = ((x * r[:, None]).astype(F32) * np.asarray(w, dtype=F32)).astype(F32)
    return round_to(y, dtype)


# ---------------------------------------------------------------------------
# K1 QK-RMSNorm + interleaved-pair RoPE   (fused_qknorm_rope_3d_kernel.cu:56-143)
# ---------------------------------------------------------------------------


def qk_norm_rope(x, w, cos, sin, seq_len, num_heads, eps):
    """x: [B, L*H, D] bf16-valued; w: [D]; cos/sin: [L, D/2] bf16-valued.

    r = rsqrt(sum(x^2)/D + eps)                        :98-112
    e = x * (r * w)                                    :114-118
    (o0, o1) = (e0*c - e1*s, e0*s + e1*c) per pair     :120-131
    output rounded to bf16                             :133-141
    """
    x = np.asarray(x, dtype=F32)
    B, LH, D = x.shape
    xv = x.reshape(B, seq_len, num_heads, D)
    ss = (xv.astype(np.float64) ** 2).sum(axis=-1).astype(F32)
    r = (F32(1) / np.sqrt((ss / F32(D) + F32(eps)).astype(F32))).astype(F32)
    rw = (r[..., None] * np.asarray(w, dtype=F32)).astype(F32)
    e = (xv * rw).astype(F32)
    c = np.asarray(cos, dtype=F32)[None, :, None, :]
    s = np.asarray(sin, dtype=F32)[None, :, None, :]
    e0, e1 = e[..., 0::2], e[..., 1::2]
    o = np.empty_like(e)
    o[..., 0::2] = (e0 * c).astype(F32) - (e1 * s).astype(F32)
    o[..., 1::2] = (e0 * s).astype(F32) + (e1 * c).astype(F32)
    return round_bf16(o).reshape(B, LH, D)


def rope_tables_3d(grid, axes_dims=(44, 42, 42), theta=10000.0):
    """cos/sin [T*H*W, D/2] as the shim hands them to the kernel.

    Per axis of width d: f_j = 1/theta^(2j/d), angle = pos*f_j in fp32, cos/sin
    then repeat_interleave(2) (deploy/xvideo/models/dit/rope.py:31-52); axes are
    concatenated t|h|w over the row-major (t,h,w) grid (dit.py:745-783) and the
    de-duplicated [..., ::2] half is rounded to bf16 (sgl_fused_ops.py:87-94).
    """
    T, H, W = grid
    tt, hh, ww = np.meshgrid(np.arange(T), np.arange(H), np.arange(W), indexing="ij")
    pos = [tt.reshape(-1).astype(F32), hh.reshape(-1).astype(F32), ww.reshape(-1).astype(F32)]
    cs, ss = [], []
    for p, d in zip(pos, axes_dims):
        j = np.arange(0, d, 2, dtype=F32)[: d // 2]
        f = (F32(1.0) / (F32(theta) ** (j / F32(d)))).astype(F32)
        ang = np.outer(p, f).astype(F32)
        cs.append(np.cos(ang).astype(F32))
        ss.append(np.sin(ang).astype(F32))
    return round_bf16(np.concatenate(cs, axis=1)), round_bf16(np.concatenate(ss, axis=1))


def rope_apply(x, cos, sin):
    """RoPE of bf16-valued keys with fp32 tables, the pre-RoPE KV-cache path
    (deploy/xvideo/models/dit/rope.py:14-28 apply_rotary_emb, called on
    cached pre-RoPE keys at dit.py:211-217 and at graph commit,
    deploy/xvideo/serving/graph_runner.py:137-142).

    x: [L, H, D] bf16-valued; cos, sin: [L, D/2] fp32 (the de-duplicated half of
    the repeat_interleaved tables).  Per pair (x0, x1) = (x[2j], x[2j+1]):
      rotate_half gives (-x1, x0)                        rope.py:14-18
      o0 = RN(RN(x0 * c) + RN(-x1 * s))                  rope.py:28, elementwise
      o1 = RN(RN(x1 * c) + RN( x0 * s))                  torch ops, fp32, no FMA
    then .type_as(x): bf16 round-to-nearest-even.
    """
    x = np.asarray(x, dtype=F32)
    c = np.asarray(cos, dtype=F32)[:, None, :]
    s = np.asarray(sin, dtype=F32)[:, None, :]
    x0, x1 = x[..., 0::2], x[..., 1::2]
    o = np.empty_like(x)
    o[..., 0::2] = ((x0 * c).astype(F32) + (-x1 * s).astype(F32)).astype(F32)
    o[..., 1::2] = ((x1 * c).astype(F32) + (x0 * s).astype(F32)).astype(F32)
    return round_bf16(o)


def rope_tables_3d_f32(grid, t0=0, axes_dims=(44, 42, 42), theta=10000.0):
    """fp32 cos/sin [T*H*W, D/2] for a (t, h, w) grid whose temporal positions
    start at t0 (the cached-key tables of the pre-RoPE path: get_1d_rotary_pos_embed,
    rope.py:31-52, over shifted temporal ids, dit.py:955-973), not rounded."""
    T, H, W = grid
    tt, hh, ww = np.meshgrid(np.arange(T) + t0, np.arange(H), np.arange(W), indexing="ij")
    pos = [tt.reshape(-1).astype(F32), hh.reshape(-1).astype(F32), ww.reshape(-1).astype(F32)]
    cs, ss = [], []
    for p, d in zip(pos, axes_dims):
        j = np.arange(0, d, 2, dtype=F32)[: d // 2]
        f = (F32(1.0) / (F32(theta) ** (j / F32(d)))).astype(F32)
        ang = np.outer(p, f).astype(F32)
        cs.append(np.cos(ang).astype(F32))
        ss.append(np.sin(ang).astype(F32))
    return np.concatenate(cs, axis=1), np.concatenate(ss, axis=1)


# ---------------------------------------------------------------------------
# K5 FP8 scaled GEMM   (fp8_gemm.cu:834-860 epilogue; fp8_linear.py:100-110 weights)
# ---------------------------------------------------------------------------


def quantize_weight_per_channel(w, on_cuda=False):
    """w: [N, K] bf16-valued -> (codes [N, K] uint8 (= column-major [K, N]), scale f32 [N]).

    scale = max(absmax_k |W[n,:]|, 1e-8) / 448 ; q = e4m3(clamp(W / scale, +-448))
    (deploy/xvideo/models/dit/fp8_linear.py:100-110; fp32 division).

    on_cuda=True follows the same torch code run on a GPU: ATen's CUDA true
    division by a Python scalar multiplies by the scalar's fp32 reciprocal, so
    the scale there is RN(absmax * RN(1/448)) (up to one ulp away from the
    quotient); the division of W by the scale tensor stays an IEEE division.
    """
    w = np.asarray(w, dtype=F32)
    amax = np.maximum(np.abs(w).max(axis=1), F32(1e-8)).astype(F32)
    s = (amax * (F32(1.0) / FP8_MAX)).astype(F32) if on_cuda else (amax / FP8_MAX).astype(F32)
    v = (w / s[:, None]).astype(F32)
    v = np.clip(v, -FP8_MAX, FP8_MAX)
    return e4m3_encode(v), s


def gelu_tanh(y):
    """0.5*y*(1+tanh(sqrt(2/pi)*(y+0.044715*y^3))) in float64, as F.gelu(approximate='tanh')."""
    y = np.asarray(y, dtype=np.float64)
    return 0.5 * y * (1.0 + np.tanh(math.sqrt(2.0 / math.pi) * (y + 0.044715 * y ** 3)))


def fp8_scaled_mm(a_codes, b_codes_nk, sa, sb, bias=None, out="bf16", epilogue="none"):
    """D[m,n] = out(sa[m] * (sb[n] * acc[m,n]) + bias[n]), acc = sum_k A[m,k] B[k,n].

    b_codes_nk is the column-major [K, N] weight stored as N rows of K codes.
    acc is computed exactly (float64) and rounded to fp32 like the tensor-core
    fp32 accumulator; the epilogue follows the CUTLASS visitor tree of
    fp8_gemm.cu:834-860: t = fp32(sb*acc), D = round(fma(sa, t, bias)).
    epilogue='gelu_tanh' applies GELU to the rounded output and rounds again
    (dit.py:90-92 applies F.gelu after fp8_scaled_mm).
    """
    A = e4m3_decode(a_codes).astype(np.float64)
    B = e4m3_decode(b_codes_nk).astype(np.float64)
    acc = (A @ B.T).astype(F32)
    t = (np.asarray(sb, dtype=F32)[None, :] * acc).astype(F32)
    z = np.asarray(sa, dtype=F32)[:, None].astype(np.float64) * t.astype(np.float64)
    if bias is not None:
        z = z + np.asarray(bias, dtype=F32)[None, :].astype(np.float64)
    y = round_to(z.astype(F32), out)
    if epilogue == "gelu_tanh":
        y = round_to(gelu_tanh(y).astype(F32), out)
    return y
