"""CPU checks of the oracle itself: its number-format encoders against PyTorch's
casts, its per-op formulas against independent torch restatements of the
reference's eager code, and (when present) against golden fixtures produced by
the reference's own CUDA kernels."""
import glob
import os

import numpy as np
import pytest
import torch

import joyomni_oracle as O
from _util import assert_close_ulp, randn

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _special_values():
    rng = np.random.default_rng(0)
    parts = [rng.standard_normal(50000).astype(np.float32) * s for s in (1e-5, 1e-3, 1.0, 40.0, 400.0)]
    parts.append(np.array([0.0, -0.0, 448, -448, 449, 464, 465, 480, 1e30, -1e30, 2 ** -6, 2 ** -7, 2 ** -9,
                           2 ** -10, 3 * 2 ** -11, np.nan, np.inf, -np.inf], np.float32))
    return np.concatenate(parts)


def test_e4m3_encoder_matches_torch():
    x = np.clip(_special_values(), -448, 448)
    ref = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(O.e4m3_encode(x), ref)


def test_e4m3_encoder_midpoints_round_to_even():
    vals = O.E4M3_TABLE[:0x7F].astype(np.float64)
    mids = ((vals[1:] + vals[:-1]) / 2).astype(np.float32)
    for sgn in (1, -1):
        m = mids * sgn
        ref = torch.from_numpy(m).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
        assert np.array_equal(O.e4m3_encode(m), ref)


def test_e4m3_encoder_saturates():
    assert O.e4m3_encode(np.array([500.0, -1e9, np.inf], np.float32)).tolist() == [0x7E, 0xFE, 0x7E]


def test_e4m3_decode_table():
    t = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    same = (t == O.E4M3_TABLE) | (np.isnan(t) & np.isnan(O.E4M3_TABLE))
    assert same.all()


def test_bf16_rounding_matches_torch():
    x = _special_values()
    ref = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    got = O.round_bf16(x)
    assert np.array_equal(got, ref, equal_nan=True)


def _torch_quant_restatement(x):
    """The reference kernel's formulas (per_token_quant_fp8.cu:55-78) restated in torch."""
    xt = torch.from_numpy(x)
    amax = torch.nan_to_num(xt.abs(), nan=0.0).amax(dim=1).clamp_min(0)
    s = amax / 448.0
    inv = torch.where(s == 0, torch.zeros_like(s), 1.0 / s)
    v = xt * inv[:, None]
    v = torch.where(torch.isnan(v), torch.full_like(v, 448.0), v)   # fminf(NaN, 448) = 448
    v = v.clamp(-448, 448)
    return v.to(torch.float8_e4m3fn).view(torch.uint8).numpy(), s.numpy()


@pytest.mark.parametrize("M,K", [(1, 4), (7, 128), (64, 5120), (33, 1000)])
def test_quant_oracle_matches_torch_restatement(M, K):
    rng = np.random.default_rng(M * 1000 + K)
    x = randn(rng, (M, K), 3.0)
    x[0, : min(K, 3)] = [np.float32(300.0), np.float32(-2.0), np.float32(0.0)][: min(K, 3)]
    if M > 2:
        x[1] = 0.0
    q, s = O.per_token_quant_fp8(x)
    q2, s2 = _torch_quant_restatement(x)
    assert np.array_equal(s, s2)
    assert np.array_equal(q, q2)


def test_quant_oracle_edge_rows():
    x = np.zeros((4, 8), np.float32)
    x[1, 3] = np.nan                    # NaN is ignored by the amax, then maps to 448
    x[1, 0] = 2.0
    x[2, 2] = -0.0
    x[3, :] = 1e-40                     # subnormal input row
    q, s = O.per_token_quant_fp8(x)
    assert s[0] == 0 and (q[0] == 0).all()
    assert s[1] == np.float32(2.0) / np.float32(448.0)
    assert q[1, 3] == 0x7E and q[1, 0] == 0x7E
    assert q[2, 2] == 0x80               # -0 keeps its sign
    assert s[3] > 0


def _torch_norm(x, g, b, sc, sh, nt, eps):
    """fp32 torch formulas from deploy/joyomni_ops/tests/test_parity_light.py:42-51 (layer)
    and the RMS branch of fused_norm_scale_shift.cu:118,136-139."""
    xf = torch.from_numpy(x).double()
    if nt == 0:
        mean = xf.mean(-1, keepdim=True)
        var = (xf - mean).pow(2).mean(-1, keepdim=True)
        n = (xf - mean) * torch.rsqrt(var + eps)
    else:
        n = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    if g is not None:
        n = n * torch.from_numpy(g).double()
        if nt == 0 and b is not None:
            n = n + torch.from_numpy(b).double()
    y = n * (1 + torch.from_numpy(sc).double()) + torch.from_numpy(sh).double()
    return y.float().numpy()


@pytest.mark.parametrize("nt", [0, 1])
@pytest.mark.parametrize("affine", [False, True])
def test_norm_oracle_vs_fp64(nt, affine):
    rng = np.random.default_rng(5 + nt)
    M, N = 37, 512
    x = randn(rng, (M, N))
    g = randn(rng, (N,)) if affine else None
    b = randn(rng, (N,)) if affine else None
    sc = randn(rng, (M, N), 0.1)
    sh = randn(rng, (M, N), 0.1)
    y = O.fused_norm_scale_shift(x, g, b, sc, sh, nt, 1e-6)
    assert_close_ulp(y, O.round_bf16(_torch_norm(x, g, b, sc, sh, nt, 1e-6)), max_ulp=1)


def test_rmsnorm_oracle_vs_fp64():
    rng = np.random.default_rng(11)
    x = randn(rng, (100, 128))
    w = randn(rng, (128,))
    xf = torch.from_numpy(x).double()
    ref = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * torch.from_numpy(w).double()).float()
    assert_close_ulp(O.rmsnorm(x, w, 1e-6), O.round_bf16(ref.numpy()), max_ulp=1)


def test_qk_norm_rope_oracle_vs_fp32_reference():
    """Against the interleaved-pair fp32 reference of test_parity_light.py:77-87."""
    rng = np.random.default_rng(3)
    B, L, H, D = 1, 16, 4, 128
    x = randn(rng, (B, L * H, D))
    w = randn(rng, (D,))
    c = randn(rng, (L, D // 2))
    s = randn(rng, (L, D // 2))
    got = O.qk_norm_rope(x, w, c, s, L, H, 1e-6)
    xf = torch.from_numpy(x).double().view(B, L, H, D)
    xn = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * torch.from_numpy(w).double()
    cc = torch.from_numpy(c).double().view(L, 1, D // 2)
    ss = torch.from_numpy(s).double().view(L, 1, D // 2)
    o = torch.empty_like(xn)
    o[..., 0::2] = xn[..., 0::2] * cc - xn[..., 1::2] * ss
    o[..., 1::2] = xn[..., 0::2] * ss + xn[..., 1::2] * cc
    assert_close_ulp(got, O.round_bf16(o.float().numpy().reshape(B, L * H, D)), max_ulp=2)


def _torch_rope_1d(dim, pos, theta):
    """deploy/xvideo/models/dit/rope.py:31-52 restated."""
    freqs = 1.0 / (theta ** (torch.arange(0, dim, 2)[: (dim // 2)].float() / dim))
    freqs = torch.outer(pos.float(), freqs)
    return freqs.cos().repeat_interleave(2, dim=1), freqs.sin().repeat_interleave(2, dim=1)


def test_rope_tables_match_reference_formula():
    T, H, W = 2, 4, 6
    c, s = O.rope_tables_3d((T, H, W))
    tt, hh, ww = torch.meshgrid(torch.arange(T), torch.arange(H), torch.arange(W), indexing="ij")
    cs, sn = [], []
    for p, d in zip((tt, hh, ww), (44, 42, 42)):
        a, b = _torch_rope_1d(d, p.reshape(-1), 10000.0)
        cs.append(a)
        sn.append(b)
    cref = torch.cat(cs, 1)[:, ::2].to(torch.bfloat16).float().numpy()
    sref = torch.cat(sn, 1)[:, ::2].to(torch.bfloat16).float().numpy()
    # numpy and torch cos/sin may differ by an fp32 ulp before the bf16 rounding
    assert np.abs(c - cref).max() <= 2 ** -8 and np.abs(s - sref).max() <= 2 ** -8
    assert (c != cref).mean() < 0.01


def test_weight_quant_oracle_matches_fp8_linear_formula():
    """deploy/xvideo/models/dit/fp8_linear.py:100-110 restated in torch."""
    rng = np.random.default_rng(9)
    w = randn(rng, (48, 64), 0.02)
    q, s = O.quantize_weight_per_channel(w)
    wt = torch.from_numpy(w).t().contiguous()
    amax = wt.abs().amax(dim=0).float().clamp_min(1e-8)
    sc = amax / 448.0
    wq = (wt / sc.unsqueeze(0)).clamp(-448, 448).to(torch.float8_e4m3fn)
    assert np.array_equal(s, sc.numpy())
    assert np.array_equal(q, wq.t().contiguous().view(torch.uint8).numpy())


def test_gemm_oracle_small_exact():
    rng = np.random.default_rng(1)
    M, N, K = 5, 7, 32
    a, sa = O.per_token_quant_fp8(randn(rng, (M, K)))
    b, sb = O.quantize_weight_per_channel(randn(rng, (N, K), 0.02))
    bias = randn(rng, (N,), 0.01)
    y = O.fp8_scaled_mm(a, b, sa, sb, bias)
    A = O.e4m3_decode(a).astype(np.float64)
    B = O.e4m3_decode(b).astype(np.float64)
    ref = (A @ B.T) * sb[None, :].astype(np.float64) * sa[:, None].astype(np.float64) + bias[None, :]
    assert_close_ulp(y, O.round_bf16(ref.astype(np.float32)), max_ulp=1)


# --------------------------------------------------------------------------
# golden fixtures from the reference's own kernels (tests/golden/*.npz)
# --------------------------------------------------------------------------
GOLDEN_FILES = sorted(glob.glob(os.path.join(GOLDEN, "*.npz")))


@pytest.mark.skipif(not GOLDEN_FILES, reason="no golden fixtures generated yet")
@pytest.mark.parametrize("path", GOLDEN_FILES, ids=[os.path.basename(p) for p in GOLDEN_FILES])
def test_oracle_against_reference_golden(path):
    import golden_cases
    golden_cases.check_oracle(path)


def test_torch_eager_cpu_path_agrees_with_oracle():
    """The eager-torch CPU baseline (oracle/torch_eager.py) computes the same
    config-2 chain as the oracle: scales to fp32 rounding, codes almost all equal."""
    import torch_eager
    rng = np.random.default_rng(12)
    M, N = 64, 1024
    x = randn(rng, (M, N))
    w = O.round_bf16(1 + 0.1 * rng.standard_normal(N).astype(np.float32))
    sh, sc = randn(rng, (N,), 0.1), randn(rng, (N,), 0.1)
    T = lambda a: torch.from_numpy(a).to(torch.bfloat16)  # noqa: E731
    q, s = torch_eager.cfg2_chain(T(x), T(w), T(sh), T(sc))
    y = O.fused_norm_scale_shift(x, w, None, sc, sh, 1, 1e-6)
    oq, os_ = O.per_token_quant_fp8(y)
    assert np.allclose(s.view(-1).numpy(), os_, rtol=1e-5)
    assert (q.view(torch.uint8).numpy() != oq).mean() < 2e-3


def _rn32(fr):
    """Round an exact rational to float32 (nearest, ties to even)."""
    from fractions import Fraction
    f = np.float32(float(fr))
    best, bd = f, abs(Fraction(float(f)) - fr)
    for c in (np.nextafter(f, np.float32(np.inf)), np.nextafter(f, np.float32(-np.inf))):
        d = abs(Fraction(float(c)) - fr)
        if d < bd or (d == bd and (c.view(np.uint32) & 1) == 0):
            best, bd = c, d
    return best


def test_div448_fma_sequence_exact_for_16bit_inputs():
    """The staged kernel forms the per-token scale amax / 448 as
    q = a * RN(1/448); r = fma(-q, 448, a); q + r * RN(1/448) (each step one
    IEEE rounding).  For every finite positive bf16 / fp16 amax that equals the
    correctly rounded quotient the reference computes."""
    from fractions import Fraction as F
    c = _rn32(F(1, 448))
    assert c == np.float32(1) / np.float32(448)
    for vals in ((np.arange(1, 0x7f80, dtype=np.uint32) << 16).view(np.float32),
                 np.arange(1, 0x7c00, dtype=np.uint16).view(np.float16).astype(np.float32)):
        for a in vals:
            A = F(float(a))
            q = _rn32(A * F(float(c)))
            r = _rn32(A - F(float(q)) * 448)
            assert _rn32(F(float(r)) * F(float(c)) + F(float(q))) == _rn32(A / 448), a


def test_rope_apply_oracle_matches_reference_formula():
    """O.rope_apply equals apply_rotary_emb of deploy/xvideo/models/dit/rope.py:14-28
    restated in torch (fp32 elementwise ops, bf16 result), bit for bit."""
    import torch
    rng = np.random.default_rng(5)
    L, H, D = 37, 3, 128
    x = O.round_bf16(rng.standard_normal((L, H, D)).astype(np.float32) * 3)
    c, s = O.rope_tables_3d_f32((1, 37, 1), t0=4)
    xt = torch.from_numpy(x).to(torch.bfloat16)
    cos = torch.from_numpy(c).repeat_interleave(2, dim=1)[:, None, :]
    sin = torch.from_numpy(s).repeat_interleave(2, dim=1)[:, None, :]
    xr, xi = xt.float().reshape(L, H, -1, 2).unbind(-1)
    rot = torch.stack([-xi, xr], dim=-1).flatten(-2)
    ref = (xt.float() * cos + rot * sin).to(torch.bfloat16).float().numpy()
    assert np.array_equal(O.rope_apply(x, c, s), ref)
