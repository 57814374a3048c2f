"""Parity at the shipped model's shapes, which differ from BASELINE's synthetic
ones: hidden 4096, 32 heads x 128, FFN 16384 (deploy/xvideo/config.py:22-25,
dit.py:268) and the steady-state DiT sequence of 1560 tokens
(deploy/joyomni_ops/tests/test_bench.py:113).  LayerNorm without affine is the
model's norm (dit.py:271-273 -> sgl_fused_ops.py:53); RMS is checked too.
Same tolerances as the other parity tests: codes and scales bit-exact against
quantising this repository's own norm output, norm outputs within 2 bf16 ulps
of the oracle, GEMMs within 1e-3 relative RMS of the exact-dequant oracle."""
import numpy as np
import pytest
import torch

import joyomni_oracle as O
from _util import assert_close_ulp, codes_np, outlier_activations, randn, to_np, to_torch

pytestmark = pytest.mark.gpu

L, D, H, FFN = 1560, 4096, 32, 16384


@pytest.fixture(scope="module")
def jo(cuda):
    import joyomni_ops
    return joyomni_ops


@pytest.mark.parametrize("nt", [0, 1])
def test_norm_modulate_quant_hidden_4096(jo, cuda, nt):
    rng = np.random.default_rng(40 + nt)
    x = outlier_activations(rng, L, D)
    sc, sh = randn(rng, (D,), 0.1), randn(rng, (D,), 0.1)
    T = lambda a: to_torch(a, "bf16", cuda)  # noqa: E731
    yo = O.fused_norm_scale_shift(x, None, None, sc, sh, nt, 1e-6)
    y = jo.fused_norm_scale_shift(T(x), None, None, T(sc).expand(L, D), T(sh).expand(L, D), nt, 1e-6)
    assert_close_ulp(to_np(y), yo)
    q = torch.empty((L, D), dtype=torch.float8_e4m3fn, device=cuda)
    s = torch.empty(L, dtype=torch.float32, device=cuda)
    jo.norm_modulate_quant_fp8(T(x), None, None, T(sc), T(sh), nt, 1e-6, q, s)
    rq, rs = O.per_token_quant_fp8(to_np(y))
    assert np.array_equal(s.cpu().numpy(), rs)
    assert np.array_equal(codes_np(q), rq)
    oq, _ = O.per_token_quant_fp8(yo)
    assert (codes_np(q) != oq).mean() <= 1e-4


@pytest.mark.parametrize("K", [D, FFN])
def test_per_token_quant_shipped(jo, cuda, K):
    rng = np.random.default_rng(K)
    x = outlier_activations(rng, 257, K)
    q = torch.empty((257, K), dtype=torch.float8_e4m3fn, device=cuda)
    s = torch.empty((257, 1), dtype=torch.float32, device=cuda)
    jo.sgl_per_token_quant_fp8(to_torch(x, "bf16", cuda), q, s)
    rq, rs = O.per_token_quant_fp8(x)
    assert np.array_equal(s.view(-1).cpu().numpy().view(np.uint32), rs.view(np.uint32))
    assert np.array_equal(codes_np(q), rq)


def test_qk_norm_rope_seq1560_32_heads(jo, cuda):
    """The kernel bench's steady-state shape: L = 1560 (a 1 x 30 x 52 token grid), 32 heads."""
    rng = np.random.default_rng(1560)
    q, k = randn(rng, (1, L * H, 128)), randn(rng, (1, L * H, 128))
    qw = O.round_bf16(1 + 0.1 * rng.standard_normal(128).astype(np.float32))
    kw = O.round_bf16(1 + 0.1 * rng.standard_normal(128).astype(np.float32))
    c, s = O.rope_tables_3d((1, 30, 52))
    qt, kt = to_torch(q, "bf16", cuda), to_torch(k, "bf16", cuda)
    jo.fused_qk_norm_rope_3d_paired(qt, kt, L, H, 1e-6, to_torch(qw, "bf16", cuda), to_torch(kw, "bf16", cuda),
                                    to_torch(c, "bf16", cuda), to_torch(s, "bf16", cuda))
    assert_close_ulp(to_np(qt), O.qk_norm_rope(q, qw, c, s, L, H, 1e-6))
    assert_close_ulp(to_np(kt), O.qk_norm_rope(k, kw, c, s, L, H, 1e-6))


@pytest.mark.parametrize("N,K,gelu", [(3 * D, D, False), (FFN, D, True), (D, FFN, False)])
def test_fp8_gemm_shipped_shapes(jo, cuda, N, K, gelu):
    """QKV projection, FFN up (+ GELU) and FFN down of the shipped model at
    1560 tokens, on a row sample checked against the oracle."""
    if not jo.has_fp8():
        pytest.skip("GEMM not built")
    rng = np.random.default_rng(N + K)
    a, sa = O.per_token_quant_fp8(randn(rng, (L, K)))
    b, sb = O.quantize_weight_per_channel(randn(rng, (N, K), 0.02))
    bias = randn(rng, (N,), 0.01)
    f = jo.fp8_scaled_mm_gelu if gelu else jo.fp8_scaled_mm
    y = f(torch.from_numpy(a).to(cuda).view(torch.float8_e4m3fn),
          torch.from_numpy(b).to(cuda).view(torch.float8_e4m3fn).t(), torch.from_numpy(sa).to(cuda),
          torch.from_numpy(sb).to(cuda), torch.bfloat16, to_torch(bias, "bf16", cuda)).float().cpu().numpy()
    rows = np.unique(np.concatenate([rng.integers(0, L, 20), [0, 255, 256, L - 1]]))
    ref = O.fp8_scaled_mm(a[rows], b, sa[rows], sb, bias, epilogue="gelu_tanh" if gelu else "none")
    if gelu:
        from test_gemm_gpu import assert_close_gelu
        assert_close_gelu(y[rows], ref, O.fp8_scaled_mm(a[rows], b, sa[rows], sb, bias))
    else:
        assert_close_ulp(y[rows], ref, max_ulp=2, rel_rms=1e-3)
    assert np.isfinite(y).all()
