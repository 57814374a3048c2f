"""Drop-in check through the reference's own, unmodified glue.

The reference's model calls the operators only through two modules:
``deploy/xvideo/models/dit/sgl_fused_ops.py`` (``from joyomni_ops import
fused_norm_scale_shift, fused_qk_norm_rope_3d_paired, rmsnorm``, line 22) and
``deploy/xvideo/models/dit/fp8_linear.py`` (``from joyomni_ops import
fp8_scaled_mm, sgl_per_token_quant_fp8``, line 9).  This test imports those two
files by path from the reference checkout named by ``$JO_REFERENCE_ROOT`` (it
is skipped when that variable is unset or the files are absent; nothing of the
reference is kept in this repository), with this repository's ``joyomni_ops``
first on the import path, and runs the calls the DiT block makes:

* ``fused_layernorm_modulate`` with ``[B, D]`` modulation (the glue expands it
  to ``[B, L, D]`` and makes it contiguous, sgl_fused_ops.py:44-51);
* ``fused_qk_norm_rope_3d`` with ``[L, 128]`` repeat-interleaved tables (the
  glue keeps ``[..., ::2]`` and casts to bf16, sgl_fused_ops.py:87-96) on q/k
  that are strided views of a QKV buffer (dit.py:358-359);
* ``rmsnorm_qk_bf16`` on the pre-RoPE keys (dit.py:360-363);
* ``Fp8Linear.from_linear`` + ``forward`` (weight quantised by the reference's
  torch code on the GPU, fp8_linear.py:100-110; activation quant + GEMM
  through this repository, fp8_linear.py:143-167, ``[M, 1]`` activation
  scales).

Each result is compared with the CPU oracle under the suite's tolerances:
norm / RoPE outputs within 2 bf16 ulps and 2e-3 relative RMS, the weight codes
and scales bit-exact, the linear within 1e-3 relative RMS of the exact
dequantised product."""
from __future__ import annotations

import importlib.util
import os
import sys

import numpy as np
import pytest
import torch

import joyomni_oracle as O
from _util import assert_close_ulp, randn, rel_rms, to_np, to_torch

pytestmark = pytest.mark.gpu

_GLUE = ("sgl_fused_ops", "fp8_linear")


def _glue_dir():
    root = os.environ.get("JO_REFERENCE_ROOT")
    if not root:
        return None
    d = os.path.join(root, "deploy", "xvideo", "models", "dit")
    return d if all(os.path.isfile(os.path.join(d, g + ".py")) for g in _GLUE) else None


@pytest.fixture(scope="module")
def glue(cuda):
    d = _glue_dir()
    if d is None:
        pytest.skip("reference glue not found (set JO_REFERENCE_ROOT to the reference checkout)")
    import joyomni_ops  # this repository's package, already first on sys.path
    assert "joyai-video-edit_b200" in os.path.dirname(joyomni_ops.__file__)
    mods = {}
    for g in _GLUE:
        spec = importlib.util.spec_from_file_location("_ref_glue_" + g, os.path.join(d, g + ".py"))
        m = importlib.util.module_from_spec(spec)
        sys.modules[spec.name] = m
        spec.loader.exec_module(m)
        mods[g] = m
    assert mods["sgl_fused_ops"].available()
    return mods


def test_layernorm_modulate_through_glue(glue, cuda):
    B, L, D = 2, 300, 3072
    rng = np.random.default_rng(71)
    x = randn(rng, (B, L, D))
    sh, sc = randn(rng, (B, D), 0.1), randn(rng, (B, D), 0.1)
    T = lambda a: to_torch(a, "bf16", cuda)  # noqa: E731
    y = glue["sgl_fused_ops"].fused_layernorm_modulate(T(x), T(sh), T(sc), eps=1e-6)
    assert y.shape == (B, L, D) and y.dtype == torch.bfloat16
    ref = np.concatenate([O.fused_norm_scale_shift(x[b], None, None, np.broadcast_to(sc[b], (L, D)),
                                                   np.broadcast_to(sh[b], (L, D)), 0, 1e-6) for b in range(B)])
    assert_close_ulp(to_np(y).reshape(B * L, D), ref)


def test_qk_norm_rope_through_glue(glue, cuda):
    grid = (2, 8, 12)
    L, H, D = grid[0] * grid[1] * grid[2], 8, 128
    rng = np.random.default_rng(72)
    qkv = randn(rng, (1, L, 3, H, D))
    qw = 1 + 0.1 * rng.standard_normal(D).astype(np.float32)     # fp32 weights, cast by the glue
    kw = 1 + 0.1 * rng.standard_normal(D).astype(np.float32)
    c, s = O.rope_tables_3d(grid)                                 # [L, 64] bf16-exact
    cf, sf = np.repeat(c, 2, axis=1), np.repeat(s, 2, axis=1)    # the model's [L, 128] form
    t = to_torch(qkv, "bf16", cuda)
    q, k = t[:, :, 0], t[:, :, 1]                                 # strided views, as dit.py:358-359
    freqs = (torch.from_numpy(cf).to(cuda), torch.from_numpy(sf).to(cuda))
    q2, k2 = glue["sgl_fused_ops"].fused_qk_norm_rope_3d(q, k, torch.from_numpy(qw).to(cuda),
                                                         torch.from_numpy(kw).to(cuda), freqs, eps=1e-6)
    qwb, kwb = O.round_bf16(qw), O.round_bf16(kw)
    rq = O.qk_norm_rope(qkv[:, :, 0].reshape(1, L * H, D), qwb, c, s, L, H, 1e-6)
    rk = O.qk_norm_rope(qkv[:, :, 1].reshape(1, L * H, D), kwb, c, s, L, H, 1e-6)
    assert_close_ulp(to_np(q2).reshape(1, L * H, D), rq)
    assert_close_ulp(to_np(k2).reshape(1, L * H, D), rk)


def test_rmsnorm_qk_through_glue(glue, cuda):
    L, H, D = 777, 8, 128
    rng = np.random.default_rng(73)
    k = randn(rng, (1, L, H, D))
    w = 1 + 0.1 * rng.standard_normal(D).astype(np.float32)
    out = glue["sgl_fused_ops"].rmsnorm_qk_bf16(to_torch(k, "bf16", cuda), torch.from_numpy(w).to(cuda), 1e-6)
    assert out.shape == (1, L, H, D)
    ref = O.rmsnorm(k.reshape(-1, D), O.round_bf16(w), 1e-6)
    assert_close_ulp(to_np(out).reshape(-1, D), ref)


@pytest.mark.parametrize("gelu_after", [False, True])
def test_fp8_linear_through_glue(glue, cuda, gelu_after):
    fl = glue["fp8_linear"]
    if getattr(fl, "_FAST_ACCUM", False):
        pytest.skip("JOYOMNI_FP8_FAST_ACCUM selects the GeForce Triton branch, not this operator set")
    B, L, K, N = 1, 1000, 1024, 768
    rng = np.random.default_rng(74 + gelu_after)
    w = randn(rng, (N, K), 0.02)
    b = randn(rng, (N,), 0.01)
    x = randn(rng, (B, L, K))
    lin = torch.nn.Linear(K, N, bias=True).to(cuda)
    with torch.no_grad():
        lin.weight.copy_(torch.from_numpy(w))
        lin.bias.copy_(torch.from_numpy(b))
    m = fl.Fp8Linear.from_linear(lin)
    # the reference's own weight quantisation, run by torch on the GPU, agrees
    # with the oracle's restatement of it (scale by reciprocal multiply there)
    wq, ws = O.quantize_weight_per_channel(w, on_cuda=True)
    assert m.weight_fp8.shape == (K, N) and m.weight_fp8.stride() == (1, K)
    assert np.array_equal(m.weight_fp8.t().contiguous().view(torch.uint8).cpu().numpy(), wq)
    assert np.array_equal(m.weight_scale.cpu().numpy(), ws)
    y = m(to_torch(x, "bf16", cuda))
    assert y.shape == (B, L, N) and y.dtype == torch.bfloat16
    aq, sa = O.per_token_quant_fp8(x.reshape(-1, K))
    ref = O.fp8_scaled_mm(aq, wq, sa, ws, b)
    got = to_np(y).reshape(-1, N)
    if gelu_after:  # the model applies F.gelu(tanh) to the bf16 linear output (dit.py:90-92)
        got = to_np(torch.nn.functional.gelu(y, approximate="tanh")).reshape(-1, N)
        ref = O.gelu_tanh(ref)
        assert rel_rms(got, ref) <= 2e-3
    else:
        assert rel_rms(got, ref) <= 1e-3
