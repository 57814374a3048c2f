"""Parity at the benchmarked configurations themselves (not only at small
shapes):

* the headline step of bench.py -- BASELINE config 2, x bf16 [10530, 5120]
  seed 2 with 1 % x50 outliers, RMS norm with a bf16 weight, [N] shift/scale --
  through the fused entry norm_modulate_quant_fp8, against the oracle chain
  fused_norm_scale_shift -> per_token_quant_fp8 (the reference model's
  dit.py:351-357 -> fp8_linear.py:143-167).  The fraction of differing codes
  and scales is printed and bounded by 1e-4;
* the same input through the reference API: K2 with the modulation expanded to
  a dense [M, N] tensor (sgl_fused_ops.py:44-51), then K4; the codes and scales
  must be bit-identical to quantising that K2 output, and K2 within the stated
  norm tolerance of the oracle;
* one MMDiT block at BASELINE config 4 dims (hidden 5120, 40 heads x 128, FFN
  13824, 10530 image + 512 text tokens, 21060 cached keys) against the eager
  restatement of the reference block, relative RMS <= 1e-2.
"""
import numpy as np
import pytest
import torch

import joyomni_oracle as O
from _util import assert_close_ulp, codes_np, rel_rms, to_np

pytestmark = pytest.mark.gpu

M, N = 10530, 5120


@pytest.fixture(scope="module")
def jo(cuda):
    import joyomni_ops
    return joyomni_ops


@pytest.fixture(scope="module")
def cfg2(cuda):
    from bench import make_cfg2_inputs
    x, w, sh, sc = make_cfg2_inputs(torch, "cpu", 2)
    xn, wn, shn, scn = (t.float().numpy() for t in (x, w, sh, sc))
    y = O.fused_norm_scale_shift(xn, wn, None, scn, shn, 1, 1e-6)
    oq, os_ = O.per_token_quant_fp8(y)
    dev = [t.to(cuda) for t in (x, w, sh, sc)]
    return dev, y, oq, os_


def test_headline_fused_entry_matches_oracle_chain(jo, cuda, cfg2):
    (x, w, sh, sc), y, oq, os_ = cfg2
    q = torch.empty((M, N), dtype=torch.float8_e4m3fn, device=cuda)
    s = torch.empty(M, dtype=torch.float32, device=cuda)
    jo.norm_modulate_quant_fp8(x, w, None, sc, sh, "rms", 1e-6, q, s)
    codes = codes_np(q)
    scales = s.cpu().numpy()
    code_frac = float((codes != oq).mean())
    scale_frac = float((scales.view(np.uint32) != os_.view(np.uint32)).mean())
    print(f"\nheadline cfg2 fused entry vs oracle chain: differing codes {code_frac:.3e} "
          f"({int((codes != oq).sum())} of {codes.size}), differing scales {scale_frac:.3e} "
          f"({int((scales != os_).sum())} of {M})")
    assert code_frac <= 1e-4
    assert scale_frac <= 1e-3


def test_headline_reference_api_chain(jo, cuda, cfg2):
    (x, w, sh, sc), y, oq, os_ = cfg2
    # the shim of the reference model materialises [M, N] modulation rows
    y_k2 = jo.fused_norm_scale_shift(x, w, None, sc.expand(M, N).contiguous(), sh.expand(M, N).contiguous(),
                                     "rms", 1e-6)
    yk = to_np(y_k2)
    assert_close_ulp(yk, y)
    print(f"\nK2 [M,N] modulation: bf16 outputs differing from the oracle {float((yk != y).mean()):.3e}")
    q = torch.empty((M, N), dtype=torch.float8_e4m3fn, device=cuda)
    s = torch.empty((M, 1), dtype=torch.float32, device=cuda)
    jo.sgl_per_token_quant_fp8(y_k2, q, s)
    rq, rs = O.per_token_quant_fp8(yk)
    assert np.array_equal(s.view(-1).cpu().numpy().view(np.uint32), rs.view(np.uint32))
    assert np.array_equal(codes_np(q), rq)
    print(f"K2 -> K4 chain vs oracle chain: differing codes {float((codes_np(q) != oq).mean()):.3e}")


def test_block_at_config4_dims(cuda):
    import stack_reference as R
    from joyomni_stack import Stack, StackConfig
    cfg = StackConfig(layers=1)
    st = Stack(cfg, cuda)
    gen = torch.Generator(device=cuda).manual_seed(3)
    st.kv[0].fill_random(gen, cfg.cache_chunks)
    img, txt = st.inputs(7)
    img = img.to(torch.bfloat16)
    vec = st.timestep_vec(1000)
    kv = st.kv[0]
    assert kv.valid == 21060
    ck = kv.k[kv.cur: kv.cur + kv.valid].clone()
    cv = kv.v[kv.cur: kv.cur + kv.valid].clone()
    out_img, out_txt = st.blocks[0].forward(img, txt, vec, st.cos, st.sin, kv, st.sp)
    torch.cuda.synchronize()
    ref_img, ref_txt, _, _ = R.block_forward(st.blocks[0], img, txt, vec, st.cos, st.sin, ck, cv)
    ri, rt = rel_rms(to_np(out_img), to_np(ref_img)), rel_rms(to_np(out_txt), to_np(ref_txt))
    print(f"\nconfig-4 block vs eager restatement: rel RMS img {ri:.3e} txt {rt:.3e}")
    assert torch.isfinite(out_img).all() and torch.isfinite(out_txt).all()
    assert ri <= 1e-2 and rt <= 1e-2
    st.close()
