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
  restatement of the reference block, whole (bounded by the spread between
  two valid attention kernels) and stage by stage.
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


@pytest.fixture(scope="module")
def block4(cuda):
    """One block at config-4 dims with a full 2-chunk cache (21060 keys) and its inputs."""
    from joyomni_stack import Stack, StackConfig
    cfg = StackConfig(layers=1)
    st = Stack(cfg, cuda)
    gen = torch.Generator(device=cuda).manual_seed(3)
    st.kv[0].fill_random(gen, cfg.cache_chunks)
    img, txt = st.inputs(7)
    yield st, img.to(torch.bfloat16), txt, st.timestep_vec(1000)
    st.close()


def test_block_at_config4_dims(cuda, block4):
    """The whole block against its eager restatement.  Any two valid bf16
    attention kernels differ by bf16 rounding flips, which the per-token FP8
    requantisations that follow amplify; the bound is therefore set by the
    spread between two valid references: the restatement with torch's bf16
    SDPA (the reference model's own fallback, dit.py:150-158) against the same
    restatement with fp32 attention.  This repository's block (tcgen05
    attention) must be at least as close to the fp32-attention restatement as
    the SDPA one is (x1.25 + 1e-3); as a sanity bound, within 5e-2 of both
    (measured: 2.6e-2 against fp32 attention, where SDPA sits at 2.55e-2, and
    1.5e-2 against the SDPA restatement)."""
    import stack_reference as R
    st, img, txt, vec = block4
    kv = st.kv[0]
    assert kv.valid == 21060
    ck = kv.k[kv.cur: kv.cur + kv.valid].clone()
    cv = kv.v[kv.cur: kv.cur + kv.valid].clone()
    st.cfg.attention = "joyomni"
    out_img, out_txt = st.blocks[0].forward(img, txt, vec, st.cos, st.sin, kv, st.sp)
    out_img, out_txt = out_img.clone(), out_txt.clone()
    torch.cuda.synchronize()
    sd_img, sd_txt, _, _ = R.block_forward(st.blocks[0], img, txt, vec, st.cos, st.sin, ck, cv, attn="sdpa")
    f_img, f_txt, _, _ = R.block_forward(st.blocks[0], img, txt, vec, st.cos, st.sin, ck, cv, attn="fp32")
    e_ours = max(rel_rms(to_np(out_img), to_np(f_img)), rel_rms(to_np(out_txt), to_np(f_txt)))
    e_sdpa = max(rel_rms(to_np(sd_img), to_np(f_img)), rel_rms(to_np(sd_txt), to_np(f_txt)))
    e_vs_sdpa = max(rel_rms(to_np(out_img), to_np(sd_img)), rel_rms(to_np(out_txt), to_np(sd_txt)))
    print(f"\nconfig-4 block rel RMS: ours vs fp32-attention restatement {e_ours:.3e}, SDPA restatement vs "
          f"fp32-attention restatement {e_sdpa:.3e}, ours vs SDPA restatement {e_vs_sdpa:.3e}")
    assert torch.isfinite(out_img).all() and torch.isfinite(out_txt).all()
    assert e_ours <= 1.25 * e_sdpa + 1e-3
    assert e_ours <= 5e-2 and e_vs_sdpa <= 5e-2


def test_block_stages_at_config4_dims(jo, cuda, block4):
    """Stage by stage at config-4 dims, each stage fed the restatement's own
    input so that nothing upstream is amplified: norm -> modulate -> FP8 codes,
    the FP8 GEMMs with their fused epilogues (bias, GELU, gated residual)."""
    import stack_reference as R
    from joyomni_stack.mmdit import norm_mod_quant
    st, img, txt, vec = block4
    blk = st.blocks[0]
    im = (blk.img.mod + vec).unbind(0)

    def rel(a, b):
        return rel_rms(to_np(a), to_np(b))
    yref = R.ln_mod(img, im[0], im[1])
    qr, sr = R.quant(yref)
    xq, xs = norm_mod_quant(img, im[0], im[1])
    code_frac = (xq.float() != qr).float().mean().item()
    qkv_ref = R.lin(qr, sr, blk.img.qkv)
    qkv = blk.img.qkv(qr.to(torch.float8_e4m3fn), sr.contiguous())
    attn = torch.randn(img.shape[0], st.cfg.hidden, generator=torch.Generator(device=cuda).manual_seed(9),
                       device=cuda).to(torch.bfloat16)
    aq, as_ = R.quant(attn)
    pr_ref = torch.addcmul(img, R.lin(aq, as_, blk.img.proj), im[2])
    pr = blk.img.proj.residual(aq.to(torch.float8_e4m3fn), as_.contiguous(), img, im[2])
    hq, hs = R.quant(R.ln_mod(pr_ref, im[3], im[4]))
    up_ref = R.lin(hq, hs, blk.img.up, gelu=True)
    up = blk.img.up(hq.to(torch.float8_e4m3fn), hs.contiguous(), gelu=True)
    h2q, h2s = R.quant(up_ref)
    dn_ref = torch.addcmul(pr_ref, R.lin(h2q, h2s, blk.img.down), im[5])
    dn = blk.img.down.residual(h2q.to(torch.float8_e4m3fn), h2s.contiguous(), pr_ref.clone(), im[5])
    res = {"norm_mod_quant_code_frac": code_frac, "qkv": rel(qkv, qkv_ref), "proj_resid": rel(pr, pr_ref),
           "up_gelu": rel(up, up_ref), "down_resid": rel(dn, dn_ref)}
    print("\nconfig-4 stages:", {k: f"{v:.2e}" for k, v in res.items()})
    assert res["norm_mod_quant_code_frac"] <= 1e-4
    assert res["qkv"] <= 1e-3 and res["proj_resid"] <= 1e-3 and res["down_resid"] <= 1e-3
    assert res["up_gelu"] <= 2e-3
