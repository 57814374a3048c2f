"""GPU parity of the pre-RoPE KV-cache path (the reference's
kv_cache_pre_rope=True mode): keys are cached after the per-head RMSNorm
(rmsnorm_qk_bf16, deploy/xvideo/models/dit/dit.py:360-363) and rotated at the
positions they take in the attention window when the cache is assembled
(apply_rotary_emb, rope.py:21-28, at dit.py:211-217 and
deploy/xvideo/serving/graph_runner.py:137-142).

* joyomni_ops.rope_apply against the oracle restatement of apply_rotary_emb:
  bit-exact (fp32 products and sums rounded as torch's elementwise ops do);
* the stack in pre-RoPE mode over several chunks: the staged keys equal the
  oracle RMSNorm of the raw keys (2 bf16 ulps, the norm tolerance), and every
  cached slot of the attention buffer equals the oracle rotation of its stored
  keys at its shifted window position, bit for bit (given the same fp32
  tables)."""
import numpy as np
import pytest
import torch

import joyomni_oracle as O
from _util import assert_close_ulp, randn, to_np, to_torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def jo(cuda):
    import joyomni_ops
    return joyomni_ops


@pytest.mark.parametrize("L,H,D,t0", [(37, 3, 128, 0), (10, 2, 64, 5), (6, 1, 256, 2), (1170, 4, 128, 6)])
def test_rope_apply_bitexact(jo, cuda, L, H, D, t0):
    rng = np.random.default_rng(L + H + D)
    x = randn(rng, (L, H, D), 2.0)
    if D == 128:
        c, s = O.rope_tables_3d_f32((1, L, 1), t0=t0)
    else:
        ang = rng.standard_normal((L, D // 2)).astype(np.float32) * 3
        c, s = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    ct, st = torch.from_numpy(c).to(cuda), torch.from_numpy(s).to(cuda)
    got = jo.rope_apply(to_torch(x, "bf16", cuda), ct, st)
    assert np.array_equal(to_np(got), O.rope_apply(x, c, s))


def test_rope_apply_strided_and_in_place(jo, cuda):
    rng = np.random.default_rng(3)
    L, H, D = 50, 4, 128
    big = to_torch(randn(rng, (L, 3, H, D)), "bf16", cuda)   # k third of a [L, 3, H, D] buffer
    k = big[:, 1]
    ref = O.rope_apply(to_np(k), *O.rope_tables_3d_f32((1, 5, 10), t0=1))
    c, s = (torch.from_numpy(t).to(cuda) for t in O.rope_tables_3d_f32((1, 5, 10), t0=1))
    before_q = big[:, 0].clone()
    jo.rope_apply(k, c, s, out=k)
    assert np.array_equal(to_np(big[:, 1]), ref)
    assert torch.equal(big[:, 0], before_q)


def test_stack_pre_rope_cache(jo, cuda):
    from joyomni_stack import Stack, StackConfig
    cfg = StackConfig(hidden=512, heads=4, ffn=1376, layers=2, img_tokens=130, txt_tokens=24, grid=(1, 10, 13),
                      cache_chunks=2, seed=11, kv_cache_pre_rope=True)
    st = Stack(cfg, cuda)
    for kv in st.kv:
        kv.keep_q = True
    x, txt = st.inputs(1)
    for chunk in range(3):
        x = st.denoise_chunk(x, txt)
        for li, kv in enumerate(st.kv):
            # staged keys (last step of the chunk) = RMSNorm of the raw image keys
            raw = to_np(kv.last_k_raw[:cfg.img_tokens]).reshape(-1, cfg.head_dim)
            kn = to_np(st.blocks[li].img.k_norm)
            assert_close_ulp(to_np(kv.stage).reshape(-1, cfg.head_dim), O.rmsnorm(raw, kn, 1e-6))
            # every cached slot = rotation of its stored keys at its window position
            assert kv.slot_age and len(kv.slot_age) == min(chunk + 1, 2)
            for age, slot in enumerate(kv.slot_age):
                r0 = slot * cfg.img_tokens
                # the same fp32 table tensors the kernel consumed (torch's cos / sin
                # may differ from numpy's by an ulp; the oracle restates the rotation)
                c, s = (t.cpu().numpy() for t in st.window_tables(age))
                want = O.rope_apply(to_np(kv.kpre[r0:r0 + cfg.img_tokens]), c, s)
                got = to_np(kv.k[kv.cur + r0: kv.cur + r0 + cfg.img_tokens])
                assert np.array_equal(got, want), (chunk, li, age)
    assert torch.isfinite(x).all()
    # the newest slot holds the last chunk's staged keys
    kv = st.kv[0]
    newest = kv.slot_age[-1]
    assert torch.equal(kv.kpre[newest * cfg.img_tokens:(newest + 1) * cfg.img_tokens], kv.stage)
    st.close()


def test_stack_pre_rope_step_graph(cuda):
    """The pre-RoPE mode captures into the step graph and replays like eager."""
    from joyomni_stack import Stack, StackConfig
    cfg = StackConfig(hidden=512, heads=4, ffn=1376, layers=2, img_tokens=130, txt_tokens=24, grid=(1, 10, 13),
                      cache_chunks=2, seed=11, kv_cache_pre_rope=True)
    outs = []
    for use_graph in (False, True):
        st = Stack(cfg, cuda)
        gen = torch.Generator(device=cuda).manual_seed(3)
        for kv in st.kv:
            kv.fill_random(gen, 2, st.window_tables)
        x, txt = st.inputs(4)
        if use_graph:
            assert st.capture(txt), getattr(st, "capture_error", "")
        x = st.denoise_chunk(x, txt)
        x = st.denoise_chunk(x, txt)
        outs.append(x)
        st.close()
    a, b = outs[1].float(), outs[0].float()
    assert ((a - b).pow(2).mean().sqrt() / b.pow(2).mean().sqrt()).item() < 1e-6
