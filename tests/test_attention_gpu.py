"""GPU parity of the tcgen05 attention kernel (joyomni_ops.attention, the
replacement of the reference block's FA4 / SDPA call, dit.py:150-178) against
an fp32 torch reference of the same op: softmax(q k^T / sqrt(128)) v.

Tolerance: relative RMS error <= 4e-3 against fp32, and at most 1.5x (+1e-4)
the error of torch's own bf16 SDPA on the same inputs; the kernel rounds P to
bf16 before the PV product and the output to bf16, as flash attention kernels do.
Cases cover ragged query and key counts (partial tiles on both sides), a
single key, strided NHD views, batches, keys whose scale grows along the
sequence (the running-max rescale path), and the config-4 shape of the block
(11042 queries x 32102 keys, 40 heads) on sampled heads and rows."""
import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def jo(cuda):
    import joyomni_ops
    return joyomni_ops


def ref_attn(q, k, v, scale=None):
    """fp32 reference over [B, L, H, D] tensors."""
    sc = 1.0 / math.sqrt(q.shape[-1]) if scale is None else scale
    qf, kf, vf = (t.float().permute(0, 2, 1, 3) for t in (q, k, v))
    p = torch.softmax((qf @ kf.transpose(-1, -2)) * sc, dim=-1)
    return (p @ vf).permute(0, 2, 1, 3)


def sdpa_bf16(q, k, v):
    return F.scaled_dot_product_attention(q.permute(0, 2, 1, 3), k.permute(0, 2, 1, 3),
                                          v.permute(0, 2, 1, 3)).permute(0, 2, 1, 3)


def rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).pow(2).mean().sqrt() / b.pow(2).mean().sqrt()).item()


def check(got, q, k, v):
    ref = ref_attn(q, k, v)
    e = rel(got, ref)
    e_sdpa = rel(sdpa_bf16(q, k, v), ref)
    assert torch.isfinite(got).all()
    assert e <= 4e-3 and e <= 1.5 * e_sdpa + 1e-4, (e, e_sdpa)
    return e, e_sdpa


@pytest.mark.parametrize("B,Lq,Lk,H", [(1, 100, 77, 2), (1, 256, 256, 1), (2, 300, 513, 3), (1, 1, 1, 1),
                                       (1, 257, 129, 2), (1, 1000, 3000, 4), (3, 64, 700, 1)])
def test_attention_matches_fp32(jo, cuda, B, Lq, Lk, H):
    g = torch.Generator(device=cuda).manual_seed(B * 1000 + Lq + Lk + H)
    q = torch.randn(B, Lq, H, 128, generator=g, device=cuda).to(torch.bfloat16)
    k = torch.randn(B, Lk, H, 128, generator=g, device=cuda).to(torch.bfloat16)
    v = torch.randn(B, Lk, H, 128, generator=g, device=cuda).to(torch.bfloat16)
    check(jo.attention(q, k, v), q, k, v)


def test_attention_strided_views_and_out(jo, cuda):
    """q, k, v as the thirds of a [L, 3, H, 128] QKV buffer (token stride 3*H*128),
    output into a strided slice of a larger buffer."""
    g = torch.Generator(device=cuda).manual_seed(5)
    L, H = 333, 4
    qkv = torch.randn(1, L, 3, H, 128, generator=g, device=cuda).to(torch.bfloat16)
    q, k, v = qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]
    big = torch.full((1, L, 2 * H, 128), 7.0, dtype=torch.bfloat16, device=cuda)
    out = big[:, :, H:]
    jo.attention(q, k, v, out=out)
    check(out, q, k, v)
    assert bool((big[:, :, :H] == 7.0).all())


def test_attention_growing_scores(jo, cuda):
    """Key norms grow 40x along the sequence, so the running max rises many
    times across key tiles (the lazy O rescale in tensor memory)."""
    g = torch.Generator(device=cuda).manual_seed(9)
    Lq, Lk, H = 256, 2048, 2
    q = torch.randn(1, Lq, H, 128, generator=g, device=cuda)
    k = torch.randn(1, Lk, H, 128, generator=g, device=cuda) * torch.linspace(0.1, 4.0, Lk, device=cuda)[None, :, None,
                                                                                                         None]
    v = torch.randn(1, Lk, H, 128, generator=g, device=cuda)
    q, k, v = (t.to(torch.bfloat16) for t in (q, k, v))
    check(jo.attention(q, k, v), q, k, v)


def test_attention_3d_views_and_errors(jo, cuda):
    q = torch.randn(50, 2, 128, device=cuda).to(torch.bfloat16)
    out = jo.attention(q, q, q)
    assert out.shape == (50, 2, 128)
    check(out[None], q[None], q[None], q[None])
    with pytest.raises(RuntimeError):
        jo.attention(q.float(), q.float(), q.float())
    with pytest.raises(RuntimeError):
        jo.attention(q[..., :64], q[..., :64], q[..., :64])


def test_attention_config4_shape(jo, cuda):
    """BASELINE config 4 at P = 1: 10530 + 512 queries, 2 x 10530 cached + 11042
    current keys, 40 heads; fp32 reference on 3 heads x 1024 sampled queries."""
    g = torch.Generator(device=cuda).manual_seed(4)
    Lq, Lk, H = 11042, 32102, 40
    q = torch.randn(Lq, H, 128, generator=g, device=cuda).to(torch.bfloat16)
    k = torch.randn(Lk, H, 128, generator=g, device=cuda).to(torch.bfloat16)
    v = torch.randn(Lk, H, 128, generator=g, device=cuda).to(torch.bfloat16)
    out = jo.attention(q, k, v)
    torch.cuda.synchronize()
    rows = torch.randperm(Lq, generator=torch.Generator().manual_seed(1))[:1024].to(cuda)
    for h in (0, 17, 39):
        qs = q[rows, h:h + 1][None]
        ks, vs = k[:, h:h + 1][None], v[:, h:h + 1][None]
        e, e_sdpa = check(out[rows, h:h + 1][None], qs, ks, vs)
        print(f"head {h}: rel RMS vs fp32 {e:.2e} (torch bf16 SDPA {e_sdpa:.2e})")
    jo.check_gemm_fault(cuda)


def test_attention_scatter_emulated_ranks(jo, cuda):
    """The scattering epilogue (jo_attention_fwd_scatter) on one GPU with three
    emulated ranks: every query row lands, bit-identical to attention(), at its
    owner's token row and at heads head0 .. head0 + h of the owner's
    [tokens, all heads, 128] buffer; nothing else in the buffers changes."""
    g = torch.Generator(device=cuda).manual_seed(21)
    Lq, Lk, h, total, head0 = 700, 1500, 2, 6, 2
    segs = [0, 250, 450, 700]
    cap = 260
    q = torch.randn(Lq, h, 128, generator=g, device=cuda).to(torch.bfloat16)
    k = torch.randn(Lk, h, 128, generator=g, device=cuda).to(torch.bfloat16)
    v = torch.randn(Lk, h, 128, generator=g, device=cuda).to(torch.bfloat16)
    ref = jo.attention(q, k, v)
    dst = [torch.full((cap, total, 128), -7.0, dtype=torch.bfloat16, device=cuda) for _ in range(3)]
    for rep in range(2):
        jo.attention_scatter(q, k, v, [d.data_ptr() for d in dst], segs, head0, total, cap)
        torch.cuda.synchronize()
        for r in range(3):
            n = segs[r + 1] - segs[r]
            assert torch.equal(dst[r][:n, head0:head0 + h], ref[segs[r]:segs[r + 1]])
            assert bool((dst[r][:n, :head0] == -7.0).all()) and bool((dst[r][:n, head0 + h:] == -7.0).all())
            assert bool((dst[r][n:] == -7.0).all())
    with pytest.raises(RuntimeError):
        jo.attention_scatter(q, k, v, [d.data_ptr() for d in dst], segs, head0, total, 249)
    jo.check_gemm_fault(cuda)
