"""Eager-torch restatement of one MMDiT double-stream block forward
(deploy/xvideo/models/dit/dit.py:314-481 with FP8 linears, fp8_linear.py:138-169),
used only as the checker for joyomni_stack.  fp32 math, reference grouping,
the same FP8 weights as the block under test."""
import torch
import torch.nn.functional as F

EPS = 1e-6


def quant(y):
    """per_token_quant_fp8.cu:55-78 in torch: y bf16 [M, K] -> (codes as float, scale [M, 1])."""
    yf = y.float()
    amax = yf.abs().amax(-1, keepdim=True)
    s = (amax.double() / 448.0).float()   # IEEE amax/448 (torch's GPU scalar division multiplies by 1/448)
    # correctly rounded 1/s (the kernel's IEEE reciprocal); float64 then round
    inv = torch.where(s == 0, torch.zeros_like(s), (1.0 / s.double()).float())
    q = (yf * inv).clamp(-448, 448).to(torch.float8_e4m3fn).float()
    return q, s


def ln_mod(x, shift, scale):
    xf = x.float()
    mu = xf.mean(-1, keepdim=True)
    var = ((xf - mu) ** 2).mean(-1, keepdim=True)
    return (((xf - mu) * torch.rsqrt(var + EPS)) * (1 + scale.float()) + shift.float()).to(torch.bfloat16)


def lin(q, s, W, gelu=False):
    acc = q @ W.codes.float().t()
    y = ((acc * W.scale[None, :]) * s + W.b.float()).to(torch.bfloat16)
    if gelu:
        y = F.gelu(y.float(), approximate="tanh").to(torch.bfloat16)
    return y


def qk_norm(x, w, cos=None, sin=None):
    """x [L, H, D] -> per-head RMSNorm * w, then interleaved-pair RoPE (rope.py:14-28)."""
    xf = x.float()
    e = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + EPS) * w.float()
    if cos is not None:
        c, s = cos.float()[:, None, :], sin.float()[:, None, :]
        o = torch.empty_like(e)
        o[..., 0::2] = e[..., 0::2] * c - e[..., 1::2] * s
        o[..., 1::2] = e[..., 0::2] * s + e[..., 1::2] * c
        e = o
    return e.to(torch.bfloat16)


def attention_fp32(q, k, v):
    """softmax(q k^T / sqrt(d)) v in fp32, one head at a time; q [Lq, H, D], k/v [Lk, H, D]."""
    out = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    sc = 1.0 / (q.shape[-1] ** 0.5)
    for h in range(q.shape[1]):
        p = torch.softmax((q[:, h].float() @ k[:, h].float().t()) * sc, dim=-1)
        out[:, h] = p @ v[:, h].float()
        del p
    return out


def block_forward(blk, img, txt, vec, cos, sin, cache_k=None, cache_v=None, attn="sdpa"):
    H, Dh, D = blk.cfg.heads, blk.cfg.head_dim, blk.cfg.hidden
    Li = img.shape[0]
    im = (blk.img.mod + vec).unbind(0)
    tm = (blk.txt.mod + vec).unbind(0)
    iqkv = lin(*quant(ln_mod(img, im[0], im[1])), blk.img.qkv).view(Li, 3, H, Dh)
    tqkv = lin(*quant(ln_mod(txt, tm[0], tm[1])), blk.txt.qkv).view(txt.shape[0], 3, H, Dh)
    q = torch.cat((qk_norm(iqkv[:, 0], blk.img.q_norm, cos, sin), qk_norm(tqkv[:, 0], blk.txt.q_norm)), 0)
    k = torch.cat((qk_norm(iqkv[:, 1], blk.img.k_norm, cos, sin), qk_norm(tqkv[:, 1], blk.txt.k_norm)), 0)
    v = torch.cat((iqkv[:, 2], tqkv[:, 2]), 0)
    if cache_k is not None:
        k = torch.cat((k, cache_k), 0)
        v = torch.cat((v, cache_v), 0)
    if attn == "fp32":
        o = attention_fp32(q, k, v)
    else:
        # bf16 attention, as the reference model runs it (FA4 / SDPA in bf16, dit.py:162-178)
        o = F.scaled_dot_product_attention(q.permute(1, 0, 2)[None], k.permute(1, 0, 2)[None],
                                           v.permute(1, 0, 2)[None])[0].permute(1, 0, 2)
    o = o.reshape(-1, D).to(torch.bfloat16)

    def tail(st, m, x, attn):
        x = torch.addcmul(x, lin(*quant(attn), st.proj), m[2])
        h = lin(*quant(ln_mod(x, m[3], m[4])), st.up, gelu=True)
        return torch.addcmul(x, lin(*quant(h), st.down), m[5])

    return tail(blk.img, im, img, o[:Li]), tail(blk.txt, tm, txt, o[Li:]), k, v
