"""Eager-torch CPU path of the joyomni_ops hot path — TEST/MEASUREMENT INFRASTRUCTURE.

The reference has no CPU implementation of its CUDA kernels; its model code
runs the same math as eager torch (deploy/xvideo/models/dit/sgl_fused_ops.py,
fp8_linear.py).  This module restates the config-2 chain in eager torch, fp32
math, on the host's cores, as the CPU baseline bench.py reports
(`cpu_baseline`, `--impl reference`):

  y = bf16(RMSNorm(x) * w * (1 + scale) + shift)            (fused_norm_scale_shift.cu:99-139, RMS)
  s = amax(|y|) / 448 ; q = e4m3(clamp(y * (1/s), +-448))    (per_token_quant_fp8.cu:55-78)
"""
import torch


def cfg2_chain(x, w, shift, scale, eps=1e-6):
    """x bf16 [M, N]; w, shift, scale bf16 [N] -> (codes e4m3 [M, N], scales fp32 [M, 1])."""
    xf = x.float()
    r = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    y = (((xf * r) * w.float()) * (1 + scale.float()) + shift.float()).to(torch.bfloat16)
    yf = y.float()
    s = yf.abs().amax(-1, keepdim=True) / 448.0
    inv = torch.where(s == 0, torch.zeros_like(s), 1.0 / s)
    q = (yf * inv).clamp(-448, 448).to(torch.float8_e4m3fn)
    return q, s


def cfg1_qk_norm_rope(q, k, qw, kw, cos, sin, num_heads, eps=1e-6):
    """Config 1 in eager torch, fp32 math (the interleaved-pair formula of
    fused_qknorm_rope_3d_kernel.cu:98-141 and test_parity_light.py:77-87):
    q, k bf16 [L*H, D]; qw, kw bf16 [D]; cos, sin bf16 [L, D/2] -> new q, k bf16."""
    def one(x, w):
        xf = x.float()
        xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()
        L = cos.shape[0]
        xf = xf.view(L, num_heads, -1, 2)
        c = cos.float().view(L, 1, -1)
        s = sin.float().view(L, 1, -1)
        x1, x2 = xf[..., 0], xf[..., 1]
        return torch.stack((x1 * c - x2 * s, x1 * s + x2 * c), -1).reshape(x.shape).to(torch.bfloat16)
    return one(q, qw), one(k, kw)


def cfg3_fp8_scaled_mm(a, b_nk, sa, sb, bias):
    """Config 3 in eager torch: e4m3 A [M, K] and W [N, K] dequantised to fp32,
    fp32 matmul, then bf16(sa * (sb * acc) + bias) (fp8_gemm.cu:833-860 of the
    reference for the epilogue)."""
    acc = a.float() @ b_nk.float().t()
    return (sa.view(-1, 1) * (sb.view(1, -1) * acc) + bias.float()).to(torch.bfloat16)


def _quant(y):
    """Per-token e4m3 quantisation of a bf16 [M, K] activation (per_token_quant_fp8.cu:55-78)."""
    yf = y.float()
    s = yf.abs().amax(-1, keepdim=True) / 448.0
    inv = torch.where(s == 0, torch.zeros_like(s), 1.0 / s)
    return (yf * inv).clamp(-448, 448).to(torch.float8_e4m3fn), s


def _lin(y, lw, gelu=False):
    """Fp8Linear.forward (fp8_linear.py:138-169): quantise, dequantised fp32 matmul, epilogue."""
    q, s = _quant(y)
    out = cfg3_fp8_scaled_mm(q, lw["codes"], s, lw["scale"], lw["bias"])
    if gelu:
        out = torch.nn.functional.gelu(out.float(), approximate="tanh").to(torch.bfloat16)
    return out


def _ln_mod(x, shift, scale, eps=1e-6):
    xf = x.float()
    mu = xf.mean(-1, keepdim=True)
    var = (xf - mu).pow(2).mean(-1, keepdim=True)
    return (((xf - mu) * torch.rsqrt(var + eps)) * (1 + scale.float()) + shift.float()).to(torch.bfloat16)


def _qk_norm(x, w, cos=None, sin=None, eps=1e-6):
    xf = x.float()
    e = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()
    if cos is not None:
        c, s = cos.float()[:, None, :], sin.float()[:, None, :]
        e1, e2 = e[..., 0::2], e[..., 1::2]
        e = torch.stack((e1 * c - e2 * s, e1 * s + e2 * c), -1).flatten(-2)
    return e.to(torch.bfloat16)


def cfg4_block(img, txt, mods, layers, cache_k, cache_v, cos, sin, heads):
    """Config 4 (one MMDiT double-stream block, dit.py:314-481) in eager torch on
    the host: adaLN LayerNorm-modulate, FP8 linears dequantised to fp32, QK
    RMSNorm with RoPE on the image stream, fp32 attention of [img | txt] queries
    over [img | txt | cache] keys one head at a time, gated residuals and the
    GELU-tanh MLP.  img [Li, D], txt [Lt, D] bf16; mods[stream] = six [D]
    modulation vectors; layers[stream] = dict of qkv / proj / up / down
    (codes e4m3 [N, K], scale fp32 [N], bias bf16 [N]) and q_norm / k_norm [Dh];
    cache_k / cache_v [Lc, H, Dh] bf16.  Returns the two stream outputs."""
    D = img.shape[1]
    Dh = D // heads
    qs, ks, vs = [], [], []
    for x, st in ((img, "img"), (txt, "txt")):
        m, lw = mods[st], layers[st]
        qkv = _lin(_ln_mod(x, m[0], m[1]), lw["qkv"]).view(x.shape[0], 3, heads, Dh)
        rc = (cos, sin) if st == "img" else (None, None)
        qs.append(_qk_norm(qkv[:, 0], lw["q_norm"], *rc))
        ks.append(_qk_norm(qkv[:, 1], lw["k_norm"], *rc))
        vs.append(qkv[:, 2])
    q = torch.cat(qs, 0)
    k = torch.cat(ks + [cache_k], 0)
    v = torch.cat(vs + [cache_v], 0)
    o = torch.empty(q.shape, dtype=torch.float32)
    sc = 1.0 / (Dh ** 0.5)
    for h in range(heads):
        p = torch.softmax((q[:, h].float() @ k[:, h].float().t()) * sc, dim=-1)
        o[:, h] = p @ v[:, h].float()
        del p
    o = o.reshape(-1, D).to(torch.bfloat16)
    outs = []
    for x, st, oo in ((img, "img", o[:img.shape[0]]), (txt, "txt", o[img.shape[0]:])):
        m, lw = mods[st], layers[st]
        x = torch.addcmul(x.float(), _lin(oo, lw["proj"]).float(), m[2].float()).to(torch.bfloat16)
        hdn = _lin(_ln_mod(x, m[3], m[4]), lw["up"], gelu=True)
        outs.append(torch.addcmul(x.float(), _lin(hdn, lw["down"]).float(), m[5].float()).to(torch.bfloat16))
    return outs[0], outs[1]
