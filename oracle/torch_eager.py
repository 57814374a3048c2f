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
