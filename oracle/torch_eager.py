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
