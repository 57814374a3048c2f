"""Shared helpers for the parity tests: seeded inputs, dtype conversion between
numpy (oracle) and torch (kernels), and the stated tolerances."""
from __future__ import annotations

import numpy as np
import torch

import joyomni_oracle as O

TDT = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


def randn(rng, shape, scale=1.0, dtype="bf16"):
    return O.round_to(rng.standard_normal(shape).astype(np.float32) * np.float32(scale), dtype)


def to_torch(a, dtype="bf16", device="cpu"):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(TDT[dtype]).to(device)


def to_np(t):
    return t.detach().float().cpu().numpy()


def codes_np(t):
    return t.detach().view(torch.uint8).cpu().numpy()


def ulp(v, dtype="bf16"):
    """Spacing of the 16-bit format at |v| (mantissa bits: bf16 7, fp16 10)."""
    mb = {"bf16": 7, "f16": 10, "f32": 23}[dtype]
    a = np.abs(np.asarray(v, dtype=np.float64))
    e = np.floor(np.log2(np.maximum(a, 2.0 ** -126)))
    return np.ldexp(1.0, (e - mb).astype(np.int64))


def assert_close_ulp(got, ref, dtype="bf16", max_ulp=2, rel_rms=2e-3, atol=1e-6):
    """Max-abs within ``max_ulp`` units in the last place of the larger of the two
    values, and relative RMS error below ``rel_rms`` (the stated tolerance for the
    norm / RoPE / GEMM outputs)."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    if got.size == 0:
        return
    fin = np.isfinite(ref)
    assert np.array_equal(np.isfinite(got), fin), "non-finite pattern differs"
    d = np.abs(got[fin] - ref[fin])
    tol = max_ulp * ulp(np.maximum(np.abs(got[fin]), np.abs(ref[fin])), dtype) + atol
    bad = d > tol
    assert not bad.any(), (
        f"{bad.sum()} of {d.size} elements beyond {max_ulp} ulp; worst diff {d.max():.3e} "
        f"at ref {ref[fin][np.argmax(d)]:.4e}")
    rr = np.sqrt(np.mean((got[fin] - ref[fin]) ** 2)) / max(np.sqrt(np.mean(ref[fin] ** 2)), 1e-30)
    assert rr <= rel_rms, f"relative RMS {rr:.3e} > {rel_rms}"


def rel_rms(got, ref):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.sqrt(np.mean((got - ref) ** 2)) / max(np.sqrt(np.mean(ref ** 2)), 1e-30))


def outlier_activations(rng, M, N, frac=0.01, mult=50.0, dtype="bf16"):
    """N(0,1) with a Bernoulli(frac) mask scaled by ``mult`` (BASELINE config 2 inputs)."""
    x = rng.standard_normal((M, N)).astype(np.float32)
    mask = rng.random((M, N)) < frac
    x[mask] *= np.float32(mult)
    return O.round_to(x, dtype)
