"""Golden-fixture cases for the joyomni_ops hot path.

``make_inputs()`` builds small seeded inputs for every op; ``run_ops(ops, ...)``
runs them through any object exposing the reference's five op signatures
(the reference library loaded from oracle/_ref, or this repository's
joyomni_ops).  ``tests/golden/make_golden.py`` stores the reference's outputs as
``tests/golden/<case>.npz``; ``check_oracle`` and ``check_kernel`` compare the
CPU oracle and our kernels with them.

Bit-exactness expectations:
  * per-token quant codes and scales: exact (oracle and kernel);
  * qk-norm-rope: kernel exact by construction (same reduction tree), oracle <= 2 ulp;
  * norm / rmsnorm / GEMM: <= 2 bf16 ulp, relative RMS <= 2e-3 (GEMM: 1e-3... see tol).
"""
from __future__ import annotations

import numpy as np

import joyomni_oracle as O

# name -> (op, params)
CASES = {
    "quant_bf16_cfg2": ("quant", dict(M=24, K=5120, dtype="bf16", outliers=True, seed=21)),
    "quant_bf16_warp": ("quant", dict(M=2400, K=64, dtype="bf16", outliers=False, seed=22)),
    "quant_f16_k1000": ("quant", dict(M=19, K=1000, dtype="f16", outliers=True, seed=23)),
    "quant_bf16_k12": ("quant", dict(M=9, K=12, dtype="bf16", outliers=False, seed=24)),
    "quant_bf16_special": ("quant_special", dict(seed=25)),
    "norm_rms_bf16_5120": ("norm", dict(M=16, N=5120, nt=1, affine=True, dtype="bf16", seed=31)),
    "norm_layer_bf16_5120": ("norm", dict(M=16, N=5120, nt=0, affine=False, dtype="bf16", seed=32)),
    "norm_layer_bf16_1024_affine": ("norm", dict(M=24, N=1024, nt=0, affine=True, dtype="bf16", seed=33)),
    "norm_rms_f32_512": ("norm", dict(M=8, N=512, nt=1, affine=False, dtype="f32", seed=34)),
    "norm_layer_f16_768": ("norm", dict(M=8, N=768, nt=0, affine=True, dtype="f16", seed=35)),
    "rmsnorm_bf16_128": ("rmsnorm", dict(M=1000, N=128, dtype="bf16", seed=41)),
    "rmsnorm_bf16_5120": ("rmsnorm", dict(M=8, N=5120, dtype="bf16", seed=42)),
    "rmsnorm_f32_96": ("rmsnorm", dict(M=20, N=96, dtype="f32", seed=43)),
    "qkrope_d128_grid": ("qkrope", dict(B=1, grid=(2, 4, 8), H=8, D=128, seed=51)),
    "qkrope_d64_rand": ("qkrope", dict(B=2, grid=(1, 3, 5), H=3, D=64, seed=52)),
    "qkrope_d256_rand": ("qkrope", dict(B=1, grid=(1, 2, 9), H=2, D=256, seed=53)),
    "gemm_bias_300x256x512": ("gemm", dict(M=300, N=256, K=512, bias=True, seed=61)),
    "gemm_nobias_130x384x256": ("gemm", dict(M=130, N=384, K=256, bias=False, seed=62)),
    "gemm_bias_16x128x1024": ("gemm", dict(M=16, N=128, K=1024, bias=True, seed=63)),
    "gemm_bias_1x64x128": ("gemm", dict(M=1, N=64, K=128, bias=True, seed=64)),
}


def _outliers(rng, M, N, dtype):
    x = rng.standard_normal((M, N)).astype(np.float32)
    x[rng.random((M, N)) < 0.01] *= np.float32(50.0)
    return O.round_to(x, dtype)


def make_inputs(name):
    op, p = CASES[name]
    rng = np.random.default_rng(p.get("seed", 0))
    d = {"op": np.array(op)}
    if op == "quant":
        d["x"] = _outliers(rng, p["M"], p["K"], p["dtype"]) if p["outliers"] else \
            O.round_to(rng.standard_normal((p["M"], p["K"])).astype(np.float32) * 2, p["dtype"])
        d["dtype"] = np.array(p["dtype"])
    elif op == "quant_special":
        x = O.round_bf16(rng.standard_normal((8, 64)).astype(np.float32))
        x[0] = 0.0
        x[1, 5] = np.nan
        x[2, :] = np.float32(1e-39)
        x[3, 7] = np.inf
        x[4, :] = -0.0
        x[5, :] = np.float32(3e38)
        x[6, ::2] = np.float32(448.0)
        d["x"] = O.round_bf16(x)
        d["dtype"] = np.array("bf16")
        d["op"] = np.array("quant")
    elif op == "norm":
        M, N, dt = p["M"], p["N"], p["dtype"]
        d["x"] = _outliers(rng, M, N, dt)
        d["scale"] = O.round_to(rng.standard_normal((M, N)).astype(np.float32) * 0.1, dt)
        d["shift"] = O.round_to(rng.standard_normal((M, N)).astype(np.float32) * 0.1, dt)
        if p["affine"]:
            d["gamma"] = O.round_to(1 + 0.1 * rng.standard_normal(N).astype(np.float32), dt)
            d["beta"] = O.round_to(0.1 * rng.standard_normal(N).astype(np.float32), dt)
        d["nt"] = np.array(p["nt"])
        d["eps"] = np.array(1e-6, np.float32)
        d["dtype"] = np.array(dt)
    elif op == "rmsnorm":
        M, N, dt = p["M"], p["N"], p["dtype"]
        d["x"] = O.round_to(rng.standard_normal((M, N)).astype(np.float32), dt)
        d["w"] = O.round_to(1 + 0.1 * rng.standard_normal(N).astype(np.float32), dt)
        d["eps"] = np.array(1e-6, np.float32)
        d["dtype"] = np.array(dt)
    elif op == "qkrope":
        B, (T, Hh, W), H, D = p["B"], p["grid"], p["H"], p["D"]
        L = T * Hh * W
        d["q"] = O.round_bf16(rng.standard_normal((B, L * H, D)).astype(np.float32))
        d["k"] = O.round_bf16(rng.standard_normal((B, L * H, D)).astype(np.float32))
        d["qw"] = O.round_bf16(1 + 0.1 * rng.standard_normal(D).astype(np.float32))
        d["kw"] = O.round_bf16(1 + 0.1 * rng.standard_normal(D).astype(np.float32))
        if D == 128:
            c, s = O.rope_tables_3d((T, Hh, W))
        else:
            c = O.round_bf16(rng.standard_normal((L, D // 2)).astype(np.float32))
            s = O.round_bf16(rng.standard_normal((L, D // 2)).astype(np.float32))
        d["cos"], d["sin"] = c, s
        d["L"], d["H"] = np.array(L), np.array(H)
        d["eps"] = np.array(1e-6, np.float32)
    elif op == "gemm":
        M, N, K = p["M"], p["N"], p["K"]
        a, sa = O.per_token_quant_fp8(O.round_bf16(rng.standard_normal((M, K)).astype(np.float32)))
        w = O.round_bf16(rng.standard_normal((N, K)).astype(np.float32) * 0.02)
        b, sb = O.quantize_weight_per_channel(w)
        d["a"], d["sa"], d["b_nk"], d["sb"] = a, sa, b, sb
        if p["bias"]:
            d["bias"] = O.round_bf16(rng.standard_normal(N).astype(np.float32) * 0.01)
    return d


# ------------------------------------------------------------------ running --
def _t(a, dtype, dev):
    import torch
    tdt = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[str(dtype)]
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(tdt).to(dev)


def run_ops(ops, d, dev="cuda"):
    """Run case ``d`` through ``ops`` (reference signatures); return numpy outputs."""
    import torch
    op = str(d["op"])
    out = {}
    if op == "quant":
        x = _t(d["x"], d["dtype"], dev)
        q = torch.empty(x.shape, dtype=torch.float8_e4m3fn, device=dev)
        s = torch.empty((x.shape[0], 1), dtype=torch.float32, device=dev)
        ops.sgl_per_token_quant_fp8(x, q, s)
        out["codes"] = q.view(torch.uint8).cpu().numpy()
        out["scales"] = s.view(-1).cpu().numpy()
    elif op == "norm":
        dt = d["dtype"]
        g = _t(d["gamma"], dt, dev) if "gamma" in d else None
        b = _t(d["beta"], dt, dev) if "beta" in d else None
        y = ops.fused_norm_scale_shift(_t(d["x"], dt, dev), g, b, _t(d["scale"], dt, dev),
                                       _t(d["shift"], dt, dev), int(d["nt"]), float(d["eps"]))
        out["y"] = y.float().cpu().numpy()
    elif op == "rmsnorm":
        dt = d["dtype"]
        y = ops.rmsnorm(_t(d["x"], dt, dev), _t(d["w"], dt, dev), float(d["eps"]))
        out["y"] = y.float().cpu().numpy()
    elif op == "qkrope":
        q, k = _t(d["q"], "bf16", dev), _t(d["k"], "bf16", dev)
        ops.fused_qk_norm_rope_3d_paired(q, k, int(d["L"]), int(d["H"]), float(d["eps"]), _t(d["qw"], "bf16", dev),
                                         _t(d["kw"], "bf16", dev), _t(d["cos"], "bf16", dev),
                                         _t(d["sin"], "bf16", dev))
        out["q_out"] = q.float().cpu().numpy()
        out["k_out"] = k.float().cpu().numpy()
    elif op == "gemm":
        a = torch.from_numpy(d["a"]).to(dev).view(torch.float8_e4m3fn)
        b = torch.from_numpy(d["b_nk"]).to(dev).view(torch.float8_e4m3fn).t()   # [K, N] column-major
        bias = _t(d["bias"], "bf16", dev) if "bias" in d else None
        y = ops.fp8_scaled_mm(a, b, torch.from_numpy(d["sa"]).to(dev), torch.from_numpy(d["sb"]).to(dev),
                              torch.bfloat16, bias)
        out["y"] = y.float().cpu().numpy()
    return out


def oracle_outputs(d):
    op = str(d["op"])
    if op == "quant":
        q, s = O.per_token_quant_fp8(d["x"])
        return {"codes": q, "scales": s}
    if op == "norm":
        return {"y": O.fused_norm_scale_shift(d["x"], d.get("gamma"), d.get("beta"), d["scale"], d["shift"],
                                              int(d["nt"]), float(d["eps"]), str(d["dtype"]))}
    if op == "rmsnorm":
        return {"y": O.rmsnorm(d["x"], d["w"], float(d["eps"]), str(d["dtype"]))}
    if op == "qkrope":
        L, H = int(d["L"]), int(d["H"])
        return {"q_out": O.qk_norm_rope(d["q"], d["qw"], d["cos"], d["sin"], L, H, float(d["eps"])),
                "k_out": O.qk_norm_rope(d["k"], d["kw"], d["cos"], d["sin"], L, H, float(d["eps"]))}
    if op == "gemm":
        return {"y": O.fp8_scaled_mm(d["a"], d["b_nk"], d["sa"], d["sb"], d.get("bias"))}
    raise ValueError(op)


def load(path):
    z = np.load(path, allow_pickle=False)
    d = {k: z[k] for k in z.files}
    inputs = {k[3:]: v for k, v in d.items() if k.startswith("in_")}
    ref = {k[4:]: v for k, v in d.items() if k.startswith("ref_")}
    return inputs, ref


def _dtype_of(inputs):
    return str(inputs["dtype"]) if "dtype" in inputs else "bf16"


def compare(got, ref, inputs, exact_quant=True, max_ulp=2):
    from _util import assert_close_ulp
    op = str(inputs["op"])
    if op == "quant":
        assert np.array_equal(got["scales"].view(np.uint32), ref["scales"].view(np.uint32)), "scales differ"
        assert np.array_equal(got["codes"], ref["codes"]), \
            f"{int((got['codes'] != ref['codes']).sum())} codes differ"
        return
    dt = _dtype_of(inputs)
    for k in ref:
        if dt == "f32":
            assert_close_ulp(got[k], ref[k], dtype="f32", max_ulp=64, rel_rms=1e-5, atol=1e-6)
        else:
            assert_close_ulp(got[k], ref[k], dtype=dt, max_ulp=max_ulp)


def check_oracle(path):
    inputs, ref = load(path)
    compare(oracle_outputs(inputs), ref, inputs)


def exact_fraction(got, ref):
    fr = {}
    for k in ref:
        a, b = np.asarray(got[k]), np.asarray(ref[k])
        fr[k] = float(np.mean((a == b) | (np.isnan(a) & np.isnan(b))))
    return fr
