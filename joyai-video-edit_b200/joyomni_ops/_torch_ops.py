"""Registers ``torch.ops.joyomni_ops.*`` with the reference's schema strings
(deploy/joyomni_ops/csrc/pybind.cpp:33-47), CUDA dispatch key only, so code that
calls the registered ops (or CUDA-graph-captures / torch.compile-traces them as
opaque ops) keeps working.  Each implementation is the Python wrapper in
``joyomni_ops/__init__.py``, i.e. the sm_100a kernels behind the C ABI.
"""
from __future__ import annotations

import torch


_lib_def = None


def _register():
    global _lib_def
    import joyomni_ops as jo

    try:
        lib = torch.library.Library("joyomni_ops", "DEF")
    except RuntimeError:
        # Already defined in this process (e.g. the module was reloaded).
        return
    lib.define("fused_qk_norm_rope_3d_paired(Tensor! q, Tensor! k, int seq_len, int num_heads, float eps, "
               "Tensor q_weight, Tensor k_weight, Tensor cos, Tensor sin) -> ()")
    lib.define("fused_norm_scale_shift(Tensor x, Tensor? gamma_opt, Tensor? beta_opt, "
               "Tensor scale, Tensor shift, int norm_type, float eps) -> Tensor")
    lib.define("rmsnorm(Tensor x, Tensor weight, float eps) -> Tensor")
    lib.define("sgl_per_token_quant_fp8(Tensor input, Tensor! output_q, Tensor! output_s) -> ()")
    lib.define("fp8_scaled_mm(Tensor mat_a, Tensor mat_b, Tensor scales_a, Tensor scales_b, "
               "ScalarType out_dtype, Tensor? bias) -> Tensor")
    lib.impl("fused_qk_norm_rope_3d_paired", jo.fused_qk_norm_rope_3d_paired, "CUDA")
    lib.impl("fused_norm_scale_shift",
             lambda x, g, b, sc, sh, nt, eps: jo.fused_norm_scale_shift(x, g, b, sc, sh, int(nt), eps), "CUDA")
    lib.impl("rmsnorm", jo.rmsnorm, "CUDA")
    lib.impl("sgl_per_token_quant_fp8", jo.sgl_per_token_quant_fp8, "CUDA")
    lib.impl("fp8_scaled_mm", jo.fp8_scaled_mm, "CUDA")
    _lib_def = lib


_register()
