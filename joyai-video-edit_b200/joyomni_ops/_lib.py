"""ctypes binding of ``libjoyomni_b200.so`` (the C ABI in include/joyomni_b200.h).

Loading fails loudly (ImportError) when the library has not been built: there is
no CPU or eager-PyTorch fallback for any operator.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("JOYOMNI_B200_LIB", os.path.join(_HERE, "libjoyomni_b200.so"))

if not os.path.exists(LIB_PATH):
    raise ImportError(
        f"joyomni_b200 CUDA library not found at {LIB_PATH}; build it first "
        "(python -c 'import __graft_entry__ as g; g.build()' or python joyomni_ops/_build.py)")

lib = ctypes.CDLL(LIB_PATH)

JO_OK = 0
JO_ERR_INVALID = -1
JO_ERR_DTYPE = -2
JO_ERR_ALIGN = -3
JO_ERR_ARCH = -4
JO_ERR_CUDA = -5

JO_DTYPE_F32 = 0
JO_DTYPE_F16 = 1
JO_DTYPE_BF16 = 2
JO_DTYPE_E4M3 = 3

JO_NORM_LAYER = 0
JO_NORM_RMS = 1

JO_EPI_NONE = 0
JO_EPI_GELU_TANH = 1
JO_EPI_RESID_GATE = 2

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_f32 = ctypes.c_float

# name -> argtypes, in declaration order of include/joyomni_b200.h
SIGNATURES = {
    "jo_version": [],
    "jo_last_error": [],
    "jo_device_arch": [_i32],
    "jo_fused_qk_norm_rope_3d_paired": [_p, _p, _i64, _i64, _i64, _i64, _f32, _p, _p, _p, _p, _p],
    "jo_qk_norm_rope_strided": [_p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _p, _p, _p, _p, _p],
    "jo_fused_norm_scale_shift": [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i32, _f32, _i32, _p],
    "jo_rmsnorm": [_p, _p, _p, _i64, _i64, _i64, _f32, _i32, _p],
    "jo_per_token_quant_fp8": [_p, _i32, _p, _p, _i64, _i64, _p],
    "jo_norm_modulate_quant_fp8": [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i32, _f32, _i32, _p, _p, _p],
    "jo_fp8_scaled_mm": [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i32, _i32, _p],
    "jo_fp8_scaled_mm_ex": [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i32, _i32, _p, _p, _p],
    "jo_rope_apply": [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _p],
    "jo_attention_fwd": [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, ctypes.POINTER(_i64), ctypes.POINTER(_i64),
                         ctypes.POINTER(_i64), ctypes.POINTER(_i64), _f32, _i32, _p],
    "jo_attention_fwd_scatter": [_p, _p, _p, _i64, _i64, _i64, _i64, ctypes.POINTER(_i64), ctypes.POINTER(_i64),
                                 ctypes.POINTER(_i64), _p, ctypes.POINTER(_i64), _i32, _i64, _i64, _i64, _f32, _i32,
                                 _p],
    "jo_attention_last_fault": [_i32],
    "jo_gemm_last_fault": [_i32],
    "jo_fp8_scaled_mm_scatter": [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i32, _p, _i32, _i32, _i32, _i32, _i64, _i64,
                                 _p],
    "jo_ipc_get_handle": [_p, _p, ctypes.POINTER(_i64)],
    "jo_ipc_open": [_p, ctypes.POINTER(_p)],
    "jo_ipc_close": [_p],
}

for _name, _args in SIGNATURES.items():
    _fn = getattr(lib, _name, None)
    if _fn is None:
        continue
    _fn.argtypes = _args
    _fn.restype = ctypes.c_char_p if _name == "jo_last_error" else ctypes.c_int


def has(name: str) -> bool:
    return getattr(lib, name, None) is not None


def last_error() -> str:
    return lib.jo_last_error().decode(errors="replace")


def check(status: int) -> None:
    """Raise the exception the reference op would raise for a failed call."""
    if status == JO_OK:
        return
    msg = last_error()
    if status == JO_ERR_ARCH:
        raise NotImplementedError(msg)
    raise RuntimeError(msg)
