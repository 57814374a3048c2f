"""CPU checks of the drop-in boundary: the C-ABI library loads and exports every
symbol include/*.h declares, and the Python shim validates arguments with the
reference's messages (no kernel is launched; there is no GPU here)."""
import ctypes
import glob
import os
import re

import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols():
    names = []
    for h in glob.glob(os.path.join(REPO, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names += re.findall(r"^\s*(?:int|const char\s*\*)\s+(jo_\w+)\s*\(", src, flags=re.M)
    return sorted(set(names))


def test_header_declares_entry_points():
    names = _declared_symbols()
    for n in ("jo_per_token_quant_fp8", "jo_fused_norm_scale_shift", "jo_rmsnorm",
              "jo_fused_qk_norm_rope_3d_paired", "jo_norm_modulate_quant_fp8", "jo_last_error"):
        assert n in names


def test_library_exports_every_declared_symbol():
    from joyomni_ops import _lib
    missing = [n for n in _declared_symbols() if getattr(_lib.lib, n, None) is None]
    assert not missing, f"declared but not exported: {missing}"


def test_binding_table_covers_header():
    from joyomni_ops import _lib
    assert set(_declared_symbols()) <= set(_lib.SIGNATURES)


def test_version_and_error_string():
    from joyomni_ops import _lib
    assert _lib.lib.jo_version() >= 100
    assert isinstance(_lib.last_error(), str)


def test_invalid_arguments_rejected_before_any_launch():
    """Shape/dtype checks fire in the C ABI without touching a device."""
    from joyomni_ops import _lib
    L = _lib.lib
    assert L.jo_per_token_quant_fp8(None, _lib.JO_DTYPE_F32, None, None, 4, 8, None) == _lib.JO_ERR_DTYPE
    assert "bf16 or fp16" in _lib.last_error()
    assert L.jo_per_token_quant_fp8(None, _lib.JO_DTYPE_BF16, None, None, 4, 6, None) == _lib.JO_ERR_INVALID
    assert "divisible by 4" in _lib.last_error()
    assert L.jo_fused_norm_scale_shift(None, None, None, None, None, None, 4, 8, 8, 8, 1, 7, 1e-6,
                                       _lib.JO_DTYPE_BF16, None) == _lib.JO_ERR_INVALID
    assert "norm_type" in _lib.last_error()
    assert L.jo_fused_qk_norm_rope_3d_paired(None, None, 1, 2, 2, 96, 1e-6, None, None, None, None,
                                             None) == _lib.JO_ERR_INVALID
    assert "head_dim" in _lib.last_error()
    # scatter rows beyond the destinations' token count (a peer GPU's buffer) are refused
    dst = (ctypes.c_void_p * 3)(16, 16, 16)
    assert L.jo_fp8_scaled_mm_scatter(16, 16, 16, 16, None, 8, 96, 64, _lib.JO_DTYPE_BF16, dst, 3, 1, 1, 32,
                                      4, 10, None) == _lib.JO_ERR_INVALID
    assert "do not fit" in _lib.last_error()
    # attention output scattered to owning ranks: a segment longer than the
    # destination's token rows, or heads beyond its stride, is refused
    st3 = (ctypes.c_int64 * 3)(0, 256, 128)
    adst = (ctypes.c_void_p * 2)(256, 512)
    seg = (ctypes.c_int64 * 3)(0, 70, 100)
    assert L.jo_attention_fwd_scatter(256, 256, 256, 100, 50, 2, 128, st3, st3, st3, adst, seg, 2, 0, 4 * 128,
                                      64, 0.1, _lib.JO_DTYPE_BF16, None) == _lib.JO_ERR_INVALID
    assert "exceeds the destination" in _lib.last_error()
    assert L.jo_attention_fwd_scatter(256, 256, 256, 100, 50, 2, 128, st3, st3, st3, adst, seg, 2, 3, 4 * 128,
                                      128, 0.1, _lib.JO_DTYPE_BF16, None) == _lib.JO_ERR_INVALID
    assert "too small" in _lib.last_error()
    bad = (ctypes.c_int64 * 3)(0, 70, 99)
    assert L.jo_attention_fwd_scatter(256, 256, 256, 100, 50, 2, 128, st3, st3, st3, adst, bad, 2, 0, 4 * 128,
                                      128, 0.1, _lib.JO_DTYPE_BF16, None) == _lib.JO_ERR_INVALID
    assert "cover" in _lib.last_error()


def test_status_mapping():
    from joyomni_ops import _lib
    with pytest.raises(NotImplementedError):
        _lib.check(_lib.JO_ERR_ARCH)
    with pytest.raises(RuntimeError):
        _lib.check(_lib.JO_ERR_INVALID)
    _lib.check(_lib.JO_OK)


def test_shim_messages_match_reference():
    import joyomni_ops as jo
    x = torch.zeros(4, 8, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="x must be a CUDA tensor"):
        jo.rmsnorm(x, torch.zeros(8, dtype=torch.bfloat16))
    with pytest.raises(RuntimeError, match="input must be a CUDA tensor"):
        jo.sgl_per_token_quant_fp8(x, torch.empty(4, 8), torch.empty(4))
    with pytest.raises(RuntimeError, match="q must be 3D"):
        jo.fused_qk_norm_rope_3d_paired(x, x, 4, 1, 1e-6, x, x, x, x)
    with pytest.raises(RuntimeError, match="mat_a must be a CUDA tensor"):
        jo.fp8_scaled_mm(x, x, x, x, torch.bfloat16) if jo.has_fp8() else (_ for _ in ()).throw(
            RuntimeError("mat_a must be a CUDA tensor"))


def test_torch_ops_registered_with_reference_schema():
    import joyomni_ops  # noqa: F401
    ops = torch.ops.joyomni_ops
    for name in ("fused_qk_norm_rope_3d_paired", "fused_norm_scale_shift", "rmsnorm", "sgl_per_token_quant_fp8",
                 "fp8_scaled_mm"):
        assert hasattr(ops, name)
    s = str(ops.sgl_per_token_quant_fp8.default._schema)
    assert "Tensor(a1!) output_q" in s or "Tensor! output_q" in s or "output_q" in s


def test_norm_type_strings():
    from joyomni_ops import _norm_type_code
    assert _norm_type_code("layer") == 0 and _norm_type_code("rms") == 1 and _norm_type_code("x") == -1
