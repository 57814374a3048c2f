"""Build recipe for ``oracle/_ref``: the reference's own joyomni_ops kernels.

This is test infrastructure only.  It compiles the reference CUDA sources
in place (never copying them) into ``oracle/_ref/joyomni_ref.so`` with nvcc for
sm_100a, using our own build line instead of the reference's ``setup.py``.  The
resulting library registers ``torch.ops.joyomni_ops.*`` exactly as the reference
extension does (``deploy/joyomni_ops/csrc/pybind.cpp:33-58``), so it must be
loaded in a process that does NOT also import this repository's ``joyomni_ops``
shim.  It is used to generate golden fixtures on a GPU box
(``tests/golden/make_golden.py``) and to time the reference's CUTLASS FP8 GEMM.

The FP8 GEMM (``fp8_gemm.cu``) needs CUTLASS headers.  The reference pins CUTLASS
commit dcf215af (``deploy/joyomni_ops/README.md:43``), which is not available
here; the CUTLASS 4.5.0 header tree that ships inside the installed flashinfer
wheel is used instead (unpinned).  Set ``JO_REF_NO_FP8=1`` to build without it.
"""
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")


def reference_root():
    """Root of the reference checkout: $JO_REFERENCE_ROOT, else the
    `reference_path` that BASELINE.json at the repository root records; None
    when neither names an existing directory (the reference is then absent,
    as on a GPU box, and nothing is built)."""
    root = os.environ.get("JO_REFERENCE_ROOT")
    if not root:
        try:
            import json
            root = json.load(open(os.path.join(os.path.dirname(HERE), "BASELINE.json"))).get("reference_path")
        except (OSError, ValueError):
            root = None
    return root if root and os.path.isdir(root) else None


def ops_dir():
    root = reference_root()
    d = os.path.join(root, "deploy", "joyomni_ops") if root else None
    return d if d and os.path.isdir(d) else None


def _cutlass_dir():
    import importlib.util
    spec = importlib.util.find_spec("flashinfer")
    if spec is None or not spec.submodule_search_locations:
        return None
    d = os.path.join(list(spec.submodule_search_locations)[0], "data", "cutlass")
    return d if os.path.isdir(os.path.join(d, "include")) else None


def build(no_fp8=None, verbose=False):
    REF = ops_dir()
    if REF is None:
        raise FileNotFoundError("reference sources not found (set JO_REFERENCE_ROOT)")
    from torch.utils.cpp_extension import load
    if no_fp8 is None:
        no_fp8 = os.environ.get("JO_REF_NO_FP8", "") == "1"
    os.makedirs(OUT, exist_ok=True)
    srcs = ["csrc/pybind.cpp", "csrc/fused_qknorm_rope_3d_kernel.cu",
            "csrc/fused_norm_scale_shift.cu", "csrc/rmsnorm.cu"]
    inc = [os.path.join(REF, "include")]
    flags = ["-O3", "-std=c++17", "--expt-relaxed-constexpr", "--expt-extended-lambda",
             "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
             "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
             "-gencode=arch=compute_100a,code=sm_100a"]
    cflags = ["-O3", "-std=c++17"]
    if no_fp8:
        flags.append("-DJOYOMNI_OPS_NO_FP8")
        cflags.append("-DJOYOMNI_OPS_NO_FP8")
        name = "joyomni_ref_light"
    else:
        cd = _cutlass_dir()
        if cd is None:
            raise RuntimeError("no CUTLASS header tree found for the reference FP8 GEMM")
        inc += [os.path.join(cd, "include"), os.path.join(cd, "tools", "util", "include")]
        srcs += ["csrc/per_token_quant_fp8.cu", "csrc/fp8_gemm.cu"]
        name = "joyomni_ref"
    os.environ.setdefault("MAX_JOBS", str(os.cpu_count() or 4))
    # torch's extension builder waits forever on a lock file left by a build
    # that was killed; a lock older than an hour cannot belong to a live build.
    lock = os.path.join(OUT, "lock")
    if os.path.exists(lock) and time.time() - os.path.getmtime(lock) > 3600:
        os.remove(lock)
    load(name=name, sources=[os.path.join(REF, s) for s in srcs],
         extra_include_paths=inc, extra_cflags=cflags, extra_cuda_cflags=flags,
         build_directory=OUT, is_python_module=False, verbose=verbose)
    return os.path.join(OUT, name + ".so")


if __name__ == "__main__":
    print(build(no_fp8=("--no-fp8" in sys.argv), verbose=True))
