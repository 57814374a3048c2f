"""Generate the golden fixtures tests/golden/<case>.npz from the REFERENCE's own
CUDA kernels (deploy/joyomni_ops, compiled unmodified into oracle/_ref by
oracle/build_ref.py).  Runs on a B200 box:

    python tests/golden/make_golden.py [outdir]

Each fixture stores the case inputs (``in_*``) and the reference outputs
(``ref_*``).  Only the reference library is loaded in this process (it registers
torch.ops.joyomni_ops, the same namespace as this repository's shim).
"""
import glob
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [os.path.join(REPO, "tests"), os.path.join(REPO, "oracle")]

import golden_cases  # noqa: E402


def main(outdir):
    libs = sorted(glob.glob(os.path.join(REPO, "oracle", "_ref", "joyomni_ref*.so")))
    if not libs:
        raise SystemExit("oracle/_ref/joyomni_ref*.so not built (python oracle/build_ref.py)")
    torch.ops.load_library(libs[0])
    ops = torch.ops.joyomni_ops
    has_fp8 = hasattr(ops, "fp8_scaled_mm")
    os.makedirs(outdir, exist_ok=True)
    for name in golden_cases.CASES:
        d = golden_cases.make_inputs(name)
        if str(d["op"]) in ("gemm", "quant") and not has_fp8:
            print("skip", name, "(reference built without FP8)")
            continue
        out = golden_cases.run_ops(ops, d, "cuda")
        torch.cuda.synchronize()
        arrs = {f"in_{k}": np.asarray(v) for k, v in d.items()}
        arrs.update({f"ref_{k}": v for k, v in out.items()})
        np.savez_compressed(os.path.join(outdir, name + ".npz"), **arrs)
        print("wrote", name)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else HERE)
