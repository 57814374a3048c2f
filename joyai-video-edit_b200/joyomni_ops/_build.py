"""In-tree build of the joyomni_b200 C-ABI library (``libjoyomni_b200.so``).

Every ``csrc/*.cu`` file is compiled by nvcc for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``) into ``_build/`` and linked into a
shared library next to this file.  No fast-math: the quantisation and
normalisation kernels rely on IEEE division and reciprocal to match the
reference bit for bit.  Rebuilds only what changed (mtime of the .cu file or
of any header in csrc/ and include/).
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG_DIR)                      # joyai-video-edit_b200/
REPO = os.path.dirname(ROOT)
CSRC = os.path.join(ROOT, "csrc")
INCLUDE = os.path.join(REPO, "include")
BUILD = os.path.join(ROOT, "_build")
LIB_NAME = "libjoyomni_b200.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
              "--expt-relaxed-constexpr", "-I", INCLUDE, "-I", CSRC]


def nvcc_path() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    p = os.path.join(home, "bin", "nvcc")
    return p if os.path.exists(p) else (shutil.which("nvcc") or "nvcc")


def _headers_mtime() -> float:
    t = 0.0
    for d in (CSRC, INCLUDE):
        for f in os.listdir(d):
            if f.endswith((".h", ".cuh", ".hpp")):
                t = max(t, os.path.getmtime(os.path.join(d, f)))
    return t


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _compile(src: str, obj: str, extra) -> None:
    cmd = [nvcc_path(), *ARCH_FLAGS, *NVCC_FLAGS, *extra, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")


def build(force: bool = False, verbose: bool = False, extra_flags=()) -> str:
    os.makedirs(BUILD, exist_ok=True)
    hdr = _headers_mtime()
    srcs = sources()
    jobs = []
    objs = []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s)[:-3] + ".o")
        objs.append(o)
        if force or not os.path.exists(o) or os.path.getmtime(o) < max(os.path.getmtime(s), hdr):
            jobs.append((s, o))
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            futs = [ex.submit(_compile, s, o, list(extra_flags)) for s, o in jobs]
            for f in futs:
                f.result()
            if verbose:
                print(f"[joyomni_b200] compiled {len(jobs)} file(s)", file=sys.stderr)
    newest = max(os.path.getmtime(o) for o in objs)
    if force or jobs or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < newest:
        tmp = LIB_PATH + ".tmp"
        cmd = [nvcc_path(), *ARCH_FLAGS, "-shared", "-Xcompiler", "-fPIC", *objs, "-o", tmp]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
