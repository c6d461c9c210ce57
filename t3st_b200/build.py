"""Build libdfc_b200.so in-tree from t3st_b200/csrc with nvcc (sm_100a only).

    python -m t3st_b200.build            # build if any source is newer
    python -m t3st_b200.build --force    # rebuild
    python -m t3st_b200.build --verbose  # also print ptxas register/spill report

The library is a plain C-ABI shared object (no PyTorch headers, CUDA runtime
linked statically), loaded with ctypes by t3st_b200/_lib.py.
"""

from __future__ import annotations

import argparse
import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(REPO, "include")
LIB_PATH = os.path.join(PKG, "libdfc_b200.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    # no contraction, IEEE divide and sqrt, denormals kept: the step must round
    # exactly like the reference's separate eager ops
    "-fmad=false", "-prec-div=true", "-prec-sqrt=true", "-ftz=false",
    "-Xcompiler", "-fPIC,-O2,-fvisibility=hidden",
    "-shared", "-cudart", "static",
]


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _stale() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    deps = sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + [os.path.join(INCLUDE, "dfc_b200.h")]
    return any(os.path.getmtime(d) > t for d in deps)


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.sep not in cand or os.path.exists(cand)):
            return cand
    return "nvcc"


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile every .cu under csrc into libdfc_b200.so; return its path."""
    if not force and not _stale():
        return LIB_PATH
    tmp = LIB_PATH + f".tmp{os.getpid()}"
    cmd = [nvcc(), *NVCC_FLAGS, f"-I{INCLUDE}", f"-I{CSRC}", "-o", tmp, *sources()]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError("nvcc failed building libdfc_b200.so")
    if verbose:
        sys.stderr.write(proc.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
