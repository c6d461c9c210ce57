"""Build the two native pieces in-tree (sm_100a only):

- libdfc_b200.so from t3st_b200/csrc/*.cu with nvcc: the kernels behind the
  C ABI of include/dfc_b200.h (no PyTorch headers, CUDA runtime linked
  statically), loaded with ctypes by t3st_b200/_lib.py;
- _dfc_host (a CPython extension) from t3st_b200/csrc/dfc_host_plan.cpp with
  g++ against PyTorch's headers: the steady-state host path of
  DFCAdamW.step(), which calls dfc_mt_step through the C ABI.

    python -m t3st_b200.build            # build what any source is newer than
    python -m t3st_b200.build --force    # rebuild
    python -m t3st_b200.build --verbose  # also print ptxas register/spill report
"""

from __future__ import annotations

import argparse
import glob
import os
import subprocess
import sys
import sysconfig

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(REPO, "include")
LIB_PATH = os.path.join(PKG, "libdfc_b200.so")
HOST_SRC = os.path.join(CSRC, "dfc_host_plan.cpp")
HOST_PATH = os.path.join(PKG, "_dfc_host" + sysconfig.get_config_var("EXT_SUFFIX"))

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


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _lib_deps() -> list[str]:
    return sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + [os.path.join(INCLUDE, "dfc_b200.h")]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.sep not in cand or os.path.exists(cand)):
            return cand
    return "nvcc"


def build_host(force: bool = False) -> str:
    """Compile the DFCAdamW host plan (CPython extension); return its path."""
    if not force and not _stale(HOST_PATH, [HOST_SRC, os.path.join(INCLUDE, "dfc_b200.h")]):
        return HOST_PATH
    import torch
    from torch.utils import cpp_extension

    cuda_home = cpp_extension.CUDA_HOME or "/usr/local/cuda"
    incs = [sysconfig.get_paths()["include"], *cpp_extension.include_paths(),
            os.path.join(cuda_home, "include"), INCLUDE]
    libdir = os.path.join(os.path.dirname(torch.__file__), "lib")
    tmp = HOST_PATH + f".tmp{os.getpid()}"
    cmd = [os.environ.get("CXX", "g++"), "-O2", "-std=c++17", "-shared", "-fPIC",
           "-fvisibility=hidden", f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
           *[f"-I{d}" for d in incs], HOST_SRC, "-o", tmp, f"-L{libdir}", f"-Wl,-rpath,{libdir}",
           "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_python"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError("g++ failed building the DFCAdamW host plan")
    os.replace(tmp, HOST_PATH)
    return HOST_PATH


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile every .cu under csrc into libdfc_b200.so; return its path."""
    if not force and not _stale(LIB_PATH, _lib_deps()):
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
    print(build_host(force=a.force))
