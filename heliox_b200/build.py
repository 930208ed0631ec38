"""Build recipe for the native library ``heliox_b200/libhx_b200.so`` (sm_100a).

Compiled in-tree with nvcc so the shared object travels with the repository
snapshot.  ``--fmad=false`` keeps device arithmetic uncontracted, the GPU
counterpart of the reference CPU build's ``-ffp-contract=off``
(CMakeLists.txt:26-31), so the solver and assembly round exactly like the
reference's CPU integrator.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libhx_b200.so")
SOURCES = ["hx_kernels.cu", "hx_split.cu", "hx_runtime.cu", "hx_runtime_net.cu", "hx_runtime_lib.cu", "hx_netstim.cpp", "hx_plan.cpp", "hx_noalloc.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    p = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(p):
        raise RuntimeError("nvcc not found")
    return p


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)] + [os.path.join(ROOT, "include", "heliox_b200.h"), __file__]
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not _stale():
        return LIB
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    objs = []
    common = [
        "-O3",
        "-std=c++17",
        "-lineinfo",
        "--fmad=false",
        "-Xcompiler",
        "-fPIC,-ffp-contract=off",
        "-I" + os.path.join(ROOT, "include"),
        "-I" + CSRC,
    ] + ARCH
    for src in SOURCES:
        obj = os.path.join(objdir, src + ".o")
        cmd = [nvcc(), "-c", os.path.join(CSRC, src), "-o", obj] + common
        if verbose:
            cmd.append("-Xptxas=-v")
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        if verbose:
            sys.stderr.write(r.stderr)
        objs.append(obj)
    tmp = LIB + ".tmp"
    cmd = [nvcc(), "-shared", "-o", tmp] + objs + ARCH + ["-cudart", "static", "-Xcompiler", "-fPIC"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
