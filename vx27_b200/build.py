"""Builds libvx27cuda.so in-tree (vx27_b200/libvx27cuda.so) for sm_100a.

nvcc compiles every csrc/*.cu for `-gencode arch=compute_100a,code=sm_100a` with line
info; csrc/host_ref.c (the host-side reference-arithmetic entry points) is compiled as
ISO C11 without floating-point contraction so its results match the reference bit for
bit. The CUDA runtime is linked statically, so the library needs only the driver.
Objects are rebuilt when their source or any header changed.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libvx27cuda.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
              "-Xcompiler", "-fPIC,-ffp-contract=off", "-Xptxas", "-warn-spills"]
CC_FLAGS = ["-std=c11", "-O2", "-fPIC", "-ffp-contract=off", "-Wall"]


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libvx27cuda")


def _headers() -> list[str]:
    return (glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) +
            glob.glob(os.path.join(ROOT, "include", "*.h")))


def _stale(out: str, deps: list[str]) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("build failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
    if r.stderr.strip():
        # ptxas spill warnings and the like are worth seeing
        print(r.stderr.strip())


def build(verbose: bool = False, jobs: int | None = None) -> str:
    os.makedirs(OBJ, exist_ok=True)
    nvcc = _nvcc()
    hdrs = _headers()
    cmds, objs = [], []
    for src in sorted(glob.glob(os.path.join(CSRC, "*.cu"))):
        obj = os.path.join(OBJ, os.path.basename(src) + ".o")
        objs.append(obj)
        if _stale(obj, [src] + hdrs):
            cmds.append([nvcc, *ARCH, *NVCC_FLAGS, "-c", src, "-o", obj])
    for src in sorted(glob.glob(os.path.join(CSRC, "*.c"))):
        obj = os.path.join(OBJ, os.path.basename(src) + ".o")
        objs.append(obj)
        if _stale(obj, [src] + hdrs):
            cmds.append(["gcc", *CC_FLAGS, "-c", src, "-o", obj])
    if cmds:
        with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
            for c in cmds:
                if verbose:
                    print(" ".join(c))
            list(ex.map(_run, cmds))
    if cmds or _stale(LIB, objs):
        _run([nvcc, *ARCH, "-shared", "-o", LIB, *objs, "-lm"])
    return LIB


if __name__ == "__main__":
    print(build(verbose=True))
