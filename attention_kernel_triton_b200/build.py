"""Build the sm_100a shared library ``libakt.so`` in-tree with nvcc.

``python -m attention_kernel_triton_b200.build`` compiles every ``csrc/*.cu``
to an object under ``_build/`` (in parallel) and links
``attention_kernel_triton_b200/libakt.so``.  No torch headers are involved:
the library is plain CUDA C++ behind the C ABI in ``include/akt.h``.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(PKG, "libakt.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
                     "-I" + os.path.join(ROOT, "include"), "--expt-relaxed-constexpr"]
# Files compiled as whole-program device code: ptxas ignores setmaxnreg in
# relocatable device code, and the prefill kernel's warpgroup register split
# depends on it.  They reference no device symbol of another file.
WHOLE_PROGRAM = {"prefill.cu"}


def flags_for(src: str):
    return NVCC_FLAGS + ([] if os.path.basename(src) in WHOLE_PROGRAM else ["-rdc=true"])


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _needs(obj: str, deps) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, force: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = (glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) +
               glob.glob(os.path.join(ROOT, "include", "*.h")))
    cc = nvcc()
    jobs = []
    objs = []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s)[:-3] + ".o")
        objs.append(o)
        if force or _needs(o, [s] + headers):
            jobs.append([cc] + flags_for(s) + ["-c", s, "-o", o])

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        return r

    with ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 4))) as ex:
        list(ex.map(run, jobs))
    if force or jobs or _needs(LIB, objs):
        run([cc] + ARCH + ["-shared", "-rdc=true", "-Xcompiler", "-fPIC", "-o", LIB] + objs + ["-lcudart"])
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
