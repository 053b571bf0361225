"""Build libsparsl_cuda.so in-tree with nvcc for sm_100a.

Run ``python -m sparsl_b200.build`` (or call :func:`build`).  Objects go to
``sparsl_b200/_build/``; the shared library lands beside this file so it
travels with the source tree.  Every translation unit is recompiled when it
or any header changed.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
ROOT = os.path.dirname(HERE)
OUT = os.path.join(HERE, "libsparsl_cuda.so")
BUILD = os.path.join(HERE, "_build")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# -fmad=false: no FMA contraction anywhere (the reference never contracts);
# no --use_fast_math, so no flush-to-zero and IEEE division.
NVFLAGS = ["-O3", "-lineinfo", "-fmad=false", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O2"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libsparsl_cuda")


def _nccl_include() -> str:
    try:
        import nvidia.nccl  # type: ignore

        inc = os.path.join(list(nvidia.nccl.__path__)[0], "include")
        if os.path.exists(os.path.join(inc, "nccl.h")):
            return inc
    except Exception:
        pass
    if os.path.exists("/usr/include/nccl.h"):
        return "/usr/include"
    raise RuntimeError("nccl.h not found")


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))


def _headers():
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.hpp"))
                  + glob.glob(os.path.join(ROOT, "include", "*.h")))


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, jobs: int | None = None) -> str:
    nvcc = _nvcc()
    inc = ["-I" + _nccl_include(), "-I" + os.path.join(ROOT, "include")]
    os.makedirs(BUILD, exist_ok=True)
    headers = _headers()
    objs = []
    todo = []
    for src in _sources():
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        objs.append(obj)
        if _stale(obj, [src] + headers):
            cmd = [nvcc] + ARCH + NVFLAGS + inc + ["-c", src, "-o", obj]
            if src.endswith(".cpp"):
                cmd = [nvcc] + NVFLAGS + inc + ["-x", "c++", "-c", src, "-o", obj]
            todo.append(cmd)

    def run(cmd):
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("nvcc failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
        return r

    with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 1)) as ex:
        list(ex.map(run, todo))
    if todo or _stale(OUT, objs):
        tmp = OUT + ".tmp"
        run([nvcc] + ARCH + ["-shared", "-o", tmp] + objs + ["-ldl", "-lpthread"])
        os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
