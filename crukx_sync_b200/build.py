"""Build the in-tree CUDA library ``crukx_sync_b200/libcrukx_b200.so`` for sm_100a with nvcc.

    python -m crukx_sync_b200.build [--force] [--verbose]

Objects go to ``crukx_sync_b200/_build/``; a file is recompiled when it or any header is newer
than its object.  The library exports the C ABI declared in ``include/crukx_b200.h``.
"""

from __future__ import annotations

import concurrent.futures
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libcrukx_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3", "-I", os.path.join(ROOT, "include"),
         "--expt-relaxed-constexpr"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the crukx_sync_b200 CUDA library cannot be built")


def cxx() -> str:
    return os.environ.get("CXX") or shutil.which("g++") or "g++"


def _headers():
    return glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(ROOT, "include", "*.h"))


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    newest_header = max((os.path.getmtime(h) for h in _headers()), default=0.0)
    cc = nvcc()
    jobs = []
    objs = []
    for src in srcs:
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        objs.append(obj)
        stale = force or not os.path.exists(obj) or os.path.getmtime(obj) < max(os.path.getmtime(src), newest_header)
        if stale:
            cmd = [cc, *ARCH, *FLAGS, *(extra or []), "-c", src, "-o", obj]
            if src.endswith(".cpp"):
                cmd = [cxx(), "-O3", "-std=c++17", "-fPIC", "-Wall", "-I", os.path.join(ROOT, "include"),
                       "-c", src, "-o", obj]
            jobs.append(cmd)

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout + r.stderr, flush=True)

    with concurrent.futures.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        list(ex.map(run, jobs))
    if jobs or not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        tmp = LIB + ".tmp"
        run([cc, *ARCH, "-shared", "-o", tmp, *objs, "-lcudart"])
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="--verbose" in sys.argv)
    print(LIB)
