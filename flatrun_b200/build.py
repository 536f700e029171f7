"""Build libfrcuda.so in-tree with nvcc for sm_100a.

    python -m flatrun_b200.build [--verbose] [--ptxas-info]

Each ``csrc/*.cu`` compiles to an object under ``flatrun_b200/_build`` (in
parallel, skipped when up to date), and the objects link into
``flatrun_b200/libfrcuda.so`` against the CUDA runtime.  No GPU is needed.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libfrcuda.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O2",
    "--expt-relaxed-constexpr", "-I" + os.path.join(REPO, "include"),
]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found (CUDA toolkit required to build libfrcuda.so)")
    return cand


def _deps() -> list[str]:
    out = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    out.append(os.path.join(REPO, "include", "frcuda.h"))
    return out


def _compile(src: str, obj: str, extra: list[str], verbose: bool) -> str:
    cmd = [nvcc(), *NVCC_FLAGS, *extra, "-c", src, "-o", obj]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{res.stdout}\n{res.stderr}")
    return res.stderr


def build(verbose: bool = False, ptxas_info: bool = False, force: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    sources = sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))
    dep_mtime = max(os.path.getmtime(p) for p in _deps())
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    jobs = []
    objs = []
    for f in sources:
        src = os.path.join(CSRC, f)
        obj = os.path.join(BUILD, f[:-3] + ".o")
        objs.append(obj)
        stale = force or ptxas_info or not os.path.exists(obj) or \
            os.path.getmtime(obj) < max(os.path.getmtime(src), dep_mtime)
        if stale:
            jobs.append((src, obj))
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            futs = {ex.submit(_compile, s, o, extra, verbose): s for s, o in jobs}
            for fut in cf.as_completed(futs):
                log = fut.result()
                if ptxas_info and log:
                    print(f"== {os.path.basename(futs[fut])}\n{log}")
    lib_stale = force or not os.path.exists(LIB) or \
        os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs)
    if lib_stale:
        cmd = [nvcc(), *ARCH, "-shared", "-o", LIB, *objs, "-lcudart"]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(a.verbose, a.ptxas_info, a.force))


if __name__ == "__main__":
    sys.exit(main())
