"""Build ``libfdwt_b200.so`` (the C-ABI library of sm_100a kernels) in-tree with nvcc.

    python -m pytorch_morlet_fdwt_b200._build [--force] [--verbose]

Every ``csrc/*.cu`` is compiled for ``sm_100a`` (``-gencode arch=compute_100a,code=sm_100a``)
into ``_build/*.o`` (in parallel, incrementally: an object is rebuilt when its source or any
header is newer) and linked into ``libfdwt_b200.so`` next to this file, with the CUDA runtime
linked statically so the library carries no dependency on a particular libcudart.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
ROOT = os.path.dirname(HERE)
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(HERE, "libfdwt_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
              "-Xcompiler", "-fPIC", "-Xcompiler", "-O3", "-Xptxas", "-O3", "-I", INCLUDE]


def nvcc() -> str:
    exe = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(exe):
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libfdwt_b200.so")
    return exe


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))


def _stale(obj: str, src: str) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(f) > t for f in [src] + _headers())


def build(force: bool = False, verbose: bool = False, extra_flags=()) -> str:
    os.makedirs(BUILD, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    jobs = []
    for src in sources:
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        if force or _stale(obj, src):
            cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *extra_flags, "-c", src, "-o", obj]
            jobs.append((src, cmd))
    objs = [os.path.join(BUILD, os.path.basename(s)[:-3] + ".o") for s in sources]

    def run(job):
        src, cmd = job
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        return src, r

    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            for src, r in ex.map(run, jobs):
                if verbose and r.stderr:
                    print(r.stderr, file=sys.stderr)
                if r.returncode != 0:
                    raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
    if jobs or force or not os.path.exists(LIB) or any(
            os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        tmp = LIB + ".tmp"
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))


if __name__ == "__main__":
    main()
