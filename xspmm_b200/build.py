"""Build libxspmm_b200.so in-tree from xspmm_b200/csrc/*.cu for sm_100a.

Each translation unit is compiled by nvcc in parallel into xspmm_b200/_build/, then linked into
xspmm_b200/libxspmm_b200.so (the CUDA runtime is linked statically, so the library does not depend
on which libcudart another package loads). Rebuilds only what changed (object newer than its
source and every header).

    python -m xspmm_b200.build [--force] [--verbose]
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
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libxspmm_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-I" + os.path.join(ROOT, "include"),
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build xspmm_b200")


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h"))


def _stale(obj: str, src: str, headers) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(d) > t for d in [src] + list(headers))


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = _headers()
    cc = nvcc()
    jobs = []
    for src in srcs:
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        if force or _stale(obj, src, headers):
            jobs.append((src, obj))

    def run(job):
        src, obj = job
        cmd = [cc] + NVCC_FLAGS + ["-c", src, "-o", obj]
        if verbose:
            cmd += ["-Xptxas", "-v"]
        p = subprocess.run(cmd, capture_output=True, text=True)
        return src, p.returncode, p.stdout + p.stderr

    failed = []
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            for src, rc, out in ex.map(run, jobs):
                if verbose or rc != 0:
                    sys.stderr.write(f"--- {os.path.basename(src)}\n{out}")
                if rc != 0:
                    failed.append(src)
    if failed:
        raise RuntimeError("nvcc failed for: " + ", ".join(os.path.basename(f) for f in failed))
    objs = [os.path.join(BUILD, os.path.basename(s)[:-3] + ".o") for s in srcs]
    if force or jobs or not os.path.exists(LIB) or any(
            os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        tmp = LIB + ".tmp"
        cmd = [cc] + ARCH + ["-shared", "-cudart", "static", "-o", tmp] + objs
        p = subprocess.run(cmd, capture_output=True, text=True)
        if p.returncode != 0:
            raise RuntimeError("link failed:\n" + p.stdout + p.stderr)
        os.replace(tmp, LIB)
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))


if __name__ == "__main__":
    main()
