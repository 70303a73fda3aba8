"""Build libcbx_ops.so in-tree with nvcc for sm_100a only.

    python -m chatterbox_amdvulkan_b200.build [--force] [--verbose-ptxas]

Each csrc/*.cu is compiled to an object under _build/ (in parallel), then the
objects are linked into chatterbox_amdvulkan_b200/libcbx_ops.so with the CUDA
runtime linked statically, so the library only needs the driver at run time.
Only the symbols declared CBX_API in include/cbx_ops.h are exported.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(ROOT, "_build", "cbx_ops")
LIB = os.path.join(PKG, "libcbx_ops.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
              "-Xcompiler", "-fPIC,-fvisibility=hidden,-O3,-ffp-contract=off", "-I", INCLUDE, "-I", CSRC]


def nvcc() -> str:
    cand = [os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"]
    for c in cand:
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found (set NVCC)")


def _deps() -> list[str]:
    return (glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cuh"))
            + glob.glob(os.path.join(INCLUDE, "*.h")))


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose_ptxas: bool = False, jobs: int | None = None) -> str:
    """Compile every CUDA source for sm_100a and link libcbx_ops.so; returns its path."""
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))
    cc = nvcc()
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []

    def compile_one(src: str) -> tuple[str, str]:
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        if force or verbose_ptxas or _stale(obj, [src] + headers):
            cmd = [cc, *ARCH, *NVCC_FLAGS, *extra, "-c", src, "-o", obj]
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
            return obj, r.stdout + r.stderr
        return obj, ""

    jobs = jobs or min(len(srcs), os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        results = list(ex.map(compile_one, srcs))
    objs = [o for o, _ in results]
    if verbose_ptxas:
        for (o, log) in results:
            sys.stdout.write(f"== {os.path.basename(o)}\n{log}")
    if force or _stale(LIB, objs):
        cmd = [cc, *ARCH, "-shared", "-o", LIB, *objs, "-Xcompiler", "-fPIC"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose_ptxas=a.verbose_ptxas))
