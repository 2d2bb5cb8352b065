"""Build libspx.so (the C-ABI CUDA library) in-tree for sm_100a.

    python unsloth-spectral_b200/csrc/build.py [--jobs N] [--force]

Objects go to ``csrc/_build/``; the shared library is written next to the Python
package (``unsloth_spectral/libspx.so``) so it travels with the source tree.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

CSRC = os.path.dirname(os.path.abspath(__file__))
PKG_ROOT = os.path.dirname(CSRC)
REPO = os.path.dirname(PKG_ROOT)
INCLUDE = os.path.join(REPO, "include")
OUT = os.path.join(PKG_ROOT, "unsloth_spectral", "libspx.so")
BUILD = os.path.join(CSRC, "_build")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-I", INCLUDE, "-I", CSRC]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(obj: str, deps) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(d) > t for d in deps)


def build(jobs: int = 0, force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))
    cc = nvcc()
    cmds = []
    objs = []
    for src in sources:
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if force or _stale(obj, [src] + headers):
            extra = ["-Xptxas", "-v"] if ptxas_verbose else []
            cmds.append([cc, *ARCH, *FLAGS, *extra, "-c", src, "-o", obj])
    jobs = jobs or min(len(cmds) or 1, os.cpu_count() or 4)

    def run(cmd):
        r = subprocess.run(cmd, capture_output=True, text=True)
        return cmd, r

    failed = []
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        for cmd, r in ex.map(run, cmds):
            if verbose or r.returncode != 0 or ptxas_verbose:
                sys.stderr.write(r.stdout + r.stderr)
            if r.returncode != 0:
                failed.append(cmd[-3])
    if failed:
        raise RuntimeError(f"nvcc failed for: {failed}")
    if cmds or not os.path.exists(OUT) or force:
        link = [cc, *ARCH, "-shared", "-Xcompiler", "-fPIC", *objs, "-o", OUT]
        r = subprocess.run(link, capture_output=True, text=True)
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("link failed")
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--jobs", type=int, default=0)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="print -Xptxas -v register/smem usage")
    a = ap.parse_args()
    print(build(a.jobs, a.force, a.verbose, a.ptxas))
