"""Build the CUDA library of the package in-tree: ``belt_b200/libbelt_b200.so`` for sm_100a.

    python -m belt_b200.build [--force] [--jobs N]

nvcc compiles every ``csrc/*.cu`` with ``-gencode arch=compute_100a,code=sm_100a`` (cross-compiles without a GPU)
and links them into one shared library with the C ABI of ``include/belt_b200.h``. Objects are rebuilt only when a
source or header is newer than the library.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB = os.path.join(PKG, "libbelt_b200.so")
OBJ_DIR = os.path.join(PKG, "_build")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr", "-cudart", "shared",
         "-I" + os.path.join(ROOT, "include"), "-I" + CSRC]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _newest_input() -> float:
    files = sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(ROOT, "include", "*.h"))
    return max(os.path.getmtime(f) for f in files)


def build(force: bool = False, jobs: int = 8, verbose: bool = False) -> str:
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= _newest_input():
        return LIB
    os.makedirs(OBJ_DIR, exist_ok=True)
    cc = nvcc()

    def compile_one(src):
        obj = os.path.join(OBJ_DIR, os.path.basename(src) + ".o")
        cmd = [cc, *ARCH, *FLAGS, "-c", src, "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{r.stderr}")
        return obj, r.stderr

    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        results = list(ex.map(compile_one, sources()))
    if verbose:
        for obj, err in results:
            if err.strip():
                print(err)
    tmp = LIB + ".tmp"
    cmd = [cc, *ARCH, "-shared", "-cudart", "shared", "-o", tmp, *[o for o, _ in results]]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=8)
    ap.add_argument("-v", "--verbose", action="store_true", help="print ptxas resource usage")
    a = ap.parse_args()
    print(build(a.force, a.jobs, a.verbose))


if __name__ == "__main__":
    main()
