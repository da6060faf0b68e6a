"""Build libsage_b200.so (the C-ABI library of include/sage_b200.h) with nvcc for sm_100a, in-tree.

    python rdna4-sageattention_b200/build_ext.py [--verbose] [--debug]

Compiles csrc/*.cu to objects under _build/ and links rdna4_sage/libsage_b200.so next to the Python
package that loads it.  Cross-compiles without a GPU.  Objects are rebuilt only when a source or
header is newer.  --debug builds the same sources with SAGE_DEBUG (device-side checks of every store,
TMA coordinate and varlen offset, recorded instead of trapping) into rdna4_sage/libsage_b200_debug.so,
which RDNA4_SAGE_LIB selects at import.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(HERE, "rdna4_sage", "libsage_b200.so")
DEBUG_LIB = os.path.join(HERE, "rdna4_sage", "libsage_b200_debug.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-I", os.path.join(ROOT, "include")]


def _headers() -> list[str]:
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(ROOT, "include", "*.h"))


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, debug: bool = False) -> str:
    build_dir = os.path.join(BUILD, "debug") if debug else BUILD
    lib_path = DEBUG_LIB if debug else LIB
    flags = FLAGS + (["-DSAGE_DEBUG"] if debug else [])
    os.makedirs(build_dir, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = _headers()
    jobs = []
    objects = []
    for src in sources:
        obj = os.path.join(build_dir, os.path.basename(src).replace(".cu", ".o"))
        objects.append(obj)
        if _stale(obj, [src] + headers):
            cmd = [NVCC, *ARCH, *flags, "-c", src, "-o", obj]
            if verbose:
                cmd += ["-Xptxas", "-v"]
            jobs.append(cmd)

    def run(cmd):
        r = subprocess.run(cmd, capture_output=True, text=True)
        return cmd, r

    with cf.ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 1))) as ex:
        for cmd, r in ex.map(run, jobs):
            if verbose or r.returncode != 0:
                sys.stderr.write(r.stdout + r.stderr)
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed: {' '.join(cmd)}")
    if jobs or _stale(lib_path, objects):
        cmd = [NVCC, *ARCH, "-shared", "-o", lib_path, *objects]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("link failed")
    return lib_path


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--debug", action="store_true")
    args = ap.parse_args()
    print(build(args.verbose, args.debug))
