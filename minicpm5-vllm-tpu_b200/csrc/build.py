"""Build libminicpm5_mk.so (sm_100a) in-tree next to the Python package.

    python minicpm5-vllm-tpu_b200/csrc/build.py [--force] [--verbose]

nvcc cross-compiles for sm_100a without a GPU.  The library links the CUDA runtime statically and
takes the driver entry point it needs (cuTensorMapEncodeTiled) through cudaGetDriverEntryPoint, so
it does not depend on torch or on libcuda at link time.
"""

from __future__ import annotations

import argparse
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG_ROOT = os.path.dirname(HERE)
REPO = os.path.dirname(PKG_ROOT)
OUT = os.path.join(PKG_ROOT, "minicpm5_mk", "libminicpm5_mk.so")
SOURCES = [os.path.join(HERE, "mk_api.cu")]
NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
              "-shared", "-Xptxas", "-v"]


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _inputs():
    return sorted(glob.glob(os.path.join(HERE, "*.cu")) + glob.glob(os.path.join(HERE, "*.cuh")) +
                  glob.glob(os.path.join(REPO, "include", "*.h")) + [os.path.abspath(__file__)])


def up_to_date() -> bool:
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    return all(os.path.getmtime(p) <= t for p in _inputs())


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return OUT
    cmd = [_nvcc(), *NVCC_FLAGS, "-o", OUT + ".tmp", *SOURCES]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"nvcc failed ({r.returncode})")
    if verbose:
        sys.stdout.write(r.stderr)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.verbose))
