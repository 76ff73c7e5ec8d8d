"""Build liblncc_sm100.so (the C-ABI CUDA library) in-tree for sm_100a.

Usage: python fused-lncc_b200/build.py [--force] [--checked]

--checked builds the bounds-checked variant (LNCC_CHECKED=1) into liblncc_sm100_checked.so beside
the product library: every kernel access is range-checked and entry points report violations as
LNCC_ERR_CHECK (include/lncc.h, lncc_checked_build).

The reference builds a pybind torch extension for sm_70..sm_120 without sm_100
(reference setup.py:16-23,42-49). This builds a plain shared library for sm_100a only, with -O3
and -lineinfo and, like the reference, without --use_fast_math (the variance terms
Spp - Sp^2/n cancel and fast-math would cost accuracy). cudart is linked statically so that the
library carries its own runtime.
"""
import argparse
import os
import subprocess
import sys

PKG_ROOT = os.path.dirname(os.path.abspath(__file__))
REPO_ROOT = os.path.dirname(PKG_ROOT)
SRC = os.path.join(PKG_ROOT, "csrc", "lncc_sm100.cu")
INCLUDE = os.path.join(REPO_ROOT, "include")
LIB_DIR = os.path.join(PKG_ROOT, "fused_lncc")
LIB_NAME = "liblncc_sm100.so"
LIB_PATH = os.path.join(LIB_DIR, LIB_NAME)
CHECKED_LIB_PATH = os.path.join(LIB_DIR, "liblncc_sm100_checked.so")
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path():
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = os.path.join(home, "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def sources():
    csrc = os.path.join(PKG_ROOT, "csrc")
    return sorted(os.path.join(csrc, f) for f in os.listdir(csrc) if f.endswith((".cu", ".cuh", ".h")))


def _stale(out):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    deps = sources() + [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE)]
    return any(os.path.getmtime(d) > t for d in deps)


def build_library(force=False, checked=False, verbose=False, out=None):
    """Compile the library if it is missing or older than its sources; return its path."""
    out = out or (CHECKED_LIB_PATH if checked else LIB_PATH)
    if not force and not _stale(out):
        return out
    cmd = [nvcc_path(), *ARCH_FLAGS, "-lineinfo", "-O3", "-std=c++17", "-I", INCLUDE,
           "-Xcompiler", "-fPIC", "-shared", "-o", out + ".tmp", SRC]
    if checked:
        cmd.insert(1, "-DLNCC_CHECKED=1")
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed building {out}:\n{r.stdout}\n{r.stderr}")
    os.replace(out + ".tmp", out)
    return out


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--checked", action="store_true")
    args = ap.parse_args()
    p = build_library(force=args.force, checked=args.checked, verbose=True)
    print(p)
    sys.exit(0)
