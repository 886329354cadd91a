"""Builds libgqa_sm100.so (the C-ABI library) in-tree for sm_100a.

    python gqa-flash-attn-rtx3060_b200/build.py [--force] [--debug]

The library is one translation unit (csrc/gqa_sm100.cu) compiled by nvcc with
`-gencode arch=compute_100a,code=sm_100a` and the static CUDA runtime; it does
not link libcuda (the driver's tensor-map encoder is looked up at run time),
so it loads on a machine without a GPU driver.
"""
import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
OUT = os.path.join(HERE, "gqa_kernels", "libgqa_sm100.so")
# Debug variant: in-kernel address/coordinate checks (GQA_DEBUG_CHECKS) that report
# GQA_ERR_DEBUG_CHECK instead of faulting; selected at run time with
# GQA_KERNELS_LIB=debug.
OUT_DEBUG = os.path.join(HERE, "gqa_kernels", "libgqa_sm100_debug.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "-cudart", "static",
]


def _sources():
    return sorted(
        [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cuh"))]
        + [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    )


def up_to_date(out=OUT):
    if not os.path.exists(out):
        return False
    t = os.path.getmtime(out)
    return all(os.path.getmtime(s) <= t for s in _sources())


def nvcc():
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libgqa_sm100.so")
    return path


def build(force=False, verbose=False, debug=False):
    """Compiles the library (or, with debug, its checked variant) unless it is newer
    than every source. Returns its path."""
    out = OUT_DEBUG if debug else OUT
    if not force and up_to_date(out):
        return out
    tmp = out + ".tmp"
    cmd = [nvcc(), *NVCC_FLAGS, *(["-DGQA_DEBUG_CHECKS"] if debug else []), "-I", INCLUDE, "-o", tmp,
           os.path.join(CSRC, "gqa_sm100.cu")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, out)
    return out


if __name__ == "__main__":
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--debug", action="store_true", help="build libgqa_sm100_debug.so (in-kernel checks)")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose, debug=a.debug))
    sys.exit(0)
