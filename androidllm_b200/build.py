"""Build libandroidllm_b200.so in-tree with nvcc for sm_100a.

    python -m androidllm_b200.build [--verbose]

The library is a single shared object with a plain C ABI
(include/androidllm_b200.h); it links only the CUDA runtime.
"""
import argparse
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libandroidllm_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-I", os.path.join(ROOT, "include"),
]


def sources():
    return sorted(glob.glob(os.path.join(HERE, "csrc", "*.cu")))


def headers():
    return sorted(glob.glob(os.path.join(HERE, "csrc", "*.cuh")) +
                  glob.glob(os.path.join(ROOT, "include", "*.h")))


def up_to_date():
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(f) <= t for f in sources() + headers() + [__file__])


def build(force=False, verbose=False, ptxas_info=False):
    if not force and up_to_date():
        return LIB
    cmd = [NVCC, *FLAGS, "-shared", "-o", LIB + ".tmp", *sources(), "-lcudart"]
    if ptxas_info:
        cmd.insert(1, "-Xptxas=-v")
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if ptxas_info or verbose:
        print(res.stderr, file=sys.stderr)
    os.replace(LIB + ".tmp", LIB)
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose, ptxas_info=a.ptxas_info))


if __name__ == "__main__":
    main()
