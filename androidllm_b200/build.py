"""Build libandroidllm_b200.so in-tree with nvcc for sm_100a.

    python -m androidllm_b200.build [--verbose]

The library is a single shared object with a plain C ABI
(include/androidllm_b200.h); it links only the CUDA runtime (NCCL, for
tensor parallelism, is opened at run time).  The measurement
probes (probes/*.cu: tensor-core instruction rates, the graph launch floor)
build into a separate libalm_probes.so that only `bench.py --mma-rate` loads.
"""
import argparse
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libandroidllm_b200.so")
PROBES_LIB = os.path.join(HERE, "libalm_probes.so")
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


def probe_sources():
    return sorted(glob.glob(os.path.join(HERE, "probes", "*.cu")))


def headers():
    return sorted(glob.glob(os.path.join(HERE, "csrc", "*.cuh")) +
                  glob.glob(os.path.join(ROOT, "include", "*.h")))


def up_to_date():
    for lib, srcs in ((LIB, sources()), (PROBES_LIB, probe_sources())):
        if not os.path.exists(lib):
            return False
        t = os.path.getmtime(lib)
        if not all(os.path.getmtime(f) <= t for f in srcs + headers() + [__file__]):
            return False
    return True


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    return subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)


def _finish(proc):
    out, err = proc.communicate()
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed ({proc.returncode}):\n{out}\n{err}")
    return err


def build(force=False, verbose=False, ptxas_info=False):
    """Compile every translation unit in parallel, then link the library."""
    if not force and up_to_date():
        return LIB
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    extra = ["-Xptxas=-v"] if ptxas_info else []
    jobs, objs, probe_objs = [], [], []
    for src in sources() + probe_sources():
        obj = os.path.join(objdir, os.path.basename(src) + ".o")
        (probe_objs if src in probe_sources() else objs).append(obj)
        jobs.append(_run([NVCC, *extra, *FLAGS, "-c", src, "-o", obj], verbose))
    errs = [_finish(p) for p in jobs]
    if ptxas_info or verbose:
        print("".join(errs), file=sys.stderr)
    for lib, o in ((LIB, objs), (PROBES_LIB, probe_objs)):
        _finish(_run([NVCC, *FLAGS, "-shared", "-o", lib + ".tmp", *o, "-lcudart", "-ldl"], verbose))
        os.replace(lib + ".tmp", lib)
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
