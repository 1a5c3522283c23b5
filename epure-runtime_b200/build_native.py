"""Build libepq.so (the C-ABI CUDA library) in-tree for sm_100a.

    python epure-runtime_b200/build_native.py [--verbose-ptxas]

Compiles every csrc/*.cu with nvcc into epure/libepq.so next to the Python
package, so the library travels with the source tree.  Object files go to
csrc/_build/.  A source is recompiled only when it or a header is newer than
its object.  The CPU kernel (csrc_cpu/epq_cpu.cpp, include/epq_cpu.h) is built
with g++/OpenMP into epure/libepq_cpu.so.
"""
import argparse
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(CSRC, "_build")
OUT = os.path.join(HERE, "epure", "libepq.so")
CPU_SRC = os.path.join(HERE, "csrc_cpu", "epq_cpu.cpp")
CPU_OUT = os.path.join(HERE, "epure", "libepq_cpu.so")
INCLUDE = os.path.join(ROOT, "include")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
    "-I", INCLUDE, "-I", CSRC,
]


def _nvcc():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.isabs(cand) and os.path.exists(cand) or not os.path.isabs(cand)):
            return cand
    return "nvcc"


def build(verbose_ptxas=False, force=False, quiet=False):
    os.makedirs(OBJ, exist_ok=True)
    headers = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))
    newest_header = max((os.path.getmtime(h) for h in headers), default=0)
    objs = []
    for src in sorted(glob.glob(os.path.join(CSRC, "*.cu"))):
        obj = os.path.join(OBJ, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if not force and os.path.exists(obj) and \
                os.path.getmtime(obj) >= max(os.path.getmtime(src), newest_header):
            continue
        cmd = [_nvcc(), *NVCC_FLAGS, "-c", src, "-o", obj]
        if verbose_ptxas:
            cmd.insert(1, "-Xptxas=-v")
        if not quiet:
            print(" ".join(os.path.relpath(c, ROOT) if c.startswith(ROOT) else c for c in cmd),
                  flush=True)
        subprocess.check_call(cmd)
    if force or not os.path.exists(OUT) or \
            os.path.getmtime(OUT) < max(os.path.getmtime(o) for o in objs):
        cmd = [_nvcc(), "-shared", "-gencode", "arch=compute_100a,code=sm_100a",
               *objs, "-o", OUT, "-lcudart_static", "-lrt", "-ldl", "-lpthread"]
        subprocess.check_call(cmd)
    build_cpu(force=force, quiet=quiet)
    return OUT


def _cxx():
    """A g++ with OpenMP: EPURE_CXX, else the system g++ (a toolchain named by CXX
    may lack libgomp)."""
    for cand in (os.environ.get("EPURE_CXX"), "/usr/bin/g++", "g++"):
        if cand and (not os.path.isabs(cand) or os.path.exists(cand)):
            return cand
    return "g++"


def build_cpu(force=False, quiet=False):
    """libepq_cpu.so: -ffp-contract=off keeps the reference's unfused multiply-then-add."""
    header = os.path.join(INCLUDE, "epq_cpu.h")
    newest = max(os.path.getmtime(CPU_SRC), os.path.getmtime(header))
    if not force and os.path.exists(CPU_OUT) and os.path.getmtime(CPU_OUT) >= newest:
        return CPU_OUT
    cmd = [_cxx(), "-O3", "-std=c++17", "-fPIC", "-shared", "-fopenmp",
           "-ffp-contract=off", "-I", INCLUDE, CPU_SRC, "-o", CPU_OUT]
    if not quiet:
        print(" ".join(os.path.relpath(c, ROOT) if c.startswith(ROOT) else c for c in cmd), flush=True)
    subprocess.check_call(cmd)
    return CPU_OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose-ptxas", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(verbose_ptxas=a.verbose_ptxas, force=a.force))
    sys.exit(0)
