"""Build librokoko_b200.so in-tree with nvcc for sm_100a.

    python -m rokoko_b200.build [--force]

Every translation unit under rokoko_b200/csrc is compiled with
`-gencode arch=compute_100a,code=sm_100a -lineinfo -O3` and linked into one
shared library (static cudart, no cuBLAS/cuDNN/CUTLASS).  The C++ model seam
of the reference (rokoko_b200/cpp, include/rokoko/weights.h) is compiled with
g++ into librokoko_compat.so on top of it.  Objects are cached in
rokoko_b200/_build and rebuilt when a source or header is newer.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "librokoko_b200.so")
COMPAT = os.path.join(HERE, "librokoko_compat.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-I", INCLUDE, "-ccbin", "/usr/bin/g++"]


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))


def _stale(out: str, deps: list[str]) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = _sources()
    hdrs = _headers()
    objs = []
    jobs = []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s) + ".o")
        objs.append(o)
        if force or _stale(o, [s] + hdrs):
            cmd = [NVCC, *ARCH, *FLAGS, "-c", s, "-o", o]
            jobs.append(cmd)
    def run(cmd):
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("nvcc failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
        if verbose and (r.stdout or r.stderr):
            print(r.stdout + r.stderr)
    with cf.ThreadPoolExecutor(max(1, min(8, os.cpu_count() or 1))) as ex:
        list(ex.map(run, jobs))
    if jobs or force or _stale(LIB, objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-ccbin", "/usr/bin/g++", "-Xcompiler", "-fPIC"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n" + r.stdout + r.stderr)
    build_compat(force)
    return LIB


def build_compat(force: bool = False) -> str:
    """librokoko_compat.so: the reference's C++ model seam (include/rokoko/weights.h)
    and phonemizer class (include/rokoko/g2p.h) on top of librokoko_b200.so,
    compiled with the system g++."""
    src = os.path.join(HERE, "cpp", "rokoko_compat.cpp")
    hdrs = [os.path.join(INCLUDE, "rokoko", "weights.h"), os.path.join(INCLUDE, "rokoko", "g2p.h"),
            os.path.join(INCLUDE, "rokoko", "tokens.h"), os.path.join(INCLUDE, "rk_b200.h")]
    if not force and not _stale(COMPAT, [src, LIB] + hdrs):
        return COMPAT
    cuda = os.path.dirname(os.path.dirname(NVCC))
    cmd = ["/usr/bin/g++", "-std=c++17", "-O2", "-fPIC", "-shared", "-Wall", "-I", os.path.join(INCLUDE, "rokoko"),
           "-I", os.path.join(cuda, "include"), src, "-o", COMPAT, "-L", HERE, "-lrokoko_b200",
           "-L", os.path.join(cuda, "lib64"), "-lcudart_static", "-ldl", "-lpthread", "-lrt",
           "-Wl,-rpath,$ORIGIN"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("compat library build failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
    return COMPAT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
