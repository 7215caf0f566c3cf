"""Build libvesper_c.so (the B200 IVF-PQ engine and its C ABI) in-tree.

CUDA sources are compiled for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``);
host sources with g++ -std=c++23.  Objects go to vesper_db_b200/_build/ and are rebuilt
only when a source or header is newer than the object.  The CUDA runtime is linked
statically so the library has no dependency on the toolkit's shared libraries.

    python -m vesper_db_b200.build        # or: python vesper_db_b200/build.py
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libvesper_c.so")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA, "bin", "nvcc")
CXX = "g++"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr",
]
CXX_FLAGS = ["-std=c++23", "-O2", "-fPIC", "-fvisibility=hidden", "-ffp-contract=off",
             "-Wall", "-Wextra", f"-I{CUDA}/include", f"-I{ROOT}/include"]


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.hpp")) + \
        glob.glob(os.path.join(ROOT, "include", "*.h"))


def _stale(obj: str, src: str, deps) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(p) > t for p in [src, *deps])


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {' '.join(cmd[:3])} ... {cmd[-1]}")
    return r


def build(verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    deps = _headers()
    objs, jobs = [], []
    for src in sorted(glob.glob(os.path.join(CSRC, "*.cu"))):
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        if _stale(obj, src, deps):
            jobs.append(("nvcc", [NVCC, *NVCC_FLAGS, "-c", src, "-o", obj]))
        objs.append(obj)
    for src in sorted(glob.glob(os.path.join(CSRC, "*.cpp"))):
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        if _stale(obj, src, deps):
            jobs.append(("g++ ", [CXX, *CXX_FLAGS, "-c", src, "-o", obj]))
        objs.append(obj)
    if jobs:
        # translation units are independent: compile them concurrently
        from concurrent.futures import ThreadPoolExecutor

        def one(job):
            if verbose:
                print(job[0], os.path.basename(job[1][-3]), flush=True)
            return _run(job[1])

        with ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 1))) as pool:
            list(pool.map(one, jobs))
    if jobs or not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        _run([NVCC, "-shared", "-Xlinker", "--no-undefined", "-gencode", "arch=compute_100a,code=sm_100a", "-cudart", "static",
              "-o", LIB, *objs, "-lpthread", "-ldl", "-lrt"])
    return LIB


if __name__ == "__main__":
    print(build(verbose=True))
