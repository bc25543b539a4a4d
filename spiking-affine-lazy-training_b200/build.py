"""Builds libsalt_b200.so (the CUDA kernels and the C ABI of include/salt_b200.h) in-tree.

The library is compiled for sm_100a only; nvcc cross-compiles without a GPU.  The built file
sits next to this module so that it travels with the source tree.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
import tempfile
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libsalt_b200.so")
NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
              "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr"]


def sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = sources() + [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cuh")]
    deps.append(os.path.join(HERE, "..", "include", "salt_b200.h"))
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the library if any source is newer than it; returns its path.

    Each source compiles to its own object in parallel (no device code crosses files, so no
    relocatable device code is needed), then one link step writes the shared library.
    """
    if not force and not _stale():
        return LIB
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    tmp = LIB + ".tmp"
    with tempfile.TemporaryDirectory(prefix="salt_b200_build_") as obj_dir:
        jobs = []
        for src in sources():
            obj = os.path.join(obj_dir, os.path.basename(src) + ".o")
            jobs.append(([nvcc, *NVCC_FLAGS, "-c", "-o", obj, src], obj))

        def compile_one(job):
            cmd, _ = job
            if verbose:
                print(" ".join(cmd), file=sys.stderr)
            subprocess.run(cmd, check=True)

        with ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 1))) as ex:
            list(ex.map(compile_one, jobs))
        link = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", tmp,
                *(obj for _, obj in jobs)]
        if verbose:
            print(" ".join(link), file=sys.stderr)
        subprocess.run(link, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
