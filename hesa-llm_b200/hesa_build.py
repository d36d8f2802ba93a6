"""Build recipe of the hesa-b200 CUDA backend (in-tree, sm_100a only).

``build_cuda()`` compiles ``csrc/*.cu`` with nvcc into ``libhesa_cuda.so``
next to this file: the C ABI of include/hesa_cuda.h with every kernel, built
``-gencode arch=compute_100a,code=sm_100a -lineinfo`` and linked against the
static CUDA runtime. nvcc cross-compiles, so this runs without a GPU.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
CUDA_SO = os.path.join(HERE, "libhesa_cuda.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
              "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden"]


def _run(cmd):
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("build failed: " + " ".join(cmd) + "\n" + res.stdout + res.stderr)
    return res


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps():
    return (_sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
            + glob.glob(os.path.join(INCLUDE, "*.h")) + [os.path.abspath(__file__)])


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build_cuda(force: bool = False, verbose: bool = False) -> str:
    if not (force or _stale(CUDA_SO, _deps())):
        return CUDA_SO
    objs = []
    build_dir = os.path.join(HERE, "_build")
    os.makedirs(build_dir, exist_ok=True)
    for src in _sources():
        obj = os.path.join(build_dir, os.path.basename(src)[:-3] + ".o")
        cmd = [NVCC, *ARCH_FLAGS, *NVCC_FLAGS, "-I", INCLUDE, "-c", src, "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        res = _run(cmd)
        if verbose:
            sys.stderr.write(res.stderr)
        objs.append(obj)
    tmp = CUDA_SO + ".tmp"
    _run([NVCC, *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", tmp, *objs])
    os.replace(tmp, CUDA_SO)
    return CUDA_SO


def build_all(force: bool = False) -> None:
    build_cuda(force)


if __name__ == "__main__":
    build_cuda(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(CUDA_SO)
