"""hesa::CudaBackend (hesa-llm_b200/backend/cuda_backend.cpp), the C++ drop-in
for the reference's Backend interface (include/hesa/backend.hpp:28-65), built
against the reference's own headers, Tensor and CPU_Backend sources (the
copies oracle/build.py prepares under oracle/_ref/src) and checked op by op
against CPU_Backend by tests/cpp/test_cuda_backend.cpp.

The build runs on CPU (it only needs g++ and the CUDA runtime's headers); the
comparison runs on the GPU."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_SRC = os.path.join(ROOT, "oracle", "_ref", "src")
OUT_DIR = os.path.join(ROOT, "tests", "cpp", "_build")
EXE = os.path.join(OUT_DIR, "test_cuda_backend")
SOURCES = [
    os.path.join(ROOT, "tests", "cpp", "test_cuda_backend.cpp"),
    os.path.join(ROOT, "hesa-llm_b200", "backend", "cuda_backend.cpp"),
    os.path.join(REF_SRC, "src", "tensor", "tensor.cpp"),
    os.path.join(REF_SRC, "src", "backend", "cpu_backend.cpp"),
]
HEADERS = [
    os.path.join(ROOT, "hesa-llm_b200", "backend", "cuda_backend.hpp"),
    os.path.join(ROOT, "include", "hesa_cuda.h"),
]


def _libs():
    import hesa_cuda as H
    from oracle import build as B
    H.lib()   # builds libhesa_cuda.so when it is missing or stale
    return H.library_path(), B.build_oracle()


def build_test_program() -> str:
    if not os.path.isdir(REF_SRC):
        pytest.skip("the reference's CPU backend sources are not prepared (oracle/_ref/src)")
    cuda_lib, oracle_lib = _libs()
    inputs = SOURCES + HEADERS + [cuda_lib, oracle_lib]
    if os.path.exists(EXE) and all(os.path.getmtime(p) <= os.path.getmtime(EXE) for p in inputs):
        return EXE
    os.makedirs(OUT_DIR, exist_ok=True)
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    lib_dirs = [os.path.dirname(cuda_lib), os.path.dirname(oracle_lib)]
    cmd = ["g++", "-std=c++23", "-O2", "-ffp-contract=off", "-pthread",
           # the reference's sources rely on these two headers arriving transitively
           "-include", "algorithm", "-include", "cstring",
           "-DHESA_ARCH_x86_64=1", "-DHESA_PLATFORM_linux=1",
           "-I", os.path.join(REF_SRC, "include"), "-I", os.path.join(REF_SRC, "src"),
           "-I", os.path.join(ROOT, "hesa-llm_b200"), "-I", os.path.join(ROOT, "include"),
           "-I", os.path.join(ROOT, "oracle"), "-I", os.path.join(cuda_home, "include"),
           *SOURCES, "-o", EXE,
           "-L", lib_dirs[0], "-lhesa_cuda", "-L", lib_dirs[1], "-loracle",
           "-L", os.path.join(cuda_home, "lib64"), "-lcudart",
           "-Wl,-rpath," + ":".join(lib_dirs)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr[-4000:]
    return EXE


def test_backend_builds_against_reference_headers():
    assert os.access(build_test_program(), os.X_OK)


@pytest.mark.gpu
def test_backend_ops_match_cpu_backend():
    exe = build_test_program()
    res = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    print(res.stdout)
    lines = res.stdout.splitlines()
    assert any(l.startswith("PASS matmul Q4_K") for l in lines), res.stdout + res.stderr
    failed = [l for l in lines if l.startswith("FAIL")]
    assert res.returncode == 0 and not failed, "\n".join(failed) + res.stderr
