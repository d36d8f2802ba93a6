"""Build recipe for the oracle (test infrastructure only).

* ``build_oracle()`` compiles the CPU restatement ``hesa_oracle.c`` into
  ``oracle/liboracle.so`` (gcc, -O2 -ffp-contract=off, OpenMP).
* ``build_ref()`` compiles hesa-llm's own CPU kernels -- the reference's
  ``src/backend/cpu_backend.cpp`` and ``src/tensor/tensor.cpp`` -- together
  with ``ref_shim.cpp`` into ``oracle/_ref/libhesa_ref.so``. The reference does
  not compile as shipped; the recipe copies the files it needs into
  ``oracle/_ref/src`` (git-ignored) and applies the two one-line header fixes
  listed in ``REF_FIXES``, plus ``-include`` of two standard headers. It only
  runs where the reference tree is present; elsewhere the prebuilt library is
  used as is.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REF_ROOT = os.environ.get("HESA_REFERENCE_ROOT", "/root/reference")
REF_OUT = os.path.join(HERE, "_ref")
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(REF_OUT, "libhesa_ref.so")

# (file, text as shipped, compile fix). Each fix is the smallest edit that
# lets the header compile with g++ -std=c++23; semantics are unchanged.
REF_FIXES = [
    ("include/hesa/tensor.hpp",
     "return {strides_.data(), ndim()};",   # tensor.hpp:92, .data() on a C array
     "return {strides_, ndim()};"),
    ("include/hesa/tensor.hpp",
     "return Tensor(Dtype::F32, shape, b);",  # tensor.hpp:156, ambiguous constructor
     "return Tensor(Dtype::F32, Shape(shape), b);"),
    ("src/backend/cpu_backend.cpp",
     "return error(Error::INVALID_ARGUMENT);",  # cpu_backend.cpp:137, Result<void> as Result<Tensor>
     "return std::unexpected{make_error_code(Error::INVALID_ARGUMENT)};"),
    ("src/backend/cpu_backend.cpp",
     "return error(Error::BACKEND_NOT_AVAILABLE);",  # cpu_backend.cpp:301, same
     "return std::unexpected{make_error_code(Error::BACKEND_NOT_AVAILABLE)};"),
]

REF_FILES = [
    "include/hesa/backend.hpp",
    "include/hesa/result.hpp",
    "include/hesa/tensor.hpp",
    "src/backend/cpu_backend.hpp",
    "src/backend/cpu_backend.cpp",
    "src/tensor/tensor.cpp",
]


def _run(cmd: list[str]) -> None:
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("command failed: " + " ".join(cmd) + "\n" + res.stdout + res.stderr)


def _stale(target: str, sources: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources if os.path.exists(s))


def build_oracle(force: bool = False) -> str:
    src = os.path.join(HERE, "hesa_oracle.c")
    hdr = os.path.join(HERE, "hesa_oracle.h")
    if force or _stale(ORACLE_SO, [src, hdr, __file__]):
        _run(["gcc", "-std=c11", "-O2", "-ffp-contract=off", "-fopenmp", "-fPIC",
              "-shared", "-Wall", "-Wno-misleading-indentation", src, "-o", ORACLE_SO, "-lm"])
    return ORACLE_SO


def prepare_ref_sources(dst: str) -> None:
    """Copy the reference files the CPU kernels need and apply REF_FIXES."""
    for rel in REF_FILES:
        s = os.path.join(REF_ROOT, rel)
        d = os.path.join(dst, rel)
        os.makedirs(os.path.dirname(d), exist_ok=True)
        shutil.copyfile(s, d)
        os.chmod(d, 0o644)
    for rel, old, new in REF_FIXES:
        p = os.path.join(dst, rel)
        with open(p) as f:
            text = f.read()
        if old not in text:
            raise RuntimeError(f"reference fix no longer applies: {rel}: {old!r}")
        with open(p, "w") as f:
            f.write(text.replace(old, new, 1))


def build_ref(force: bool = False) -> str | None:
    """Build oracle/_ref/libhesa_ref.so from the reference's own sources.

    Returns the library path, or None when neither the reference tree nor a
    prebuilt library is available.
    """
    shim = os.path.join(HERE, "ref_shim.cpp")
    if not os.path.isdir(os.path.join(REF_ROOT, "src")):
        return REF_SO if os.path.exists(REF_SO) else None
    srcdir = os.path.join(REF_OUT, "src")
    ref_inputs = [os.path.join(REF_ROOT, r) for r in REF_FILES] + [shim, __file__]
    if not (force or _stale(REF_SO, ref_inputs)):
        return REF_SO
    os.makedirs(REF_OUT, exist_ok=True)
    prepare_ref_sources(srcdir)
    # The reference's CMake builds with C++20 plus -mavx512f -mfma; <expected>
    # needs C++23 with g++ 13. -ffp-contract=off keeps `sum += a*b` as a
    # separate multiply and add, the arithmetic the oracle restates.
    _run(["g++", "-std=c++23", "-O2", "-ffp-contract=off", "-fPIC", "-shared", "-pthread",
          "-include", "algorithm", "-include", "cstring",
          "-DHESA_ARCH_x86_64=1", "-DHESA_PLATFORM_linux=1",
          "-I", os.path.join(srcdir, "include"), "-I", os.path.join(srcdir, "src"),
          os.path.join(srcdir, "src/backend/cpu_backend.cpp"),
          os.path.join(srcdir, "src/tensor/tensor.cpp"),
          shim, "-o", REF_SO])
    return REF_SO


def build_all(force: bool = False) -> None:
    build_oracle(force)
    build_ref(force)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv)
    print(ORACLE_SO)
    print(REF_SO if os.path.exists(REF_SO) else "(reference library unavailable)")
