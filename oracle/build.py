"""Build recipe for the oracle libraries (TEST INFRASTRUCTURE ONLY).

    python oracle/build.py            # both, when the reference tree is present

* ``oracle/_build/liboracle.so`` -- the C restatement in ``hlkv_oracle.c``.
* ``oracle/_ref/libhlkv_ref_cuda.so`` -- the reference's own GPU kernel
  (project2_quant/src/dequant_kernel.cu, flat FP8 -> FP16) compiled for sm_100a
  with ``ref_cuda_shim.cu``: the GPU comparison point for this library's drop-in.
* ``oracle/_ref/libhlkv_ref.so`` -- the reference's own CPU library compiled
  straight from its sources (hl_quant: cpu_quant.cpp, cpu_dequant.cpp,
  quant_types.cpp; hl_allocator: hetero_block_table.cpp, id_arena.cpp,
  status.cpp) with g++, plus ``ref_shim.cpp`` (extern "C" wrappers) and
  ``table_trace.cpp`` (the API random walk).  Built only where the reference
  tree exists; the reference's own CMake build is not used.  Outputs go to
  ``oracle/_ref/`` only, which is git-ignored and travels with the tree.

Both are built without -ffast-math and with -ffp-contract=off, like the
reference's own build (project2_quant/CMakeLists.txt keeps fast-math off).
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
# The reference tree: HLKV_REFERENCE_ROOT, else a checkout named "reference" beside
# this repository.  Where neither exists (a machine that only runs the prebuilt
# libraries), nothing of the reference is built.
REF_ROOT = os.environ.get("HLKV_REFERENCE_ROOT") or os.path.normpath(
    os.path.join(HERE, os.pardir, os.pardir, "reference"))
BUILD_DIR = os.path.join(HERE, "_build")
REF_DIR = os.path.join(HERE, "_ref")
ORACLE_SO = os.path.join(BUILD_DIR, "liboracle.so")
REF_SO = os.path.join(REF_DIR, "libhlkv_ref.so")
REF_CUDA_SO = os.path.join(REF_DIR, "libhlkv_ref_cuda.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
# The reference's one GPU kernel (flat FP8 -> FP16) and what it links against.
REF_CUDA_SOURCES = ["project2_quant/src/dequant_kernel.cu", "project2_quant/src/quant_types.cpp"]

REF_SOURCES = [
    "project2_quant/src/cpu_quant.cpp",
    "project2_quant/src/cpu_dequant.cpp",
    "project2_quant/src/quant_types.cpp",
    "project1_allocator/src/hetero_block_table.cpp",
    "project1_allocator/src/id_arena.cpp",
    "project1_allocator/src/status.cpp",
]


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def _run(cmd: list[str]) -> None:
    subprocess.run(cmd, check=True)


def build_oracle(force: bool = False) -> str:
    src = os.path.join(HERE, "hlkv_oracle.c")
    if force or _stale(ORACLE_SO, [src, __file__]):
        os.makedirs(BUILD_DIR, exist_ok=True)
        tmp = ORACLE_SO + f".tmp{os.getpid()}"
        _run(["gcc", "-std=c11", "-O2", "-fPIC", "-shared", "-ffp-contract=off",
              "-fno-fast-math", "-fvisibility=hidden", "-o", tmp, src, "-lm", "-lpthread"])
        os.replace(tmp, ORACLE_SO)
    return ORACLE_SO


def reference_available() -> bool:
    return all(os.path.exists(os.path.join(REF_ROOT, s)) for s in REF_SOURCES)


def build_ref(force: bool = False) -> str | None:
    """Compiles the reference CPU library into oracle/_ref; None without the tree."""
    if not reference_available():
        return REF_SO if os.path.exists(REF_SO) else None
    srcs = [os.path.join(REF_ROOT, s) for s in REF_SOURCES]
    mine = [os.path.join(HERE, "ref_shim.cpp"), os.path.join(HERE, "table_trace.cpp")]
    if force or _stale(REF_SO, srcs + mine + [__file__]):
        os.makedirs(REF_DIR, exist_ok=True)
        tmp = REF_SO + f".tmp{os.getpid()}"
        _run(["g++", "-std=c++20", "-O2", "-fPIC", "-shared", "-ffp-contract=off",
              "-fno-fast-math",
              "-I", os.path.join(REF_ROOT, "project1_allocator/include"),
              "-I", os.path.join(REF_ROOT, "project2_quant/include"),
              "-I", os.path.join(REF_ROOT, "project2_quant/src"),
              "-o", tmp, *srcs, *mine, "-lpthread"])
        os.replace(tmp, REF_SO)
    return REF_SO


def build_ref_cuda(force: bool = False) -> str | None:
    """Compiles the reference's FP8 -> FP16 kernel (its own source, sm_100a only, no
    fast-math) with oracle/ref_cuda_shim.cu into oracle/_ref; None without the tree."""
    srcs = [os.path.join(REF_ROOT, s) for s in REF_CUDA_SOURCES]
    if not all(os.path.exists(s) for s in srcs):
        return REF_CUDA_SO if os.path.exists(REF_CUDA_SO) else None
    shim = os.path.join(HERE, "ref_cuda_shim.cu")
    if force or _stale(REF_CUDA_SO, srcs + [shim, __file__]):
        os.makedirs(REF_DIR, exist_ok=True)
        tmp = REF_CUDA_SO + f".tmp{os.getpid()}"
        _run([NVCC, "-std=c++20", "-O3", "-shared", "-Xcompiler", "-fPIC",
              "-gencode", "arch=compute_100a,code=sm_100a",
              "-I", os.path.join(REF_ROOT, "project2_quant/include"),
              "-I", os.path.join(REF_ROOT, "project2_quant/src"),
              "-o", tmp, *srcs, shim])
        os.replace(tmp, REF_CUDA_SO)
    return REF_CUDA_SO


def build_all(force: bool = False) -> None:
    build_oracle(force)
    build_ref(force)
    build_ref_cuda(force)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv)
    print(ORACLE_SO, REF_SO if os.path.exists(REF_SO) else "(reference not built)")
