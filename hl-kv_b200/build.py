"""Builds libhlkv.so (the CUDA kernels, the C++ host library and the C ABI).

    python hl-kv_b200/build.py [--force] [--verbose-ptxas]

Every .cu file is compiled for sm_100a only (``-gencode
arch=compute_100a,code=sm_100a``), without fast-math: the kernels must round
exactly like the reference's CPU code.  Objects go to hl-kv_b200/_build/ and
the library to hl-kv_b200/hlkv/libhlkv.so, inside the tree, so it travels with
the repository to the GPU machine.  Rebuilds only what changed (sources or
headers newer than the object).
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OBJ_DIR = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "hlkv", "libhlkv.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
INCLUDES = ["-I", os.path.join(ROOT, "include"), "-I", os.path.join(CSRC, "kernels")]


def _sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "**", "*.cu"), recursive=True) +
                  glob.glob(os.path.join(CSRC, "**", "*.cpp"), recursive=True))


def _headers() -> list[str]:
    return (glob.glob(os.path.join(ROOT, "include", "**", "*.h*"), recursive=True) +
            glob.glob(os.path.join(CSRC, "**", "*.cuh"), recursive=True) +
            glob.glob(os.path.join(CSRC, "**", "*.hpp"), recursive=True))


def _obj(src: str) -> str:
    rel = os.path.relpath(src, CSRC).replace(os.sep, "__")
    return os.path.join(OBJ_DIR, rel + ".o")


def _compile(src: str, verbose_ptxas: bool) -> str:
    obj = _obj(src)
    tmp = obj + f".tmp{os.getpid()}"
    if src.endswith(".cu"):
        cmd = [NVCC, "-std=c++20", "-O3", "-Xcompiler", "-fPIC", *INCLUDES, *ARCH, "-lineinfo",
               "--expt-relaxed-constexpr", "-Xcompiler", "-Wall"]
        if verbose_ptxas:
            cmd += ["-Xptxas", "-v"]
        cmd += ["-c", src, "-o", tmp]
    else:
        cmd = ["g++", "-std=c++20", "-O3", "-fPIC", "-Wall", "-Wextra", "-ffp-contract=off",
               "-I", "/usr/local/cuda/include", *INCLUDES, "-c", src, "-o", tmp]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {src}\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, obj)
    return (r.stdout + r.stderr).strip()


def build(force: bool = False, verbose_ptxas: bool = False, quiet: bool = True) -> str:
    os.makedirs(OBJ_DIR, exist_ok=True)
    srcs = _sources()
    newest_header = max((os.path.getmtime(h) for h in _headers()), default=0.0)
    stale = [s for s in srcs if force or verbose_ptxas or not os.path.exists(_obj(s)) or
             os.path.getmtime(_obj(s)) < max(os.path.getmtime(s), newest_header)]
    if stale:
        with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
            for src, log in zip(stale, ex.map(lambda s: _compile(s, verbose_ptxas), stale)):
                if log and (verbose_ptxas or not quiet):
                    print(f"== {os.path.relpath(src, ROOT)}\n{log}")
    objs = [_obj(s) for s in srcs]
    if stale or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(map(os.path.getmtime, objs)):
        tmp = LIB + f".tmp{os.getpid()}"
        cmd = [NVCC, "-shared", *ARCH, "-o", tmp, *objs, "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose_ptxas="--verbose-ptxas" in sys.argv,
                quiet=False))
