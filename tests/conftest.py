"""Test configuration: the `gpu` marker, import paths and on-demand builds.

`-m "not gpu"` runs on any machine (oracle vs golden vectors, host table,
C-ABI exports).  `-m gpu` needs a CUDA device and runs the CUDA kernels
through the C ABI against the CPU oracle.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "hl-kv_b200")
for p in (ROOT, PKG, os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def hlkv_lib():
    """libhlkv.so, built from the tree when missing or stale."""
    import runpy
    runpy.run_path(os.path.join(PKG, "build.py"))["build"]()
    import hlkv
    return hlkv


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def ref():
    from oracle.oracle import Ref, ref_available
    if not ref_available():
        pytest.skip("the reference tree is not present (golden fixtures cover this case)")
    return Ref()


@pytest.fixture(scope="session")
def cuda_device(hlkv_lib):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.init()
    return torch.device("cuda:0")
