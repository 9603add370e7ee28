"""Shared pytest set-up: markers, in-tree builds, GPU fixtures.

`-m "not gpu"` tests run anywhere (no GPU); `-m gpu` tests need a B200 and call the CUDA library
through its C-ABI. The product library and the CPU oracle are built in place when missing
(nvcc cross-compiles sm_100a without a GPU), so a fresh checkout can run the CPU suite directly.
"""
from __future__ import annotations

import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 GPU (sm_100a)")
    config.addinivalue_line("markers", "slow: full-size workloads")


def _ensure_built():
    from grouped_gemm_gpu_kernel_b200 import build as gbuild

    if not os.path.exists(gbuild.LIB_PATH):
        gbuild.build()
    if not os.path.exists(os.path.join(REPO, "oracle", "liboracle.so")):
        import subprocess

        subprocess.run(["make", "-C", os.path.join(REPO, "oracle"), "oracle"], check=True, capture_output=True)


_ensure_built()


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.init()
    return torch.device("cuda:0")
