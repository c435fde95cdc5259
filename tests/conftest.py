"""Shared pytest setup: the `gpu` marker and import paths.

`-m "not gpu"` runs on a CPU-only machine: the oracle against the golden
fixtures, the host logic and the C-ABI surface of libdial_cuda.so.
`-m gpu` runs the CUDA kernels through the C ABI and checks them against the
oracle (tests/ is the only place besides __graft_entry__.smoke() and the CPU
baseline leg of bench.py that imports the oracle).
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "dial-8b-orin_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (B200)")


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, _ = torch.cuda.get_device_capability(0)
    if major < 10:
        pytest.skip("needs sm_100")
    return torch.device("cuda:0")
