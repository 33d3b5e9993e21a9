"""Test configuration: the `gpu` marker, import paths, and shared helpers.

CPU tests (-m "not gpu") cover the oracle against the golden vectors, the host-side logic,
and that libkt_gguf_b200.so loads and exports its C ABI. GPU tests (-m gpu) are the parity
tests of the CUDA kernels against the oracle and need an sm_100 GPU.
"""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT, ROOT / "kt-prefill-lend_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("gpu test without a CUDA device")
    return torch.device("cuda", 0)
