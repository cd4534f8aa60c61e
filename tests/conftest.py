import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


def golden(name):
    return torch.load(os.path.join(GOLDEN, name), weights_only=True)


def rel_err(a, b):
    """max |a - b| / max |b| (0 when both are empty)."""
    a = a.detach().to(torch.float64).cpu()
    b = b.detach().to(torch.float64).cpu()
    if b.numel() == 0 and a.numel() == 0:
        return 0.0
    den = b.abs().max().clamp_min(1e-30)
    return float((a - b).abs().max() / den)


@pytest.fixture(scope="session")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
