import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def rel_l2(a, b):
    """Relative L2 error ||a - b|| / ||b|| computed in float64."""
    import torch
    a = a.detach().to("cpu", torch.complex128 if (a.is_complex() or b.is_complex()) else torch.float64)
    b = b.detach().to("cpu", a.dtype)
    den = torch.linalg.vector_norm(b).item()
    num = torch.linalg.vector_norm(a - b).item()
    return num / den if den > 0 else num


@pytest.fixture(scope="session")
def golden():
    import torch
    def load(name):
        return torch.load(os.path.join(GOLDEN, name), weights_only=False)
    return load
