"""FNOStaged through the CUDA path: forward equals the reference's output on its own checkpoint, and a
training step reaches every parameter."""

import os

import pytest
import torch

import neuraloperator_b200 as nb
from neuraloperator_b200 import _lib
from conftest import GOLDEN, rel_l2

pytestmark = pytest.mark.gpu

CASES = torch.load(os.path.join(GOLDEN, "staged_cases.pt"), weights_only=False)


@pytest.fixture(autouse=True)
def _fp32_torch():
    saved = torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = torch.backends.cudnn.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = saved


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_fnostaged_forward_matches_reference(case):
    model = nb.FNOStaged(**case["kwargs"])
    model.load_state_dict(case["state_dict"])
    model = model.cuda()
    with torch.no_grad():
        y = model(case["x"].cuda())
    assert rel_l2(y.cpu(), case["y"]) <= 1e-5
    x = case["x"].cuda().requires_grad_(True)
    model(x).square().mean().backward()
    assert x.grad is not None and all(p.grad is not None for p in model.parameters())
    assert _lib.device_status() == 0
