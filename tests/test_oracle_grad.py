"""The CPU oracle's backward reproduces the reference's gradients (golden vectors) — pins the oracle
for the backward of SpectralConv / FNO / TFNO.

The reference trains through torch autograd of its forward (neuralop/training/trainer.py:629-700 calls
``loss.backward()``); the oracle's backward is torch autograd of its restated forward, so the two must
agree to float32 rounding.  ``tests/golden/grad_cases.pt`` holds, per case, x, the weights, a seeded
dL/dy and the reference's dL/dx, dL/dW (per weight factor) and dL/dbias.
"""

import os

import pytest
import torch

import oracle
from conftest import GOLDEN, rel_l2
from test_oracle_golden import fno_cfg, run_oracle_case

TOL = 1e-5

GRAD = torch.load(os.path.join(GOLDEN, "grad_cases.pt"), weights_only=False)
LAYERS = GRAD["layers"]
MODELS = GRAD["models"]


def leaves(obj):
    """Deep copy of a payload (tensors / lists / tuples / dicts) with every tensor a grad-requiring leaf."""
    if isinstance(obj, torch.Tensor):
        return obj.detach().clone().requires_grad_(True)
    if isinstance(obj, dict):
        return {k: leaves(v) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        return type(obj)(leaves(v) for v in obj)
    return obj


def pairs(ours, ref, path=""):
    """(path, our leaf's grad, reference grad) for every tensor of matching payload structures."""
    if isinstance(ref, torch.Tensor):
        yield path, ours.grad, ref
    elif isinstance(ref, dict):
        for k in ref:
            yield from pairs(ours[k], ref[k], f"{path}/{k}")
    elif isinstance(ref, (list, tuple)):
        for i, (a, b) in enumerate(zip(ours, ref)):
            yield from pairs(a, b, f"{path}[{i}]")


@pytest.mark.parametrize("case", LAYERS, ids=[c["name"] for c in LAYERS])
def test_spectral_conv_grads_match_reference(case):
    c = dict(case)
    c["x"] = case["x"].clone().requires_grad_(True)
    c["weight"] = leaves(case["weight"])
    c["bias"] = None if case["bias"] is None else case["bias"].clone().requires_grad_(True)
    y = run_oracle_case(c)
    y.backward(case["grad_y"])
    assert rel_l2(c["x"].grad, case["grad_x"]) <= TOL
    for path, g, ref in pairs(c["weight"], case["grad_weight"], "weight"):
        assert g is not None and g.shape == ref.shape, path
        assert rel_l2(g, ref) <= TOL, path
    if case["bias"] is not None:
        assert rel_l2(c["bias"].grad, case["grad_bias"]) <= TOL


@pytest.mark.parametrize("case", MODELS, ids=[m["name"] for m in MODELS])
def test_model_grads_match_reference(case):
    params = leaves(case["params"])
    x = case["x"].clone().requires_grad_(True)
    y = oracle.fno_forward(x, params, fno_cfg(case))
    y.backward(case["grad_y"])
    assert rel_l2(x.grad, case["grad_x"]) <= TOL
    n = 0
    for path, g, ref in pairs(params, case["grads"]):
        if ref is None:
            continue
        assert g is not None, path
        assert rel_l2(g, ref) <= TOL, path
        n += 1
    assert n > 0
    # the reference's own model test: every parameter receives a gradient
    assert case["n_params_with_grad"] == case["n_params"]
