"""The per-mode contraction on the tcgen05 tensor cores against the CUDA-core kernel and the oracle.

The fused engine runs its contraction on the tensor cores (three-pass tf32 for fp32, kind::f16 for
the bf16 contraction).  NOP_CONTRACTION=simt (read at plan creation) selects the CUDA-core kernel,
which computes the same sums in plain fp32 FMAs; the two must agree to fp32 rounding
(relative L2 <= 2e-6) on shapes that exercise every tile edge: batch not a multiple of 64, channel
counts not multiples of 8 / 32 / 64, more than one output tile, factorized weights, 1D / 2D / 3D.
The tensor-core kernel loads its operands and stores its results with tensor copies (TMA), its
weights pre-split into tf32 hi / lo tiles when they are packed; NOP_MIX_TMA=0 (read at plan creation)
selects its per-thread-gather twin on the float4 packing, which must give bit-identical results (the
same MMAs on the same operands in the same order).
Every run must leave the device status word at 0 (no bounded wait expired).
"""

import os

import pytest
import torch

import neuraloperator_b200 as nb
import oracle
from conftest import rel_l2
from neuraloperator_b200 import _lib, ops

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True, scope="module")
def _needs_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _forward(conv, x, simt):
    old = os.environ.get("NOP_CONTRACTION")
    try:
        if simt:
            os.environ["NOP_CONTRACTION"] = "simt"
        else:
            os.environ.pop("NOP_CONTRACTION", None)
        ops.clear_plans()
        conv.__dict__.pop("_nop_pack_cache", None)
        with torch.no_grad():
            y = conv(x)
        torch.cuda.synchronize()
        return y
    finally:
        if old is None:
            os.environ.pop("NOP_CONTRACTION", None)
        else:
            os.environ["NOP_CONTRACTION"] = old
        ops.clear_plans()


CASES = [
    # (batch, ci, co, grid, modes, kwargs)
    (2, 4, 4, (128, 128), (16, 16), {}),
    (70, 40, 72, (128, 128), (32, 32), {}),
    (3, 3, 5, (128, 128), (20, 12), {}),
    (65, 64, 64, (256, 256), (64, 64), {}),
    (16, 33, 31, (128, 128), (16, 16), {}),
    (16, 64, 96, (8192,), (16,), {}),
    (2, 32, 32, (256, 256, 256), (32, 32, 32), {}),
    (8, 16, 24, (128, 128), (32, 32), dict(factorization="tucker", rank=0.5)),
    (8, 64, 64, (256, 256), (64, 64), dict(contraction_precision="bf16")),
    (5, 20, 36, (128, 128), (16, 16), dict(contraction_precision="bf16")),
]


@pytest.mark.parametrize("case", CASES, ids=[f"B{c[0]}_ci{c[1]}_co{c[2]}_{len(c[3])}d_{'_'.join(c[5])}" for c in CASES])
def test_tensor_core_contraction_matches_cuda_core_kernel(case):
    batch, ci, co, grid, modes, kw = case
    torch.manual_seed(0)
    conv = nb.SpectralConv(ci, co, modes, **kw).cuda()
    if "factorization" not in kw:
        with torch.no_grad():
            w = conv.weight.tensor
            w.copy_(torch.complex(torch.randn_like(w.real), torch.randn_like(w.real)) * 0.1)
    x = torch.randn((batch, ci, *grid), device="cuda")
    _lib.device_status(clear=True)
    y_tc = _forward(conv, x, simt=False)
    assert _lib.device_status(clear=True) == 0
    y_simt = _forward(conv, x, simt=True)
    assert rel_l2(y_tc, y_simt) <= 2e-6


def test_tensor_core_contraction_against_oracle_fp32():
    torch.manual_seed(1)
    conv = nb.SpectralConv(24, 40, (24, 24)).cuda()
    with torch.no_grad():
        w = conv.weight.tensor
        w.copy_(torch.complex(torch.randn_like(w.real), torch.randn_like(w.real)) * 0.1)
    x = torch.randn((9, 24, 128, 128))
    y = _forward(conv, x.cuda(), simt=False).cpu()
    ref = oracle.spectral_conv(x, conv.weight.tensor.detach().cpu(), conv.bias.detach().cpu(), (24, 24))
    assert rel_l2(y, ref) <= 1e-5
    assert _lib.device_status(clear=True) == 0


def _forward_tma(conv, x, tma):
    old = os.environ.get("NOP_MIX_TMA")
    try:
        if tma:
            os.environ.pop("NOP_MIX_TMA", None)
        else:
            os.environ["NOP_MIX_TMA"] = "0"
        ops.clear_plans()
        conv.__dict__.pop("_nop_pack_cache", None)
        with torch.no_grad():
            y = conv(x)
        torch.cuda.synchronize()
        return y
    finally:
        if old is None:
            os.environ.pop("NOP_MIX_TMA", None)
        else:
            os.environ["NOP_MIX_TMA"] = old
        ops.clear_plans()


@pytest.mark.parametrize("case", CASES, ids=[f"B{c[0]}_ci{c[1]}_co{c[2]}_{len(c[3])}d_{'_'.join(c[5])}" for c in CASES])
def test_tma_contraction_bit_identical_to_gather_kernel(case):
    batch, ci, co, grid, modes, kw = case
    torch.manual_seed(0)
    conv = nb.SpectralConv(ci, co, modes, **kw).cuda()
    x = torch.randn((batch, ci, *grid), device="cuda")
    _lib.device_status(clear=True)
    y_tma = _forward_tma(conv, x, tma=True)
    y_gather = _forward_tma(conv, x, tma=False)
    assert _lib.device_status(clear=True) == 0
    assert torch.equal(y_tma, y_gather)
