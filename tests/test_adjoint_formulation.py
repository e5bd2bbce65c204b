"""The backward recipe the CUDA path uses, written out in float64 with explicit DFTs, equals the
reference's autograd (golden gradients) — the math of the backward, checked without a GPU.

Recipe (include/nop_spectral.h, backward section):
  dL/dx    = forward of the adjoint geometry on dL/dy with the conjugate-transposed weights
  dL/dW    = d_t * sum_b conj(Xh) * Gh   (Xh: kept spectrum of x, Gh: of dL/dy under the adjoint geometry)
  dL/dbias = Re(DC mode of Gh) / (adjoint fwd_scale), summed over the batch
and the package's host logic (adjoint_geometry, adjoint_operands, the chain rule from the dense weight
gradient to the weight's parameters) is what runs here.
"""

import os

import pytest
import torch

import neuraloperator_b200 as nb
from neuraloperator_b200 import ops
from neuraloperator_b200.geometry import adjoint_geometry
from neuraloperator_b200.spectral_convolution import _cp_full, _tucker_full
from oracle import dft_formulation as dft
from conftest import GOLDEN, rel_l2
from helpers import build_spectral_conv

GRAD = torch.load(os.path.join(GOLDEN, "grad_cases.pt"), weights_only=False)
LAYERS = GRAD["layers"]
TOL = 1e-5


def _dense(kind, ws):
    if kind == "dense":
        return ws[0]
    return _tucker_full(ws[0], ws[1:]) if kind == "tucker" else _cp_full(ws[0], ws[1:])


def _geo_args(g):
    return dict(n_in=g.n_in, n_out=g.n_out, kept=g.kept, fwd_off=g.fwd_off, inv_off=g.inv_off,
                fwd_scale=g.fwd_scale, inv_scale=g.inv_scale, complex_data=g.complex_data,
                zero_imag_bins=g.zero_imag_bins)


def _param_grads(conv):
    w = conv.weight
    if hasattr(w, "tensor"):
        return w.tensor.grad
    if hasattr(w, "core"):
        return {"core": w.core.grad, "factors": [f.grad for f in w.factors]}
    if hasattr(w, "weights"):
        return {"weights": w.weights.grad, "factors": [f.grad for f in w.factors]}
    return {"factors": [f.grad for f in w.factors]}


def _walk(a, b, path="weight"):
    if isinstance(b, torch.Tensor):
        yield path, a, b
    elif isinstance(b, dict):
        for k in b:
            yield from _walk(a[k], b[k], f"{path}/{k}")
    else:
        for i, (x, y) in enumerate(zip(a, b)):
            yield from _walk(x, y, f"{path}[{i}]")


@pytest.mark.parametrize("case", LAYERS, ids=[c["name"] for c in LAYERS])
def test_backward_recipe_matches_reference(case):
    conv = build_spectral_conv(case, device="cpu")
    x, gy = case["x"], case["grad_y"]
    geo = conv.geometry(list(x.shape[2:]))
    adj = adjoint_geometry(geo)
    kind, ws, ranks = conv.kernel_operands(geo)
    sep = conv.separable

    # dL/dx: the adjoint forward with the package's adjoint operands (reconstructed to dense here)
    adj_ws, _ = ops.adjoint_operands(kind, [w.detach() for w in ws], ranks, sep)
    w_adj = _dense(kind, adj_ws) if kind != "dense" else adj_ws[0]
    gx = dft.spectral_conv_direct(gy, w_adj, None, separable=sep, **_geo_args(adj))
    assert rel_l2(gx.to(case["grad_x"].dtype), case["grad_x"]) <= TOL

    # dL/dW of the sliced dense weight, then the chain rule to the parameters as the package does it
    xs = dft.forward_spectrum(x, geo.n_in, geo.kept, geo.fwd_off, geo.fwd_scale, geo.complex_data)
    gs = dft.forward_spectrum(gy, adj.n_in, adj.kept, adj.fwd_off, adj.fwd_scale, adj.complex_data)
    gw = dft.weight_grad_direct(xs, gs, geo.kept, geo.n_out, geo.complex_data, sep).to(torch.complex64)
    torch.autograd.backward(_dense(kind, ws), gw)
    for path, g, ref in _walk(_param_grads(conv), case["grad_weight"]):
        assert g is not None, path
        assert rel_l2(g, ref) <= TOL, path

    # dL/dbias from the DC mode of the adjoint spectrum
    if case["bias"] is not None:
        dc = tuple(adj.fwd_off)
        gb = gs[(slice(None), slice(None)) + dc].real.sum(0) / adj.fwd_scale
        assert rel_l2(gb.to(torch.float32), case["grad_bias"].reshape(-1)) <= TOL


@pytest.mark.parametrize("shape, ranks", [((16, 16, 12, 9), (6, 5, 4, 3)), ((5, 6, 7), (2, 3, 4)), ((4, 9), (3, 5))])
def test_tucker_grads_equal_autograd_of_reconstruction(shape, ranks):
    """The direct Tucker factor gradients (shared half-mode projections) equal torch autograd through
    the reconstructed weight, the route the reference's TFNO backward takes."""
    from neuraloperator_b200.spectral_convolution import _tucker_grads
    g = torch.Generator().manual_seed(len(shape))
    c = lambda *s: torch.complex(torch.randn(s, generator=g, dtype=torch.float64),
                                 torch.randn(s, generator=g, dtype=torch.float64))
    core, facs, gw = c(*ranks), [c(n, r) for n, r in zip(shape, ranks)], c(*shape)
    leaves = [core.clone().requires_grad_()] + [f.clone().requires_grad_() for f in facs]
    ref = torch.autograd.grad(_tucker_full(leaves[0], leaves[1:]), leaves, gw)
    for a, b in zip(_tucker_grads(core, facs, gw), ref):
        assert rel_l2(a, b) <= 1e-12
