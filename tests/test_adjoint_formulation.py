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


def _mode_dot(t, u, k):
    """t x_k conj(u): mode k (size n) of t against u [n, r] (k_mode_dot of csrc/tucker_grad.cu)."""
    return torch.tensordot(t, u.conj(), dims=([k], [0])).movedim(-1, k)


def _mode_gram(t, c, k):
    """sum over every mode but k of t[.., x, ..] * c[.., a, ..] -> [x, a] (k_mode_gram)."""
    other = [j for j in range(t.ndim) if j != k]
    return torch.tensordot(t, c, dims=(other, other))


def tucker_grads_recipe(core, factors, gw):
    """float64 restatement of nop_tucker_grads' orchestration: gw projected on the right half of the
    modes (A_right) and on the left half (A_left), each half largest reduction first; the core gradient
    is A_right projected on the left half, factor k's gram takes the other modes of k's half projected
    from A_right (k left) or A_left (k right) against conj(core)."""
    n = len(factors)

    def proj(t, modes):
        for k in sorted(modes, key=lambda j: -(factors[j].shape[0] - factors[j].shape[1])):
            t = _mode_dot(t, factors[k], k)
        return t

    left, right = list(range(n // 2)), list(range(n // 2, n))
    a_right, a_left = proj(gw, right), proj(gw, left)
    g_fac = []
    for k in range(n):
        t = proj(a_right, [j for j in left if j != k]) if k in left else proj(a_left, [j for j in right if j != k])
        g_fac.append(_mode_gram(t, core.conj(), k))
    return [proj(a_right, left)] + g_fac


@pytest.mark.parametrize("shape, ranks", [((16, 16, 12, 9), (6, 5, 4, 3)), ((5, 6, 7), (2, 3, 4)), ((4, 9), (3, 5)),
                                          ((6, 5, 4, 3, 7), (2, 2, 3, 3, 4))])
def test_tucker_grads_equal_autograd_of_reconstruction(shape, ranks):
    """The Tucker factor-gradient recipe of the CUDA kernels (shared half-mode projections, then one
    gram per factor) equals torch autograd through the reconstructed weight, the route the reference's
    TFNO backward takes."""
    g = torch.Generator().manual_seed(len(shape))
    c = lambda *s: torch.complex(torch.randn(s, generator=g, dtype=torch.float64),
                                 torch.randn(s, generator=g, dtype=torch.float64))
    core, facs, gw = c(*ranks), [c(n, r) for n, r in zip(shape, ranks)], c(*shape)
    leaves = [core.clone().requires_grad_()] + [f.clone().requires_grad_() for f in facs]
    ref = torch.autograd.grad(_tucker_full(leaves[0], leaves[1:]), leaves, gw)
    for a, b in zip(tucker_grads_recipe(core, facs, gw), ref):
        assert rel_l2(a, b) <= 1e-12
