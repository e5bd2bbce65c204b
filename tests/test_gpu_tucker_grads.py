"""Tucker factor gradients on the library's kernels (nop_tucker_grads) against torch autograd through the
float64 reconstruction of the weight (the route of the reference's TFNO backward through
_contract_tucker, neuralop/layers/spectral_convolution.py:76-103).

Tolerance: relative L2 <= 2e-5 per gradient (fp32 products with fp32 accumulation over up to 10^7 terms
against float64).  The C4 case is the TFNO Navier-Stokes layer's weight (64 x 64 channels, 64 x 33
kept modes, ranks of rank=0.1); the golden TFNO gradients in grad_cases.pt run through the same
kernels in test_gpu_backward.py.
"""

import pytest
import torch

import neuraloperator_b200 as nb
from neuraloperator_b200 import _lib, ops
from neuraloperator_b200.spectral_convolution import _tucker_full
from conftest import rel_l2

pytestmark = pytest.mark.gpu

TOL = 2e-5


@pytest.fixture(autouse=True, scope="module")
def _needs_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _autograd(core, facs, gw):
    leaves = [core.to(torch.complex128).requires_grad_()] + [f.to(torch.complex128).requires_grad_() for f in facs]
    return torch.autograd.grad(_tucker_full(leaves[0], leaves[1:]), leaves, gw.to(torch.complex128))


def _rand(g, *s):
    return torch.complex(torch.randn(s, generator=g), torch.randn(s, generator=g))


@pytest.mark.parametrize("shape, ranks", [((16, 16, 12, 9), (6, 5, 4, 3)), ((5, 6, 7), (2, 3, 4)), ((4, 9), (3, 5)),
                                          ((6, 5, 4, 3, 7, 5), (2, 2, 3, 3, 4, 1)), ((8, 300, 20), (40, 17, 33)),
                                          ((3, 4, 5, 6), (5, 6, 7, 8))],
                         ids=["4_modes", "3_modes", "2_modes", "6_modes", "long_mode_and_ranks_over_16",
                              "ranks_above_sizes"])
def test_tucker_grads_match_autograd(shape, ranks):
    g = torch.Generator().manual_seed(sum(shape))
    core, facs, gw = _rand(g, *ranks), [_rand(g, n, r) for n, r in zip(shape, ranks)], _rand(g, *shape)
    got = ops.tucker_grads(core.cuda(), [f.cuda() for f in facs], gw.cuda())
    torch.cuda.synchronize()
    for i, (a, b) in enumerate(zip(got, _autograd(core, facs, gw))):
        assert a.shape == b.shape, i
        assert rel_l2(a.cpu().to(torch.complex128), b) <= TOL, i


def test_tucker_grads_c4_layer_weight():
    """The C4 TFNO layer's own factor shapes; two calls agree bit for bit (fixed reduction order)."""
    torch.manual_seed(0)
    conv = nb.SpectralConv(64, 64, (64, 64), factorization="tucker", implementation="factorized", rank=0.1).cuda()
    geo = conv.geometry([512, 512])
    kind, ws, _ = conv.kernel_operands(geo)
    assert kind == "tucker"
    core, facs = ws[0].detach(), [u.detach() for u in ws[1:]]
    g = torch.Generator(device="cuda").manual_seed(1)
    shape = tuple(u.shape[0] for u in facs)
    gw = torch.complex(torch.randn(shape, generator=g, device="cuda"), torch.randn(shape, generator=g, device="cuda"))
    got = ops.tucker_grads(core, facs, gw)
    again = ops.tucker_grads(core, facs, gw)
    torch.cuda.synchronize()
    for a, b in zip(got, again):
        assert torch.equal(a, b)
    for i, (a, b) in enumerate(zip(got, _autograd(core.cpu(), [f.cpu() for f in facs], gw.cpu()))):
        assert rel_l2(a.cpu().to(torch.complex128), b) <= TOL, i
    assert _lib.device_status() == 0
