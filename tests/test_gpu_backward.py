"""Backward of the spectral block through the CUDA kernels.

* Golden cases (``tests/golden/grad_cases.pt``): dL/dx, dL/dW (per weight factor) and dL/dbias of
  SpectralConv layers, and every parameter gradient of small FNO / TFNO models, equal the reference's
  autograd (rel-L2 <= 1e-5 in fp32, <= 2e-2 with the bf16 contraction).
* Benchmark-size layers (the five configurations' grids and modes at full batch where memory allows):
  size-independent identities of a linear map and its adjoint, accumulated in float64:
    <y(x) - bias, g> = <x, dL/dx>                         (input gradient is the adjoint)
    <y_{W = dW}(x), g> = Re <dL/dW, dW>                   (y is linear in each weight operand)
    dL/dbias = sum of g over batch and space
"""

import os

import pytest
import torch

import neuraloperator_b200 as nb
from neuraloperator_b200 import _lib
from conftest import GOLDEN, rel_l2
from helpers import build_fno, build_spectral_conv

pytestmark = pytest.mark.gpu

GRAD = torch.load(os.path.join(GOLDEN, "grad_cases.pt"), weights_only=False)
LAYERS = GRAD["layers"]
MODELS = GRAD["models"]
TOL = 1e-5
TOL_BF16 = 2e-2


def _param_grads(conv):
    w = conv.weight
    if hasattr(w, "tensor"):
        return w.tensor.grad
    if hasattr(w, "core"):
        return {"core": w.core.grad, "factors": [f.grad for f in w.factors]}
    if hasattr(w, "weights"):
        return {"weights": w.weights.grad, "factors": [f.grad for f in w.factors]}
    return {"factors": [f.grad for f in w.factors]}


def _walk(a, b, path=""):
    if isinstance(b, torch.Tensor):
        yield path, a, b
    elif isinstance(b, dict):
        for k in b:
            yield from _walk(a[k], b[k], f"{path}/{k}")
    elif isinstance(b, (list, tuple)):
        for i, (x, y) in enumerate(zip(a, b)):
            yield from _walk(x, y, f"{path}[{i}]")


def _check_layer(case, tol, **extra):
    conv = build_spectral_conv(case, **extra)
    x = case["x"].cuda().requires_grad_(True)
    y = conv(x)
    y.backward(case["grad_y"].cuda())
    torch.cuda.synchronize()
    assert rel_l2(x.grad.cpu(), case["grad_x"]) <= tol
    for path, g, ref in _walk(_param_grads(conv), case["grad_weight"], "weight"):
        assert g is not None, path
        assert rel_l2(g.cpu(), ref) <= tol, path
    if case["bias"] is not None:
        assert rel_l2(conv.bias.grad.cpu(), case["grad_bias"]) <= tol
    assert _lib.device_status() == 0


@pytest.mark.parametrize("engine", ["auto", "generic"])
@pytest.mark.parametrize("case", LAYERS, ids=[c["name"] for c in LAYERS])
def test_layer_grads_match_reference(case, engine):
    _check_layer(case, TOL, engine=engine)


@pytest.mark.parametrize("case", [c for c in LAYERS if c["name"].startswith("g_fast")],
                         ids=[c["name"] for c in LAYERS if c["name"].startswith("g_fast")])
def test_layer_grads_bf16_contraction(case):
    _check_layer(case, TOL_BF16, contraction_precision="bf16")


def _model_grads(model):
    def lin(fcs):
        return [(fc.weight.grad, fc.bias.grad) for fc in fcs]
    fb = model.fno_blocks
    blocks = []
    for i in range(fb.n_layers):
        sk = fb.fno_skips[i]
        blocks.append({"weight": _param_grads(fb.convs[i]), "bias": fb.convs[i].bias.grad,
                       "fno_skip": (sk.conv.weight if hasattr(sk, "conv") else sk.weight).grad,
                       "mlp": lin(fb.channel_mlp[i].fcs), "mlp_skip": fb.channel_mlp_skips[i].weight.grad})
    return {"lifting": lin(model.lifting.fcs), "projection": lin(model.projection.fcs), "blocks": blocks}


@pytest.fixture
def fp32_torch_layers():
    """The training path runs the per-pixel layers as torch Conv1d, which cuDNN computes in TF32 by
    default; these tests check the spectral kernels' precision, so torch's layers run in fp32 here."""
    saved = torch.backends.cudnn.allow_tf32, torch.backends.cuda.matmul.allow_tf32
    torch.backends.cudnn.allow_tf32 = torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cudnn.allow_tf32, torch.backends.cuda.matmul.allow_tf32 = saved


@pytest.mark.parametrize("case", MODELS, ids=[m["name"] for m in MODELS])
def test_model_grads_match_reference(case, fp32_torch_layers):
    model = build_fno(case)
    x = case["x"].cuda().requires_grad_(True)
    y = model(x)
    assert y.grad_fn is not None
    y.backward(case["grad_y"].cuda())
    torch.cuda.synchronize()
    assert rel_l2(x.grad.cpu(), case["grad_x"]) <= TOL
    n = 0
    for path, g, ref in _walk(_model_grads(model), case["grads"]):
        assert g is not None, path
        assert rel_l2(g.cpu(), ref) <= TOL, path
        n += 1
    assert n > 0
    # the reference's model test: every parameter receives a gradient
    assert all(p.grad is not None for p in model.parameters())
    assert _lib.device_status() == 0


def _dot(a, b):
    """Re <a, b> accumulated in float64 (complex: Re sum conj(a) b)."""
    if a.is_complex():
        return (a.conj().to(torch.complex128) * b.to(torch.complex128)).real.sum().item()
    return (a.double() * b.double()).sum().item()


def _weight_operands(conv):
    w = conv.weight
    if hasattr(w, "tensor"):
        return [w.tensor]
    if hasattr(w, "core"):
        return [w.core, w.factors[0]]
    return [w.factors[0]]


CONFIGS = [
    # (name, batch, channels, n_modes, grid, kwargs)
    ("c1_darcy_128", 16, 32, (16, 16), (128, 128), {}),
    ("c2_micro_256", 64, 64, (64, 64), (256, 256), {}),
    ("c3_burgers_8192", 256, 64, (16,), (8192,), {}),
    ("c4_tfno_512", 8, 64, (64, 64), (512, 512), dict(factorization="tucker", implementation="factorized",
                                                        rank=0.1)),
    ("c5_fno3d_256", 1, 32, (32, 32, 32), (256, 256, 256), {}),
]


@pytest.mark.parametrize("cfg", CONFIGS, ids=[c[0] for c in CONFIGS])
def test_adjoint_identities_at_config_sizes(cfg):
    name, batch, ch, modes, grid, kw = cfg
    torch.manual_seed(0)
    conv = nb.SpectralConv(ch, ch, modes, **kw).cuda()
    x = torch.randn(batch, ch, *grid, device="cuda", requires_grad=True)
    y = conv(x)
    g = torch.randn_like(y)
    y.backward(g)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    bias = conv.bias.detach()
    # input gradient: <y - bias, g> = <x, gx>
    lhs = _dot(y.detach() - bias, g)
    rhs = _dot(x.detach(), x.grad)
    assert abs(lhs - rhs) <= 1e-5 * max(abs(lhs), 1.0) * 10, (lhs, rhs)
    # bias gradient
    gb_ref = g.double().sum(dim=[0] + list(range(2, g.ndim))).reshape(bias.shape)
    assert rel_l2(conv.bias.grad.double().cpu(), gb_ref.cpu()) <= TOL
    # each weight operand: y is linear in it (bias excluded)
    for p in _weight_operands(conv):
        grad = p.grad.detach().clone()
        dp = torch.randn_like(p) * p.detach().abs().mean()
        saved = p.detach().clone()
        with torch.no_grad():
            y0 = conv(x.detach())
            p.copy_(saved + dp)
            y1 = conv(x.detach())
            p.copy_(saved)
        lhs = _dot(y1 - y0, g)
        rhs = _dot(grad, dp)
        assert abs(lhs - rhs) <= 1e-4 * max(abs(lhs), abs(rhs), 1e-3), (name, lhs, rhs)
        del y0, y1
    assert _lib.device_status() == 0


def test_backward_of_resampling_call_raises():
    conv = nb.SpectralConv(2, 2, (4, 4), resolution_scaling_factor=2).cuda()
    x = torch.randn(1, 2, 8, 8, device="cuda", requires_grad=True)
    with pytest.raises(NotImplementedError):
        conv(x)
    with torch.no_grad():
        assert conv(x).shape == (1, 2, 16, 16)


def test_no_graph_without_grad():
    conv = nb.SpectralConv(2, 2, (4, 4)).cuda()
    x = torch.randn(1, 2, 8, 8, device="cuda")
    with torch.no_grad():
        y = conv(x)
    assert y.grad_fn is None
    conv.requires_grad_(False)
    assert conv(x).grad_fn is None


@pytest.mark.parametrize("batch, ci, co, modes", [
    (64, 64, 64, (64, 64)),   # the C2 layer's weight gradient (one input / output tile, aligned stores)
    (40, 80, 48, (62, 61)),   # two input tiles, a partial output tile, batch not a multiple of 8,
                              # Mt = 62 * 31 not a multiple of 4 (per-mode stores)
])
def test_tensor_core_weight_grad_matches_cuda_cores(batch, ci, co, modes, monkeypatch):
    """dL/dW from the tcgen05 kernel equals the CUDA-core kernel's (NOP_CONTRACTION=simt) on shapes that
    select it (batch >= 32, a tile per SM)."""
    from neuraloperator_b200 import ops
    torch.manual_seed(1)
    x = torch.randn(batch, ci, 256, 256, device="cuda")
    g = torch.randn(batch, co, 256, 256, device="cuda")
    grads = {}
    for mode in ("simt", "tc"):
        if mode == "simt":
            monkeypatch.setenv("NOP_CONTRACTION", "simt")
        else:
            monkeypatch.delenv("NOP_CONTRACTION", raising=False)
        ops.clear_plans()
        torch.manual_seed(2)
        conv = nb.SpectralConv(ci, co, modes).cuda()
        y = conv(x)
        (gw,) = torch.autograd.grad(y, [conv.weight.tensor], g)
        grads[mode] = gw
    ops.clear_plans()
    assert rel_l2(grads["tc"].cpu(), grads["simt"].cpu()) <= 1e-5
    assert _lib.device_status() == 0
