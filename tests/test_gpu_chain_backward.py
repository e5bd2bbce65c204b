"""Backward of the per-pixel chain (nop_chain_backward) against autograd of the reference modules.

Reference: the same layers composed from torch ops in float64 on the CPU (test_gpu_pointwise._reference:
the linear skip, ChannelMLP with exact GELU, SoftGating, GridEmbeddingND's channels), differentiated by
torch autograd -- what the reference's trainer (neuralop/training/trainer.py:629-700) gets from
loss.backward().  Tolerance: relative L2 <= 2e-5 per gradient (fp32 arithmetic; the weight gradients
sum over up to 10^5 points).  The FNO-level test checks a whole training step through the fused path
against the module path (torch Conv1d layers, TF32 off) on the same weights.
"""

import pytest
import torch

from conftest import rel_l2
from neuraloperator_b200 import _lib, pointwise
from test_gpu_pointwise import CASES, _operands, _reference

pytestmark = pytest.mark.gpu

TOL = 2e-5
NAMES = ("x", "s", "w0", "w1", "b1", "w2", "b2", "gate_w", "gate_b")


@pytest.fixture(autouse=True, scope="module")
def _needs_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


BWD_CASES = [c for c in CASES if c[11] is None]  # the backward takes chains without the projection


def _reference_grads(case, ops, dy):
    name, batch, spatial, cx, hidden, cy, skip, grid, gate, gate_bias, acts, proj = case
    leaves = {k: v.double().requires_grad_() for k, v in ops.items()}
    mat = lambda t: None if t is None else t.reshape(t.shape[0], -1)  # noqa: E731
    vec = lambda t: None if t is None else t.reshape(-1)  # noqa: E731
    y = _reference(leaves["x"], mat(leaves["w1"]), leaves["b1"], mat(leaves["w2"]), leaves["b2"], s=leaves.get("s"),
                   w0=mat(leaves.get("w0")), act_skip=acts, act_out=acts, g=vec(leaves.get("gate_w")),
                   gb=vec(leaves.get("gate_b")), grid=grid)
    y.backward(dy.double())
    return {k: v.grad for k, v in leaves.items()}


@pytest.mark.parametrize("case", BWD_CASES, ids=[c[0] for c in BWD_CASES])
def test_chain_backward_matches_autograd(case):
    ops = _operands(case, seed=5)
    name, batch, spatial, cx, hidden, cy, skip, grid, gate, gate_bias, acts, proj = case
    g = torch.Generator().manual_seed(6)
    dy = torch.randn(batch, cy, *spatial, generator=g)
    ref = _reference_grads(case, ops, dy)
    dev = {k: v.cuda().requires_grad_() for k, v in ops.items()}
    gp = pointwise.grid_params(grid, spatial) if grid is not None else None
    y = pointwise.chain(dev["x"], dev["w1"], dev["b1"], dev["w2"], dev["b2"], s=dev.get("s"), w0=dev.get("w0"),
                        act_skip=acts, act_out=acts, gate_w=dev.get("gate_w"), gate_b=dev.get("gate_b"), grid=gp)
    y.backward(dy.cuda())
    torch.cuda.synchronize()
    for k in dev:
        assert dev[k].grad is not None, k
        assert dev[k].grad.shape == ops[k].shape, k
        assert rel_l2(dev[k].grad.cpu().double(), ref[k]) <= TOL, (k, rel_l2(dev[k].grad.cpu().double(), ref[k]))
    assert _lib.device_status() == 0


def test_chain_backward_is_deterministic():
    """Two backward calls give bit-identical gradients (per-CTA sums added in a fixed order)."""
    case = CASES[1]  # block_h64_2d
    ops = {k: v.cuda() for k, v in _operands(case).items()}
    dy = torch.randn(case[1], case[5], *case[2], device="cuda")
    kw = dict(s=ops["s"], w0=ops["w0"], act_skip=True, act_out=True, gate_w=ops["gate_w"])
    a = pointwise.chain_backward(dy, ops["x"], ops["w1"], ops["b1"], ops["w2"], ops["b2"], **kw)
    b = pointwise.chain_backward(dy, ops["x"], ops["w1"], ops["b1"], ops["w2"], ops["b2"], **kw)
    torch.cuda.synchronize()
    for k in a:
        if a[k] is not None:
            assert torch.equal(a[k], b[k]), k


def test_fno_training_step_fused_matches_module_path(monkeypatch):
    """One FNO training step (loss.backward()) through the fused path -- chain kernels forward and
    backward, the spectral layers' own backward -- gives the module path's parameter gradients."""
    import neuraloperator_b200 as nb
    old = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    try:
        torch.manual_seed(0)
        model = nb.FNO(n_modes=(12, 12), in_channels=1, out_channels=1, hidden_channels=32, n_layers=4).cuda()
        x = torch.randn(3, 1, 64, 64, device="cuda", requires_grad=True)
        target = torch.randn(3, 1, 64, 64, device="cuda")

        def step():
            model.zero_grad(set_to_none=True)
            x.grad = None
            loss = ((model(x) - target) ** 2).mean()
            loss.backward()
            grads = {n: p.grad.clone() for n, p in model.named_parameters()}
            grads["input"] = x.grad.clone()  # through every block's two gradient paths of its input
            return loss.item(), grads

        assert model.fused_plan(x) is not None  # a gradient is recorded: the fused path must take it
        loss_f, g_f = step()
        monkeypatch.setattr(pointwise, "supported", lambda *a, **k: False)
        assert model.fused_plan(x) is None
        loss_m, g_m = step()
        assert abs(loss_f - loss_m) <= 1e-5 * abs(loss_m)
        for n in g_m:
            assert rel_l2(g_f[n], g_m[n]) <= 1e-4, (n, rel_l2(g_f[n], g_m[n]))
    finally:
        torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = old
