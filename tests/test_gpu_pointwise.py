"""The fused per-pixel channel-MLP kernel (nop_pointwise_forward) against the reference modules.

Reference: the same layers composed from torch ops in float64 on the CPU -- Conv1d(k=1) layers with
exact GELU (neuralop/layers/channel_mlp.py:82-119), soft-gating (skip_connections.py:53-94), the
linear skip (skip_connections.py:96-127), grid channels as GridEmbeddingND
(embeddings.py:147-164).  Tolerance: relative L2 <= 1e-5 (fp32 kernel).  The full FNO / TFNO
models, which run these kernels for lifting, blocks and projection, are checked against the
reference's golden outputs in test_gpu_parity.py.
"""

import pytest
import torch
import torch.nn.functional as F

from conftest import rel_l2
from neuraloperator_b200 import _lib, pointwise

pytestmark = pytest.mark.gpu

TOL = 1e-5


@pytest.fixture(autouse=True, scope="module")
def _needs_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _grid(spatial, bounds):
    axes = [torch.linspace(lo, hi, n + 1, dtype=torch.float64)[:-1] for n, (lo, hi) in zip(spatial, bounds)]
    return torch.meshgrid(*axes, indexing="ij")


def _reference(x, w1, b1, w2, b2, grid=None, act_hidden=True, act_out=False, r=None, g=None, gb=None, w3=None):
    x = x.double()
    if grid is not None:
        gs = [t.expand(x.shape[0], 1, *t.shape) for t in (a.unsqueeze(0) for a in _grid(x.shape[2:], grid))]
        x = torch.cat((x, *[t.reshape(x.shape[0], 1, *x.shape[2:]) for t in gs]), dim=1)
    flat = x.reshape(x.shape[0], x.shape[1], -1)

    def lin(v, w, b):
        out = torch.einsum("oi,bip->bop", w.double(), v)
        return out if b is None else out + b.double()[None, :, None]

    h = flat
    if w1 is not None:
        h = lin(flat, w1, b1)
        if act_hidden:
            h = F.gelu(h)
    y = lin(h, w2, b2)
    if r is not None:
        y = y + g.double()[None, :, None] * r.double().reshape(y.shape)
        if gb is not None:
            y = y + gb.double()[None, :, None]
    if act_out:
        y = F.gelu(y)
    z = None if w3 is None else lin(y, w3, None)
    shape = lambda t: t.reshape(t.shape[0], t.shape[1], *x.shape[2:])  # noqa: E731
    return shape(y), (None if z is None else shape(z))


CASES = [
    # name, batch, spatial, cin, hidden, cout, cnext, grid, gate, gate_bias, act_out
    ("block_mlp_2d", 3, (32, 64), 64, 32, 64, 64, None, True, False, True),
    ("block_last_2d", 2, (64, 32), 32, 16, 32, 0, None, True, False, False),
    ("lifting_grid_2d", 2, (128, 128), 1, 64, 32, 32, ((0.0, 1.0), (0.0, 1.0)), False, False, False),
    ("lifting_grid_1d", 4, (8192,), 1, 128, 64, 64, ((0.0, 1.0),), False, False, False),
    ("lifting_grid_3d", 1, (32, 32, 32), 3, 64, 32, 32, ((0.0, 1.0),) * 3, False, False, False),
    ("projection", 2, (64, 64), 64, 128, 1, 0, None, False, False, False),
    ("odd_channels_gate_bias", 3, (384,), 7, 5, 9, 11, None, True, True, True),
    ("single_layer_skip", 2, (32, 32), 48, 0, 48, 0, None, False, False, False),
]


@pytest.fixture(params=["cuda_cores", "tensor_cores"])
def engine(request, monkeypatch):
    """Both per-pixel kernels: the CUDA-core one (default) and tcgen05 (NOP_POINTWISE=tc)."""
    if request.param == "tensor_cores":
        monkeypatch.setenv("NOP_POINTWISE", "tc")
    else:
        monkeypatch.delenv("NOP_POINTWISE", raising=False)
    return request.param


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_fused_channel_mlp_matches_reference(case, engine):
    name, batch, spatial, cin, hidden, cout, cnext, grid, gate, gate_bias, act_out = case
    g = torch.Generator().manual_seed(3)
    ku = cin + (len(spatial) if grid is not None else 0)
    rnd = lambda *s: torch.randn(*s, generator=g)  # noqa: E731
    x = rnd(batch, cin, *spatial)
    w1 = rnd(hidden, ku, 1) / ku ** 0.5 if hidden else None
    b1 = rnd(hidden) * 0.1 if hidden else None
    kin = hidden if hidden else ku
    w2 = rnd(cout, kin, 1) / kin ** 0.5
    b2 = rnd(cout) * 0.1 if name != "single_layer_skip" else None
    r = rnd(batch, cout, *spatial) if gate else None
    gw = rnd(1, cout, *(1,) * len(spatial)) if gate else None
    gbv = rnd(1, cout, *(1,) * len(spatial)) if gate_bias else None
    w3 = rnd(cnext, cout, 1) / cout ** 0.5 if cnext else None
    assert pointwise.supported(x.cuda(), cin, hidden, cout, cnext, grid)
    dev = lambda t: None if t is None else t.cuda()  # noqa: E731
    y, z = pointwise.channel_mlp(dev(x), dev(w1), dev(b1), dev(w2), dev(b2), grid=grid, act_hidden=True,
                                 act_out=act_out, residual=dev(r), gate_w=dev(gw), gate_b=dev(gbv), next_w=dev(w3))
    torch.cuda.synchronize()
    y_ref, z_ref = _reference(x, None if w1 is None else w1[..., 0], b1, w2[..., 0], b2, grid=grid,
                              act_out=act_out, r=r, g=None if gw is None else gw.reshape(-1),
                              gb=None if gbv is None else gbv.reshape(-1), w3=None if w3 is None else w3[..., 0])
    assert y.shape == y_ref.shape
    assert rel_l2(y.cpu(), y_ref) <= TOL
    if cnext:
        assert rel_l2(z.cpu(), z_ref) <= TOL
    from neuraloperator_b200 import _lib
    assert _lib.device_status() == 0


def test_fused_fno_matches_module_path(monkeypatch):
    """FNO forward with the fused lifting / blocks / projection equals the module path (torch
    Conv1d layers in fp32, TF32 off) on the same weights, at the Darcy configuration's size."""
    import neuraloperator_b200 as nb
    old = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    try:
        torch.manual_seed(0)
        model = nb.FNO(n_modes=(16, 16), in_channels=1, out_channels=1, hidden_channels=32, n_layers=4).cuda()
        x = torch.randn(4, 1, 128, 128, device="cuda")
        with torch.no_grad():
            y_fused = model(x)
            monkeypatch.setattr(pointwise, "supported_dims", lambda *a, **k: False)
            y_modules = model(x)
        assert rel_l2(y_fused, y_modules) <= TOL
    finally:
        torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = old
