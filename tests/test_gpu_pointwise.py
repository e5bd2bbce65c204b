"""The per-pixel tensor-core chain kernel (nop_chain_forward) against the reference modules.

Reference: the same layers composed from torch ops in float64 on the CPU -- the linear skip
(skip_connections.py:96-127) added to a given spectral output, Conv1d(k=1) layers with exact GELU
(neuralop/layers/channel_mlp.py:82-119), soft-gating (skip_connections.py:53-94), grid channels as
GridEmbeddingND (embeddings.py:147-164) and the projection ChannelMLP (fno.py:404-406).  Tolerance:
relative L2 <= 1e-5 (fp32 results from three-pass tf32 MMAs).  The full FNO / TFNO models, which run
this kernel for lifting, blocks and projection, are checked against the reference's golden outputs in
test_gpu_parity.py and against the oracle at the configurations' own widths in test_gpu_configs.py.
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


def _lin(v, w, b=None):
    out = torch.einsum("oi,bip->bop", w.double(), v)
    return out if b is None else out + b.double()[None, :, None]


def _reference(x, w1, b1, w2, b2, *, s=None, w0=None, act_skip=False, act_out=False, g=None, gb=None,
               grid=None, w3=None, b3=None, w4=None, b4=None):
    """float64 restatement of the chain (the reference modules' arithmetic)."""
    batch, spatial = x.shape[0], x.shape[2:]
    xd = x.double()
    flat_x = xd.reshape(batch, x.shape[1], -1)
    if s is not None:
        u = _lin(flat_x, w0) + s.double().reshape(batch, s.shape[1], -1)
        if act_skip:
            u = F.gelu(u)
    else:
        u = flat_x
        if grid is not None:
            gs = [a.reshape(1, 1, -1).expand(batch, 1, -1) for a in _grid(spatial, grid)]
            u = torch.cat((u, *gs), dim=1)
    h = F.gelu(_lin(u, w1, b1))
    y = _lin(h, w2, b2)
    if g is not None:
        y = y + g.double()[None, :, None] * flat_x
        if gb is not None:
            y = y + gb.double()[None, :, None]
    if act_out:
        y = F.gelu(y)
    if w3 is not None:
        y = _lin(F.gelu(_lin(y, w3, b3)), w4, b4)
    return y.reshape(batch, y.shape[1], *spatial)


# name, batch, spatial, Cx, hidden, Cy, skip stage, grid, gate, gate bias, activations, (proj hidden, proj out)
CASES = [
    ("block_h32_3d", 2, (16, 16, 32), 32, 16, 32, True, None, True, False, True, None),
    ("block_h64_2d", 3, (32, 64), 64, 32, 64, True, None, True, False, True, None),
    ("last_block_h32", 2, (64, 32), 32, 16, 32, True, None, True, False, False, None),
    ("last_block_projection_h32_3d", 2, (16, 16, 16), 32, 16, 32, True, None, True, False, False, (64, 3)),
    ("last_block_projection_h64", 1, (64, 64), 64, 32, 64, True, None, True, False, False, (128, 1)),
    ("lifting_grid_2d", 2, (128, 128), 1, 64, 32, False, ((0.0, 1.0), (0.0, 1.0)), False, False, False, None),
    ("lifting_grid_1d", 4, (8192,), 1, 128, 64, False, ((0.0, 1.0),), False, False, False, None),
    ("lifting_grid_3d", 1, (32, 32, 32), 3, 64, 32, False, ((0.0, 1.0),) * 3, False, False, False, None),
    ("projection", 2, (64, 64), 64, 128, 1, False, None, False, False, False, None),
    ("odd_channels_gate_bias_partial_tile", 3, (3, 124), 7, 5, 7, True, None, True, True, True, None),
    ("no_gate", 2, (40, 36), 24, 40, 24, True, None, False, False, True, None),
    # lifting with a hidden width that is not a multiple of 16 (40 -> 48 columns), a partial last tile
    ("lifting_odd_partial_tile", 3, (3, 124), 2, 40, 24, False, ((0.0, 1.0), (-1.0, 1.0)), False, False, True, None),
]


def _operands(case, seed=3):
    name, batch, spatial, cx, hidden, cy, skip, grid, gate, gate_bias, acts, proj = case
    g = torch.Generator().manual_seed(seed)
    rnd = lambda *s: torch.randn(*s, generator=g)  # noqa: E731
    ku = cy if skip else cx + (len(spatial) if grid is not None else 0)
    ops = dict(x=rnd(batch, cx, *spatial), w1=rnd(hidden, ku, 1) / ku ** 0.5, b1=rnd(hidden) * 0.1,
               w2=rnd(cy, hidden, 1) / hidden ** 0.5, b2=rnd(cy) * 0.1)
    if skip:
        ops.update(s=rnd(batch, cy, *spatial), w0=rnd(cy, cx, 1) / cx ** 0.5)
    if gate:
        ops["gate_w"] = rnd(1, cy, *(1,) * len(spatial))
        if gate_bias:
            ops["gate_b"] = rnd(1, cy, *(1,) * len(spatial))
    if proj:
        ph, po = proj
        ops.update(w3=rnd(ph, cy, 1) / cy ** 0.5, b3=rnd(ph) * 0.1, w4=rnd(po, ph, 1) / ph ** 0.5, b4=rnd(po) * 0.1)
    return ops


def _run(case, ops):
    name, batch, spatial, cx, hidden, cy, skip, grid, gate, gate_bias, acts, proj = case
    dev = {k: v.cuda() for k, v in ops.items()}
    kw = {k: dev[k] for k in ("s", "w0", "gate_w", "gate_b", "w3", "b3", "w4", "b4") if k in dev}
    gp = pointwise.grid_params(grid, spatial) if grid is not None else None
    y = pointwise.chain(dev["x"], dev["w1"], dev["b1"], dev["w2"], dev["b2"], act_skip=acts, act_out=acts,
                        grid=gp, **kw)
    torch.cuda.synchronize()
    return y


def _expect(case, ops):
    name, batch, spatial, cx, hidden, cy, skip, grid, gate, gate_bias, acts, proj = case
    mat = lambda t: None if t is None else t.reshape(t.shape[0], -1)  # noqa: E731
    vec = lambda t: None if t is None else t.reshape(-1)  # noqa: E731
    return _reference(ops["x"], mat(ops["w1"]), ops["b1"], mat(ops["w2"]), ops["b2"], s=ops.get("s"),
                      w0=mat(ops.get("w0")), act_skip=acts, act_out=acts, g=vec(ops.get("gate_w")),
                      gb=vec(ops.get("gate_b")), grid=grid, w3=mat(ops.get("w3")), b3=ops.get("b3"),
                      w4=mat(ops.get("w4")), b4=ops.get("b4"))


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_chain_matches_reference(case):
    ops = _operands(case)
    y = _run(case, ops)
    y_ref = _expect(case, ops)
    assert y.shape == y_ref.shape
    assert rel_l2(y.cpu(), y_ref) <= TOL
    assert _lib.device_status() == 0


def test_chain_grid_offset_places_a_slab():
    """Grid channels of a slab (x planes [16, 32) of a 32^3 grid) equal the same planes of the whole grid."""
    case = CASES[7]
    ops = _operands(case)
    d = {k: v.cuda() for k, v in ops.items()}
    full = pointwise.chain(d["x"], d["w1"], d["b1"], d["w2"], d["b2"],
                           grid=pointwise.grid_params(case[7], (32, 32, 32)))
    slab = pointwise.chain(d["x"][:, :, 16:].contiguous(), d["w1"], d["b1"], d["w2"], d["b2"],
                           grid=pointwise.grid_params(case[7], (32, 32, 32)), grid_offset=(16, 0, 0))
    torch.cuda.synchronize()
    assert torch.equal(slab, full[:, :, 16:])


def test_chain_is_deterministic_and_writes_every_point():
    """Two calls into NaN-filled outputs agree bit for bit (every point written, no race between the
    tiles in flight)."""
    case = CASES[0]
    ops = _operands(case)
    name, batch, spatial, cx, hidden, cy, *_ = case
    a = torch.full((batch, cy, *spatial), float("nan"), device="cuda")
    b = torch.full_like(a, float("nan"))
    d = {k: v.cuda() for k, v in ops.items()}
    for out in (a, b):
        pointwise.chain(d["x"], d["w1"], d["b1"], d["w2"], d["b2"], s=d["s"], w0=d["w0"], act_skip=True,
                        act_out=True, gate_w=d["gate_w"], out=out)
    torch.cuda.synchronize()
    assert torch.isfinite(a).all() and torch.equal(a, b)


def test_fused_fno_matches_module_path(monkeypatch):
    """FNO forward through the chain kernels equals the module path (torch Conv1d layers in fp32, TF32
    off) on the same weights, at the Darcy configuration's size."""
    import neuraloperator_b200 as nb
    old = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    try:
        torch.manual_seed(0)
        model = nb.FNO(n_modes=(16, 16), in_channels=1, out_channels=1, hidden_channels=32, n_layers=4).cuda()
        x = torch.randn(4, 1, 128, 128, device="cuda")
        with torch.no_grad():
            assert model.fused_plan(x) is not None
            y_fused = model(x)
            monkeypatch.setattr(pointwise, "supported", lambda *a, **k: False)
            assert model.fused_plan(x) is None
            y_modules = model(x)
        assert rel_l2(y_fused, y_modules) <= TOL
    finally:
        torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = old


def test_chain_large_block_wide_form_with_stash_gate():
    """A C5-shaped block chain large enough (16384 tiles) for the planner's wide MMA form with the gate
    reading x from the two-buffer shared-memory stash, against the float64 reference."""
    case = ("block_h32_3d_large", 1, (128, 128, 128), 32, 16, 32, True, None, True, False, True, None)
    assert pointwise.query(pointwise.make_desc(1, (128, 128, 128), 32, 16, 32, skip=32, act_skip=True,
                                               act_out=True, gate=True)) == 4  # the wide form
    ops = _operands(case)
    y = _run(case, ops)
    y_ref = _expect(case, ops)
    assert rel_l2(y.cpu(), y_ref) <= TOL
    assert _lib.device_status() == 0


@pytest.mark.parametrize("wide", ["0", "1"])
def test_chain_lifting_many_tiles_per_group(monkeypatch, wide):
    """The C5 lifting shape (3 channels + 3 grid channels -> 64 -> 32) over 4096 tiles, several per group
    (the barrier phases and x-stash reuse carry across tiles), in both MMA forms, against the float64
    reference."""
    monkeypatch.setenv("NOP_CHAIN_WIDE", wide)
    case = ("lifting_3d_many_tiles", 2, (64, 64, 64), 3, 64, 32, False, ((0.0, 1.0),) * 3, False, False, False, None)
    assert pointwise.query(pointwise.make_desc(2, (64, 64, 64), 3, 64, 32, grid=[(0.0, 1 / 64)] * 3)) == \
        (5 if wide == "0" else 3)
    ops = _operands(case)
    y = _run(case, ops)
    y_ref = _expect(case, ops)
    assert rel_l2(y.cpu(), y_ref) <= TOL
    assert _lib.device_status() == 0
