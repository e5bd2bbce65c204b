"""Parity of the CUDA spectral block with the reference (golden vectors) and the oracle.

Tolerances (the benchmark's stated bars): relative L2 <= 1e-5 in fp32, <= 2e-2 with the bf16
contraction.  TF32 is switched off in torch so the host-side ChannelMLP / skip GEMMs run in
full fp32 like the reference's CPU path.
"""

import os

import pytest
import torch

import neuraloperator_b200 as nb
import oracle
from conftest import GOLDEN, rel_l2
from helpers import build_fno, build_spectral_conv, case_scaling
from neuraloperator_b200 import _lib, ops

pytestmark = pytest.mark.gpu

TOL_FP32 = 1e-5
TOL_BF16 = 2e-2

SPECTRAL = torch.load(os.path.join(GOLDEN, "spectral_cases.pt"), weights_only=False)
CONFIG = torch.load(os.path.join(GOLDEN, "config_layers.pt"), weights_only=False)
FNO_CASES = torch.load(os.path.join(GOLDEN, "fno_cases.pt"), weights_only=False)


@pytest.fixture(autouse=True, scope="module")
def _fp32_torch():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    old = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = old


def _run(case, **extra):
    conv = build_spectral_conv(case, **extra)
    x = case["x"].cuda()
    with torch.no_grad():
        y = conv(x, **case["forward_kwargs"])
    torch.cuda.synchronize()
    return y


@pytest.mark.parametrize("engine", ["auto", "generic"])
@pytest.mark.parametrize("case", SPECTRAL, ids=[c["name"] for c in SPECTRAL])
def test_spectral_conv_golden(case, engine):
    y = _run(case, engine=engine)
    assert y.shape == case["y"].shape and y.dtype == case["y"].dtype
    assert rel_l2(y, case["y"]) <= TOL_FP32


@pytest.mark.parametrize("engine", ["auto", "generic"])
@pytest.mark.parametrize("case", CONFIG, ids=[c["name"] for c in CONFIG])
def test_config_layers_golden(case, engine):
    y = _run(case, engine=engine)
    assert rel_l2(y, case["y"]) <= TOL_FP32


@pytest.mark.parametrize("case", [c for c in SPECTRAL + CONFIG if not c["kwargs"].get("complex_data")],
                         ids=[c["name"] for c in SPECTRAL + CONFIG if not c["kwargs"].get("complex_data")])
def test_bf16_contraction_tolerance(case):
    y = _run(case, contraction_precision="bf16")
    assert rel_l2(y, case["y"]) <= TOL_BF16


@pytest.mark.parametrize("case", [c for c in FNO_CASES if c["model"] != "FNOBlocks"],
                         ids=[c["name"] for c in FNO_CASES if c["model"] != "FNOBlocks"])
def test_fno_end_to_end_golden(case):
    model = build_fno(case)
    with torch.no_grad():
        y = model(case["x"].cuda())
    assert rel_l2(y, case["y"]) <= TOL_FP32


def test_fnoblocks_fused_epilogue_golden():
    """Skip add + GELU fused into the inverse epilogue (fno_block.py:356-361)."""
    case = [c for c in FNO_CASES if c["model"] == "FNOBlocks"][0]
    from helpers import load_block
    fb = nb.FNOBlocks(**case["kwargs"])
    for i, blk in enumerate(case["params"]["blocks"]):
        load_block(fb, i, blk, "dense")
    fb = fb.cuda()
    h = case["x"].cuda()
    with torch.no_grad():
        for i in range(2):
            assert fb._fusable(i, h, None)
            h = fb(h, i)
            assert rel_l2(h, case["y"][i]) <= TOL_FP32


def _oracle_case(shape, modes, ci, co, batch, seed, **kw):
    g = torch.Generator().manual_seed(seed)
    conv = nb.SpectralConv(ci, co, modes, **kw)
    with torch.no_grad():
        conv.weight.tensor.copy_(torch.complex(torch.randn(conv.weight.shape, generator=g),
                                               torch.randn(conv.weight.shape, generator=g)) * 0.2)
        conv.bias.copy_(torch.randn(conv.bias.shape, generator=g))
    x = torch.randn((batch, ci, *shape), generator=g)
    ref = oracle.spectral_conv(x, conv.weight.tensor.detach(), conv.bias.detach(), modes)
    return conv, x, ref


@pytest.mark.parametrize("shape, modes, ci, co, batch", [
    ((256, 256), (64, 64), 8, 8, 2),      # micro config grid / modes
    ((512, 512), (64, 64), 4, 4, 1),      # TFNO config grid / modes
    ((8192,), (16,), 8, 8, 4),            # Burgers config
    ((128, 128), (16, 16), 8, 8, 3),      # Darcy config
    ((64, 64, 64), (32, 32, 32), 2, 3, 1),
    ((32, 48), (12, 20), 3, 5, 2),        # non-square
    ((1, 16), (1, 8), 2, 2, 1),           # degenerate axis of length 1
])
def test_random_against_oracle(shape, modes, ci, co, batch):
    conv, x, ref = _oracle_case(shape, modes, ci, co, batch, seed=sum(shape) + ci)
    conv = conv.cuda()
    with torch.no_grad():
        y = conv(x.cuda())
    assert rel_l2(y, ref) <= TOL_FP32


def test_linearity_and_bias():
    """Size-independent property: conv(a x1 + b x2) - bias = a (conv(x1)-bias) + b (conv(x2)-bias)."""
    conv = nb.SpectralConv(8, 8, (64, 64)).cuda()
    x1 = torch.randn(2, 8, 256, 256, device="cuda")
    x2 = torch.randn(2, 8, 256, 256, device="cuda")
    with torch.no_grad():
        b = conv.bias
        y1, y2, y12 = conv(x1) - b, conv(x2) - b, conv(0.5 * x1 - 2.0 * x2) - b
    assert rel_l2(y12, 0.5 * y1 - 2.0 * y2) <= 1e-5


def test_batch_zero_and_errors():
    conv = nb.SpectralConv(2, 3, (4, 4)).cuda()
    with torch.no_grad():
        y = conv(torch.empty(0, 2, 8, 8, device="cuda"))
    assert y.shape == (0, 3, 8, 8)
    with pytest.raises(TypeError):
        conv(torch.randn(1, 2, 8, 8, device="cuda", dtype=torch.float64))


def test_backward_through_fused_gelu_raises():
    """The fused GELU epilogue keeps no pre-activation, so a call that needs a gradient must not use it."""
    conv = nb.SpectralConv(2, 2, (4, 4)).cuda()
    x = torch.randn(1, 2, 8, 8, device="cuda", requires_grad=True)
    with pytest.raises(NotImplementedError):
        conv(x, apply_gelu=True)


def test_nonzero_stream_and_repeat():
    """Launches go on torch's current stream; repeated calls give identical results."""
    conv = nb.SpectralConv(4, 4, (16, 16)).cuda()
    x = torch.randn(2, 4, 64, 64, device="cuda")
    s = torch.cuda.Stream()
    with torch.no_grad():
        y0 = conv(x)
        with torch.cuda.stream(s):
            y1 = conv(x)
        s.synchronize()
    assert torch.equal(y0, y1)


def test_workspace_too_small_is_rejected():
    geo = nb.SpectralConv(2, 2, (4, 4)).geometry([8, 8])
    desc = ops.make_desc(geo, 1, 2, 2)
    plan = _lib.Plan(desc)
    import ctypes
    x = torch.randn(1, 2, 8, 8, device="cuda")
    w = torch.zeros(2, 2, 4, 3, dtype=torch.complex64, device="cuda")
    y = torch.empty_like(x)
    ws = torch.empty(16, dtype=torch.uint8, device="cuda")
    arr = (ctypes.c_void_p * 1)(w.data_ptr())
    rc = _lib.library().nop_spectral_forward(plan.handle, ctypes.c_void_p(x.data_ptr()), arr, 1, None, None, 0,
                                             ctypes.c_void_p(y.data_ptr()), ctypes.c_void_p(ws.data_ptr()), 16, None)
    if plan.workspace_bytes > 16:
        assert rc == -4 and "workspace" in _lib.last_error()


@pytest.mark.parametrize("n, modes, ci, co, batch", [
    (128, (16, 16), 3, 70, 17),     # Darcy grid; Co > 64 (two output tiles), batch not a multiple of 16
    (256, (64, 64), 8, 8, 2),       # micro config grid / modes
    (512, (64, 64), 4, 5, 1),       # TFNO grid / modes
    (256, (30, 20), 5, 3, 3),       # odd kept counts (My=30, Kx=11)
    (128, (128, 64), 2, 2, 1),      # every y bin kept (offset 64), Kx = 33
    (256, (8, 2), 2, 2, 1),         # tiny mode counts (Kx = 2)
])
def test_fast_engine_against_oracle(n, modes, ci, co, batch):
    conv, x, ref = _oracle_case((n, n), modes, ci, co, batch, seed=n + ci + co)
    conv.engine = "fast"
    conv = conv.cuda()
    with torch.no_grad():
        y = conv(x.cuda())
    assert rel_l2(y, ref) <= TOL_FP32


@pytest.mark.parametrize("n", [128, 256, 512])
def test_fast_engine_fused_epilogue(n):
    conv, x, ref = _oracle_case((n, n), (32, 32), 4, 4, 2, seed=n)
    g = torch.Generator().manual_seed(n + 1)
    skip = torch.randn(ref.shape, generator=g)
    conv.engine = "fast"
    conv = conv.cuda()
    with torch.no_grad():
        y = conv(x.cuda(), addend=skip.cuda(), apply_gelu=True)
    assert rel_l2(y, torch.nn.functional.gelu(ref + skip)) <= TOL_FP32


def test_fast_engine_bf16_contraction():
    conv, x, ref = _oracle_case((256, 256), (64, 64), 16, 16, 2, seed=5)
    conv.engine = "fast"
    conv.contraction_precision = "bf16"
    conv = conv.cuda()
    with torch.no_grad():
        y = conv(x.cuda())
    err = rel_l2(y, ref)
    assert 1e-5 < err <= TOL_BF16  # visibly reduced precision, inside the bf16 bound


def test_fast_engine_rejects_uncovered_shape():
    conv = nb.SpectralConv(2, 2, (6, 6), engine="fast").cuda()
    with pytest.raises(_lib.NopError):
        conv(torch.randn(1, 2, 12, 12, device="cuda"))


def test_fast_plan_unpacked_entry_matches_packed():
    """nop_spectral_forward on a fused plan packs internally; same result as the packed path."""
    import ctypes
    conv, x, ref = _oracle_case((256, 256), (64, 64), 4, 6, 3, seed=11)
    conv = conv.cuda()
    xd = x.cuda()
    with torch.no_grad():
        y_mod = conv(xd)
    geo = conv.geometry([256, 256])
    _, weights, _ = conv.kernel_operands(geo)
    w = weights[0].detach().contiguous()
    b = conv.bias.detach().reshape(-1).contiguous()
    plan = ops.get_plan(ops.make_desc(geo, 3, 4, 6), 0)
    assert plan.is_fast and plan.packed_bytes > 0
    ws = torch.empty(plan.workspace_bytes, dtype=torch.uint8, device="cuda")
    y = torch.empty_like(y_mod)
    arr = (ctypes.c_void_p * 1)(w.data_ptr())
    rc = _lib.library().nop_spectral_forward(plan.handle, ctypes.c_void_p(xd.data_ptr()), arr, 1,
                                             ctypes.c_void_p(b.data_ptr()), None, 0, ctypes.c_void_p(y.data_ptr()),
                                             ctypes.c_void_p(ws.data_ptr()), plan.workspace_bytes,
                                             ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, _lib.last_error()
    torch.cuda.synchronize()
    assert torch.equal(y, y_mod)
    assert rel_l2(y, ref) <= TOL_FP32


def test_packed_weights_follow_in_place_updates():
    conv, x, _ = _oracle_case((128, 128), (16, 16), 4, 4, 2, seed=3)
    conv = conv.cuda()
    xd = x.cuda()
    with torch.no_grad():
        y0 = conv(xd)
        conv.weight.tensor.mul_(2.0)   # in-place update bumps the version counter -> repack
        y1 = conv(xd)
    b = conv.bias.detach()
    assert rel_l2(y1 - b, 2.0 * (y0 - b)) <= 1e-6


@pytest.mark.parametrize("n, modes, ranks", [(256, (64, 64), 0.1), (128, (16, 16), 0.5)])
def test_fast_tucker_against_oracle(n, modes, ranks):
    g = torch.Generator().manual_seed(n)
    conv = nb.SpectralConv(8, 8, modes, factorization="tucker", implementation="factorized", rank=ranks)
    with torch.no_grad():
        for prm in conv.weight.parameters():
            prm.copy_(torch.complex(torch.randn(prm.shape, generator=g), torch.randn(prm.shape, generator=g)) * 0.5)
    x = torch.randn((2, 8, n, n), generator=g)
    w = {"core": conv.weight.core.detach(), "factors": [f.detach() for f in conv.weight.factors]}
    ref = oracle.spectral_conv(x, w, conv.bias.detach(), modes, weight_kind="tucker")
    conv.engine = "fast"
    conv = conv.cuda()
    with torch.no_grad():
        y = conv(x.cuda())
    assert rel_l2(y, ref) <= TOL_FP32


def _assert_fast(conv, x):
    geo = conv.geometry(list(x.shape[2:]))
    kind, _, ranks = conv.kernel_operands(geo)
    plan = ops.get_plan(ops.make_desc(geo, x.shape[0], conv.in_channels, conv.out_channels, weight_kind=kind,
                                      ranks=ranks), 0)
    assert plan.is_fast


@pytest.mark.parametrize("n, modes, ci, co, batch", [
    (8192, (16,), 8, 6, 5),    # Burgers config length / modes (9 kept bins)
    (2048, (32,), 3, 4, 3),    # 17 kept bins (fold of bin 16 onto the 16-point transform)
    (16384, (16,), 2, 2, 2),
])
def test_fast_1d_against_oracle(n, modes, ci, co, batch):
    conv, x, ref = _oracle_case((n,), modes, ci, co, batch, seed=n + ci)
    g = torch.Generator().manual_seed(n)
    skip = torch.randn(ref.shape, generator=g)
    conv.engine = "fast"
    conv = conv.cuda()
    _assert_fast(conv, x)
    with torch.no_grad():
        y = conv(x.cuda())
        yf = conv(x.cuda(), addend=skip.cuda(), apply_gelu=True)
    assert rel_l2(y, ref) <= TOL_FP32
    assert rel_l2(yf, torch.nn.functional.gelu(ref + skip)) <= TOL_FP32


@pytest.mark.parametrize("modes, ci, co", [((32, 32, 32), 2, 3), ((64, 64, 64), 1, 2)])
def test_fast_3d_against_oracle(modes, ci, co):
    conv, x, ref = _oracle_case((256, 256, 256), modes, ci, co, 1, seed=sum(modes) + co)
    conv.engine = "fast"
    conv = conv.cuda()
    _assert_fast(conv, x)
    with torch.no_grad():
        y = conv(x.cuda())
    assert rel_l2(y, ref) <= TOL_FP32
    skip = torch.randn(ref.shape, generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        yf = conv(x.cuda(), addend=skip.cuda(), apply_gelu=True)
    assert rel_l2(yf, torch.nn.functional.gelu(ref + skip)) <= TOL_FP32


def test_fast_3d_tucker():
    g = torch.Generator().manual_seed(9)
    conv = nb.SpectralConv(4, 4, (32, 32, 32), factorization="tucker", implementation="factorized", rank=0.2)
    with torch.no_grad():
        for prm in conv.weight.parameters():
            prm.copy_(torch.complex(torch.randn(prm.shape, generator=g), torch.randn(prm.shape, generator=g)) * 0.5)
    x = torch.randn((1, 4, 256, 256, 256), generator=g)
    w = {"core": conv.weight.core.detach(), "factors": [f.detach() for f in conv.weight.factors]}
    ref = oracle.spectral_conv(x, w, conv.bias.detach(), (32, 32, 32), weight_kind="tucker")
    conv.engine = "fast"
    conv = conv.cuda()
    with torch.no_grad():
        y = conv(x.cuda())
    assert rel_l2(y, ref) <= TOL_FP32
