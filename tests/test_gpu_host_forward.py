"""Forward from host memory (nop_spectral_forward_host): chunked, copies overlapped with kernels.

Every sample is computed by the same kernels as the device forward with a smaller batch per launch,
so the result must equal the device forward on the same inputs to fp32 rounding (relative L2
<= 1e-6; the contraction sums run over channels only, never over the batch).
"""

import ctypes

import pytest
import torch

import neuraloperator_b200 as nb
from conftest import rel_l2
from neuraloperator_b200 import _lib, ops

pytestmark = pytest.mark.gpu

TOL = 1e-6
NOP_E_INVALID, NOP_E_WORKSPACE = -1, -4   # nop_status values (include/nop_spectral.h)


@pytest.fixture(autouse=True, scope="module")
def _needs_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _conv(ci, co, modes, seed=0, **kw):
    torch.manual_seed(seed)
    conv = nb.SpectralConv(ci, co, modes, **kw).cuda()
    if kw.get("factorization") is None:
        with torch.no_grad():
            w = conv.weight.tensor
            w.copy_(torch.complex(torch.randn_like(w.real), torch.randn_like(w.real)) * 0.05)
    with torch.no_grad():
        if conv.bias is not None:
            conv.bias.copy_(torch.randn_like(conv.bias) * 0.1)
    return conv


CASES = [
    ("fast2d_256", dict(ci=4, co=6, modes=(64, 64)), (8, 256, 256), 2, 3),
    ("fast2d_128_tucker", dict(ci=8, co=8, modes=(16, 16), factorization="tucker", rank=0.5), (6, 128, 128), 3, 2),
    ("fast1d_8192", dict(ci=4, co=4, modes=(16,)), (16, 8192), 4, 3),
    ("fast3d_256", dict(ci=2, co=2, modes=(32, 32, 32)), (2, 256, 256, 256), 1, 2),
    ("generic2d_odd", dict(ci=3, co=5, modes=(12, 10)), (6, 60, 44), 2, 3),
    ("generic1d_cp", dict(ci=4, co=4, modes=(8,), factorization="cp", rank=0.5), (4, 40), 1, 4),
]


@pytest.mark.parametrize("name,kw,shape,chunk,streams", CASES, ids=[c[0] for c in CASES])
def test_host_forward_matches_device_forward(name, kw, shape, chunk, streams):
    kw = dict(kw)
    conv = _conv(kw.pop("ci"), kw.pop("co"), kw.pop("modes"), **kw)
    g = torch.Generator().manual_seed(3)
    batch = shape[0]
    x = torch.randn((batch, conv.in_channels, *shape[1:]), generator=g).pin_memory()
    with torch.no_grad():
        ref = conv(x.cuda()).cpu()
    y = conv.forward_host(x, chunk=chunk, n_streams=streams)
    assert y.shape == ref.shape and not y.is_cuda
    assert rel_l2(y, ref) <= TOL


def test_host_forward_fused_epilogue_and_out_buffer():
    conv = _conv(4, 4, (64, 64), seed=2)
    g = torch.Generator().manual_seed(5)
    x = torch.randn((8, 4, 256, 256), generator=g).pin_memory()
    skip = torch.randn((8, 4, 256, 256), generator=g).pin_memory()
    with torch.no_grad():
        ref = conv(x.cuda(), addend=skip.cuda(), apply_gelu=True).cpu()
    out = torch.full((8, 4, 256, 256), float("nan")).pin_memory()
    y = conv.forward_host(x, addend=skip, apply_gelu=True, chunk=2, n_streams=2, out=out)
    assert y.data_ptr() == out.data_ptr()
    assert rel_l2(y, ref) <= TOL


def test_host_forward_unpacked_weights_on_fused_plan():
    """The C entry point packs unpacked weights once for fused plans (no Python-side packing)."""
    conv = _conv(4, 4, (64, 64), seed=4)
    geo = conv.geometry([256, 256])
    kind, weights, ranks = conv.kernel_operands(geo)
    ws = [w.detach().to(torch.complex64).contiguous() for w in weights]
    desc = ops.make_desc(geo, 2, 4, 4, weight_kind=kind, ranks=ranks)
    plan = ops.get_plan(desc, 0)
    assert plan.is_fast
    lib = _lib.library()
    size = ctypes.c_size_t()
    _lib.check(lib.nop_spectral_host_workspace_size(plan.handle, 2, ctypes.byref(size)))
    x = torch.randn((8, 4, 256, 256)).pin_memory()
    y = torch.empty((8, 4, 256, 256)).pin_memory()
    workspace = torch.empty(size.value, dtype=torch.uint8, device="cuda")
    arr = (ctypes.c_void_p * len(ws))(*[w.data_ptr() for w in ws])
    b = conv.bias.detach().reshape(-1).contiguous()
    stream = torch.cuda.current_stream()
    _lib.check(lib.nop_spectral_forward_host(plan.handle, ctypes.c_void_p(x.data_ptr()), 8, arr, len(ws), None, 0,
                                             ctypes.c_void_p(b.data_ptr()), None, 0, ctypes.c_void_p(y.data_ptr()),
                                             ctypes.c_void_p(workspace.data_ptr()), size.value, 2,
                                             ctypes.c_void_p(stream.cuda_stream)))
    stream.synchronize()
    with torch.no_grad():
        ref = conv(x.cuda()).cpu()
    assert rel_l2(y, ref) <= TOL


def test_host_forward_argument_errors():
    conv = _conv(2, 2, (16, 16))
    x = torch.randn((6, 2, 128, 128))
    with pytest.raises(ValueError):
        conv.forward_host(x, chunk=4)                      # 4 does not divide 6
    geo = conv.geometry([128, 128])
    desc = ops.make_desc(geo, 4, 2, 2)
    plan = ops.get_plan(desc, 0)
    lib = _lib.library()
    size = ctypes.c_size_t()
    assert lib.nop_spectral_host_workspace_size(plan.handle, 0, ctypes.byref(size)) == NOP_E_INVALID
    assert lib.nop_spectral_host_workspace_size(plan.handle, 9, ctypes.byref(size)) == NOP_E_INVALID
    _lib.check(lib.nop_spectral_host_workspace_size(plan.handle, 2, ctypes.byref(size)))
    workspace = torch.empty(size.value, dtype=torch.uint8, device="cuda")
    y = torch.empty((6, 2, 128, 128))
    packed = torch.empty(plan.packed_bytes, dtype=torch.uint8, device="cuda")
    rc = lib.nop_spectral_forward_host(plan.handle, ctypes.c_void_p(x.data_ptr()), 6, None, 0,
                                       ctypes.c_void_p(packed.data_ptr()), plan.packed_bytes, None, None, 0,
                                       ctypes.c_void_p(y.data_ptr()), ctypes.c_void_p(workspace.data_ptr()),
                                       size.value, 2, None)
    assert rc == NOP_E_INVALID and b"multiple" in lib.nop_last_error()
    rc = lib.nop_spectral_forward_host(plan.handle, ctypes.c_void_p(x.data_ptr()), 4, None, 0,
                                       ctypes.c_void_p(packed.data_ptr()), plan.packed_bytes, None, None, 0,
                                       ctypes.c_void_p(y.data_ptr()), ctypes.c_void_p(workspace.data_ptr()),
                                       size.value - 256, 2, None)
    assert rc == NOP_E_WORKSPACE


@pytest.mark.parametrize("chunk", [1, 2, 3, 6])
def test_fno_forward_host_matches_device(chunk):
    """FNO.forward_host (three-stage copy / forward / copy pipeline over chunks of the batch) returns
    exactly the device forward, for every chunk size, into a caller-owned pinned output."""
    import neuraloperator_b200 as nb
    torch.manual_seed(0)
    model = nb.FNO(n_modes=(8, 8), in_channels=1, out_channels=1, hidden_channels=32, n_layers=4).cuda().eval()
    x = torch.randn(6, 1, 64, 64)
    with torch.no_grad():
        ref = model(x.cuda()).cpu()
        out = torch.full((6, 1, 64, 64), float("nan")).pin_memory()
        y = model.forward_host(x.pin_memory(), out=out, chunk=chunk)
    assert y.data_ptr() == out.data_ptr()
    assert torch.equal(y, ref)
