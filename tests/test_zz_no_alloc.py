"""The allocation-free entry point agrees with the regular one and with the oracle.

nop_spectral_forward_static serves callers that cannot allocate device memory (a host runtime
that owns all device memory and passes only input/output buffers, or a loop that cannot risk the
device-wide stall of a cudaMalloc).  It keeps its scratch in a fixed area inside the library, so
every call reuses memory that the previous call left behind.  Each case runs twice in a row and is
checked against nop_spectral_forward and against the oracle (the reference's forward restated on
the CPU); the cases run from the largest scratch footprint to the smallest, so a region that a
smaller problem failed to rewrite would still hold a larger problem's values.  Dense, Tucker and CP
weights, complex data and 1D / 2D / 3D grids cover every scratch region (twiddle tables, spectra,
factor intermediates).  This file is collected last so that a failure here never hides the other
tests.
"""

import ctypes

import pytest
import torch

import neuraloperator_b200 as nb
import oracle
from conftest import rel_l2
from neuraloperator_b200 import _lib, ops

pytestmark = pytest.mark.gpu

TOL_FP32 = 1e-5


def _static_fn():
    lib = _lib.library()
    fn = lib.nop_spectral_forward_static
    fn.restype = ctypes.c_int32
    fn.argtypes = [ctypes.POINTER(_lib.NopSpectralDesc), ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p),
                   ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p,
                   ctypes.c_void_p]
    return fn


# name, grid, n_modes, channels (in, out), batch, factorization, complex data, fused skip + GELU;
# ordered from the largest scratch footprint to the smallest
CASES = [
    ("dense2d_128", (128, 128), (32, 32), (8, 8), 2, None, False, True),
    ("tucker3d_32", (32, 32, 32), (12, 12, 12), (6, 6), 2, "tucker", False, False),
    ("dense2d_64", (64, 64), (16, 16), (4, 4), 2, None, False, True),
    ("cp2d_48", (48, 40), (12, 10), (5, 3), 2, "cp", False, False),
    ("complex2d_32", (32, 24), (10, 8), (3, 4), 1, None, True, False),
    ("dense1d_256", (256,), (20,), (4, 6), 3, None, False, True),
]


def _conv(case, seed):
    name, grid, modes, (ci, co), batch, fact, cplx, fused = case
    g = torch.Generator().manual_seed(seed)
    kw = {}
    if fact:
        kw = dict(factorization=fact, implementation="factorized", rank=0.5)
    conv = nb.SpectralConv(ci, co, modes, complex_data=cplx, **kw)
    with torch.no_grad():
        for p in conv.weight.parameters():
            p.copy_(torch.complex(torch.randn(p.shape, generator=g), torch.randn(p.shape, generator=g)) * 0.3)
        conv.bias.copy_(torch.randn(conv.bias.shape, generator=g))
    if cplx:
        x = torch.complex(torch.randn((batch, ci, *grid), generator=g), torch.randn((batch, ci, *grid), generator=g))
    else:
        x = torch.randn((batch, ci, *grid), generator=g)
    skip = torch.randn((batch, co, *grid), generator=g) if fused else None
    return conv, x, skip


def _oracle(conv, case, x, skip):
    name, grid, modes, _, _, fact, cplx, fused = case
    w = conv.weight
    if fact == "tucker":
        payload, kind = {"core": w.core.detach().cpu(), "factors": [f.detach().cpu() for f in w.factors]}, "tucker"
    elif fact == "cp":
        payload, kind = {"weights": w.weights.detach().cpu(), "factors": [f.detach().cpu() for f in w.factors]}, "cp"
    else:
        payload, kind = w.tensor.detach().cpu(), "dense"
    y = oracle.spectral_conv(x, payload, conv.bias.detach().cpu(), modes, weight_kind=kind, complex_data=cplx)
    if fused:
        y = torch.nn.functional.gelu(y + skip)
    return y


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")
def test_static_entry_matches_regular_entry_and_oracle():
    fn = _static_fn()
    stream = torch.cuda.current_stream().cuda_stream
    for seed, case in enumerate(CASES):
        name, grid, modes, (ci, co), batch, fact, cplx, fused = case
        conv, x_cpu, skip_cpu = _conv(case, seed)
        with torch.no_grad():
            expect_oracle = _oracle(conv, case, x_cpu, skip_cpu)
        conv = conv.cuda()
        x = x_cpu.cuda()
        skip = skip_cpu.cuda() if fused else None
        geo = conv.geometry(list(grid))
        kind, weights, ranks = conv.kernel_operands(geo)
        ws = [w.detach().to(torch.complex64).contiguous() for w in weights]
        b = conv.bias.detach().reshape(-1).contiguous()
        with torch.no_grad():
            expect = ops.spectral_forward(x, geo, ws, out_channels=co, weight_kind=kind, ranks=ranks, bias=b,
                                          addend=skip, apply_gelu=fused)
        torch.cuda.synchronize()
        assert rel_l2(expect, expect_oracle) <= TOL_FP32, name
        desc = ops.make_desc(geo, batch, ci, co, weight_kind=kind, ranks=ranks)
        arr = (ctypes.c_void_p * len(ws))(*[w.data_ptr() for w in ws])
        for call in range(2):  # the second call runs on the scratch the first one left behind
            y = torch.full_like(expect, float("nan"))
            rc = fn(ctypes.byref(desc), ctypes.c_void_p(x.data_ptr()), arr, len(ws), ctypes.c_void_p(b.data_ptr()),
                    None if skip is None else ctypes.c_void_p(skip.data_ptr()), int(fused),
                    ctypes.c_void_p(y.data_ptr()), ctypes.c_void_p(stream))
            assert rc == 0, (name, call, _lib.last_error())
            torch.cuda.synchronize()
            assert rel_l2(y, expect) <= TOL_FP32, (name, call)
            assert rel_l2(y, expect_oracle) <= TOL_FP32, (name, call)


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")
def test_static_entry_rejects_problems_beyond_its_scratch():
    fn = _static_fn()
    conv = nb.SpectralConv(64, 64, (64, 64))
    geo = conv.geometry([256, 256])
    desc = ops.make_desc(geo, 64, 64, 64)
    dummy = torch.empty(8, device="cuda")
    arr = (ctypes.c_void_p * 1)(dummy.data_ptr())
    rc = fn(ctypes.byref(desc), ctypes.c_void_p(dummy.data_ptr()), arr, 1, None, None, 0,
            ctypes.c_void_p(dummy.data_ptr()), None)
    assert rc == -4
    assert "static scratch" in _lib.last_error()


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")
def test_static_entry_rejects_the_fast_engine():
    fn = _static_fn()
    conv = nb.SpectralConv(4, 4, (16, 16))
    geo = conv.geometry([64, 64])
    desc = ops.make_desc(geo, 1, 4, 4, engine="fast")
    dummy = torch.empty(8, device="cuda")
    arr = (ctypes.c_void_p * 1)(dummy.data_ptr())
    rc = fn(ctypes.byref(desc), ctypes.c_void_p(dummy.data_ptr()), arr, 1, None, None, 0,
            ctypes.c_void_p(dummy.data_ptr()), None)
    assert rc == -2  # NOP_E_UNSUPPORTED
    assert "generic engine" in _lib.last_error()
