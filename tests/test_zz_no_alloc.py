"""The allocation-free entry point agrees with the regular one.

nop_spectral_forward_static serves callers that cannot allocate device memory (a host runtime
that owns all device memory and passes only input/output buffers, or a loop that cannot risk the
device-wide stall of a cudaMalloc).  It keeps its scratch in a fixed area inside the library, so
two calls in a row reuse the same memory; both must match nop_spectral_forward.  This file is
collected last so that a failure here never hides the other tests.
"""

import ctypes

import pytest
import torch

from conftest import rel_l2
from neuraloperator_b200 import _lib, ops
import neuraloperator_b200 as nb

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


def _case(seed, shape=(64, 64), modes=(16, 16), ci=4, co=4, batch=2):
    g = torch.Generator().manual_seed(seed)
    conv = nb.SpectralConv(ci, co, modes)
    with torch.no_grad():
        conv.weight.tensor.copy_(torch.complex(torch.randn(conv.weight.shape, generator=g),
                                               torch.randn(conv.weight.shape, generator=g)) * 0.3)
        conv.bias.copy_(torch.randn(conv.bias.shape, generator=g))
    conv = conv.cuda()
    x = torch.randn((batch, ci, *shape), generator=g).cuda()
    skip = torch.randn((batch, co, *shape), generator=g).cuda()
    return conv, x, skip


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")
def test_static_entry_matches_regular_entry_twice():
    fn = _static_fn()
    conv, x, skip = _case(0)
    geo = conv.geometry(list(x.shape[2:]))
    _, weights, _ = conv.kernel_operands(geo)
    w = weights[0].detach().contiguous()
    b = conv.bias.detach().reshape(-1).contiguous()
    with torch.no_grad():
        expect = ops.spectral_forward(x, geo, [w], out_channels=4, bias=b, addend=skip, apply_gelu=True)
    desc = ops.make_desc(geo, x.shape[0], 4, 4)
    stream = torch.cuda.current_stream().cuda_stream
    arr = (ctypes.c_void_p * 1)(w.data_ptr())
    for _ in range(2):  # the second call runs on the scratch the first one left behind
        y = torch.full_like(expect, float("nan"))
        rc = fn(ctypes.byref(desc), ctypes.c_void_p(x.data_ptr()), arr, 1, ctypes.c_void_p(b.data_ptr()),
                ctypes.c_void_p(skip.data_ptr()), 1, ctypes.c_void_p(y.data_ptr()), ctypes.c_void_p(stream))
        assert rc == 0, _lib.last_error()
        torch.cuda.synchronize()
        assert rel_l2(y, expect) <= TOL_FP32


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
