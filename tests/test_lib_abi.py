"""CPU checks of the C ABI: the library loads, exports every declared symbol, and rejects
malformed descriptors on the host (no GPU needed: validation runs before any CUDA call)."""

import ctypes
import os
import re

import pytest

from conftest import ROOT
from neuraloperator_b200 import _lib
from neuraloperator_b200.geometry import active_modes, compute_geometry
from neuraloperator_b200.ops import make_desc


def declared_functions():
    names = []
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            text = open(os.path.join(ROOT, "include", fn)).read()
            names += re.findall(r"^\s*(?:int32_t|void|const char\*)\s+(nop_\w+)\s*\(", text, re.M)
    return sorted(set(names))


def test_library_exports_every_declared_symbol():
    lib = _lib.library()
    names = declared_functions()
    assert names, "no declarations found in include/*.h"
    for n in names:
        assert hasattr(lib, n), f"{n} is declared in include/ but not exported"
    assert set(_lib.EXPORTED_SYMBOLS) <= set(names)


def test_abi_version_and_struct_layout():
    lib = _lib.library()
    assert lib.nop_abi_version() == _lib.ABI_VERSION
    # 8 int32 + 3 int64 + 5*4 int64 + 6 int64 + 3 int64 + 2 double
    assert ctypes.sizeof(_lib.NopSpectralDesc) == 8 * 4 + 3 * 8 + 20 * 8 + 6 * 8 + 3 * 8 + 2 * 8


def _desc(**over):
    geo = compute_geometry([16, 16], active_modes((8, 8), False), active_modes((8, 8), False))
    d = make_desc(geo, 2, 3, 4)
    for k, v in over.items():
        if isinstance(v, tuple):
            arr = getattr(d, k)
            for i, e in enumerate(v):
                arr[i] = e
        else:
            setattr(d, k, v)
    return d


@pytest.mark.parametrize("over, msg", [
    (dict(abi_version=99), "abi_version"),
    (dict(ndim=0), "ndim"),
    (dict(ndim=5), "ndim"),
    (dict(batch=-1), "batch"),
    (dict(in_channels=0), "channel"),
    (dict(separable=1), "separable"),
    (dict(weight_kind=7), "weight_kind"),
    (dict(precision=3), "precision"),
    (dict(engine=9), "engine"),
    (dict(kept=(17, 5)), "kept modes"),
    (dict(kept=(8, 10)), "kept modes"),
    (dict(fwd_off=(16, 0)), "offsets"),
    (dict(fwd_off=(4, 1)), "real last axis"),
    (dict(n_in=(0, 16)), "spatial sizes"),
    (dict(n_zero_imag=4), "n_zero_imag"),
    (dict(weight_kind=1), "ranks"),
])
def test_plan_create_rejects_bad_descriptors(over, msg):
    lib = _lib.library()
    d = _desc(**over)
    h = ctypes.c_void_p()
    rc = lib.nop_spectral_plan_create(ctypes.byref(d), ctypes.byref(h))
    assert rc == -1, (rc, _lib.last_error())
    assert msg in _lib.last_error()
    assert not h.value


def test_null_arguments():
    lib = _lib.library()
    h = ctypes.c_void_p()
    assert lib.nop_spectral_plan_create(None, ctypes.byref(h)) == -1
    assert "NULL" in _lib.last_error()
    assert lib.nop_spectral_forward(None, None, None, 0, None, None, 0, None, None, 0, None) == -1
    size = ctypes.c_size_t()
    assert lib.nop_spectral_workspace_size(None, ctypes.byref(size)) == -1
    lib.nop_spectral_plan_destroy(None)  # no-op


def test_fast_engine_request_reports_unsupported_shape():
    """engine=FAST on a shape the fused kernels do not cover fails before any CUDA call."""
    lib = _lib.library()
    geo = compute_geometry([9, 7], active_modes((4, 4), False), active_modes((4, 4), False))
    d = make_desc(geo, 1, 2, 2, engine="fast")
    h = ctypes.c_void_p()
    rc = lib.nop_spectral_plan_create(ctypes.byref(d), ctypes.byref(h))
    assert rc == -2, _lib.last_error()
    assert "fused FFT engine" in _lib.last_error()


def _chain_desc(**over):
    from neuraloperator_b200 import pointwise
    d = pointwise.make_desc(2, (16, 32), 32, 16, 32, skip=32, act_skip=True, act_out=True, gate=True)
    for k, v in over.items():
        setattr(d, k, v)
    return d


def test_chain_desc_layout():
    from neuraloperator_b200.pointwise import NopChainDesc, NopChainOperands
    # 2 int32, int64 batch, 4 int64 spatial, 2 int32, 8 float, 4 int64 offsets, 8 int32
    assert ctypes.sizeof(NopChainDesc) == 8 + 8 + 32 + 8 + 32 + 32 + 32
    assert ctypes.sizeof(NopChainOperands) == 14 * 8


@pytest.mark.parametrize("over, code", [
    (dict(), 0),
    (dict(abi_version=7), -1),
    (dict(ndim=0), -1),
    (dict(grid_dims=2), -1),          # grid channels only without the skip stage
    (dict(x_channels=0), -1),
    (dict(hidden_channels=0), -1),
    (dict(out_channels=300, gate=0), -2),
    (dict(hidden_channels=257), -2),
    (dict(batch=-1), -1),
    (dict(out_channels=16), -1),      # the gate needs x_channels == out_channels
    (dict(proj_hidden=64, proj_out=0), -1),
])
def test_chain_desc_validation_on_host(over, code):
    from neuraloperator_b200 import pointwise
    lib = _lib.library()
    pointwise._declare(lib)
    groups = ctypes.c_int32()
    assert lib.nop_chain_query(ctypes.byref(_chain_desc(**over)), ctypes.byref(groups)) == code, _lib.last_error()


def test_chain_rejects_points_not_multiple_of_4():
    from neuraloperator_b200 import pointwise
    lib = _lib.library()
    pointwise._declare(lib)
    d = _chain_desc()
    d.spatial[0], d.spatial[1] = 15, 33
    assert lib.nop_chain_query(ctypes.byref(d), None) == -2
    assert b"multiple of 4" in lib.nop_last_error()


@pytest.mark.parametrize("name, kw, groups", [
    ("block_h32", dict(cx=32, hidden=16, cout=32, skip=32, gate=True), 5),
    ("block_h64", dict(cx=64, hidden=32, cout=64, skip=64, gate=True), 2),
    ("lifting_3d_h32", dict(cx=3, hidden=64, cout=32, grid=[(0.0, 1 / 256)] * 3), 5),
    ("lifting_2d_h64", dict(cx=1, hidden=128, cout=64, grid=[(0.0, 1 / 512)] * 2), 4),
    ("last_block_proj_h32", dict(cx=32, hidden=16, cout=32, skip=32, gate=True, proj_hidden=64, proj_out=3), 4),
])
def test_chain_planner_tiles_in_flight(name, kw, groups):
    """The planner fits the FNO shapes with several tiles in flight per SM (tensor memory 512 columns,
    227 KB of shared memory)."""
    from neuraloperator_b200 import pointwise
    nd = 3 if "3d" in name else 2
    assert pointwise.query(pointwise.make_desc(2, (64,) * nd, **kw)) == groups


def test_chain_planner_mma_form(monkeypatch):
    """The C5 block chain (8 x 256^3 points) runs in the wide MMA form (two MMAs per K step) with 4 tiles
    in flight; a small problem (2 x 64^3) and a forced-narrow one keep 5, and the lifting stays narrow
    with 5 (wide would leave 3)."""
    from neuraloperator_b200 import pointwise
    block = pointwise.make_desc(8, (256,) * 3, 32, 16, 32, skip=32, gate=True)
    small = pointwise.make_desc(2, (64,) * 3, 32, 16, 32, skip=32, gate=True)
    lifting = pointwise.make_desc(8, (256,) * 3, 3, 64, 32, grid=[(0.0, 1 / 256)] * 3)
    assert pointwise.query(block) == 4 and pointwise.query(small) == 5 and pointwise.query(lifting) == 5
    monkeypatch.setenv("NOP_CHAIN_WIDE", "0")
    assert pointwise.query(block) == 5
    monkeypatch.setenv("NOP_CHAIN_WIDE", "1")
    assert pointwise.query(lifting) == 3


def test_chain_planner_block_wide_form(monkeypatch):
    """With the projection fused, the C5 last block runs its block layers wide and the projection narrow:
    that keeps the narrow form's 4 tiles in flight (all layers wide would leave 2).  The chains of the
    training forward (the last block without its output GELU, the projection on its own) plan 4 each."""
    from neuraloperator_b200 import pointwise
    last_proj = pointwise.make_desc(8, (256,) * 3, 32, 16, 32, skip=32, act_skip=True, gate=True, proj_hidden=64,
                                    proj_out=3)
    last = pointwise.make_desc(2, (256,) * 3, 32, 16, 32, skip=32, act_skip=True, gate=True)
    proj = pointwise.make_desc(2, (256,) * 3, 32, 64, 3)
    assert pointwise.query(last_proj) == 4 and pointwise.query(last) == 4 and pointwise.query(proj) == 4
    for form, groups in (("0", 4), ("1", 2), ("2", 4)):
        monkeypatch.setenv("NOP_CHAIN_WIDE", form)
        assert pointwise.query(last_proj) == groups, form
    monkeypatch.setenv("NOP_CHAIN_WIDE", "2")  # no projection, no block-wide form: the planner's own choice
    assert pointwise.query(last) == 4


def test_tucker_grads_host_checks():
    """Workspace sizing and argument checks of nop_tucker_grads run on the host (no device call)."""
    lib = _lib.library()
    dims = (ctypes.c_int64 * 4)(64, 64, 64, 33)
    ranks = (ctypes.c_int64 * 4)(7, 7, 7, 4)
    size = ctypes.c_size_t()
    assert lib.nop_tucker_grads_workspace_size(4, dims, ranks, ctypes.byref(size)) == 0, _lib.last_error()
    # four buffers of the largest intermediate (gw projected on one mode: 64 x 64 x 64 x 4... at most gw)
    assert 0 < size.value <= 4 * 64 * 64 * 64 * 33 * 8 + (1 << 20)
    assert lib.nop_tucker_grads_workspace_size(1, dims, ranks, ctypes.byref(size)) == -1
    bad = (ctypes.c_int64 * 4)(64, 0, 64, 33)
    assert lib.nop_tucker_grads_workspace_size(4, bad, ranks, ctypes.byref(size)) == -1
    ptrs = (ctypes.c_void_p * 4)()
    rc = lib.nop_tucker_grads(4, dims, ranks, None, ptrs, None, None, ptrs, None, 0, None)
    assert rc == -1 and "NULL" in _lib.last_error()
