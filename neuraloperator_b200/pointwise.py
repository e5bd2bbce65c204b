"""Per-pixel layer chain on the tensor cores (nop_chain_forward): the FNO layers around each spectral block.

``chain(x, ...)`` evaluates, in one pass over HBM, at every spatial point

    u = act_skip(W0 x + s)      if s is given (s = the block's spectral output), else u = [x ; grid]
    h = GELU(W1 u + b1)
    y = act_out(W2 h + b2 + g * x + gb)
    out = W4 GELU(W3 y + b3) + b4      (when the projection weights are given)

with the reference modules' own parameters: the linear skip (neuralop/layers/skip_connections.py:96-127),
ChannelMLP (neuralop/layers/channel_mlp.py:82-119), SoftGating (skip_connections.py:53-94),
GridEmbeddingND (neuralop/layers/embeddings.py:147-164), and the FNO's lifting / projection ChannelMLPs
(neuralop/models/fno.py:387-406).  ``supported`` tells the caller whether the kernel takes a problem;
callers keep the module path otherwise.
"""

from __future__ import annotations

import ctypes
import os
from typing import Optional, Sequence

import torch

from . import _lib

MAX_DIMS = 4


class NopChainDesc(ctypes.Structure):
    _fields_ = [
        ("abi_version", ctypes.c_int32),
        ("ndim", ctypes.c_int32),
        ("batch", ctypes.c_int64),
        ("spatial", ctypes.c_int64 * MAX_DIMS),
        ("x_channels", ctypes.c_int32),
        ("grid_dims", ctypes.c_int32),
        ("grid_lo", ctypes.c_float * MAX_DIMS),
        ("grid_step", ctypes.c_float * MAX_DIMS),
        ("grid_offset", ctypes.c_int64 * MAX_DIMS),
        ("skip_channels", ctypes.c_int32),
        ("act_skip", ctypes.c_int32),
        ("hidden_channels", ctypes.c_int32),
        ("out_channels", ctypes.c_int32),
        ("act_out", ctypes.c_int32),
        ("gate", ctypes.c_int32),
        ("proj_hidden", ctypes.c_int32),
        ("proj_out", ctypes.c_int32),
    ]


class NopChainOperands(ctypes.Structure):
    _fields_ = [(name, ctypes.c_void_p) for name in
                ("x", "s", "w0", "w1", "b1", "w2", "b2", "g", "gb", "w3", "b3", "w4", "b4", "y")]


class NopChainGrads(ctypes.Structure):
    _fields_ = [(name, ctypes.c_void_p) for name in
                ("dy", "dx", "ds", "dw0", "dw1", "db1", "dw2", "db2", "dg", "dgb")]


def _declare(lib):
    if getattr(lib, "_chain_declared", False):
        return
    lib.nop_chain_backward_query.restype = ctypes.c_int32
    lib.nop_chain_backward_query.argtypes = [ctypes.POINTER(NopChainDesc), ctypes.POINTER(ctypes.c_size_t)]
    lib.nop_chain_backward.restype = ctypes.c_int32
    lib.nop_chain_backward.argtypes = [ctypes.POINTER(NopChainDesc), ctypes.POINTER(NopChainOperands),
                                       ctypes.POINTER(NopChainGrads), ctypes.c_void_p, ctypes.c_size_t,
                                       ctypes.c_void_p]
    lib.nop_chain_query.restype = ctypes.c_int32
    lib.nop_chain_query.argtypes = [ctypes.POINTER(NopChainDesc), ctypes.POINTER(ctypes.c_int32)]
    lib.nop_chain_forward.restype = ctypes.c_int32
    lib.nop_chain_forward.argtypes = [ctypes.POINTER(NopChainDesc), ctypes.POINTER(NopChainOperands),
                                      ctypes.c_void_p]
    lib._chain_declared = True


def _mat(w: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
    """[out, in] float32 contiguous view of a Conv1d(k=1) weight ([out, in, 1]) or a matrix."""
    if w is None:
        return None
    w = w.detach()
    if w.ndim == 3:
        w = w[..., 0]
    return w.to(torch.float32).contiguous()


def _vec(v: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
    return None if v is None else v.detach().reshape(-1).to(torch.float32).contiguous()


def grid_params(boundaries: Sequence[Sequence[float]], sizes: Sequence[int]):
    """(lo, step) per axis of GridEmbeddingND's coordinates on a grid of ``sizes`` points
    (torch.linspace(lo, hi, n + 1)[:-1], neuralop/layers/embeddings.py:351-383)."""
    return [(float(lo), (float(hi) - float(lo)) / float(n)) for (lo, hi), n in zip(boundaries, sizes)]


def make_desc(batch: int, spatial: Sequence[int], cx: int, hidden: int, cout: int, *, skip: int = 0,
              act_skip: bool = False, act_out: bool = False, gate: bool = False, grid=None, grid_offset=None,
              proj_hidden: int = 0, proj_out: int = 0) -> NopChainDesc:
    """Descriptor of one chain call.  ``grid``: per-axis (lo, step) of the coordinate channels (see
    grid_params) or None; ``grid_offset``: the index of this call's first point per axis."""
    d = NopChainDesc()
    d.abi_version = _lib.ABI_VERSION
    d.ndim = len(spatial)
    d.batch = int(batch)
    for j, n in enumerate(spatial):
        d.spatial[j] = int(n)
    d.x_channels = int(cx)
    d.grid_dims = 0 if grid is None else len(spatial)
    if grid is not None:
        for j, (lo, step) in enumerate(grid):
            d.grid_lo[j] = lo
            d.grid_step[j] = step
            d.grid_offset[j] = int(grid_offset[j]) if grid_offset is not None else 0
    d.skip_channels = int(skip)
    d.act_skip = int(bool(act_skip))
    d.hidden_channels = int(hidden)
    d.out_channels = int(cout)
    d.act_out = int(bool(act_out))
    d.gate = int(bool(gate))
    d.proj_hidden = int(proj_hidden)
    d.proj_out = int(proj_out)
    return d


def query(desc: NopChainDesc) -> int:
    """Tiles in flight per CTA for this descriptor, or 0 when the kernel does not take it."""
    lib = _lib.library()
    _declare(lib)
    groups = ctypes.c_int32(0)
    return int(groups.value) if lib.nop_chain_query(ctypes.byref(desc), ctypes.byref(groups)) == _lib.NOP_OK else 0


def supported(batch: int, spatial: Sequence[int], cx: int, hidden: int, cout: int, min_groups: int = 1,
              **kw) -> bool:
    """Whether the kernel takes a chain of these sizes (channel counts <= 256, the weights and
    in-flight tiles fitting one CTA's tensor and shared memory, points per sample a multiple of 4) with
    at least ``min_groups`` tiles in flight per SM.  ``NOP_CHAIN=0`` in the environment (read at every
    call) reports False, so the models run their module path (A/B timing)."""
    if not 1 <= len(spatial) <= MAX_DIMS or os.environ.get("NOP_CHAIN") == "0":
        return False
    return query(make_desc(batch, spatial, cx, hidden, cout, **kw)) >= min_groups


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def chain(x: torch.Tensor, w1: torch.Tensor, b1: Optional[torch.Tensor], w2: torch.Tensor,
          b2: Optional[torch.Tensor], *, s: Optional[torch.Tensor] = None, w0: Optional[torch.Tensor] = None,
          act_skip: bool = False, act_out: bool = False, gate_w: Optional[torch.Tensor] = None,
          gate_b: Optional[torch.Tensor] = None, grid=None, grid_offset=None, w3: Optional[torch.Tensor] = None,
          b3: Optional[torch.Tensor] = None, w4: Optional[torch.Tensor] = None, b4: Optional[torch.Tensor] = None,
          out: Optional[torch.Tensor] = None, grad_relay: Optional["GradRelay"] = None) -> torch.Tensor:
    """One chain call on x's device and current stream (see the module docstring); returns y (or the
    projection's output when w3 / w4 are given).  ``gate_w`` switches on the soft-gating skip of x.
    ``grad_relay``: under autograd, dL/dx is handed to that relay instead of returned (GradRelay)."""
    if not x.is_cuda:
        raise RuntimeError("neuraloperator_b200 runs on CUDA devices only (there is no CPU path)")
    if torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in
                                       (x, s, w0, w1, b1, w2, b2, gate_w, gate_b, w3, b3, w4, b4)):
        if w3 is not None or w4 is not None:
            raise RuntimeError("the chain kernel's backward takes chains without the projection; run the "
                               "projection as its own chain call when a gradient is needed")
        if out is not None:
            raise ValueError("out= is not supported when a gradient is recorded")
        return _ChainFn.apply(x, s, w0, w1, b1, w2, b2, gate_w, gate_b,
                              (bool(act_skip), bool(act_out), grid, grid_offset, grad_relay))
    if x.dtype != torch.float32:
        raise TypeError(f"expected float32 input, got {x.dtype}")
    x = x.contiguous()
    spatial = tuple(x.shape[2:])
    m0, m1, m2, m3, m4 = _mat(w0), _mat(w1), _mat(w2), _mat(w3), _mat(w4)
    v1, v2, v3, v4 = _vec(b1), _vec(b2), _vec(b3), _vec(b4)
    g, gb = _vec(gate_w), _vec(gate_b)
    if s is not None:
        s = s.contiguous()
        if m0 is None or tuple(s.shape) != (x.shape[0], m0.shape[0], *spatial):
            raise ValueError("s must be [batch, rows of w0, *spatial] and w0 must be given")
    proj = m3 is not None
    cout = m4.shape[0] if proj else m2.shape[0]
    d = make_desc(x.shape[0], spatial, x.shape[1], m1.shape[0], m2.shape[0], skip=0 if s is None else m0.shape[0],
                  act_skip=act_skip, act_out=act_out, gate=g is not None, grid=grid, grid_offset=grid_offset,
                  proj_hidden=m3.shape[0] if proj else 0, proj_out=cout if proj else 0)
    y_shape = (x.shape[0], cout, *spatial)
    if out is None:
        out = torch.empty(y_shape, device=x.device, dtype=torch.float32)
    elif tuple(out.shape) != y_shape or not out.is_contiguous() or out.dtype != torch.float32:
        raise ValueError(f"out must be a contiguous float32 tensor of shape {y_shape}")
    ops = NopChainOperands()
    for name, t in (("x", x), ("s", s), ("w0", m0), ("w1", m1), ("b1", v1), ("w2", m2), ("b2", v2), ("g", g),
                    ("gb", gb), ("w3", m3), ("b3", v3), ("w4", m4), ("b4", v4), ("y", out)):
        setattr(ops, name, None if t is None else t.data_ptr())
    lib = _lib.library()
    _declare(lib)
    stream = ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)
    with torch.cuda.device(x.device):
        _lib.check(lib.nop_chain_forward(ctypes.byref(d), ctypes.byref(ops), stream))
    return out


def backward_supported(batch: int, spatial: Sequence[int], cx: int, hidden: int, cout: int, **kw) -> bool:
    """Whether nop_chain_backward takes a chain of these sizes (no projection, channel counts <= 128)."""
    if not 1 <= len(spatial) <= MAX_DIMS or kw.get("proj_hidden"):
        return False
    lib = _lib.library()
    _declare(lib)
    return lib.nop_chain_backward_query(ctypes.byref(make_desc(batch, spatial, cx, hidden, cout, **kw)), None) == \
        _lib.NOP_OK


def chain_backward(dy: torch.Tensor, x: torch.Tensor, w1, b1, w2, b2, *, s=None, w0=None, act_skip=False,
                   act_out=False, gate_w=None, gate_b=None, grid=None, grid_offset=None, need=None):
    """Gradients of one chain call (no projection) given dL/dy (nop_chain_backward): a dict with the keys
    x, s, w0, w1, b1, w2, b2, g, gb (each [out, in] / [channels] / the activation's shape, None where not
    applicable or not in ``need``)."""
    x = x.detach().contiguous()
    dy = dy.detach().contiguous().to(torch.float32)
    spatial = tuple(x.shape[2:])
    m0, m1, m2 = _mat(w0), _mat(w1), _mat(w2)
    v1, v2, g, gb = _vec(b1), _vec(b2), _vec(gate_w), _vec(gate_b)
    if s is not None:
        s = s.detach().contiguous()
    cy = m2.shape[0]
    d = make_desc(x.shape[0], spatial, x.shape[1], m1.shape[0], cy, skip=0 if s is None else m0.shape[0],
                  act_skip=act_skip, act_out=act_out, gate=g is not None, grid=grid, grid_offset=grid_offset)
    want = set(need) if need is not None else {"x", "s", "w0", "w1", "b1", "w2", "b2", "g", "gb"}
    dev = x.device
    e = lambda *shape: torch.empty(shape, device=dev, dtype=torch.float32)  # noqa: E731
    out = {
        "x": e(*x.shape) if "x" in want else None,
        "s": e(*s.shape) if s is not None and "s" in want else None,
        "w0": e(*m0.shape) if m0 is not None and "w0" in want else None,
        "w1": e(*m1.shape) if "w1" in want else None,
        "b1": e(m1.shape[0]) if "b1" in want else None,
        "w2": e(*m2.shape) if "w2" in want else None,
        "b2": e(cy) if "b2" in want else None,
        "g": e(cy) if g is not None and "g" in want else None,
        "gb": e(cy) if gb is not None and "gb" in want else None,
    }
    ops = NopChainOperands()
    for name, t in (("x", x), ("s", s), ("w0", m0), ("w1", m1), ("b1", v1), ("w2", m2), ("b2", v2), ("g", g),
                    ("gb", gb)):
        setattr(ops, name, None if t is None else t.data_ptr())
    grads = NopChainGrads()
    grads.dy = dy.data_ptr()
    for name, key in (("dx", "x"), ("ds", "s"), ("dw0", "w0"), ("dw1", "w1"), ("db1", "b1"), ("dw2", "w2"),
                      ("db2", "b2"), ("dg", "g"), ("dgb", "gb")):
        t = out[key]
        setattr(grads, name, None if t is None else t.data_ptr())
    lib = _lib.library()
    _declare(lib)
    size = ctypes.c_size_t()
    _lib.check(lib.nop_chain_backward_query(ctypes.byref(d), ctypes.byref(size)))
    ws = torch.empty(max(int(size.value), 1), device=dev, dtype=torch.uint8)
    with torch.cuda.device(dev):
        stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        _lib.check(lib.nop_chain_backward(ctypes.byref(d), ctypes.byref(ops), ctypes.byref(grads),
                                          ctypes.c_void_p(ws.data_ptr()), int(size.value), stream))
    return out


class _ChainFn(torch.autograd.Function):
    """One chain call (no projection) under autograd: the forward is the tensor-core kernel, the backward
    nop_chain_backward (the forward's intermediates recomputed from x and s)."""

    @staticmethod
    def forward(ctx, x, s, w0, w1, b1, w2, b2, gate_w, gate_b, cfg):
        act_skip, act_out, grid, grid_offset, _ = cfg
        with torch.no_grad():
            y = chain(x, w1, b1, w2, b2, s=s, w0=w0, act_skip=act_skip, act_out=act_out, gate_w=gate_w,
                      gate_b=gate_b, grid=grid, grid_offset=grid_offset)
        ctx.cfg = cfg
        ctx.save_for_backward(x, s, w0, w1, b1, w2, b2, gate_w, gate_b)
        return y

    @staticmethod
    def backward(ctx, gy):
        x, s, w0, w1, b1, w2, b2, gate_w, gate_b = ctx.saved_tensors
        act_skip, act_out, grid, grid_offset, relay = ctx.cfg
        names = ("x", "s", "w0", "w1", "b1", "w2", "b2", "g", "gb")
        need = [n for n, flag in zip(names, ctx.needs_input_grad[:9]) if flag]
        g = chain_backward(gy, x, w1, b1, w2, b2, s=s, w0=w0, act_skip=act_skip, act_out=act_out, gate_w=gate_w,
                           gate_b=gate_b, grid=grid, grid_offset=grid_offset, need=need)
        res = []
        for n, t in zip(names, (x, s, w0, w1, b1, w2, b2, gate_w, gate_b)):
            res.append(None if g.get(n) is None or t is None else g[n].view(t.shape).to(t.dtype))
        if relay is not None and res[0] is not None:
            relay.put(res[0])
            res[0] = None
        return (*res, None)


class GradRelay:
    """Hands dL/dx of one FNO block's chain call to the backward of the block's spectral convolution,
    which reads the same x and adds it in the epilogue of its dL/dx kernel: the two gradients of x then
    leave one kernel as one tensor, instead of autograd adding them in a separate pass over x.

    The spectral convolution's output feeds only the chain call, so its backward always runs after the
    chain's (it needs dL/ds); the chain then reports no gradient for x and the spectral backward's dL/dx
    is the whole of it."""

    __slots__ = ("grad",)

    def __init__(self):
        self.grad = None

    def put(self, g: torch.Tensor):
        self.grad = g

    def take(self) -> Optional[torch.Tensor]:
        g, self.grad = self.grad, None
        return g
