"""Fused per-pixel channel MLP (nop_pointwise_forward): the FNO layers around the spectral block.

``channel_mlp(x, fc1, fc2, ...)`` evaluates, in one pass over HBM,

    u = [x ; grid]                       (grid coordinates generated in the kernel, optional)
    y = act_out(fc2(act_hidden(fc1(u))) + g * r + gb)
    z = w3 y                             (optional)

with the reference modules' own parameters: ChannelMLP (neuralop/layers/channel_mlp.py:82-119),
SoftGating (neuralop/layers/skip_connections.py:53-94), the linear skip
(skip_connections.py:96-127) and GridEmbeddingND (neuralop/layers/embeddings.py:147-164).
``supported`` tells the caller whether the kernel takes a problem; callers keep the module path
otherwise.
"""

from __future__ import annotations

import ctypes
from typing import Optional, Sequence, Tuple

import torch

from . import _lib

MAX_DIMS = 4


class NopPointwiseDesc(ctypes.Structure):
    _fields_ = [
        ("abi_version", ctypes.c_int32),
        ("ndim", ctypes.c_int32),
        ("batch", ctypes.c_int64),
        ("spatial", ctypes.c_int64 * MAX_DIMS),
        ("in_channels", ctypes.c_int32),
        ("grid_dims", ctypes.c_int32),
        ("hidden_channels", ctypes.c_int32),
        ("out_channels", ctypes.c_int32),
        ("next_channels", ctypes.c_int32),
        ("act_hidden", ctypes.c_int32),
        ("act_out", ctypes.c_int32),
        ("gate", ctypes.c_int32),
        ("has_b1", ctypes.c_int32),
        ("has_b2", ctypes.c_int32),
        ("has_gate_bias", ctypes.c_int32),
        ("grid_lo", ctypes.c_float * MAX_DIMS),
        ("grid_hi", ctypes.c_float * MAX_DIMS),
    ]


def _declare(lib):
    if getattr(lib, "_pw_declared", False):
        return
    lib.nop_pointwise_smem_bytes.restype = ctypes.c_int32
    lib.nop_pointwise_smem_bytes.argtypes = [ctypes.POINTER(NopPointwiseDesc), ctypes.POINTER(ctypes.c_size_t)]
    lib.nop_pointwise_forward.restype = ctypes.c_int32
    lib.nop_pointwise_forward.argtypes = [ctypes.POINTER(NopPointwiseDesc)] + [ctypes.c_void_p] * 11 + \
        [ctypes.c_void_p]
    lib._pw_declared = True


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


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _desc(x, cin, hidden, cout, cnext, grid, act_hidden, act_out, gate, has_b1, has_b2, has_gb):
    d = NopPointwiseDesc()
    d.abi_version = _lib.ABI_VERSION
    d.ndim = x.ndim - 2
    d.batch = x.shape[0]
    for j, n in enumerate(x.shape[2:]):
        d.spatial[j] = n
    d.in_channels = cin
    d.grid_dims = 0 if grid is None else d.ndim
    if grid is not None:
        for j, (lo, hi) in enumerate(grid):
            d.grid_lo[j] = float(lo)
            d.grid_hi[j] = float(hi)
    d.hidden_channels = hidden
    d.out_channels = cout
    d.next_channels = cnext
    d.act_hidden = int(bool(act_hidden))
    d.act_out = int(bool(act_out))
    d.gate = int(bool(gate))
    d.has_b1 = int(bool(has_b1))
    d.has_b2 = int(bool(has_b2))
    d.has_gate_bias = int(bool(has_gb))
    return d


def supported_dims(batch: int, spatial: Sequence[int], cin: int, hidden: int, cout: int, cnext: int = 0,
                   grid=None) -> bool:
    """Whether the fused kernel takes a problem of these sizes (points per sample a multiple of 128,
    every channel count <= 256, the weights fitting one CTA's shared memory)."""
    if not 1 <= len(spatial) <= MAX_DIMS:
        return False
    pts = 1
    for n in spatial:
        pts *= int(n)
    if pts % 128:
        return False
    lib = _lib.library()
    _declare(lib)
    d = NopPointwiseDesc()
    d.abi_version = _lib.ABI_VERSION
    d.ndim = len(spatial)
    d.batch = int(batch)
    for j, n in enumerate(spatial):
        d.spatial[j] = int(n)
    d.in_channels, d.hidden_channels, d.out_channels, d.next_channels = cin, hidden, cout, cnext
    d.grid_dims = 0 if grid is None else d.ndim
    d.gate = 1  # counts the residual tile, the larger footprint
    size = ctypes.c_size_t()
    return lib.nop_pointwise_smem_bytes(ctypes.byref(d), ctypes.byref(size)) == _lib.NOP_OK


def supported(x: torch.Tensor, cin: int, hidden: int, cout: int, cnext: int = 0, grid=None) -> bool:
    """supported_dims for the CUDA fp32 tensor x (with cin channels)."""
    if not (x.is_cuda and x.dtype == torch.float32 and 3 <= x.ndim <= 2 + MAX_DIMS and x.shape[1] == cin):
        return False
    return supported_dims(x.shape[0], x.shape[2:], cin, hidden, cout, cnext, grid)


def channel_mlp(x: torch.Tensor, fc1_w: Optional[torch.Tensor], fc1_b: Optional[torch.Tensor],
                fc2_w: torch.Tensor, fc2_b: Optional[torch.Tensor], *, grid: Optional[Sequence] = None,
                act_hidden: bool = True, act_out: bool = False, residual: Optional[torch.Tensor] = None,
                gate_w: Optional[torch.Tensor] = None, gate_b: Optional[torch.Tensor] = None,
                next_w: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """(y, z) of the fused kernel on x's device and current stream (see the module docstring).

    ``fc1_w = None`` makes it a single layer y = act_out(fc2(u) + ...).  ``grid``: per-axis
    (lo, hi) boundaries of the coordinate channels appended to x, or None.
    """
    if not x.is_cuda:
        raise RuntimeError("neuraloperator_b200 runs on CUDA devices only (there is no CPU path)")
    if torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in
                                       (x, fc1_w, fc1_b, fc2_w, fc2_b, residual, gate_w, gate_b, next_w)):
        raise RuntimeError("the fused per-pixel kernel has no backward; call it under torch.no_grad() "
                           "(the FNO modules use their torch layers whenever a gradient is needed)")
    x = x.contiguous()
    w1, b1, w2, b2 = _mat(fc1_w), _vec(fc1_b), _mat(fc2_w), _vec(fc2_b)
    g, gb, w3 = _vec(gate_w), _vec(gate_b), _mat(next_w)
    cin = x.shape[1]
    hidden = 0 if w1 is None else w1.shape[0]
    cout = w2.shape[0]
    cnext = 0 if w3 is None else w3.shape[0]
    gate = residual is not None
    r = residual.contiguous() if gate else None
    if gate and g is None:
        raise ValueError("a residual needs gate weights")
    d = _desc(x, cin, hidden, cout, cnext, grid, act_hidden, act_out, gate, b1 is not None, b2 is not None,
              gb is not None)
    spatial = tuple(x.shape[2:])
    y = torch.empty((x.shape[0], cout, *spatial), device=x.device, dtype=torch.float32)
    z = torch.empty((x.shape[0], cnext, *spatial), device=x.device, dtype=torch.float32) if cnext else None
    lib = _lib.library()
    _declare(lib)
    stream = ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)
    with torch.cuda.device(x.device):
        _lib.check(lib.nop_pointwise_forward(ctypes.byref(d), _ptr(x), _ptr(w1), _ptr(b1), _ptr(w2), _ptr(b2),
                                             _ptr(r), _ptr(g), _ptr(gb), _ptr(w3), _ptr(y), _ptr(z), stream))
    return y, z
