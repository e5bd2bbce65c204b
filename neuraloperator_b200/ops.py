"""Torch-facing wrapper of the C ABI: descriptor assembly, plan cache, launch.

PyTorch provides device memory (including the workspace, from its caching allocator) and
the current stream; all arithmetic runs in libnop_b200's CUDA kernels.
"""

from __future__ import annotations

import ctypes
import threading
from typing import List, Optional, Sequence

import torch

from . import _lib
from .geometry import Geometry

_KIND = {"dense": _lib.WEIGHT_DENSE, "tucker": _lib.WEIGHT_TUCKER, "cp": _lib.WEIGHT_CP}
_PREC = {"fp32": _lib.PRECISION_FP32, "bf16": _lib.PRECISION_BF16}
_ENGINE = {"auto": _lib.ENGINE_AUTO, "generic": _lib.ENGINE_GENERIC, "fast": _lib.ENGINE_FAST}

_plans = {}
_plans_lock = threading.Lock()


def make_desc(geo: Geometry, batch: int, in_channels: int, out_channels: int, *, weight_kind: str = "dense",
              ranks: Sequence[int] = (), separable: bool = False, precision: str = "fp32",
              engine: str = "auto") -> _lib.NopSpectralDesc:
    d = _lib.NopSpectralDesc()
    d.abi_version = _lib.ABI_VERSION
    d.ndim = geo.order
    d.complex_data = int(geo.complex_data)
    d.separable = int(separable)
    d.weight_kind = _KIND[weight_kind]
    d.precision = _PREC[precision]
    d.engine = _ENGINE[engine]
    d.batch = int(batch)
    d.in_channels = int(in_channels)
    d.out_channels = int(out_channels)
    for j in range(_lib.MAX_DIMS):
        if j < geo.order:
            d.n_in[j], d.n_out[j], d.kept[j] = geo.n_in[j], geo.n_out[j], geo.kept[j]
            d.fwd_off[j], d.inv_off[j] = geo.fwd_off[j], geo.inv_off[j]
        else:
            d.n_in[j] = d.n_out[j] = d.kept[j] = 1
    for i, r in enumerate(ranks):
        d.ranks[i] = int(r)
    zb = list(geo.zero_imag_bins)
    if len(zb) > 3:
        raise ValueError("at most three last-axis bins can be forced real")
    d.n_zero_imag = len(zb)
    for i, b in enumerate(zb):
        d.zero_imag_bins[i] = int(b)
    d.fwd_scale = float(geo.fwd_scale)
    d.inv_scale = float(geo.inv_scale)
    return d


def get_plan(desc: _lib.NopSpectralDesc, device_index: int) -> _lib.Plan:
    key = (device_index, bytes(desc))
    plan = _plans.get(key)
    if plan is None:
        with _plans_lock:
            plan = _plans.get(key)
            if plan is None:
                with torch.cuda.device(device_index):
                    plan = _lib.Plan(desc)
                _plans[key] = plan
    return plan


def clear_plans():
    with _plans_lock:
        _plans.clear()


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _weight_key(sources):
    """Identity of the weight tensors as the caller passed them (before any dtype / device /
    contiguity copy): storage address, version counter (shared with the base tensor for views, so an
    in-place update of a sliced parameter is seen), shape and strides."""
    return tuple((w.data_ptr(), w._version, w.dtype, tuple(w.shape), tuple(w.stride())) for w in sources)


def _packed_weights(plan, desc, ws, arr, dev, workspace, cache, stream, sources=None):
    """Packed weight buffer of a fused plan: reused from ``cache`` while the caller's weight tensors
    (``sources``, default ``ws``) keep their storage and version counter and the plan is the same
    (the packed layout is the plan's choice), else packed now (nop_spectral_pack_weights).

    The cache entry holds references to the source tensors: while it exists their storage cannot be
    freed and handed to a new tensor, so a weight rebuilt on every call (a reconstructed factorized
    weight, a copy of a non-contiguous slice) never matches a stale entry by address and version."""
    sources = list(ws if sources is None else sources)
    key = (bytes(desc), _weight_key(sources), plan.handle.value, plan.packed_bytes)
    entry = cache.get("packed") if cache is not None else None
    if entry is not None and entry[0] == key:
        return entry[1]
    packed = torch.empty(plan.packed_bytes, device=dev, dtype=torch.uint8)
    _lib.check(_lib.library().nop_spectral_pack_weights(plan.handle, arr, len(ws), _ptr(packed), plan.packed_bytes,
                                                        _ptr(workspace), plan.workspace_bytes, stream))
    if cache is not None:  # detached: the storage stays referenced, no autograd graph is kept alive
        cache["packed"] = (key, packed, [w.detach() for w in sources])
    return packed


def spectral_forward(x: torch.Tensor, geo: Geometry, weights: List[torch.Tensor], *, out_channels: int,
                     weight_kind: str = "dense", ranks: Sequence[int] = (), separable: bool = False,
                     bias: Optional[torch.Tensor] = None, addend: Optional[torch.Tensor] = None,
                     apply_gelu: bool = False, precision: str = "fp32", engine: str = "auto",
                     out: Optional[torch.Tensor] = None, cache: Optional[dict] = None,
                     keep_spectrum: bool = False, packed: Optional[torch.Tensor] = None):
    """Run one spectral-block forward on x's device and current stream.

    Fused-engine plans use packed weights (nop_spectral_pack_weights).  With ``cache`` (a dict
    owned by the calling module) the packed buffer is kept and reused while the weight tensors
    keep their storage and version counter; any in-place update or replacement repacks.
    With ``keep_spectrum`` the kept input spectrum is kept too (nop_spectral_forward_keep) and
    ``(y, Spectrum)`` is returned, for ``weight_grad``.  ``packed``: weights already packed for this
    call's plan (``weights`` is then unused).
    """
    if not x.is_cuda:
        raise RuntimeError("neuraloperator_b200 runs on CUDA devices only (there is no CPU path); "
                           f"got a tensor on {x.device}")
    dev = x.device
    want = torch.complex64 if geo.complex_data else torch.float32
    if x.dtype != want:
        raise TypeError(f"expected {want} input, got {x.dtype}")
    x = x.contiguous()
    ws = [w.detach().to(device=dev, dtype=torch.complex64).contiguous() for w in weights]
    b = None if bias is None else bias.detach().reshape(-1).to(device=dev, dtype=torch.float32).contiguous()
    a = None if addend is None else addend.detach().to(device=dev, dtype=torch.float32).contiguous()
    batch, ci = x.shape[0], x.shape[1]
    y_shape = (batch, out_channels, *geo.n_out)
    if a is not None and tuple(a.shape) != y_shape:
        raise ValueError(f"addend shape {tuple(a.shape)} != output shape {y_shape}")
    if b is not None and b.numel() != out_channels:
        raise ValueError(f"bias has {b.numel()} entries, expected {out_channels}")
    y = out if out is not None else torch.empty(y_shape, device=dev, dtype=want)
    desc = make_desc(geo, batch, ci, out_channels, weight_kind=weight_kind, ranks=ranks, separable=separable,
                     precision=precision, engine=engine)
    plan = get_plan(desc, dev.index if dev.index is not None else torch.cuda.current_device())
    workspace = torch.empty(max(plan.workspace_bytes, 1), device=dev, dtype=torch.uint8)
    arr = (ctypes.c_void_p * len(ws))(*[w.data_ptr() for w in ws])
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    lib = _lib.library()
    spec = None
    if keep_spectrum:
        spec = torch.empty(max(plan.spectrum_bytes, 1), device=dev, dtype=torch.uint8)
    with torch.cuda.device(dev):
        if packed is None and plan.packed_bytes > 0:
            packed = _packed_weights(plan, desc, ws, arr, dev, workspace, cache, stream, sources=weights)
        if spec is not None:
            _lib.check(lib.nop_spectral_forward_keep(
                plan.handle, _ptr(x), None if packed is not None else arr, 0 if packed is not None else len(ws),
                _ptr(packed), plan.packed_bytes if packed is not None else 0, _ptr(b), _ptr(a),
                int(bool(apply_gelu)), _ptr(y), _ptr(spec), plan.spectrum_bytes, _ptr(workspace),
                plan.workspace_bytes, stream))
        elif packed is not None:
            _lib.check(lib.nop_spectral_forward_packed(
                plan.handle, _ptr(x), _ptr(packed), plan.packed_bytes, _ptr(b), _ptr(a), int(bool(apply_gelu)),
                _ptr(y), _ptr(workspace), plan.workspace_bytes, stream))
        else:
            _lib.check(lib.nop_spectral_forward(
                plan.handle, _ptr(x), arr, len(ws), _ptr(b), _ptr(a), int(bool(apply_gelu)), _ptr(y),
                _ptr(workspace), plan.workspace_bytes, stream))
    if keep_spectrum:
        return y, Spectrum(plan, spec)
    return y


class Spectrum:
    """Kept input spectrum left by a forward (``spectral_forward(..., keep_spectrum=True)``), with the
    plan whose layout it follows (nop_spectral_spectrum_layout)."""

    def __init__(self, plan, buf: torch.Tensor):
        self.plan = plan
        self.buf = buf


def _conj_copy(t: torch.Tensor, dims=None) -> torch.Tensor:
    """Contiguous conj(t) (with dims 0 and 1 swapped when ``dims`` is "T"), in one copy kernel."""
    src = t.transpose(0, 1) if dims == "T" else t
    out = torch.empty(src.shape, dtype=t.dtype, device=t.device)
    out.copy_(src.conj())
    return out


def adjoint_operands(kind: str, weights: List[torch.Tensor], ranks: Sequence[int], separable: bool):
    """Weight operands of the adjoint contraction W'[o, i, m] = conj(W[i, o, m]), in the same kind.

    Dense: the conjugate transpose.  Tucker (core [r_in, r_out, r_1..], U_in, U_out, U_1..): core with its
    first two modes swapped, in- and out-factors swapped, all conjugated.  CP (lambda, U_in, U_out, U_1..):
    in- and out-factors swapped, all conjugated.  Separable weights are diagonal: conjugated only.
    Returns (weights, ranks).
    """
    ws = [w.detach() for w in weights]
    if separable:
        return [_conj_copy(w) for w in ws], tuple(ranks)
    if kind == "dense":
        return [_conj_copy(ws[0], "T")], ()
    if kind == "tucker":
        core, u_in, u_out, *spatial = ws
        r = list(ranks)
        return ([_conj_copy(core, "T"), _conj_copy(u_out), _conj_copy(u_in)] + [_conj_copy(u) for u in spatial],
                tuple([r[1], r[0]] + r[2:]))
    if kind == "cp":
        lam, u_in, u_out, *spatial = ws
        return [_conj_copy(lam), _conj_copy(u_out), _conj_copy(u_in)] + [_conj_copy(u) for u in spatial], tuple(ranks)
    raise ValueError(f"unknown weight kind {kind!r}")


def pack_adjoint_dense(geo_adj: Geometry, batch: int, weight: torch.Tensor, *, precision: str = "fp32",
                       engine: str = "auto") -> Optional[torch.Tensor]:
    """Packed weights of the adjoint plan straight from the forward's dense weight [Ci, Co, kept...]
    (nop_spectral_pack_weights_adjoint), or None when that plan takes its weights unpacked."""
    ci, co = weight.shape[0], weight.shape[1]
    dev = weight.device
    desc = make_desc(geo_adj, batch, co, ci, weight_kind="dense", precision=precision, engine=engine)
    plan = get_plan(desc, dev.index if dev.index is not None else torch.cuda.current_device())
    if plan.packed_bytes == 0:
        return None
    w = weight.detach().to(torch.complex64).contiguous()
    packed = torch.empty(plan.packed_bytes, device=dev, dtype=torch.uint8)
    with torch.cuda.device(dev):
        stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        _lib.check(_lib.library().nop_spectral_pack_weights_adjoint(plan.handle, _ptr(w), _ptr(packed),
                                                                    plan.packed_bytes, stream))
    return packed


def weight_grad(fwd: Spectrum, adj: Spectrum, grad_w_shape: Optional[Sequence[int]], bias_channels: int = 0):
    """dL/dW (dense-equivalent, ``grad_w_shape`` complex64, or None) and dL/dbias ([bias_channels] float32,
    or None when 0) from the kept spectra of x (forward plan) and of dL/dy (adjoint plan)
    (nop_spectral_weight_grad)."""
    dev = fwd.buf.device
    gw = None if grad_w_shape is None else torch.empty(tuple(grad_w_shape), device=dev, dtype=torch.complex64)
    gb = torch.empty(bias_channels, device=dev, dtype=torch.float32) if bias_channels else None
    if gw is None and gb is None:
        return None, None
    lib = _lib.library()
    size = ctypes.c_size_t()
    _lib.check(lib.nop_spectral_weight_grad_workspace_size(fwd.plan.handle, ctypes.byref(size)))
    ws = torch.empty(int(size.value), device=dev, dtype=torch.uint8) if size.value else None
    with torch.cuda.device(dev):
        stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        _lib.check(lib.nop_spectral_weight_grad(fwd.plan.handle, _ptr(fwd.buf), adj.plan.handle, _ptr(adj.buf),
                                                _ptr(gw), _ptr(gb), _ptr(ws), int(size.value), stream))
    return gw, gb


def tucker_grads(core: torch.Tensor, factors: List[torch.Tensor], gw: torch.Tensor) -> List[torch.Tensor]:
    """[dL/dcore, dL/dU_0, ..., dL/dU_{n-1}] of the Tucker weight W = core x_0 U_0 ... x_{n-1} U_{n-1} given
    dL/dW = ``gw`` (complex64 CUDA tensors; nop_tucker_grads): the values autograd through the
    reconstruction einsum (neuralop/layers/spectral_convolution.py:76-103) gives."""
    if not gw.is_cuda:
        raise RuntimeError("neuraloperator_b200 runs on CUDA devices only (there is no CPU path)")
    n = len(factors)
    dev = gw.device
    c64 = lambda t: t.detach().to(device=dev, dtype=torch.complex64).contiguous()  # noqa: E731
    core, facs, gw = c64(core), [c64(u) for u in factors], c64(gw)
    dims = (ctypes.c_int64 * n)(*[u.shape[0] for u in facs])
    ranks = (ctypes.c_int64 * n)(*[u.shape[1] for u in facs])
    if tuple(gw.shape) != tuple(dims) or tuple(core.shape) != tuple(ranks):
        raise ValueError(f"grad_w {tuple(gw.shape)} / core {tuple(core.shape)} do not match the factors' "
                         f"sizes {tuple(dims)} / ranks {tuple(ranks)}")
    g_core = torch.empty_like(core)
    g_fac = [torch.empty_like(u) for u in facs]
    lib = _lib.library()
    size = ctypes.c_size_t()
    _lib.check(lib.nop_tucker_grads_workspace_size(n, dims, ranks, ctypes.byref(size)))
    ws = torch.empty(int(size.value), device=dev, dtype=torch.uint8)
    fptr = (ctypes.c_void_p * n)(*[u.data_ptr() for u in facs])
    gptr = (ctypes.c_void_p * n)(*[g.data_ptr() for g in g_fac])
    with torch.cuda.device(dev):
        stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        _lib.check(lib.nop_tucker_grads(n, dims, ranks, _ptr(core), fptr, _ptr(gw), _ptr(g_core), gptr, _ptr(ws),
                                        int(size.value), stream))
    return [g_core] + g_fac


def default_chunk(batch: int, target_chunks: int = 8) -> int:
    """Largest divisor of ``batch`` that cuts it into at least ``target_chunks`` chunks (or 1)."""
    limit = max(1, batch // target_chunks)
    return max(c for c in range(1, limit + 1) if batch % c == 0)


def spectral_forward_host(x: torch.Tensor, geo: Geometry, weights: List[torch.Tensor], *, out_channels: int,
                          device: torch.device, weight_kind: str = "dense", ranks: Sequence[int] = (),
                          separable: bool = False, bias: Optional[torch.Tensor] = None,
                          addend: Optional[torch.Tensor] = None, apply_gelu: bool = False, precision: str = "fp32",
                          engine: str = "auto", chunk: Optional[int] = None, n_streams: int = 3,
                          out: Optional[torch.Tensor] = None, cache: Optional[dict] = None,
                          synchronize: bool = True) -> torch.Tensor:
    """Forward of a batch held in HOST memory (nop_spectral_forward_host).

    The batch is cut into chunks of ``chunk`` samples; each chunk's host-to-device copy, kernels and
    device-to-host copy run on one of ``n_streams`` streams so that transfers in both directions
    overlap with each other and with the kernels.  ``x`` / ``addend`` / ``out`` are CPU tensors
    (page-locked for the overlap; the returned tensor is page-locked when ``out`` is None); the
    weights and bias live on ``device``.  With ``synchronize=False`` the call returns once the work
    is queued on the current stream of ``device`` and the caller synchronises before reading the result.
    """
    if x.is_cuda:
        raise ValueError("spectral_forward_host takes a host tensor; use spectral_forward for device tensors")
    dev = torch.device(device)
    want = torch.complex64 if geo.complex_data else torch.float32
    if x.dtype != want:
        raise TypeError(f"expected {want} input, got {x.dtype}")
    x = x.contiguous()
    batch, ci = x.shape[0], x.shape[1]
    chunk = default_chunk(batch) if chunk is None else int(chunk)
    if chunk < 1 or batch % chunk:
        raise ValueError(f"chunk {chunk} does not divide the batch {batch}")
    y_shape = (batch, out_channels, *geo.n_out)
    a = None
    if addend is not None:
        if addend.is_cuda or tuple(addend.shape) != y_shape:
            raise ValueError(f"addend must be a host tensor of shape {y_shape}")
        a = addend.detach().to(torch.float32).contiguous()
    ws = [w.detach().to(device=dev, dtype=torch.complex64).contiguous() for w in weights]
    b = None if bias is None else bias.detach().reshape(-1).to(device=dev, dtype=torch.float32).contiguous()
    if b is not None and b.numel() != out_channels:
        raise ValueError(f"bias has {b.numel()} entries, expected {out_channels}")
    y = out if out is not None else torch.empty(y_shape, dtype=want, pin_memory=True)
    if y.is_cuda or tuple(y.shape) != y_shape or not y.is_contiguous():
        raise ValueError(f"out must be a contiguous host tensor of shape {y_shape}")
    desc = make_desc(geo, chunk, ci, out_channels, weight_kind=weight_kind, ranks=ranks, separable=separable,
                     precision=precision, engine=engine)
    plan = get_plan(desc, dev.index if dev.index is not None else torch.cuda.current_device())
    lib = _lib.library()
    size = ctypes.c_size_t()
    _lib.check(lib.nop_spectral_host_workspace_size(plan.handle, int(n_streams), ctypes.byref(size)))
    arr = (ctypes.c_void_p * len(ws))(*[w.data_ptr() for w in ws])
    with torch.cuda.device(dev):
        stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        workspace = torch.empty(max(int(size.value), 1), device=dev, dtype=torch.uint8)
        packed = None
        if plan.packed_bytes > 0:
            pack_ws = torch.empty(max(plan.workspace_bytes, 1), device=dev, dtype=torch.uint8)
            packed = _packed_weights(plan, desc, ws, arr, dev, pack_ws, cache, stream, sources=weights)
        _lib.check(lib.nop_spectral_forward_host(
            plan.handle, _ptr(x), batch, None if packed is not None else arr, 0 if packed is not None else len(ws),
            _ptr(packed), plan.packed_bytes if packed is not None else 0, _ptr(b), _ptr(a), int(bool(apply_gelu)),
            _ptr(y), _ptr(workspace), int(size.value), int(n_streams), stream))
        if synchronize:
            torch.cuda.current_stream(dev).synchronize()
    return y
