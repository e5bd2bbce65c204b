"""Host utilities mirroring neuralop.utils: scaling-factor validation, parameter count, and the test
for whether autograd will record a call; the host-memory pipeline of the models' forward_host."""

from __future__ import annotations

from typing import Optional, Union

import torch

Number = Union[int, float]


def validate_scaling_factor(scaling_factor, n_dim: int, n_layers: Optional[int] = None):
    """Normalise a resolution scaling factor (neuralop/utils.py:154-199)."""
    if scaling_factor is None:
        return None
    if isinstance(scaling_factor, (float, int)):
        if n_layers is None:
            return [float(scaling_factor)] * n_dim
        return [[float(scaling_factor)] * n_dim] * n_layers
    if isinstance(scaling_factor, list) and scaling_factor and all(isinstance(s, (float, int))
                                                                    for s in scaling_factor):
        if n_layers is None and len(scaling_factor) == n_dim:
            return [float(s) for s in scaling_factor]
        return [[float(s)] * n_dim for s in scaling_factor]
    if isinstance(scaling_factor, list) and scaling_factor and all(isinstance(s, list) for s in scaling_factor):
        if all(all(isinstance(v, (int, float)) for v in s) for s in scaling_factor):
            return scaling_factor
    return None


def grad_needed(x: torch.Tensor, module: torch.nn.Module) -> bool:
    """True when autograd will record this call: grad mode on and x or a parameter of ``module``
    requires a gradient.  The fused per-pixel kernels and the fused GELU epilogue have no backward,
    so the models take their composable path (torch layers + SpectralConv's autograd) then."""
    if not torch.is_grad_enabled():
        return False
    return x.requires_grad or any(p.requires_grad for p in module.parameters())


def count_model_params(model) -> int:
    """Parameter count with complex entries counted twice (neuralop/utils.py:19-28)."""
    return sum(p.numel() * 2 if p.is_complex() else p.numel() for p in model.parameters())


def host_pipeline(fn, x: torch.Tensor, y: torch.Tensor, chunk: int, dev: torch.device, streams: dict,
                  n_buffers: int = 2) -> None:
    """y[k] = fn(x[k]) for the chunks of ``chunk`` samples of the pinned host tensors x / y, as a
    three-stage pipeline on three streams: host-to-device copies (running ahead by ``n_buffers`` chunks),
    ``fn`` on the device copies, device-to-host copies.  Chunk k's input copy overlaps chunk k - 1's
    kernels and chunk k - 2's output copy, so only the first input and the last output copy are not
    hidden.  Work is queued on the device's current stream (the caller synchronises).  ``streams``
    caches the three streams between calls."""
    cur = torch.cuda.current_stream(dev)
    key = (dev.index, "pipeline")
    if key not in streams:
        streams[key] = [torch.cuda.Stream(dev) for _ in range(3)]
    s_in, s_fn, s_out = streams[key]
    for st in (s_in, s_fn, s_out):
        st.wait_stream(cur)
    n = x.shape[0] // chunk
    bufs = [torch.empty((chunk, *x.shape[1:]), dtype=x.dtype, device=dev) for _ in range(min(n_buffers, n))]
    done_fn = []
    for k in range(n):
        b = bufs[k % len(bufs)]
        with torch.cuda.stream(s_in):
            if k >= len(bufs):
                s_in.wait_event(done_fn[k - len(bufs)])  # the kernels reading this buffer are done
            b.copy_(x[k * chunk:(k + 1) * chunk], non_blocking=True)
            ready = torch.cuda.Event()
            ready.record(s_in)
        with torch.cuda.stream(s_fn):
            s_fn.wait_event(ready)
            yd = fn(b)
            ev = torch.cuda.Event()
            ev.record(s_fn)
            done_fn.append(ev)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev)
            y[k * chunk:(k + 1) * chunk].copy_(yd, non_blocking=True)
            yd.record_stream(s_out)
    for b in bufs:
        b.record_stream(s_in)
        b.record_stream(s_fn)
    for st in (s_in, s_fn, s_out):
        cur.wait_stream(st)
