"""Host utilities mirroring neuralop.utils: scaling-factor validation and section timing.

``TimingProfiler`` / ``profiling`` / ``maybe_profile`` keep the reference's section names
(``fno/lifting``, ``fno_blocks/{i}/...``; neuralop/utils.py:232-366) so timings line up with
the reference's own profiler output.  CUDA sections are timed with events on the current
stream.
"""

from __future__ import annotations

import contextvars
import time
from contextlib import contextmanager, nullcontext
from typing import List, Optional, Union

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


_ACTIVE = contextvars.ContextVar("neuraloperator_b200_active_profiler", default=None)


class TimingStat:
    def __init__(self):
        self.total_s = 0.0
        self.count = 0

    def update(self, duration_s: float):
        self.total_s += duration_s
        self.count += 1


class TimingProfiler:
    """Accumulates wall / CUDA-event time per named section."""

    def __init__(self):
        self._stats = {}

    def reset(self):
        self._stats = {}

    def record(self, name: str, duration_s: float):
        self._stats.setdefault(name, TimingStat()).update(duration_s)

    def section(self, name: str, device: Optional[torch.device] = None):
        return _Section(self, name, device)

    @property
    def stats(self):
        return dict(self._stats)

    def _grouped(self, depth: Optional[int]):
        if depth is None:
            return self._stats
        out = {}
        for name, st in self._stats.items():
            parts = name.split("/")
            key = "/".join(parts[:depth]) if len(parts) >= depth else name
            agg = out.setdefault(key, TimingStat())
            agg.total_s += st.total_s
            agg.count += st.count
        return out

    def summary(self, title: Optional[str] = None, sort_by: str = "total", group_depth: Optional[int] = None):
        stats = self._grouped(group_depth)
        total = sum(s.total_s for s in stats.values())
        items = sorted(stats.items(), key=(lambda kv: kv[0]) if sort_by == "name" else (lambda kv: -kv[1].total_s))
        lines = [title] if title else []
        header = "section | total(s) | avg(ms) | pct | count"
        lines += [header, "-" * len(header)]
        for name, st in items:
            avg = st.total_s / st.count * 1e3 if st.count else 0.0
            pct = st.total_s / total * 100 if total else 0.0
            lines.append(f"{name} | {st.total_s:.4f} | {avg:.3f} | {pct:5.1f}% | {st.count}")
        return "\n".join(lines)


class _Section:
    def __init__(self, prof: TimingProfiler, name: str, device):
        self._prof, self._name, self._device = prof, name, device
        self._t0 = self._e0 = self._e1 = None

    def __enter__(self):
        if self._device is not None and torch.device(self._device).type == "cuda":
            self._e0 = torch.cuda.Event(enable_timing=True)
            self._e1 = torch.cuda.Event(enable_timing=True)
            self._e0.record()
        else:
            self._t0 = time.perf_counter()
        return self

    def __exit__(self, *exc):
        if self._e0 is not None:
            self._e1.record()
            self._e1.synchronize()
            dt = self._e0.elapsed_time(self._e1) / 1e3
        else:
            dt = time.perf_counter() - self._t0
        self._prof.record(self._name, dt)
        return False


@contextmanager
def profiling(profiler: TimingProfiler):
    token = _ACTIVE.set(profiler)
    try:
        yield profiler
    finally:
        _ACTIVE.reset(token)


def get_active_profiler() -> Optional[TimingProfiler]:
    return _ACTIVE.get()


def maybe_profile(profiler: Optional[TimingProfiler], name: str, device=None):
    return nullcontext() if profiler is None else profiler.section(name, device)
