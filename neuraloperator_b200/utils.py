"""Host utilities mirroring neuralop.utils: scaling-factor validation, parameter count, and the test
for whether autograd will record a call."""

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
