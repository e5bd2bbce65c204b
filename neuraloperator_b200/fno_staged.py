"""FNOStaged: drop-in for neuralop.models.FNOStaged (neuralop/models/fno_staged.py:24-502).

An FNO whose spectral layers each keep their own number of Fourier modes (``n_modes_per_layer``,
optionally ``max_n_modes_per_layer``), so later layers can carry fewer spectral parameters.  The block
computation is FNOBlocks' (fno_staged.py:318-440 repeats neuralop/layers/fno_block.py:327-414 per
layer), so this module is an FNO whose block stack holds one SpectralConv per layer with that layer's
modes; every layer runs on the same CUDA kernels (and, with the default layer shapes, the same fused
per-pixel kernels) as FNO.

The reference keeps the per-layer modules at the top level (``convs``, ``fno_skips``, ``channel_mlp``,
``channel_mlp_skips``); ``load_state_dict`` accepts those keys (and this module's own), so reference
checkpoints load unchanged.  ``no_br=True`` (bit-reversed spatial layout with ButterflySpectralConv, a
different spectral path) raises NotImplementedError.
"""

from __future__ import annotations

from typing import List, Optional, Tuple, Union

import torch.nn.functional as F
from torch import nn

from .fno import FNO
from .spectral_convolution import SpectralConv

Number = Union[float, int]

_BLOCK_PREFIXES = ("convs.", "fno_skips.", "channel_mlp.", "channel_mlp_skips.", "norm.")


class FNOStaged(FNO):
    def __init__(self, n_modes_per_layer: List[Tuple[int, ...]], in_channels: int, out_channels: int,
                 hidden_channels: int, n_layers: Optional[int] = None,
                 max_n_modes_per_layer: Optional[List[Tuple[int, ...]]] = None, lifting_channel_ratio: Number = 2,
                 projection_channel_ratio: Number = 2, positional_embedding: Union[str, nn.Module] = "grid",
                 non_linearity: nn.Module = F.gelu, norm=None, norm_groups: int = 1, complex_data: bool = False,
                 use_channel_mlp: bool = True, channel_mlp_dropout: float = 0, channel_mlp_expansion: float = 0.5,
                 channel_mlp_skip="soft-gating", fno_skip="linear",
                 resolution_scaling_factor: Union[Number, List[Number]] = None,
                 domain_padding: Union[Number, List[Number]] = None, fno_block_precision: str = "full",
                 stabilizer: str = None, factorization: str = None, rank: float = 1.0,
                 fixed_rank_modes: bool = False, implementation: str = "factorized",
                 decomposition_kwargs: dict = None, separable: bool = False, preactivation: bool = False,
                 conv_module: nn.Module = SpectralConv, enforce_hermitian_symmetry: bool = True, no_br: bool = False,
                 contraction_precision: str = "fp32", engine: str = "auto"):
        if n_layers is not None and n_layers != len(n_modes_per_layer):
            raise ValueError(f"Got n_layers={n_layers} but n_modes_per_layer has length {len(n_modes_per_layer)}")
        if no_br:
            raise NotImplementedError("no_br=True (bit-reversed layout with ButterflySpectralConv) is a different "
                                      "spectral path and is not provided")
        modes = [tuple(int(v) for v in m) for m in n_modes_per_layer]
        if max_n_modes_per_layer is None:
            max_n_modes_per_layer = modes
        if len(max_n_modes_per_layer) != len(modes):
            raise ValueError("max_n_modes_per_layer must be None or have the same length as n_modes_per_layer")
        max_modes = [tuple(int(v) for v in m) for m in max_n_modes_per_layer]
        if decomposition_kwargs is None:
            decomposition_kwargs = {}
        super().__init__(
            n_modes=modes[0], in_channels=in_channels, out_channels=out_channels, hidden_channels=hidden_channels,
            n_layers=len(modes), lifting_channel_ratio=lifting_channel_ratio,
            projection_channel_ratio=projection_channel_ratio, positional_embedding=positional_embedding,
            non_linearity=non_linearity, norm=norm, norm_groups=norm_groups, complex_data=complex_data,
            use_channel_mlp=use_channel_mlp, channel_mlp_dropout=channel_mlp_dropout,
            channel_mlp_expansion=channel_mlp_expansion, channel_mlp_skip=channel_mlp_skip, fno_skip=fno_skip,
            resolution_scaling_factor=resolution_scaling_factor, domain_padding=domain_padding,
            fno_block_precision=fno_block_precision, stabilizer=stabilizer, max_n_modes=max_modes[0],
            factorization=factorization, rank=rank, fixed_rank_modes=fixed_rank_modes,
            implementation=implementation, decomposition_kwargs=decomposition_kwargs, separable=separable,
            preactivation=preactivation, conv_module=conv_module,
            enforce_hermitian_symmetry=enforce_hermitian_symmetry, contraction_precision=contraction_precision,
            engine=engine)
        self.no_br = no_br
        self.n_modes_per_layer = [list(m) for m in modes]
        self.max_n_modes_per_layer = [list(m) for m in max_modes]
        # one spectral layer per stage, built with the arguments the reference passes (fno_staged.py:162-191)
        ours = isinstance(conv_module, type) and issubclass(conv_module, SpectralConv)
        extra = {"enforce_hermitian_symmetry": enforce_hermitian_symmetry} if ours else {}
        if ours:
            extra.update(contraction_precision=contraction_precision, engine=engine)
        blocks = self.fno_blocks
        scaling = blocks.resolution_scaling_factor
        blocks.convs = nn.ModuleList([
            conv_module(hidden_channels, hidden_channels, n_modes=modes[i], max_n_modes=max_modes[i],
                        resolution_scaling_factor=scaling[i] if scaling is not None else None, rank=rank,
                        fixed_rank_modes=fixed_rank_modes, implementation=implementation, separable=separable,
                        factorization=factorization, fno_block_precision=fno_block_precision,
                        decomposition_kwargs=decomposition_kwargs, complex_data=complex_data, **extra)
            for i in range(len(modes))])

    @property
    def n_modes(self):
        """Per-layer active modes (FNO's constructor reads the first layer's before the blocks exist)."""
        if "fno_blocks" not in self._modules:
            return self._n_modes
        return [list(c.n_modes) for c in self.fno_blocks.convs]

    @n_modes.setter
    def n_modes(self, n_modes_per_layer):
        if len(n_modes_per_layer) != self.n_layers:
            raise ValueError(f"expected {self.n_layers} per-layer mode tuples, got {len(n_modes_per_layer)}")
        for conv, m in zip(self.fno_blocks.convs, n_modes_per_layer):
            conv.n_modes = m
        self.n_modes_per_layer = [list(m) for m in n_modes_per_layer]

    def load_state_dict(self, state_dict, strict=True, assign=False):
        """Accepts the reference's keys (per-layer modules at the top level) and this module's own."""
        mapped = {}
        for k, v in state_dict.items():
            if k == "_metadata":
                continue
            mapped["fno_blocks." + k if k.startswith(_BLOCK_PREFIXES) else k] = v
        return nn.Module.load_state_dict(self, mapped, strict=strict, assign=assign)
