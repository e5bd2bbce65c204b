"""FNOBlocks: drop-in for neuralop.layers.fno_block.FNOBlocks (neuralop/layers/fno_block.py:18-481).

Same constructor, parameters and forward semantics.  When the block has the FNO default
shape -- ``fno_skip="linear"``, real data, no norm, no stabilizer, GELU, post-activation,
a ``SpectralConv`` of this package and no output resampling -- the skip add and the GELU
(:356-361) run inside the spectral block's inverse-transform epilogue: the skip GEMM
(a 1x1 conv) is computed first and handed to the kernel as an addend.  Every other
configuration composes the same operations as the reference around the CUDA spectral block.
Normalisation layers other than None are not provided (norm=None is the FNO default).
"""

from __future__ import annotations

from typing import List, Union

import torch
import torch.nn.functional as F
from torch import nn

from .layers import ChannelMLP, skip_connection
from .spectral_convolution import SpectralConv
from .utils import get_active_profiler, maybe_profile, validate_scaling_factor

Number = Union[int, float]


class FNOBlocks(nn.Module):
    def __init__(self, in_channels, out_channels, n_modes, resolution_scaling_factor=None, n_layers=1,
                 max_n_modes=None, fno_block_precision="full", use_channel_mlp=True, channel_mlp_dropout=0,
                 channel_mlp_expansion=0.5, non_linearity=F.gelu, stabilizer=None, norm=None, norm_groups=1,
                 ada_in_features=None, preactivation=False, fno_skip="linear", channel_mlp_skip="soft-gating",
                 complex_data=False, separable=False, factorization=None, rank=1.0, conv_module=SpectralConv,
                 fixed_rank_modes=False, implementation="factorized", decomposition_kwargs=dict(),
                 enforce_hermitian_symmetry=True, contraction_precision="fp32", engine="auto"):
        super().__init__()
        if isinstance(n_modes, int):
            n_modes = [n_modes]
        self._n_modes = n_modes
        self.n_dim = len(n_modes)
        self.resolution_scaling_factor = validate_scaling_factor(resolution_scaling_factor, self.n_dim, n_layers)
        self.max_n_modes = max_n_modes
        self.fno_block_precision = fno_block_precision
        self.in_channels = in_channels
        self.out_channels = out_channels
        self.n_layers = n_layers
        self.stabilizer = stabilizer
        self.rank = rank
        self.factorization = factorization
        self.fixed_rank_modes = fixed_rank_modes
        self.decomposition_kwargs = decomposition_kwargs
        self.fno_skip = fno_skip
        self.channel_mlp_skip = channel_mlp_skip
        self.complex_data = complex_data
        self.use_channel_mlp = use_channel_mlp
        self.channel_mlp_expansion = channel_mlp_expansion
        self.channel_mlp_dropout = channel_mlp_dropout
        self.implementation = implementation
        self.separable = separable
        self.preactivation = preactivation
        self.ada_in_features = ada_in_features
        self.enforce_hermitian_symmetry = enforce_hermitian_symmetry
        if complex_data:
            raise NotImplementedError("FNOBlocks with complex_data is not provided; SpectralConv supports "
                                      "complex data on its own")
        if norm is not None:
            raise NotImplementedError(f"norm={norm!r} is not provided (the FNO default is norm=None)")
        self.norm = None
        self.n_norms = 2
        self.non_linearity = non_linearity
        ours = isinstance(conv_module, type) and issubclass(conv_module, SpectralConv)
        extra = {"enforce_hermitian_symmetry": enforce_hermitian_symmetry} if ours else {}
        if ours:
            extra.update(contraction_precision=contraction_precision, engine=engine)
        self.convs = nn.ModuleList([
            conv_module(self.in_channels, self.out_channels, self.n_modes,
                        resolution_scaling_factor=(self.resolution_scaling_factor[i]
                                                   if resolution_scaling_factor is not None else None),
                        max_n_modes=max_n_modes, rank=rank, fixed_rank_modes=fixed_rank_modes,
                        implementation=implementation, separable=separable, factorization=factorization,
                        fno_block_precision=fno_block_precision, decomposition_kwargs=decomposition_kwargs,
                        complex_data=complex_data, **extra)
            for i in range(n_layers)])
        for i, conv in enumerate(self.convs):
            setattr(conv, "profile_prefix", f"fno_blocks/{i}/spectral_conv")
        self.fno_skips = (nn.ModuleList([skip_connection(self.in_channels, self.out_channels, skip_type=fno_skip,
                                                         n_dim=self.n_dim) for _ in range(n_layers)])
                          if fno_skip is not None else None)
        if use_channel_mlp:
            self.channel_mlp = nn.ModuleList([
                ChannelMLP(in_channels=self.out_channels, hidden_channels=round(self.out_channels * channel_mlp_expansion),
                           dropout=channel_mlp_dropout, n_dim=self.n_dim) for _ in range(n_layers)])
            self.channel_mlp_skips = (nn.ModuleList([
                skip_connection(self.in_channels, self.out_channels, skip_type=channel_mlp_skip, n_dim=self.n_dim)
                for _ in range(n_layers)]) if channel_mlp_skip is not None else None)

    def forward(self, x, index=0, output_shape=None):
        if self.preactivation:
            return self.forward_with_preactivation(x, index, output_shape)
        return self.forward_with_postactivation(x, index, output_shape)

    def _fusable(self, index, x, output_shape) -> bool:
        conv = self.convs[index]
        return (isinstance(conv, SpectralConv) and self.fno_skip is not None and self.fno_skip.lower() == "linear"
                and self.stabilizer is None and self.non_linearity is F.gelu and output_shape is None
                and conv.resolution_scaling_factor is None and x.is_cuda)

    def forward_with_postactivation(self, x, index=0, output_shape=None):
        prof = get_active_profiler()
        prefix = f"fno_blocks/{index}"
        last = index >= self.n_layers - 1
        if self.use_channel_mlp and self.channel_mlp_skips is not None:
            with maybe_profile(prof, f"{prefix}/channel_mlp_skip", x.device):
                x_skip_mlp = self.channel_mlp_skips[index](x)
                x_skip_mlp = self.convs[index].transform(x_skip_mlp, output_shape=output_shape)
        if self._fusable(index, x, output_shape):
            with maybe_profile(prof, f"{prefix}/fno_skip", x.device):
                x_skip = self.fno_skips[index](x)
            with maybe_profile(prof, f"{prefix}/spectral_conv_skip_add_activation", x.device):
                x = self.convs[index](x, addend=x_skip, apply_gelu=not last)
        else:
            if self.fno_skips is not None:
                with maybe_profile(prof, f"{prefix}/fno_skip", x.device):
                    x_skip = self.fno_skips[index](x)
                    x_skip = self.convs[index].transform(x_skip, output_shape=output_shape)
            if self.stabilizer == "tanh":
                x = torch.tanh(x)
            with maybe_profile(prof, f"{prefix}/spectral_conv", x.device):
                x_fno = self.convs[index](x, output_shape=output_shape)
            x = x_fno + x_skip if self.fno_skips is not None else x_fno
            if not last:
                x = self.non_linearity(x)
        if self.use_channel_mlp:
            with maybe_profile(prof, f"{prefix}/channel_mlp", x.device):
                x = self.channel_mlp[index](x)
                if self.channel_mlp_skips is not None:
                    x = x + x_skip_mlp
        if not last:
            with maybe_profile(prof, f"{prefix}/activation_1", x.device):
                x = self.non_linearity(x)
        return x

    def forward_with_preactivation(self, x, index=0, output_shape=None):
        x = self.non_linearity(x)
        if self.fno_skips is not None:
            x_skip = self.convs[index].transform(self.fno_skips[index](x), output_shape=output_shape)
        if self.use_channel_mlp and self.channel_mlp_skips is not None:
            x_skip_mlp = self.convs[index].transform(self.channel_mlp_skips[index](x), output_shape=output_shape)
        if self.stabilizer == "tanh":
            x = torch.tanh(x)
        x_fno = self.convs[index](x, output_shape=output_shape)
        x = x_fno + x_skip if self.fno_skips is not None else x_fno
        if index < self.n_layers - 1:
            x = self.non_linearity(x)
        if self.use_channel_mlp:
            x = self.channel_mlp[index](x)
            if self.channel_mlp_skips is not None:
                x = x + x_skip_mlp
        return x

    @property
    def n_modes(self):
        return self._n_modes

    @n_modes.setter
    def n_modes(self, n_modes):
        for i in range(self.n_layers):
            self.convs[i].n_modes = n_modes
        self._n_modes = n_modes
