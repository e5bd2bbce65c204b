"""FNOBlocks: drop-in for neuralop.layers.fno_block.FNOBlocks (neuralop/layers/fno_block.py:18-481).

Same constructor, parameters and forward semantics.  When the block has the FNO default
shape -- ``fno_skip="linear"``, real data, no norm, no stabilizer, GELU, post-activation,
a ``SpectralConv`` of this package and no output resampling -- the skip add and the GELU
(:356-361) run inside the spectral block's inverse-transform epilogue: the skip GEMM
(a 1x1 conv) is computed first and handed to the kernel as an addend.  Every other
configuration composes the same operations as the reference around the CUDA spectral block.
Normalisation layers other than None are not provided (norm=None is the FNO default).

With the default ChannelMLP (two layers, GELU, no dropout) and a soft-gating (or no) channel-MLP
skip, the rest of the block -- ChannelMLP, soft-gating skip, closing GELU (:363-381) -- and the next
block's linear skip run as one fused per-pixel kernel (``pointwise.channel_mlp``); the next block
then takes that skip instead of recomputing it.
"""

from __future__ import annotations

from typing import List, Union

import torch
import torch.nn.functional as F
from torch import nn

from . import pointwise
from .layers import ChannelMLP, SoftGating, skip_connection
from .spectral_convolution import SpectralConv
from .utils import get_active_profiler, grad_needed, maybe_profile, validate_scaling_factor

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
                and conv.resolution_scaling_factor is None and x.is_cuda and not grad_needed(x, self))

    def _mlp_fusable(self, index, x) -> bool:
        if not (self.use_channel_mlp and x.is_cuda and x.dtype == torch.float32):
            return False
        mlp = self.channel_mlp[index]
        sg = self.channel_mlp_skips[index] if self.channel_mlp_skips is not None else None
        if not (isinstance(mlp, ChannelMLP) and mlp.n_layers == 2 and mlp.dropout is None
                and mlp.non_linearity is F.gelu and (sg is None or isinstance(sg, SoftGating))):
            return False
        nxt = self.fno_skips[index + 1].conv.out_channels if index + 1 < self.n_layers else 0
        return pointwise.supported(x, self.out_channels, mlp.hidden_channels, mlp.out_channels, nxt)

    def next_skip_weight(self, index):
        """Weight [out, in, 1] of block `index`'s linear skip (None past the last block)."""
        return self.fno_skips[index].conv.weight if index < self.n_layers else None

    def set_pending_skip(self, x, index, skip):
        """Hand block `index` the linear skip of its input x computed by a fused kernel upstream."""
        self._pending_skip = (x, index, skip) if skip is not None else None

    def fused_block(self, x, index, skip=None):
        """Spectral block + skip add + GELU, then the fused ChannelMLP / soft-gating / GELU kernel, which
        also returns the next block's linear skip.  Returns (y, next block's skip or None)."""
        prof = get_active_profiler()
        prefix = f"fno_blocks/{index}"
        last = index >= self.n_layers - 1
        conv = self.convs[index]
        if skip is None:
            with maybe_profile(prof, f"{prefix}/fno_skip", x.device):
                skip, _ = pointwise.channel_mlp(x, None, None, self.fno_skips[index].conv.weight, None,
                                                act_hidden=False, act_out=False)
        with maybe_profile(prof, f"{prefix}/spectral_conv_skip_add_activation", x.device):
            s = conv(x, addend=skip, apply_gelu=not last)
        mlp = self.channel_mlp[index]
        sg = self.channel_mlp_skips[index] if self.channel_mlp_skips is not None else None
        with maybe_profile(prof, f"{prefix}/channel_mlp_skip_activation_next_skip", x.device):
            y, z = pointwise.channel_mlp(
                s, mlp.fcs[0].weight, mlp.fcs[0].bias, mlp.fcs[1].weight, mlp.fcs[1].bias, act_hidden=True,
                act_out=not last, residual=x if sg is not None else None,
                gate_w=sg.weight if sg is not None else None, gate_b=sg.bias if sg is not None else None,
                next_w=self.next_skip_weight(index + 1))
        return y, z

    def forward_with_postactivation(self, x, index=0, output_shape=None):
        if self._fusable(index, x, output_shape) and self._mlp_fusable(index, x):
            pending = getattr(self, "_pending_skip", None)
            skip = pending[2] if pending is not None and pending[0] is x and pending[1] == index else None
            self._pending_skip = None
            y, z = self.fused_block(x, index, skip)
            self.set_pending_skip(y, index + 1, z)
            return y
        self._pending_skip = None
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
