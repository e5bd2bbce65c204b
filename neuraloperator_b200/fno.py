"""FNO / TFNO: drop-ins for neuralop.models.FNO and TFNO (neuralop/models/fno.py:26-485).

Same constructor arguments and forward: grid embedding -> lifting ChannelMLP -> n_layers x
FNOBlocks -> projection ChannelMLP.  The spectral blocks run on libnop_b200's CUDA kernels; with
the default layer shapes the grid embedding + lifting (which also emits the first block's linear
skip) and the projection each run as one fused per-pixel kernel (``pointwise.channel_mlp``).
Options the reference offers outside the FNO default path raise NotImplementedError here:
``domain_padding``, ``norm``, ``complex_data`` and ``fno_block_precision`` other than "full".
"""

from __future__ import annotations

from typing import List, Tuple, Union

import torch
import torch.nn.functional as F
from torch import nn

from . import pointwise
from .fno_block import FNOBlocks
from .layers import ChannelMLP, GridEmbeddingND
from .spectral_convolution import SpectralConv
from .utils import get_active_profiler, grad_needed, maybe_profile

Number = Union[float, int]


class FNO(nn.Module):
    def __init__(self, n_modes: Tuple[int, ...], in_channels: int, out_channels: int, hidden_channels: int,
                 n_layers: int = 4, lifting_channel_ratio: Number = 2, projection_channel_ratio: Number = 2,
                 positional_embedding: Union[str, nn.Module] = "grid", non_linearity: nn.Module = F.gelu,
                 norm=None, norm_groups: int = 1, complex_data: bool = False, use_channel_mlp: bool = True,
                 channel_mlp_dropout: float = 0, channel_mlp_expansion: float = 0.5,
                 channel_mlp_skip="soft-gating", fno_skip="linear",
                 resolution_scaling_factor: Union[Number, List[Number]] = None,
                 domain_padding: Union[Number, List[Number]] = None, fno_block_precision: str = "full",
                 stabilizer: str = None, max_n_modes: Tuple[int, ...] = None, factorization: str = None,
                 rank: float = 1.0, fixed_rank_modes: bool = False, implementation: str = "factorized",
                 decomposition_kwargs: dict = None, separable: bool = False, preactivation: bool = False,
                 conv_module: nn.Module = SpectralConv, enforce_hermitian_symmetry: bool = True,
                 contraction_precision: str = "fp32", engine: str = "auto"):
        super().__init__()
        if decomposition_kwargs is None:
            decomposition_kwargs = {}
        if domain_padding is not None and ((isinstance(domain_padding, list) and sum(domain_padding) > 0) or
                                           (isinstance(domain_padding, (float, int)) and domain_padding > 0)):
            raise NotImplementedError("domain_padding is not provided")
        if complex_data:
            raise NotImplementedError("complex_data FNO is not provided")
        self.n_dim = len(n_modes)
        self._n_modes = n_modes
        self.hidden_channels = hidden_channels
        self.in_channels = in_channels
        self.out_channels = out_channels
        self.n_layers = n_layers
        self.lifting_channel_ratio = lifting_channel_ratio
        self.lifting_channels = int(lifting_channel_ratio * hidden_channels)
        self.projection_channel_ratio = projection_channel_ratio
        self.projection_channels = int(projection_channel_ratio * hidden_channels)
        self.non_linearity = non_linearity
        self.rank = rank
        self.factorization = factorization
        self.fixed_rank_modes = fixed_rank_modes
        self.decomposition_kwargs = decomposition_kwargs
        self.fno_skip = (fno_skip,)
        self.channel_mlp_skip = (channel_mlp_skip,)
        self.implementation = implementation
        self.separable = separable
        self.preactivation = preactivation
        self.complex_data = complex_data
        self.fno_block_precision = fno_block_precision
        if positional_embedding == "grid":
            self.positional_embedding = GridEmbeddingND(in_channels=in_channels, dim=self.n_dim,
                                                        grid_boundaries=[[0.0, 1.0]] * self.n_dim)
        elif isinstance(positional_embedding, GridEmbeddingND):
            self.positional_embedding = positional_embedding
        elif positional_embedding is None:
            self.positional_embedding = None
        else:
            raise ValueError(f"Error: tried to instantiate FNO positional embedding with {positional_embedding}, "
                             "expected one of 'grid', GridEmbeddingND")
        self.domain_padding = None
        if resolution_scaling_factor is not None and isinstance(resolution_scaling_factor, (float, int)):
            resolution_scaling_factor = [resolution_scaling_factor] * n_layers
        self.resolution_scaling_factor = resolution_scaling_factor
        self.fno_blocks = FNOBlocks(
            in_channels=hidden_channels, out_channels=hidden_channels, n_modes=self.n_modes,
            resolution_scaling_factor=resolution_scaling_factor, use_channel_mlp=use_channel_mlp,
            channel_mlp_dropout=channel_mlp_dropout, channel_mlp_expansion=channel_mlp_expansion,
            non_linearity=non_linearity, stabilizer=stabilizer, norm=norm, norm_groups=norm_groups,
            preactivation=preactivation, fno_skip=fno_skip, channel_mlp_skip=channel_mlp_skip,
            complex_data=complex_data, max_n_modes=max_n_modes, fno_block_precision=fno_block_precision, rank=rank,
            fixed_rank_modes=fixed_rank_modes, implementation=implementation, separable=separable,
            factorization=factorization, decomposition_kwargs=decomposition_kwargs, conv_module=conv_module,
            n_layers=n_layers, enforce_hermitian_symmetry=enforce_hermitian_symmetry,
            contraction_precision=contraction_precision, engine=engine)
        lifting_in = in_channels + (self.n_dim if self.positional_embedding is not None else 0)
        self.lifting = ChannelMLP(in_channels=lifting_in, out_channels=hidden_channels,
                                  hidden_channels=self.lifting_channels, n_layers=2, n_dim=self.n_dim,
                                  non_linearity=non_linearity)
        self.projection = ChannelMLP(in_channels=hidden_channels, out_channels=out_channels,
                                     hidden_channels=self.projection_channels, n_layers=2, n_dim=self.n_dim,
                                     non_linearity=non_linearity)

    def _mlp_ok(self, mlp, x, cin, cnext=0, grid=None):
        """mlp (2 layers, GELU, no dropout) on cin data channels (+ grid channels) fits the fused kernel."""
        ku = cin + (len(grid) if grid is not None else 0)
        return (isinstance(mlp, ChannelMLP) and mlp.n_layers == 2 and mlp.dropout is None
                and mlp.non_linearity is F.gelu and mlp.in_channels == ku
                and pointwise.supported_dims(x.shape[0], x.shape[2:], cin, mlp.hidden_channels,
                                             mlp.out_channels, cnext, grid))

    def _fused_forward(self, x):
        """Lifting (+ grid channels, + block 0's linear skip), fused blocks, projection; None when a
        layer does not fit the fused kernels (the module path then runs)."""
        pe = self.positional_embedding
        if not (x.is_cuda and x.dtype == torch.float32) or (pe is not None and not isinstance(pe, GridEmbeddingND)):
            return None
        if grad_needed(x, self):
            return None
        grid = [tuple(b) for b in pe.grid_boundaries] if pe is not None else None
        blocks = self.fno_blocks
        if not (blocks._fusable(0, x, None) and self.resolution_scaling_factor is None):
            return None
        cnext = blocks.fno_skips[0].conv.out_channels
        if not (x.shape[1] == self.in_channels and self._mlp_ok(self.lifting, x, self.in_channels, cnext, grid)
                and self._mlp_ok(self.projection, x, self.hidden_channels)):
            return None
        prof = get_active_profiler()
        with maybe_profile(prof, "fno/positional_embedding_lifting_skip0", x.device):
            fc1, fc2 = self.lifting.fcs
            h, skip = pointwise.channel_mlp(x, fc1.weight, fc1.bias, fc2.weight, fc2.bias, grid=grid,
                                            act_hidden=True, act_out=False, next_w=blocks.next_skip_weight(0))
        blocks.set_pending_skip(h, 0, skip)
        for i in range(self.n_layers):
            h = blocks(h, i)
        with maybe_profile(prof, "fno/projection", x.device):
            fc1, fc2 = self.projection.fcs
            y, _ = pointwise.channel_mlp(h, fc1.weight, fc1.bias, fc2.weight, fc2.bias, act_hidden=True,
                                         act_out=False)
        return y

    def forward(self, x, output_shape=None, **kwargs):
        if output_shape is None:
            fused = self._fused_forward(x)
            if fused is not None:
                return fused
            output_shape = [None] * self.n_layers
        elif isinstance(output_shape, tuple):
            output_shape = [None] * (self.n_layers - 1) + [output_shape]
        prof = get_active_profiler()
        if self.positional_embedding is not None:
            with maybe_profile(prof, "fno/positional_embedding", x.device):
                x = self.positional_embedding(x)
        with maybe_profile(prof, "fno/lifting", x.device):
            x = self.lifting(x)
        for i in range(self.n_layers):
            x = self.fno_blocks(x, i, output_shape=output_shape[i])
        with maybe_profile(prof, "fno/projection", x.device):
            x = self.projection(x)
        return x

    @property
    def n_modes(self):
        return self._n_modes

    @n_modes.setter
    def n_modes(self, n_modes):
        self.fno_blocks.n_modes = n_modes
        self._n_modes = n_modes

    def load_state_dict(self, state_dict, strict=True, assign=False):
        # reference checkpoints carry a '_metadata' entry with the constructor arguments
        state_dict = {k: v for k, v in state_dict.items() if k != "_metadata"}
        return super().load_state_dict(state_dict, strict=strict, assign=assign)


class TFNO(FNO):
    """FNO with Tucker-factorized spectral weights (rank 0.1 by default)."""

    def __init__(self, *args, **kwargs):
        kwargs.setdefault("factorization", "Tucker")
        kwargs.setdefault("rank", 0.1)
        super().__init__(*args, **kwargs)
