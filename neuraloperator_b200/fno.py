"""FNO / TFNO: drop-ins for neuralop.models.FNO and TFNO (neuralop/models/fno.py:26-485).

Same constructor arguments and forward: grid embedding -> lifting ChannelMLP -> n_layers x
FNOBlocks -> projection ChannelMLP.  The spectral blocks run on libnop_b200's CUDA kernels; with
the default layer shapes the grid embedding + lifting is one per-pixel tensor-core kernel
(``pointwise.chain``), every block is its spectral convolution plus one such kernel, and the
projection is fused into the last block's kernel.
Options the reference offers outside the FNO default path raise NotImplementedError here:
``domain_padding``, ``norm``, ``complex_data`` and ``fno_block_precision`` other than "full".
"""

from __future__ import annotations

from typing import List, Optional, Tuple, Union

import torch
import torch.nn.functional as F
from torch import nn

from . import ops, pointwise
from .fno_block import FNOBlocks
from .layers import ChannelMLP, GridEmbeddingND
from .spectral_convolution import SpectralConv
from .utils import grad_needed, host_pipeline

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

    @staticmethod
    def _mlp_ok(mlp) -> bool:
        """A two-layer GELU ChannelMLP without dropout (the chain kernel's form)."""
        return (isinstance(mlp, ChannelMLP) and mlp.n_layers == 2 and mlp.dropout is None
                and mlp.non_linearity is F.gelu)

    def fused_plan(self, x, grid_sizes=None, train_ok=True):
        """(grid, fuse_projection) when the fused forward takes x, else None.  ``grid_sizes``: the full
        grid's sizes when x is a slab of it (the coordinate step follows the full grid).  When autograd
        records the call (``train_ok``), every chain must also fit the chain backward kernel and the
        projection runs as its own chain call."""
        pe = self.positional_embedding
        train = grad_needed(x, self)
        if not (x.is_cuda and x.dtype == torch.float32 and x.ndim == 2 + self.n_dim) or (train and not train_ok):
            return None
        if (pe is not None and not isinstance(pe, GridEmbeddingND)) or self.resolution_scaling_factor is not None:
            return None
        if x.shape[1] != self.in_channels or not (self._mlp_ok(self.lifting) and self._mlp_ok(self.projection)):
            return None
        blocks = self.fno_blocks
        batch, spatial = x.shape[0], tuple(x.shape[2:])
        grid = pointwise.grid_params(pe.grid_boundaries, grid_sizes or spatial) if pe is not None else None
        f1, f2 = self.lifting.fcs
        if self.lifting.in_channels != self.in_channels + (self.n_dim if pe is not None else 0):
            return None
        lift = (batch, spatial, self.in_channels, f1.out_channels, f2.out_channels)
        if not pointwise.supported(*lift, grid=grid) or (train and not pointwise.backward_supported(*lift, grid=grid)):
            return None
        for i in range(self.n_layers):
            if not (blocks._fusable(i, x, None) and blocks.chain_supported(i, batch, spatial, backward=train)):
                return None
        # the projection rides in the last block's kernel unless its weights would leave one tile in flight
        # (or a gradient is recorded: the chain backward takes no projection)
        fuse_proj = not train and blocks.chain_supported(self.n_layers - 1, batch, spatial, proj=self.projection,
                                                         min_groups=2)
        if not fuse_proj:
            p1, p2 = self.projection.fcs
            proj = (batch, spatial, self.hidden_channels, p1.out_channels, p2.out_channels)
            if not pointwise.supported(*proj) or (train and not pointwise.backward_supported(*proj)):
                return None
        return grid, fuse_proj

    def fused_forward(self, x, spectral=None, grid_offset=None, grid_sizes=None):
        """Grid embedding + lifting (one chain kernel), every block as spectral convolution + one chain
        kernel, the projection fused into the last block's chain (or one more chain call); None when a
        layer does not fit the fused kernels (the module path then runs).  ``spectral(index, conv, h)``
        replaces the blocks' spectral calls and ``grid_offset`` / ``grid_sizes`` place x in a larger grid
        (the slab-decomposed forward)."""
        plan = self.fused_plan(x, grid_sizes, train_ok=spectral is None)
        if plan is None:
            return None
        grid, fuse_proj = plan
        f1, f2 = self.lifting.fcs
        h = pointwise.chain(x, f1.weight, f1.bias, f2.weight, f2.bias, grid=grid, grid_offset=grid_offset)
        last = self.n_layers - 1
        for i in range(self.n_layers):
            h = self.fno_blocks.fused_block(h, i, spectral=spectral,
                                            proj=self.projection if (i == last and fuse_proj) else None)
        if not fuse_proj:
            p1, p2 = self.projection.fcs
            h = pointwise.chain(h, p1.weight, p1.bias, p2.weight, p2.bias)
        return h

    def forward(self, x, output_shape=None, **kwargs):
        if output_shape is None:
            fused = self.fused_forward(x)
            if fused is not None:
                return fused
            output_shape = [None] * self.n_layers
        elif isinstance(output_shape, tuple):
            output_shape = [None] * (self.n_layers - 1) + [output_shape]
        if self.positional_embedding is not None:
            x = self.positional_embedding(x)
        x = self.lifting(x)
        for i in range(self.n_layers):
            x = self.fno_blocks(x, i, output_shape=output_shape[i])
        x = self.projection(x)
        return x

    @torch.no_grad()
    def forward_host(self, x: torch.Tensor, out: Optional[torch.Tensor] = None, chunk: Optional[int] = None,
                     n_streams: int = 2, synchronize: bool = True) -> torch.Tensor:
        """``forward`` of a batch held in HOST memory: the batch is cut into chunks of ``chunk`` samples
        whose host-to-device copies, forwards and device-to-host copies run as a three-stage pipeline on
        three streams (utils.host_pipeline), so the PCIe transfers in both directions overlap the kernels
        (``n_streams`` is kept for compatibility and ignored).  ``x`` and ``out``
        are CPU tensors (page-locked for the overlap; the returned tensor is page-locked when ``out`` is
        None); the parameters stay on their CUDA device.  With ``synchronize=False`` the call returns once
        the work is queued on the device's current stream.  Inference only."""
        if x.is_cuda:
            raise ValueError("forward_host takes a host tensor; call the module on device tensors")
        dev = next(self.parameters()).device
        if dev.type != "cuda":
            raise RuntimeError("neuraloperator_b200 models run on CUDA devices only (there is no CPU path)")
        batch = x.shape[0]
        chunk = ops.default_chunk(batch) if chunk is None else int(chunk)
        if chunk < 1 or batch % chunk:
            raise ValueError(f"chunk {chunk} does not divide the batch {batch}")
        y_shape = (batch, self.out_channels, *x.shape[2:])
        y = out if out is not None else torch.empty(y_shape, dtype=torch.float32, pin_memory=True)
        if y.is_cuda or tuple(y.shape) != y_shape or not y.is_contiguous():
            raise ValueError(f"out must be a contiguous host tensor of shape {y_shape}")
        host_pipeline(self, x, y, chunk, dev, self.__dict__.setdefault("_nop_host_streams", {}))
        if synchronize:
            torch.cuda.current_stream(dev).synchronize()
        return y

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
