"""FNOBlocks: drop-in for neuralop.layers.fno_block.FNOBlocks (neuralop/layers/fno_block.py:18-481).

Same constructor, parameters and forward semantics.  When a block has the FNO default shape --
``fno_skip="linear"``, real data, no norm, no stabilizer, GELU, post-activation, a ``SpectralConv`` of
this package, no output resampling, and the default ChannelMLP (two layers, GELU, no dropout) with a
soft-gating (or no) channel-MLP skip -- it runs as two launch sequences: the spectral convolution
(its own kernels, bias included), then ONE per-pixel tensor-core kernel (``pointwise.chain``) that adds
the linear skip W_skip x to the spectral output, applies GELU, the ChannelMLP, the soft-gating skip of x
and the closing GELU (:339-381).  x is read twice from HBM and the block output written once.  Every
other configuration composes the same operations as the reference around the CUDA spectral block.
Normalisation layers other than None are not provided (norm=None is the FNO default).
"""

from __future__ import annotations

from typing import List, Union

import torch
import torch.nn.functional as F
from torch import nn

from . import pointwise
from .layers import ChannelMLP, SoftGating, skip_connection
from .spectral_convolution import SpectralConv
from .utils import grad_needed, validate_scaling_factor

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
        """The spectral convolution of block `index` runs bare (no resampling) and its linear skip, GELU
        and the rest of the block can be composed around it."""
        conv = self.convs[index]
        return (isinstance(conv, SpectralConv) and self.fno_skips is not None and self.fno_skip.lower() == "linear"
                and self.stabilizer is None and self.non_linearity is F.gelu and output_shape is None
                and conv.resolution_scaling_factor is None and x.is_cuda)

    def _mlp_parts(self, index):
        """(ChannelMLP, soft-gating skip or None) of block `index` when they fit the chain kernel's form."""
        if not self.use_channel_mlp:
            return None
        mlp = self.channel_mlp[index]
        sg = self.channel_mlp_skips[index] if self.channel_mlp_skips is not None else None
        if not (isinstance(mlp, ChannelMLP) and mlp.n_layers == 2 and mlp.dropout is None
                and mlp.non_linearity is F.gelu and (sg is None or isinstance(sg, SoftGating))):
            return None
        return mlp, sg

    def chain_supported(self, index, batch, spatial, proj=None, min_groups=1, backward=False) -> bool:
        """Block `index` after its spectral convolution (and, with `proj`, the FNO projection ChannelMLP)
        fits one chain kernel call for an input of `batch` samples on a grid of `spatial` points, with at
        least `min_groups` tiles in flight per SM (and, with `backward`, the chain's backward kernel)."""
        parts = self._mlp_parts(index)
        if parts is None:
            return False
        mlp, sg = parts
        last = index >= self.n_layers - 1
        kw = {}
        if proj is not None:
            kw = dict(proj_hidden=proj.fcs[0].out_channels, proj_out=proj.fcs[1].out_channels)
        args = (batch, tuple(spatial), self.in_channels, mlp.hidden_channels, self.out_channels)
        kw.update(skip=self.out_channels, act_skip=not last, act_out=not last, gate=sg is not None)
        if backward and not pointwise.backward_supported(*args, **kw):
            return False
        return pointwise.supported(*args, min_groups=min_groups, **kw)

    def fused_block(self, x, index, spectral=None, proj=None):
        """Spectral convolution, then ONE chain kernel for the rest of the block: the linear skip added to
        the spectral output, GELU, ChannelMLP, soft-gating skip, GELU (fno_block.py:339-381) -- and, with
        `proj` (a ChannelMLP), the FNO's projection on the block output.  ``spectral(index, conv, x)``
        replaces the spectral call (the slab-decomposed path passes its own)."""
        conv = self.convs[index]
        relay = None
        if spectral is None and proj is None and type(conv) is SpectralConv and grad_needed(x, self):
            # x's two gradients (through the spectral convolution and through the chain's skip and gate)
            # leave the spectral backward's last kernel as one tensor (pointwise.GradRelay)
            relay = pointwise.GradRelay()
            conv.__dict__["_nop_grad_relay"] = relay
        try:
            s = conv(x) if spectral is None else spectral(index, conv, x)
        finally:
            unused = conv.__dict__.pop("_nop_grad_relay", None) is not None
        if relay is not None and (unused or not s.requires_grad or s.grad_fn is None):
            relay = None  # the spectral call took no relay or recorded no backward: the chain returns dL/dx
        mlp, sg = self._mlp_parts(index)
        last = index >= self.n_layers - 1
        kw = {}
        if proj is not None:
            (f1, f2) = proj.fcs
            kw = dict(w3=f1.weight, b3=f1.bias, w4=f2.weight, b4=f2.bias)
        return pointwise.chain(x, mlp.fcs[0].weight, mlp.fcs[0].bias, mlp.fcs[1].weight, mlp.fcs[1].bias, s=s,
                               w0=self.fno_skips[index].conv.weight, act_skip=not last, act_out=not last,
                               gate_w=sg.weight if sg is not None else None,
                               gate_b=sg.bias if sg is not None else None, grad_relay=relay, **kw)

    def forward_with_postactivation(self, x, index=0, output_shape=None):
        if (self._fusable(index, x, output_shape) and x.dtype == torch.float32
                and self.chain_supported(index, x.shape[0], x.shape[2:], backward=grad_needed(x, self))):
            return self.fused_block(x, index)
        last = index >= self.n_layers - 1
        if self.use_channel_mlp and self.channel_mlp_skips is not None:
            x_skip_mlp = self.channel_mlp_skips[index](x)
            x_skip_mlp = self.convs[index].transform(x_skip_mlp, output_shape=output_shape)
        if self._fusable(index, x, output_shape) and not grad_needed(x, self):  # the epilogue has no backward
            x_skip = self.fno_skips[index](x)
            x = self.convs[index](x, addend=x_skip, apply_gelu=not last)
        else:
            if self.fno_skips is not None:
                x_skip = self.fno_skips[index](x)
                x_skip = self.convs[index].transform(x_skip, output_shape=output_shape)
            if self.stabilizer == "tanh":
                x = torch.tanh(x)
            x_fno = self.convs[index](x, output_shape=output_shape)
            x = x_fno + x_skip if self.fno_skips is not None else x_fno
            if not last:
                x = self.non_linearity(x)
        if self.use_channel_mlp:
            x = self.channel_mlp[index](x)
            if self.channel_mlp_skips is not None:
                x = x + x_skip_mlp
        if not last:
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
