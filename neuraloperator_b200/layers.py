"""The FNO layers around the spectral block, mirroring the reference modules.

ChannelMLP (neuralop/layers/channel_mlp.py:6-119), skip connections
(neuralop/layers/skip_connections.py:5-127), GridEmbeddingND (neuralop/layers/embeddings.py:90-164,
351-383) and resample (neuralop/layers/resample.py:7-80).  These are per-pixel channel GEMMs,
elementwise ops and interpolation; they run as PyTorch (cuBLAS / cuDNN) ops on the device.
Parameter names match the reference so its state dicts load.
"""

from __future__ import annotations

import itertools
from typing import List

import torch
import torch.nn.functional as F
from torch import nn


class ChannelMLP(nn.Module):
    def __init__(self, in_channels, out_channels=None, hidden_channels=None, n_layers=2, n_dim=2,
                 non_linearity=F.gelu, dropout=0.0):
        super().__init__()
        self.n_layers = n_layers
        self.in_channels = in_channels
        self.out_channels = in_channels if out_channels is None else out_channels
        self.hidden_channels = in_channels if hidden_channels is None else hidden_channels
        self.non_linearity = non_linearity
        self.dropout = nn.ModuleList([nn.Dropout(dropout) for _ in range(n_layers)]) if dropout > 0.0 else None
        self.fcs = nn.ModuleList()
        for i in range(n_layers):
            cin = self.in_channels if i == 0 else self.hidden_channels
            cout = self.out_channels if i == n_layers - 1 else self.hidden_channels
            self.fcs.append(nn.Conv1d(cin, cout, 1))

    def forward(self, x):
        size = list(x.shape)
        reshaped = x.ndim > 3
        if reshaped:
            x = x.reshape((*size[:2], -1))
        for i, fc in enumerate(self.fcs):
            x = fc(x)
            if i < self.n_layers - 1:
                x = self.non_linearity(x)
            if self.dropout is not None:
                x = self.dropout[i](x)
        if reshaped:
            x = x.reshape((size[0], self.out_channels, *size[2:]))
        return x


class SoftGating(nn.Module):
    def __init__(self, in_features, out_features=None, n_dim=2, bias=False):
        super().__init__()
        if out_features is not None and in_features != out_features:
            raise ValueError(f"Got in_features={in_features} and out_features={out_features}, "
                             "but these two must be the same for soft-gating")
        self.in_features = in_features
        self.out_features = out_features
        self.weight = nn.Parameter(torch.ones(1, self.in_features, *(1,) * n_dim))
        self.bias = nn.Parameter(torch.ones(1, self.in_features, *(1,) * n_dim)) if bias else None

    def forward(self, x):
        return self.weight * x + self.bias if self.bias is not None else self.weight * x


class Flattened1dConv(nn.Module):
    def __init__(self, in_channels: int, out_channels: int, kernel_size, bias=False):
        super().__init__()
        self.conv = nn.Conv1d(in_channels=in_channels, out_channels=out_channels, kernel_size=kernel_size,
                              bias=bias)

    def forward(self, x):
        size = list(x.shape)
        x = x.view(*size[:2], -1)
        x = self.conv(x)
        return x.view(size[0], self.conv.out_channels, *size[2:])


def skip_connection(in_features, out_features, n_dim=2, bias=False, skip_type="soft-gating"):
    kind = skip_type.lower()
    if kind == "soft-gating":
        return SoftGating(in_features=in_features, out_features=out_features, bias=bias, n_dim=n_dim)
    if kind == "linear":
        return Flattened1dConv(in_channels=in_features, out_channels=out_features, kernel_size=1, bias=bias)
    if kind == "identity":
        return nn.Identity()
    raise ValueError(f"Got skip-connection type={skip_type}, expected one of {'soft-gating', 'linear', 'id'}.")


def regular_grid_nd(resolutions: List[int], grid_boundaries=None):
    if grid_boundaries is None:
        grid_boundaries = [[0, 1]] * len(resolutions)
    axes = [torch.linspace(a, b, r + 1)[:-1] for r, (a, b) in zip(resolutions, grid_boundaries)]
    grid = torch.meshgrid(*axes, indexing="ij")
    return tuple(g.repeat([1] * len(resolutions)) for g in grid)


class GridEmbeddingND(nn.Module):
    def __init__(self, in_channels: int, dim: int = 2, grid_boundaries=None):
        super().__init__()
        self.in_channels = in_channels
        self.dim = dim
        self.grid_boundaries = grid_boundaries if grid_boundaries is not None else [[0, 1]] * dim
        assert self.dim == len(self.grid_boundaries)
        self._grid = None
        self._res = None

    @property
    def out_channels(self):
        return self.in_channels + self.dim

    def grid(self, spatial_dims, device, dtype):
        if self._grid is None or self._res != spatial_dims or self._grid[0].device != torch.device(device):
            grids = regular_grid_nd(list(spatial_dims), grid_boundaries=self.grid_boundaries)
            self._grid = [g.to(device).to(dtype).unsqueeze(0).unsqueeze(0) for g in grids]
            self._res = spatial_dims
        return self._grid

    def forward(self, data, batched=True):
        if not batched and data.ndim == self.dim + 1:
            data = data.unsqueeze(0)
        b = data.shape[0]
        grids = [g.repeat(b, *[1] * (self.dim + 1)) for g in self.grid(data.shape[2:], data.device, data.dtype)]
        out = torch.cat((data, *grids), dim=1)
        if not batched and b == 1:
            return out.squeeze(0)
        return out


def resample(x, res_scale, axis, output_shape=None):
    """Linear (1D) / bicubic (2D) / spectral (>=3D) resampling (neuralop/layers/resample.py:7-80)."""
    if isinstance(res_scale, (float, int)):
        if axis is None:
            axis = list(range(2, x.ndim))
            res_scale = [res_scale] * len(axis)
        elif isinstance(axis, int):
            axis = [axis]
            res_scale = [res_scale]
        else:
            res_scale = [res_scale] * len(axis)
    old = x.shape[-len(axis):]
    new = tuple(int(round(s * r)) for s, r in zip(old, res_scale)) if output_shape is None else tuple(output_shape)
    if len(axis) == 1:
        return F.interpolate(x, size=new[0], mode="linear", align_corners=True)
    if len(axis) == 2:
        return F.interpolate(x, size=new, mode="bicubic", align_corners=True)
    X = torch.fft.rfftn(x.float(), norm="forward", dim=axis)
    nf = list(new)
    nf[-1] = nf[-1] // 2 + 1
    nfc = [min(i, j) for i, j in zip(nf, X.shape[-len(axis):])]
    out = torch.zeros([x.shape[0], x.shape[1], *nf], device=x.device, dtype=torch.cfloat)
    bounds = [((None, m // 2), (-m // 2, None)) for m in nfc[:-1]] + [((None, nfc[-1]),)]
    for b in itertools.product(*bounds):
        idx = (slice(None), slice(None)) + tuple(slice(*e) for e in b)
        out[idx] = X[idx]
    return torch.fft.irfftn(out, s=new, norm="forward", dim=axis)
