"""Spectral weight containers: dense, Tucker, CP and tensor-train (complex64).

They stand where the reference uses tensorly-torch's ``FactorizedTensor.new(...)``
(neuralop/layers/spectral_convolution.py:362-370) and expose the surface the reference
forward touches: ``name``, ``shape``, ``normal_``, ``to_tensor``, slicing, and the
``tensor`` / ``core`` / ``weights`` / ``factors`` parameters.

Rank rules for a float ``rank`` (fraction of the dense parameter count) restate the
published tensorly rules: Tucker solves ``n x^d + (sum s_i^2) x = rank n`` for ``x`` and uses
``round(s_i x)`` per mode (fixed modes keep their full size); CP uses
``round(rank prod(s) / sum(s))``; TT uses one internal rank ``r`` solving
``(s_0 + s_last) r + (sum_middle s_i) r^2 = rank prod(s)``.  Initialisations follow
tensorly-torch's ``normal_`` conventions (reconstructed entries with standard deviation
``std``).
"""

from __future__ import annotations

import math
from typing import List, Optional, Sequence

import torch
from torch import nn


def tucker_rank(shape: Sequence[int], rank, fixed_modes: Optional[Sequence[int]] = None) -> List[int]:
    if isinstance(rank, (list, tuple)):
        return [int(r) for r in rank]
    if isinstance(rank, int):
        return [rank] * len(shape)
    rank = float(rank)
    shape = list(shape)
    fixed = sorted(fixed_modes or [])
    free = [s for i, s in enumerate(shape) if i not in fixed]
    n = math.prod(shape)
    sq = sum(s * s for s in free)
    fixed_params = sum(shape[i] ** 2 for i in fixed)
    lo, hi = 0.0, max(rank, 1.0)
    for _ in range(200):
        mid = 0.5 * (lo + hi)
        if n * mid ** len(free) + sq * mid + fixed_params * mid - rank * n > 0:
            hi = mid
        else:
            lo = mid
    out = []
    for i, s in enumerate(shape):
        out.append(s if i in fixed else max(int(round(s * lo)), 1))
    return out


def cp_rank(shape: Sequence[int], rank) -> int:
    if isinstance(rank, int):
        return rank
    return max(1, int(round(float(rank) * math.prod(shape) / sum(shape))))


def tt_rank(shape: Sequence[int], rank) -> List[int]:
    if isinstance(rank, (list, tuple)):
        return [int(r) for r in rank]
    if isinstance(rank, int):
        r = rank
    else:
        order = len(shape)
        if order == 1:
            return [1, 1]
        a = float(sum(shape[1:-1]))
        b = float(shape[0] + shape[-1])
        c = float(rank) * math.prod(shape)
        r = (-b + math.sqrt(b * b + 4 * a * c)) / (2 * a) if a > 0 else c / b
        r = max(1, int(round(r)))
    return [1] + [r] * (len(shape) - 1) + [1]


class FactorizedTensor(nn.Module):
    """Base class; ``FactorizedTensor.new`` builds the container named by ``factorization``."""

    name = "Factorized"

    @classmethod
    def new(cls, shape, rank=None, factorization="Dense", fixed_rank_modes=None, dtype=torch.cfloat,
            device=None, **kwargs):
        kind = str(factorization).lower().replace("complex", "")
        if kind == "dense":
            return DenseTensor(shape, dtype=dtype, device=device)
        if kind == "tucker":
            return TuckerTensor(shape, rank, fixed_rank_modes=fixed_rank_modes, dtype=dtype, device=device)
        if kind == "cp":
            return CPTensor(shape, rank, dtype=dtype, device=device)
        if kind == "tt":
            return TTTensor(shape, rank, dtype=dtype, device=device)
        raise ValueError(f"unknown factorization {factorization!r}")

    @classmethod
    def from_tensor(cls, tensor, rank=None, factorization="ComplexDense", **kwargs):
        kind = str(factorization).lower().replace("complex", "")
        if kind != "dense":
            raise NotImplementedError("only dense from_tensor is supported")
        return DenseTensor(tensor.shape, dtype=tensor.dtype, device=tensor.device, tensor=tensor)

    @property
    def shape(self):
        return torch.Size(self._shape)

    @property
    def order(self):
        return len(self._shape)

    def __len__(self):
        return self._shape[0]


class DenseTensor(FactorizedTensor):
    name = "ComplexDense"

    def __init__(self, shape, dtype=torch.cfloat, device=None, tensor=None):
        super().__init__()
        self._shape = tuple(shape)
        data = tensor.detach().clone() if tensor is not None else torch.empty(shape, dtype=dtype, device=device)
        self.tensor = nn.Parameter(data)
        self.rank = None

    def normal_(self, mean=0.0, std=1.0):
        with torch.no_grad():
            self.tensor.normal_(mean, std)
        return self

    def to_tensor(self):
        return self.tensor

    def __getitem__(self, idx):
        return self.tensor[idx]

    def extra_repr(self):
        return f"shape={tuple(self._shape)}, rank=None"


class TuckerTensor(FactorizedTensor):
    name = "ComplexTucker"

    def __init__(self, shape, rank, fixed_rank_modes=None, dtype=torch.cfloat, device=None):
        super().__init__()
        self._shape = tuple(shape)
        self.rank = tucker_rank(shape, rank if rank is not None else 1.0, fixed_rank_modes)
        self.core = nn.Parameter(torch.empty(self.rank, dtype=dtype, device=device))
        self.factors = nn.ParameterList(
            [nn.Parameter(torch.empty(s, r, dtype=dtype, device=device)) for s, r in zip(shape, self.rank)])

    def normal_(self, mean=0.0, std=1.0):
        if mean != 0:
            raise ValueError("only mean=0 is supported")
        r = math.prod(math.sqrt(x) for x in self.rank)
        s = (std / r) ** (1.0 / (self.order + 1))
        with torch.no_grad():
            self.core.normal_(0, s)
            for f in self.factors:
                f.normal_(0, s)
        return self

    def to_tensor(self):
        t = self.core
        for mode, u in enumerate(self.factors):
            t = torch.tensordot(u, t.movedim(mode, 0), dims=([1], [0])).movedim(0, mode)
        return t

    def sliced(self, idx):
        """(core, factors) after slicing mode i with idx[i] (slices only)."""
        facs = [f[i] for f, i in zip(self.factors, idx)] + list(self.factors)[len(idx):]
        return self.core, facs

    def __getitem__(self, idx):
        core, facs = self.sliced(idx if isinstance(idx, tuple) else (idx,))
        t = core
        for mode, u in enumerate(facs):
            t = torch.tensordot(u, t.movedim(mode, 0), dims=([1], [0])).movedim(0, mode)
        return t

    def extra_repr(self):
        return f"shape={tuple(self._shape)}, rank={self.rank}"


class CPTensor(FactorizedTensor):
    name = "ComplexCP"

    def __init__(self, shape, rank, dtype=torch.cfloat, device=None):
        super().__init__()
        self._shape = tuple(shape)
        self.rank = cp_rank(shape, rank if rank is not None else 1.0)
        self.weights = nn.Parameter(torch.ones(self.rank, dtype=dtype, device=device))
        self.factors = nn.ParameterList(
            [nn.Parameter(torch.empty(s, self.rank, dtype=dtype, device=device)) for s in shape])

    def normal_(self, mean=0.0, std=1.0):
        if mean != 0:
            raise ValueError("only mean=0 is supported")
        s = (std / math.sqrt(self.rank)) ** (1.0 / self.order)
        with torch.no_grad():
            self.weights.fill_(1)
            for f in self.factors:
                f.normal_(0, s)
        return self

    def to_tensor(self):
        sy = "abcdefghijklmnop"
        eq = "z," + ",".join(sy[i] + "z" for i in range(self.order)) + "->" + sy[: self.order]
        return torch.einsum(eq, self.weights, *self.factors)

    def sliced(self, idx):
        facs = [f[i] for f, i in zip(self.factors, idx)] + list(self.factors)[len(idx):]
        return self.weights, facs

    def extra_repr(self):
        return f"shape={tuple(self._shape)}, rank={self.rank}"


class TTTensor(FactorizedTensor):
    name = "ComplexTT"

    def __init__(self, shape, rank, dtype=torch.cfloat, device=None):
        super().__init__()
        self._shape = tuple(shape)
        self.rank = tt_rank(shape, rank if rank is not None else 1.0)
        self.factors = nn.ParameterList(
            [nn.Parameter(torch.empty(self.rank[i], s, self.rank[i + 1], dtype=dtype, device=device))
             for i, s in enumerate(shape)])

    def normal_(self, mean=0.0, std=1.0):
        if mean != 0:
            raise ValueError("only mean=0 is supported")
        r = math.prod(self.rank)
        s = (std / r) ** (1.0 / self.order)
        with torch.no_grad():
            for f in self.factors:
                f.normal_(0, s)
        return self

    def to_tensor(self, factors=None):
        facs = list(self.factors) if factors is None else factors
        t = facs[0]
        for g in facs[1:]:
            t = torch.tensordot(t, g, dims=([t.ndim - 1], [0]))
        return t.squeeze(0).squeeze(-1)

    def sliced(self, idx):
        return [f[:, i, :] for f, i in zip(self.factors, idx)] + list(self.factors)[len(idx):]

    def extra_repr(self):
        return f"shape={tuple(self._shape)}, rank={self.rank}"
