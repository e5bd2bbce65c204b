"""Load the reference's own neuralop forward code in this container (golden-vector generation).

``import neuralop`` fails here: tensorly 0.9.0, tensorly-torch 0.5.0 and opt-einsum 3.4.0
(pinned in the reference's uv.lock) are not installed and there is no network.  The
reference path only touches a small surface of them, so this module installs stand-ins
written from that surface and then imports the reference files verbatim:

* ``tensorly``: ``set_backend`` (no-op), ``einsum`` (= ``torch.einsum``, which is what the
  pytorch backend dispatches to), ``ndim``; ``tensorly.plugins.use_opt_einsum`` (no-op;
  opt_einsum only chooses the contraction order, which changes rounding, not results).
* ``tltorch.factorized_tensors.core.FactorizedTensor``: ``new`` / ``from_tensor`` returning
  dense, Tucker, CP or TT containers with ``name``, ``normal_``, ``to_tensor``, ``shape``,
  ``core`` / ``weights`` / ``factors`` and slice indexing (slicing a factorized tensor
  slices the factor that carries each mode).

The ``neuralop`` package ``__init__`` files are bypassed (they pull in h5py / zencfg /
datasets), so only the modules on the FNO path are executed.  Nothing here is used at
run time by the product or by the GPU tests; it needs the reference checkout.
"""

from __future__ import annotations

import importlib
import math
import os
import sys
import types

import torch
from torch import nn

REF_ROOT = os.environ.get("NOP_REFERENCE_ROOT")  # the reference checkout (its parent of ``neuralop/``)


def _tucker_rank(shape, rank):
    """Tucker ranks for a float ``rank`` (fraction of the dense parameter count).

    Solves n * x**d + (sum_i s_i**2) * x = rank * n for x by bisection (the rule of
    tensorly's ``validate_tucker_rank``) and rounds ``s_i * x``.
    """
    if not isinstance(rank, float):
        return list(rank) if isinstance(rank, (list, tuple)) else [int(rank)] * len(shape)
    n = math.prod(shape)
    sq = sum(s * s for s in shape)
    lo, hi = 0.0, max(rank, 1.0)
    for _ in range(200):
        mid = 0.5 * (lo + hi)
        if n * mid ** len(shape) + sq * mid - rank * n > 0:
            hi = mid
        else:
            lo = mid
    return [max(int(round(s * lo)), 1) for s in shape]


class _Sliced:
    """Result of slicing a factorized stand-in: the sliced factors plus ``to_tensor``."""

    def __init__(self, rebuild, **kw):
        self.__dict__.update(kw)
        self._rebuild = rebuild

    def to_tensor(self):
        return self._rebuild(self)


class StubFactorizedTensor(nn.Module):
    """Base of the stand-in containers (the reference checks ``isinstance(w, FactorizedTensor)``)."""

    @classmethod
    def new(cls, shape, rank=None, factorization="Dense", fixed_rank_modes=None, dtype=torch.cfloat, **kw):
        kind = factorization.lower().replace("complex", "")
        if kind == "dense":
            return _StubDense(shape, dtype)
        if kind == "tucker":
            return _StubTucker(shape, rank, dtype)
        if kind == "cp":
            return _StubCP(shape, rank, dtype)
        if kind == "tt":
            return _StubTT(shape, rank, dtype)
        raise ValueError(factorization)

    @classmethod
    def from_tensor(cls, tensor, rank=None, factorization="ComplexDense", **kw):
        return _StubDense(tensor=tensor)


class _StubDense(StubFactorizedTensor):
    name = "ComplexDense"

    def __init__(self, shape=None, dtype=torch.cfloat, tensor=None):
        super().__init__()
        self.tensor = nn.Parameter(tensor.clone() if tensor is not None else torch.zeros(shape, dtype=dtype))

    @property
    def shape(self):
        return self.tensor.shape

    def normal_(self, mean=0.0, std=1.0):
        with torch.no_grad():
            self.tensor.normal_(mean, std)
        return self

    def to_tensor(self):
        return self.tensor

    def __getitem__(self, idx):
        return self.tensor[idx]


class _StubTucker(StubFactorizedTensor):
    name = "ComplexTucker"

    def __init__(self, shape, rank, dtype=torch.cfloat):
        super().__init__()
        ranks = _tucker_rank(shape, rank)
        self.core = nn.Parameter(torch.zeros(ranks, dtype=dtype))
        self.factors = nn.ParameterList([nn.Parameter(torch.zeros(s, r, dtype=dtype)) for s, r in zip(shape, ranks)])
        self._shape = tuple(shape)

    @property
    def shape(self):
        return torch.Size(self._shape)

    def normal_(self, mean=0.0, std=1.0):
        r = math.prod(math.sqrt(x) for x in self.core.shape)
        s = (std / r) ** (1.0 / (self.core.ndim + 1))
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

    def __getitem__(self, idx):
        facs = [f[i] for f, i in zip(self.factors, idx)] + list(self.factors)[len(idx):]
        return _Sliced(_StubTucker.to_tensor, core=self.core, factors=facs, shape=torch.Size([f.shape[0] for f in facs]))


class _StubCP(StubFactorizedTensor):
    name = "ComplexCP"

    def __init__(self, shape, rank, dtype=torch.cfloat):
        super().__init__()
        r = rank if isinstance(rank, int) else max(1, int(round(rank * math.prod(shape) / sum(shape))))
        self.weights = nn.Parameter(torch.ones(r, dtype=dtype))
        self.factors = nn.ParameterList([nn.Parameter(torch.zeros(s, r, dtype=dtype)) for s in shape])
        self._shape = tuple(shape)

    @property
    def shape(self):
        return torch.Size(self._shape)

    def normal_(self, mean=0.0, std=1.0):
        r = self.weights.shape[0]
        s = (std / math.sqrt(r)) ** (1.0 / len(self._shape))
        with torch.no_grad():
            for f in self.factors:
                f.normal_(0, s)
        return self

    def to_tensor(self):
        order = len(self.factors)
        sy = "abcdefghijklmnop"
        eq = "z," + ",".join(sy[i] + "z" for i in range(order)) + "->" + sy[:order]
        return torch.einsum(eq, self.weights, *self.factors)

    def __getitem__(self, idx):
        facs = [f[i] for f, i in zip(self.factors, idx)] + list(self.factors)[len(idx):]
        return _Sliced(_StubCP.to_tensor, weights=self.weights, factors=facs, shape=torch.Size([f.shape[0] for f in facs]))


class _StubTT(StubFactorizedTensor):
    name = "ComplexTT"

    def __init__(self, shape, rank, dtype=torch.cfloat):
        super().__init__()
        r = rank if isinstance(rank, int) else 3
        ranks = [1] + [r] * (len(shape) - 1) + [1]
        self.factors = nn.ParameterList(
            [nn.Parameter(torch.zeros(ranks[i], s, ranks[i + 1], dtype=dtype)) for i, s in enumerate(shape)])
        self._shape = tuple(shape)

    @property
    def shape(self):
        return torch.Size(self._shape)

    def normal_(self, mean=0.0, std=1.0):
        with torch.no_grad():
            for f in self.factors:
                f.normal_(0, std ** (1.0 / len(self._shape)))
        return self

    def to_tensor(self):
        t = self.factors[0]
        for g in list(self.factors)[1:]:
            t = torch.tensordot(t, g, dims=([t.ndim - 1], [0]))
        return t.squeeze(0).squeeze(-1)

    def __getitem__(self, idx):
        facs = [f[:, i, :] for f, i in zip(self.factors, idx)] + list(self.factors)[len(idx):]
        return _Sliced(_StubTT.to_tensor, factors=facs, shape=torch.Size([f.shape[1] for f in facs]))


_STUB_CLASSES = (_StubDense, _StubTucker, _StubCP, _StubTT)


def install(ref_root: str = REF_ROOT):
    """Install the stand-ins and shell packages; return the reference modules."""
    if not ref_root:
        raise RuntimeError("set NOP_REFERENCE_ROOT to the reference checkout (the directory holding neuralop/)")
    if not os.path.isdir(os.path.join(ref_root, "neuralop")):
        raise FileNotFoundError(f"reference checkout not found under {ref_root}")
    tl = types.ModuleType("tensorly")
    tl.set_backend = lambda *a, **k: None
    tl.einsum = torch.einsum
    tl.ndim = lambda t: t.ndim
    plugins = types.ModuleType("tensorly.plugins")
    plugins.use_opt_einsum = lambda *a, **k: None
    tl.plugins = plugins
    tlt = types.ModuleType("tltorch")
    tlt_ft = types.ModuleType("tltorch.factorized_tensors")
    tlt_core = types.ModuleType("tltorch.factorized_tensors.core")
    tlt_core.FactorizedTensor = StubFactorizedTensor
    tlt.FactorizedTensor = StubFactorizedTensor
    tlt_ft.core = tlt_core
    tlt.factorized_tensors = tlt_ft
    stubs = {
        "tensorly": tl, "tensorly.plugins": plugins, "opt_einsum": types.ModuleType("opt_einsum"),
        "tltorch": tlt, "tltorch.factorized_tensors": tlt_ft, "tltorch.factorized_tensors.core": tlt_core,
    }
    for name, mod in stubs.items():
        sys.modules.setdefault(name, mod)
    for pkg, sub in (("neuralop", "neuralop"), ("neuralop.layers", "neuralop/layers"),
                     ("neuralop.models", "neuralop/models")):
        if pkg not in sys.modules:
            m = types.ModuleType(pkg)
            m.__path__ = [os.path.join(ref_root, sub)]
            m.__package__ = pkg
            sys.modules[pkg] = m
    mods = {}
    for name in ("neuralop.utils", "neuralop.layers.spectral_convolution", "neuralop.layers.fno_block",
                 "neuralop.models.fno"):
        mods[name.rsplit(".", 1)[1]] = importlib.import_module(name)
    return mods
