"""Plain-PyTorch CPU restatement of the reference FNO spectral block (TEST INFRASTRUCTURE).

Every function below restates one piece of the reference forward path of
AnirudhG07/neuraloperator v2.0.0 and cites the reference file:line it follows.  The
arithmetic is the reference's own sequence of ``torch.fft`` / ``torch.einsum`` calls
(``tensorly.einsum`` with the pytorch backend is ``torch.einsum``), so results agree
with the reference to float32 rounding.  Parameters are passed explicitly (plain
tensors / dicts) rather than as modules, so the oracle does not depend on the product
package it checks.

Weight containers used by the oracle:

* dense:   complex tensor ``(Ci, Co, *modes)`` (or ``(C, *modes)`` when separable)
* tucker:  ``{"core": (r0, r1, *r), "factors": [U_in (Ci,r0), U_out (Co,r1), U_1 (m1,r2), ...]}``
* cp:      ``{"weights": (R,), "factors": [U_in (Ci,R), U_out (Co,R), U_1 (m1,R), ...]}``
* tt:      ``{"factors": [G_0 (1,Ci,r1), G_1 (r1,Co,r2), ..., G_last (r,m_last,1)]}``

(the separable variants drop the ``U_out`` / ``G_1`` entry, as in the reference.)
"""

from __future__ import annotations

import itertools
from typing import List, Optional, Sequence

import torch
import torch.nn.functional as F

# Index alphabet used to build einsum equations (spectral_convolution.py:18).
_SYMBOLS = "abcdefghijklmnopqrstuvwxyzABCDEFGHIJKLMNOPQRSTUVWXYZ"


# ----------------------------------------------------------------------------------
# n_modes bookkeeping
# ----------------------------------------------------------------------------------
def effective_modes(n_modes, complex_data: bool = False) -> List[int]:
    """The ``SpectralConv.n_modes`` setter (spectral_convolution.py:404-415).

    For real data the last axis keeps ``m // 2 + 1`` rFFT bins.
    """
    modes = [int(n_modes)] if isinstance(n_modes, int) else [int(m) for m in n_modes]
    if not complex_data:
        modes[-1] = modes[-1] // 2 + 1
    return modes


# ----------------------------------------------------------------------------------
# contractions (spectral_convolution.py:21-132)
# ----------------------------------------------------------------------------------
def contract_dense(x: torch.Tensor, w: torch.Tensor, separable: bool = False) -> torch.Tensor:
    """``_contract_dense`` (spectral_convolution.py:21-46) and ``_contract_dense_separable`` (:49-52).

    Non-separable: ``b i <modes>, i o <modes> -> b o <modes>``.
    """
    order = x.ndim
    xs = _SYMBOLS[:order]
    if separable:
        eq = f"{xs},{xs[1:]}->{xs}"
    else:
        o = _SYMBOLS[order]
        eq = f"{xs},{xs[1]}{o}{xs[2:]}->{xs[0]}{o}{xs[2:]}"
    return torch.einsum(eq, x, w)


def contract_tucker(x: torch.Tensor, core: torch.Tensor, factors: Sequence[torch.Tensor],
                    separable: bool = False) -> torch.Tensor:
    """``_contract_tucker`` (spectral_convolution.py:76-103).

    Non-separable 2D example: ``abcd,fghi,bf,eg,ch,di->aecd``.  The reference evaluates the equation with
    opt_einsum choosing the pairwise order; torch.einsum without opt_einsum (not installed here) would
    contract left to right and form the outer product of x and the core (hundreds of GB at the TFNO
    configuration's size).  The same sum is therefore taken in an explicit order -- the core expanded
    over the spatial factors, then the input factor, the expanded core per mode, the output factor --
    which changes only the rounding, as opt_einsum's choice does.
    """
    order = x.ndim
    xs = _SYMBOLS[:order]
    a, b, modes = xs[0], xs[1], xs[2:]
    o, ri, ro = _SYMBOLS[order:order + 3]
    lead = 1 if separable else 2
    g = core
    for j, u in enumerate(factors[lead:]):  # the core over each spatial factor: r_j -> m_j
        g = torch.tensordot(u, g.movedim(lead + j, 0), dims=([1], [0])).movedim(0, lead + j)
    if separable:
        return x * torch.einsum(f"{ri}{modes},{b}{ri}->{b}{modes}", g, factors[0])
    t = torch.einsum(f"{xs},{b}{ri}->{a}{ri}{modes}", x, factors[0])
    t = torch.einsum(f"{a}{ri}{modes},{ri}{ro}{modes}->{a}{ro}{modes}", t, g)
    return torch.einsum(f"{a}{ro}{modes},{o}{ro}->{a}{o}{modes}", t, factors[1])


def contract_cp(x: torch.Tensor, weights: torch.Tensor, factors: Sequence[torch.Tensor],
                separable: bool = False) -> torch.Tensor:
    """``_contract_cp`` (spectral_convolution.py:55-73). 2D: ``abcd,e,be,fe,ce,de->afcd``.

    Evaluated in an explicit pairwise order (input factor, the rank-wise weights and spatial factors,
    output factor) for the reason given at contract_tucker; only the rounding differs."""
    order = x.ndim
    xs = _SYMBOLS[:order]
    a, b, modes = xs[0], xs[1], xs[2:]
    o, r = _SYMBOLS[order:order + 2]
    lead = 1 if separable else 2
    # w[r, modes] = weights[r] prod_j U_j[m_j, r]
    w = weights.reshape(-1, *([1] * len(modes)))
    for j, u in enumerate(factors[lead:]):
        shape = [1] * (1 + len(modes))
        shape[0], shape[1 + j] = u.shape[1], u.shape[0]
        w = w * u.transpose(0, 1).reshape(shape)
    if separable:
        return x * torch.einsum(f"{r}{modes},{b}{r}->{b}{modes}", w, factors[0])
    t = torch.einsum(f"{xs},{b}{r}->{a}{r}{modes}", x, factors[0]) * w.unsqueeze(0)
    return torch.einsum(f"{a}{r}{modes},{o}{r}->{a}{o}{modes}", t, factors[1])


def contract_tt(x: torch.Tensor, factors: Sequence[torch.Tensor], separable: bool = False) -> torch.Tensor:
    """``_contract_tt`` (spectral_convolution.py:106-132). 2D: ``abcd,fbg,geh,hci,idj->aecd``."""
    order = x.ndim
    xs = list(_SYMBOLS[:order])
    ws = list(xs[1:])
    if not separable:
        ws.insert(1, _SYMBOLS[order])
        out = list(ws)
        out[0] = xs[0]
    else:
        out = list(xs)
    rs = list(_SYMBOLS[order + 1:])
    tts = ["".join((rs[i], s, rs[i + 1])) for i, s in enumerate(ws)]
    eq = "".join(xs) + "," + ",".join(tts) + "->" + "".join(out)
    return torch.einsum(eq, x, *factors)


def tucker_to_dense(core, factors):
    """Full tensor of a Tucker decomposition (core times each factor along its mode)."""
    t = core
    for mode, u in enumerate(factors):
        t = torch.tensordot(u, t.movedim(mode, 0), dims=([1], [0])).movedim(0, mode)
    return t


def cp_to_dense(weights, factors):
    """Full tensor of a CP decomposition: sum_r w_r  u_0[:, r] o u_1[:, r] o ..."""
    order = len(factors)
    r = _SYMBOLS[order]
    eq = r + "," + ",".join(_SYMBOLS[i] + r for i in range(order)) + "->" + _SYMBOLS[:order]
    return torch.einsum(eq, weights, *factors)


def tt_to_dense(factors):
    """Full tensor of a tensor-train decomposition (chain of 3-way cores)."""
    t = factors[0]
    for g in factors[1:]:
        t = torch.tensordot(t, g, dims=([t.ndim - 1], [0]))
    return t.squeeze(0).squeeze(-1)


def _slice_weight(weight, kind: str, mode_slices: Sequence[slice], separable: bool):
    """``self.weight[slices_w]`` (spectral_convolution.py:465-489) for each weight container.

    Slicing a factorized tensor slices the factor that carries each mode (the
    tensorly-torch ``__getitem__`` semantics for slice indices).
    """
    lead = 1 if separable else 2
    if kind == "dense":
        return weight[(slice(None),) * lead + tuple(mode_slices)]
    factors = list(weight["factors"])
    if kind == "tt":
        for j, s in enumerate(mode_slices):
            factors[lead + j] = factors[lead + j][:, s, :]
        return {"factors": factors}
    for j, s in enumerate(mode_slices):
        factors[lead + j] = factors[lead + j][s]
    out = dict(weight)
    out["factors"] = factors
    return out


def _weight_mode_shape(weight, kind: str, separable: bool) -> List[int]:
    lead = 1 if separable else 2
    if kind == "dense":
        return list(weight.shape[lead:])
    if kind == "tt":
        return [f.shape[1] for f in weight["factors"][lead:]]
    return [f.shape[0] for f in weight["factors"][lead:]]


def _contract(x, weight, kind: str, separable: bool):
    """``get_contract_fun`` dispatch (spectral_convolution.py:135-177)."""
    if kind == "dense":
        return contract_dense(x, weight, separable)
    if kind == "tucker":
        return contract_tucker(x, weight["core"], weight["factors"], separable)
    if kind == "cp":
        return contract_cp(x, weight["weights"], weight["factors"], separable)
    if kind == "tt":
        return contract_tt(x, weight["factors"], separable)
    raise ValueError(f"unknown weight kind {kind!r}")


# ----------------------------------------------------------------------------------
# SpectralConv.forward
# ----------------------------------------------------------------------------------
def spectral_conv(x: torch.Tensor, weight, bias: Optional[torch.Tensor], n_modes,
                  max_n_modes=None, *, weight_kind: str = "dense", complex_data: bool = False,
                  separable: bool = False, enforce_hermitian_symmetry: bool = True,
                  fft_norm: str = "forward", output_shape=None,
                  resolution_scaling_factor=None) -> torch.Tensor:
    """``SpectralConv.forward`` (spectral_convolution.py:417-570).

    ``n_modes`` is the user-facing value (before the ``//2+1`` of the setter);
    ``max_n_modes`` follows the constructor rule (spectral_convolution.py:317-321).
    ``resolution_scaling_factor`` is a per-axis list (already validated).
    """
    modes = effective_modes(n_modes, complex_data)
    order = len(modes)
    if max_n_modes is None:
        max_modes = list(modes)
    elif isinstance(max_n_modes, int):
        max_modes = [max_n_modes]
    else:
        max_modes = list(max_n_modes)

    batch, _, *sizes = x.shape
    fft_size = list(sizes)
    if not complex_data:
        fft_size[-1] = fft_size[-1] // 2 + 1
    dims = list(range(-order, 0))

    # :439-449  forward transform, shift non-last (or all, complex) axes
    if complex_data:
        xf = torch.fft.fftn(x, norm=fft_norm, dim=dims)
        shift_dims = dims
    else:
        xf = torch.fft.rfftn(x, norm=fft_norm, dim=dims)
        shift_dims = dims[:-1]
    if order > 1:
        xf = torch.fft.fftshift(xf, dim=shift_dims)

    # :465-489  weight slice when the active modes are below max_n_modes
    starts = [mm - min(s, m) for s, m, mm in zip(fft_size, modes, max_modes)]
    centred = starts if complex_data else starts[:-1]
    w_slices = [slice(st // 2, -st // 2) if st else slice(st, None) for st in centred]
    if not complex_data:
        w_slices.append(slice(None, -starts[-1]) if starts[-1] else slice(None))
    w = _slice_weight(weight, weight_kind, w_slices, separable)
    kept = _weight_mode_shape(w, weight_kind, separable)

    # :500-519  centred slice of the shifted spectrum; the last axis keeps the leading bins
    x_slices = [slice(None), slice(None)]
    for full, k in zip(fft_size, kept):
        c = full // 2
        x_slices.append(slice(c - k // 2, c + k // 2 + k % 2))
    x_slices[-1] = slice(None, kept[-1]) if kept[-1] < fft_size[-1] else slice(None)
    x_slices = tuple(x_slices)

    out_channels = _out_channels(w, weight_kind, separable, x.shape[1])
    out_fft = torch.zeros([batch, out_channels, *fft_size], dtype=torch.cfloat)
    out_fft[x_slices] = _contract(xf[x_slices], w, weight_kind, separable)

    # :524-529  output resolution
    mode_sizes = list(sizes)
    if resolution_scaling_factor is not None and output_shape is None:
        mode_sizes = [round(s * r) for s, r in zip(mode_sizes, resolution_scaling_factor)]
    if output_shape is not None:
        mode_sizes = list(output_shape)

    # :531-564  un-shift the non-last axes, inverse transform with the Hermitian fix-up
    if order > 1:
        out_fft = torch.fft.ifftshift(out_fft, dim=dims[:-1])
    if complex_data:
        y = torch.fft.ifftn(out_fft, s=mode_sizes, dim=dims, norm=fft_norm)
    elif enforce_hermitian_symmetry:
        out_fft = torch.fft.ifftn(out_fft, s=mode_sizes[:-1], dim=dims[:-1], norm=fft_norm)
        out_fft[..., 0].imag.zero_()
        if mode_sizes[-1] % 2 == 0:
            out_fft[..., -1].imag.zero_()
        y = torch.fft.irfft(out_fft, n=mode_sizes[-1], dim=dims[-1], norm=fft_norm)
    else:
        y = torch.fft.irfftn(out_fft, s=mode_sizes, dim=dims, norm=fft_norm)

    # :567-568  bias (Co, 1, ..., 1)
    if bias is not None:
        y = y + bias
    return y


def _out_channels(w, kind, separable, in_channels):
    if separable:
        return in_channels
    if kind == "dense":
        return w.shape[1]
    if kind == "tt":
        return w["factors"][1].shape[1]
    return w["factors"][1].shape[0]


# ----------------------------------------------------------------------------------
# resample (neuralop/layers/resample.py:7-80), used by SpectralConv.transform for skips
# ----------------------------------------------------------------------------------
def resample(x: torch.Tensor, res_scale, axis, output_shape=None) -> torch.Tensor:
    """``resample`` (resample.py:7-80): linear (1D) / bicubic (2D) / spectral (>=3D)."""
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
    out = torch.zeros([x.shape[0], x.shape[1], *nf], dtype=torch.cfloat)
    bounds = [((None, m // 2), (-m // 2, None)) for m in nfc[:-1]] + [((None, nfc[-1]),)]
    for b in itertools.product(*bounds):
        idx = (slice(None), slice(None)) + tuple(slice(*e) for e in b)
        out[idx] = X[idx]
    return torch.fft.irfftn(out, s=new, norm="forward", dim=axis)


# ----------------------------------------------------------------------------------
# FNO pieces around the spectral block
# ----------------------------------------------------------------------------------
def grid_embedding(x: torch.Tensor, boundaries=None) -> torch.Tensor:
    """``GridEmbeddingND.forward`` (embeddings.py:147-164) with ``regular_grid_nd`` (:351-383)."""
    dims = list(x.shape[2:])
    if boundaries is None:
        boundaries = [[0.0, 1.0]] * len(dims)
    axes = [torch.linspace(a, b, n + 1)[:-1] for n, (a, b) in zip(dims, boundaries)]
    grids = torch.meshgrid(*axes, indexing="ij")
    grids = [g.to(x.dtype).unsqueeze(0).unsqueeze(0).repeat(x.shape[0], *[1] * (len(dims) + 1))
             for g in grids]
    return torch.cat((x, *grids), dim=1)


def _conv1x1(h: torch.Tensor, w: torch.Tensor, b: Optional[torch.Tensor] = None) -> torch.Tensor:
    """A kernel-size-1 Conv1d ([out, in, 1] weight) on h [B, in, L] as a matrix product: the same sums as
    F.conv1d, through BLAS (conv1d's CPU kernels crashed on lines of 2^24 points in one environment)."""
    out = torch.matmul(w.reshape(w.shape[0], -1), h)
    return out if b is None else out + b.reshape(1, -1, 1)


def channel_mlp(x: torch.Tensor, layers, non_linearity=F.gelu) -> torch.Tensor:
    """``ChannelMLP.forward`` (channel_mlp.py:82-119): 1x1 Conv1d layers with GELU between."""
    size = list(x.shape)
    h = x.reshape(size[0], size[1], -1) if x.ndim > 3 else x
    for i, (w, b) in enumerate(layers):
        h = _conv1x1(h, w, b)
        if i < len(layers) - 1:
            h = non_linearity(h)
    if x.ndim > 3:
        h = h.reshape(size[0], h.shape[1], *size[2:])
    return h


def skip(x: torch.Tensor, kind: Optional[str], weight) -> torch.Tensor:
    """``skip_connection`` (skip_connections.py:5-127): linear = flattened 1x1 conv, no bias."""
    kind = kind.lower()
    if kind == "identity":
        return x
    if kind == "soft-gating":
        return weight * x
    if kind == "linear":
        size = list(x.shape)
        h = _conv1x1(x.reshape(size[0], size[1], -1), weight)
        return h.reshape(size[0], weight.shape[0], *size[2:])
    raise ValueError(kind)


def fno_block(x: torch.Tensor, blk: dict, index: int, n_layers: int, cfg: dict) -> torch.Tensor:
    """``FNOBlocks.forward_with_postactivation`` (fno_block.py:327-381), norm=None, no stabilizer.

    ``preactivation=True`` follows ``forward_with_preactivation`` (fno_block.py:383-437).
    """
    act = cfg.get("non_linearity", F.gelu)
    conv = lambda h: spectral_conv(
        h, blk["weight"], blk.get("bias"), cfg["n_modes"], cfg.get("max_n_modes"),
        weight_kind=cfg.get("weight_kind", "dense"), separable=cfg.get("separable", False),
        enforce_hermitian_symmetry=cfg.get("enforce_hermitian_symmetry", True))
    fno_skip = cfg.get("fno_skip", "linear")
    mlp_skip = cfg.get("channel_mlp_skip", "soft-gating")
    use_mlp = cfg.get("use_channel_mlp", True)
    last = index >= n_layers - 1
    if cfg.get("preactivation", False):
        x = act(x)
        xs = skip(x, fno_skip, blk.get("fno_skip")) if fno_skip else None
        xm = skip(x, mlp_skip, blk.get("mlp_skip")) if (use_mlp and mlp_skip) else None
        x = conv(x)
        x = x + xs if xs is not None else x
        if not last:
            x = act(x)
        if use_mlp:
            x = channel_mlp(x, blk["mlp"])
            if xm is not None:
                x = x + xm
        return x
    xs = skip(x, fno_skip, blk.get("fno_skip")) if fno_skip else None
    xm = skip(x, mlp_skip, blk.get("mlp_skip")) if (use_mlp and mlp_skip) else None
    x = conv(x)
    x = x + xs if xs is not None else x
    if not last:
        x = act(x)
    if use_mlp:
        x = channel_mlp(x, blk["mlp"])
        if xm is not None:
            x = x + xm
    if not last:
        x = act(x)
    return x


def fno_forward(x: torch.Tensor, params: dict, cfg: dict) -> torch.Tensor:
    """``FNO.forward`` (fno.py:342-408): grid embedding, lifting, blocks, projection.

    ``params = {"lifting": [(W, b), ...], "projection": [(W, b), ...], "blocks": [blk, ...]}``;
    each ``blk`` holds ``weight``, ``bias``, ``fno_skip``, ``mlp`` and ``mlp_skip``.
    With ``cfg["n_modes_per_layer"]`` (and optionally ``cfg["max_n_modes_per_layer"]``) block i uses its own
    modes: ``FNOStaged.forward`` (neuralop/models/fno_staged.py:456-502), whose blocks repeat FNOBlocks'.
    """
    if cfg.get("positional_embedding", "grid") == "grid":
        x = grid_embedding(x)
    x = channel_mlp(x, params["lifting"])
    n_layers = len(params["blocks"])
    per_layer = cfg.get("n_modes_per_layer")
    for i, blk in enumerate(params["blocks"]):
        c = cfg
        if per_layer is not None:
            c = dict(cfg, n_modes=per_layer[i])
            if cfg.get("max_n_modes_per_layer") is not None:
                c["max_n_modes"] = cfg["max_n_modes_per_layer"][i]
        x = fno_block(x, blk, i, n_layers, c)
    return channel_mlp(x, params["projection"])
