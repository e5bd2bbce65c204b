"""SpectralConv: drop-in for neuralop.layers.spectral_convolution.SpectralConv on B200.

Same constructor signature, parameters, ``n_modes`` property and ``forward`` /
``transform`` methods as the reference (neuralop/layers/spectral_convolution.py:183-570).
The forward runs entirely in libnop_b200's CUDA kernels: truncated forward FFT, per-mode
contraction, truncated inverse FFT and bias, with no full spectrum ever stored.  Inputs
must be CUDA tensors; there is no CPU path.

Two keyword arguments are added after the reference's:
``contraction_precision`` ("fp32" or "bf16": contraction operands rounded to bfloat16 with
float32 accumulation) and ``engine`` ("auto", "fast", "generic").

Backward (training) runs through the same kernels: the input gradient is the forward of the
adjoint plan (grids, bin maps and scales swapped, conjugate-transposed weights) and the weight /
bias gradients come from the kept spectra of x and dL/dy (nop_spectral_weight_grad); factorized
weights get their factor gradients from the reconstructed weight's gradient by the chain rule.

Differences that raise instead of silently diverging: ``fno_block_precision`` "half" /
"mixed" (complex-half einsum, neuralop/layers/einsum_utils.py) raises NotImplementedError;
backward through an output-resampling call, or through the fused GELU epilogue, raises
NotImplementedError.
"""

from __future__ import annotations

from typing import List, Optional, Tuple, Union

import torch
from torch import nn

from . import ops
from .factorized import CPTensor, DenseTensor, FactorizedTensor, TTTensor, TuckerTensor
from .geometry import Geometry, active_modes, adjoint_geometry, compute_geometry, output_sizes
from .utils import validate_scaling_factor

Number = Union[int, float]


class BaseSpectralConv(nn.Module):
    """Plugin base (neuralop/layers/base_spectral_conv.py:4-27)."""

    def __init__(self, device=None, dtype=None):
        super().__init__()
        self.dtype = dtype
        self.device = device

    def transform(self, x, output_shape=None):
        return x


class _Call:
    """One SpectralConv call: geometry, weight kind and options, with its forward and backward."""

    def __init__(self, module, geo: Geometry, kind: str, ranks, apply_gelu: bool, train: bool):
        self.module = module
        self.geo = geo
        self.kind = kind
        self.ranks = tuple(ranks)
        self.apply_gelu = apply_gelu
        self.train = train
        self.relay = None  # GradRelay of a fused FNO block: dL/dx of the block's chain call, added in backward

    def forward(self, x, weights, bias, addend, keep_spectrum=False):
        m = self.module
        cache = m.__dict__.setdefault("_nop_pack_cache", {})
        return ops.spectral_forward(x, self.geo, weights, out_channels=m.out_channels, weight_kind=self.kind,
                                    ranks=self.ranks, separable=m.separable, bias=bias, addend=addend,
                                    apply_gelu=self.apply_gelu, precision=m.contraction_precision, engine=m.engine,
                                    cache=cache, keep_spectrum=keep_spectrum)

    def backward(self, gy, weights, spec, need_x: bool, need_w: bool, need_b: bool, addend=None):
        """(dL/dx, [dL/d weight operand], dL/dbias [Co]) for dL/dy = gy; entries not needed are None.
        ``addend`` (x's shape) is added to dL/dx in the adjoint forward's last kernel."""
        m = self.module
        gy = gy.contiguous()
        adj_geo = adjoint_geometry(self.geo)
        packed = None
        if self.kind == "dense" and not m.separable:  # fused engine: conj transpose inside the packing kernel
            packed = ops.pack_adjoint_dense(adj_geo, gy.shape[0], weights[0], precision=m.contraction_precision,
                                            engine=m.engine)
        if packed is not None:
            adj_ws, adj_ranks = [], ()
        else:
            adj_ws, adj_ranks = ops.adjoint_operands(self.kind, weights, self.ranks, m.separable)
        gx, gspec = ops.spectral_forward(gy, adj_geo, adj_ws, out_channels=m.in_channels,
                                         weight_kind=self.kind, ranks=adj_ranks, separable=m.separable,
                                         precision=m.contraction_precision, engine=m.engine, keep_spectrum=True,
                                         packed=packed, addend=addend if need_x else None)
        lead = (m.in_channels,) if m.separable else (m.in_channels, m.out_channels)
        gw, gb = ops.weight_grad(spec, gspec, lead + tuple(self.geo.kept) if need_w else None,
                                 m.out_channels if need_b else 0)
        gws = None
        if need_w:
            if self.kind == "dense":
                gws = [gw.view(weights[0].shape)]
            elif self.kind == "tucker":
                gws = _tucker_grads(weights[0].detach(), [u.detach() for u in weights[1:]], gw)
            else:  # CP: chain rule through the reconstruction
                with torch.enable_grad():
                    leaves = [w.detach().requires_grad_() for w in weights]
                    gws = list(torch.autograd.grad(_cp_full(leaves[0], leaves[1:]), leaves, gw))
        return (gx if need_x else None), gws, gb


class _SpectralFn(torch.autograd.Function):
    """Forward and backward of one SpectralConv call through the CUDA kernels.

    The forward keeps the kept input spectrum when a gradient will be needed; the backward runs the
    adjoint forward on dL/dy and the weight / bias gradient kernel."""

    @staticmethod
    def forward(ctx, x, bias, addend, call, *weights):
        if not call.train:
            return call.forward(x, list(weights), bias, addend)
        if call.apply_gelu:
            raise NotImplementedError("the fused GELU epilogue has no backward; call SpectralConv without "
                                      "apply_gelu (FNOBlocks does so whenever a gradient is needed)")
        y, spec = call.forward(x, list(weights), bias, addend, keep_spectrum=True)
        ctx.call = call
        ctx.spec = spec
        ctx.bias_shape = None if bias is None else tuple(bias.shape)
        ctx.save_for_backward(*weights)
        return y

    @staticmethod
    def backward(ctx, gy):
        weights = list(ctx.saved_tensors)
        need_x, need_b, need_a = ctx.needs_input_grad[:3]
        need_w = any(ctx.needs_input_grad[4:])
        need_b = bool(need_b and ctx.bias_shape is not None)
        # a fused FNO block's chain call hands its dL/dx here (the same x), so both gradients of x leave
        # the adjoint forward's last kernel as one tensor instead of autograd adding them in another pass
        relay = ctx.call.relay.take() if ctx.call.relay is not None else None
        gx, gws, gb = ctx.call.backward(gy, weights, ctx.spec, need_x, need_w, need_b, addend=relay)
        if gb is not None:
            gb = gb.view(ctx.bias_shape)
        ga = gy if need_a else None
        gws = gws if gws is not None else [None] * len(weights)
        return (gx, gb, ga, None, *gws)


class SpectralConv(BaseSpectralConv):
    """Fourier layer: rFFT -> keep n_modes -> per-mode channel contraction -> irFFT -> + bias."""

    def __init__(self, in_channels, out_channels, n_modes, complex_data=False, max_n_modes=None, bias=True,
                 separable=False, resolution_scaling_factor: Optional[Union[Number, List[Number]]] = None,
                 fno_block_precision="full", rank=1.0, factorization=None, implementation="reconstructed",
                 enforce_hermitian_symmetry=True, fixed_rank_modes=False, decomposition_kwargs: Optional[dict] = None,
                 init_std="auto", fft_norm="forward", device=None, contraction_precision="fp32", engine="auto"):
        super().__init__(device=device)
        self.in_channels = in_channels
        self.out_channels = out_channels
        self.complex_data = complex_data
        self.n_modes = n_modes
        self.order = len(self.n_modes)
        if max_n_modes is None:
            max_n_modes = self.n_modes
        elif isinstance(max_n_modes, int):
            max_n_modes = [max_n_modes]
        self.max_n_modes = max_n_modes
        self.fno_block_precision = fno_block_precision
        self.rank = rank
        self.factorization = factorization
        self.implementation = implementation
        self.enforce_hermitian_symmetry = enforce_hermitian_symmetry
        self.resolution_scaling_factor = validate_scaling_factor(resolution_scaling_factor, self.order)
        if contraction_precision not in ("fp32", "bf16"):
            raise ValueError("contraction_precision must be 'fp32' or 'bf16'")
        self.contraction_precision = contraction_precision
        self.engine = engine
        if init_std == "auto":
            init_std = (2 / (in_channels + out_channels)) ** 0.5
        if isinstance(fixed_rank_modes, bool):
            fixed_rank_modes = [0] if fixed_rank_modes else None
        self.fft_norm = fft_norm
        if factorization is None:
            factorization = "Dense"
        if separable:
            if in_channels != out_channels:
                raise ValueError("To use separable Fourier Conv, in_channels must be equal to out_channels, "
                                 f"but got in_channels={in_channels} and out_channels={out_channels}")
            weight_shape = (in_channels, *max_n_modes)
        else:
            weight_shape = (in_channels, out_channels, *max_n_modes)
        self.separable = separable
        if implementation not in ("reconstructed", "factorized"):
            raise ValueError(f'Got implementation={implementation}, expected "reconstructed" or "factorized"')
        kwargs = decomposition_kwargs if decomposition_kwargs is not None else {}
        self.weight = FactorizedTensor.new(weight_shape, rank=self.rank, factorization=factorization,
                                           fixed_rank_modes=fixed_rank_modes, **kwargs, dtype=torch.cfloat,
                                           device=device)
        self.weight.normal_(0, init_std)
        if bias:
            self.bias = nn.Parameter(init_std * torch.randn(*((self.out_channels,) + (1,) * self.order),
                                                            device=device))
        else:
            self.bias = None

    # -- reference API -------------------------------------------------------------------------
    @property
    def n_modes(self):
        return self._n_modes

    @n_modes.setter
    def n_modes(self, n_modes):
        self._n_modes = active_modes(n_modes, self.complex_data)

    def transform(self, x, output_shape=None):
        """Resample a skip connection to the output resolution (spectral_convolution.py:383-398)."""
        in_shape = list(x.shape[2:])
        if self.resolution_scaling_factor is not None and output_shape is None:
            out_shape = tuple(round(s * r) for s, r in zip(in_shape, self.resolution_scaling_factor))
        elif output_shape is not None:
            out_shape = output_shape
        else:
            out_shape = in_shape
        if list(in_shape) == list(out_shape):
            return x
        from .layers import resample
        return resample(x, 1.0, list(range(2, x.ndim)), output_shape=out_shape)

    # -- geometry and kernel operands -------------------------------------------------------------
    def geometry(self, in_sizes, output_shape=None) -> Geometry:
        out = output_sizes(in_sizes, self.resolution_scaling_factor, output_shape)
        return compute_geometry(in_sizes, self.n_modes, self.max_n_modes, complex_data=self.complex_data,
                                enforce_hermitian_symmetry=self.enforce_hermitian_symmetry, fft_norm=self.fft_norm,
                                out_sizes=out)

    def kernel_operands(self, geo: Geometry):
        """(weight_kind, [tensors], ranks) for the kernels: the weight slice of :465-489."""
        lead = (slice(None),) * (1 if self.separable else 2)
        idx = lead + geo.weight_slices
        w = self.weight
        factorized = self.implementation == "factorized"
        if isinstance(w, DenseTensor):
            return "dense", [w.tensor[idx]], ()
        if isinstance(w, TuckerTensor):
            core, facs = w.sliced(idx)
            if factorized:
                return "tucker", [core] + facs, tuple(core.shape)
            return "dense", [_tucker_full(core, facs)], ()
        if isinstance(w, CPTensor):
            lam, facs = w.sliced(idx)
            if factorized:
                return "cp", [lam] + facs, (lam.shape[0],)
            return "dense", [_cp_full(lam, facs)], ()
        if isinstance(w, TTTensor):
            # tensor-train weights run as the reconstructed dense weight (same math, other rounding)
            return "dense", [w.to_tensor(w.sliced(idx))], ()
        if torch.is_tensor(w):
            return "dense", [w[idx]], ()
        raise ValueError(f"unexpected weight type {type(w).__name__}")

    def forward(self, x: torch.Tensor, output_shape: Optional[Tuple[int]] = None, *, addend=None,
                apply_gelu: bool = False):
        """Spectral convolution of x (batch, channels, d1, ..., dN).

        ``addend`` / ``apply_gelu`` fuse FNOBlocks' skip add and activation into the same
        kernel: returns gelu(conv(x) + addend) (neuralop/layers/fno_block.py:356-361).
        """
        if self.fno_block_precision in ("half", "mixed"):
            raise NotImplementedError("fno_block_precision='half'/'mixed' is not implemented; use "
                                      "contraction_precision='bf16' for a reduced-precision contraction")
        if not x.is_cuda:
            raise RuntimeError("neuraloperator_b200.SpectralConv needs CUDA tensors; there is no CPU path")
        geo = self.geometry(list(x.shape[2:]), output_shape)
        kind, weights, ranks = self.kernel_operands(geo)
        bias = None if self.bias is None else self.bias
        train = torch.is_grad_enabled() and any(
            t is not None and t.requires_grad for t in (x, bias, addend, *weights))
        if train and geo.n_out != geo.n_in:
            raise NotImplementedError("backward of a SpectralConv that resamples its output is not implemented; "
                                      "run it under torch.no_grad()")
        call = _Call(self, geo, kind, ranks, apply_gelu, train)
        # set by FNOBlocks.fused_block for this one call (pointwise.GradRelay); taken here so that a later
        # call of the module never sees it
        call.relay = self.__dict__.pop("_nop_grad_relay", None) if train else None
        self.__dict__.pop("_nop_grad_relay", None)
        return _SpectralFn.apply(x, bias, addend, call, *weights)

    @torch.no_grad()
    def forward_host(self, x: torch.Tensor, output_shape: Optional[Tuple[int]] = None, *, addend=None,
                     apply_gelu: bool = False, chunk: Optional[int] = None, n_streams: int = 3, out=None,
                     synchronize: bool = True):
        """``forward`` for a batch held in host memory, with the PCIe copies of one chunk of the batch
        overlapped with the kernels and copies of the others (nop_spectral_forward_host).  ``x``,
        ``addend`` and ``out`` are CPU tensors (page-locked for the overlap); this module's parameters
        stay on their CUDA device.  Inference only (no autograd graph)."""
        if self.fno_block_precision in ("half", "mixed"):
            raise NotImplementedError("fno_block_precision='half'/'mixed' is not implemented")
        geo = self.geometry(list(x.shape[2:]), output_shape)
        kind, weights, ranks = self.kernel_operands(geo)
        cache = self.__dict__.setdefault("_nop_pack_cache", {})
        return ops.spectral_forward_host(x, geo, weights, out_channels=self.out_channels, device=weights[0].device,
                                         weight_kind=kind, ranks=ranks, separable=self.separable, bias=self.bias,
                                         addend=addend, apply_gelu=apply_gelu, precision=self.contraction_precision,
                                         engine=self.engine, chunk=chunk, n_streams=n_streams, out=out, cache=cache,
                                         synchronize=synchronize)


def _tucker_full(core, factors):
    t = core
    for mode, u in enumerate(factors):
        t = torch.tensordot(u, t.movedim(mode, 0), dims=([1], [0])).movedim(0, mode)
    return t


def _cp_full(lam, factors):
    sy = "abcdefghijklmnop"
    eq = "z," + ",".join(sy[i] + "z" for i in range(len(factors))) + "->" + sy[: len(factors)]
    return torch.einsum(eq, lam, *factors)


def _tucker_grads(core, factors, gw):
    """Gradients of (core, U_0..U_{n-1}) for W = core x_0 U_0 ... x_{n-1} U_{n-1} given dL/dW = gw, on the
    library's kernels (nop_tucker_grads): dL/dcore = gw x_0 conj(U_0) ... x_{n-1} conj(U_{n-1}) and
    dL/dU_k = sum over modes j != k of (gw x_j conj(U_j) for j != k) * conj(core), the values autograd
    of the reconstruction (spectral_convolution.py:76-103) gives."""
    return ops.tucker_grads(core, factors, gw)
