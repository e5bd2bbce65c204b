"""Spectral geometry of one SpectralConv call: which modes are kept and where they map.

This is the host-side half of ``SpectralConv.forward`` that decides, from the input
shape, the active ``n_modes``, ``max_n_modes`` and the output resolution:

* which part of the weight is used (the weight slice of
  neuralop/layers/spectral_convolution.py:465-489),
* how many modes each axis keeps and which DFT bin each kept mode is
  (the fftshift / centred-slice / ifftshift bookkeeping of :443-449, :500-519, :531-532),
* which last-axis bins are forced real before the inverse real FFT (:547-559),
* the forward / inverse scale factors for ``fft_norm`` (torch.fft ``norm=``).

The CUDA kernels never see shifts or slices: they receive, per axis, the number of kept
modes ``M`` and an offset ``off`` such that kept mode ``m`` is DFT bin
``u = (m - off) mod N``.  Everything here is plain Python (no device work).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import List, Optional, Sequence, Tuple


def active_modes(n_modes, complex_data: bool) -> List[int]:
    """The ``n_modes`` setter (spectral_convolution.py:404-415)."""
    modes = [int(n_modes)] if isinstance(n_modes, int) else [int(m) for m in n_modes]
    if not complex_data:
        modes[-1] = modes[-1] // 2 + 1
    return modes


@dataclass
class Geometry:
    order: int
    complex_data: bool
    n_in: List[int]
    n_out: List[int]
    kept: List[int]                       # modes per axis (weight mode dims after slicing)
    weight_slices: Tuple[slice, ...]      # slices over the weight's mode dims
    fwd_off: List[int]                    # kept mode m  ->  forward DFT bin (m - off) mod n_in
    inv_off: List[int]                    # kept mode m  ->  inverse bin index (m - off) mod n_in
    fwd_scale: float
    inv_scale: float
    zero_imag_bins: List[int] = field(default_factory=list)  # last-axis bins forced real (real data)

    @property
    def n_modes_total(self) -> int:
        return math.prod(self.kept)


def _scales(fft_norm: str, n_in: Sequence[int], n_out: Sequence[int]):
    p_in, p_out = math.prod(n_in), math.prod(n_out)
    if fft_norm == "forward":
        return 1.0 / p_in, 1.0
    if fft_norm == "backward":
        return 1.0, 1.0 / p_out
    if fft_norm == "ortho":
        return 1.0 / math.sqrt(p_in), 1.0 / math.sqrt(p_out)
    raise ValueError(f"fft_norm must be 'forward', 'backward' or 'ortho', got {fft_norm!r}")


def output_sizes(in_sizes: Sequence[int], resolution_scaling_factor=None, output_shape=None) -> List[int]:
    """Output spatial sizes (spectral_convolution.py:524-528)."""
    sizes = list(in_sizes)
    if resolution_scaling_factor is not None and output_shape is None:
        sizes = [round(s * r) for s, r in zip(sizes, resolution_scaling_factor)]
    if output_shape is not None:
        sizes = [int(s) for s in output_shape]
    return sizes


def compute_geometry(in_sizes: Sequence[int], modes: Sequence[int], max_modes: Sequence[int], *,
                     complex_data: bool = False, enforce_hermitian_symmetry: bool = True,
                     fft_norm: str = "forward", out_sizes: Optional[Sequence[int]] = None) -> Geometry:
    """Derive the kernel geometry for one forward call.

    ``modes`` are the active modes as stored by the setter (last axis already ``//2+1`` for
    real data) and ``max_modes`` the constructor's ``max_n_modes`` (weight mode dims).
    """
    order = len(modes)
    n_in = [int(s) for s in in_sizes]
    if len(n_in) != order:
        raise ValueError(f"input has {len(n_in)} spatial dims but n_modes has {order}")
    n_out = list(n_in) if out_sizes is None else [int(s) for s in out_sizes]
    fft_size = list(n_in)
    if not complex_data:
        fft_size[-1] = fft_size[-1] // 2 + 1

    # weight slice (spectral_convolution.py:465-489)
    starts = [mm - min(s, m) for s, m, mm in zip(fft_size, modes, max_modes)]
    centred = starts if complex_data else starts[:-1]
    w_slices = [slice(st // 2, -st // 2) if st else slice(st, None) for st in centred]
    if not complex_data:
        w_slices.append(slice(None, -starts[-1]) if starts[-1] else slice(None))
    kept = []
    for mm, sl in zip(max_modes, w_slices):
        kept.append(len(range(*sl.indices(mm))))
    for k, full in zip(kept, fft_size):
        if k < 1 or k > full:
            raise ValueError(f"kept modes {kept} incompatible with spectrum size {fft_size}")

    fwd_off, inv_off = [], []
    for j in range(order):
        last = j == order - 1
        if not last:
            # shifted, centred slice, un-shifted before the inverse
            fwd_off.append(kept[j] // 2)
            inv_off.append(kept[j] // 2)
        elif not complex_data:
            fwd_off.append(0)            # rFFT bins 0..kept-1
            inv_off.append(0)
        elif order > 1:
            fwd_off.append(n_in[j] // 2)  # leading bins of the fftshifted axis
            inv_off.append(0)             # the last axis is not un-shifted (:531-532)
        else:
            fwd_off.append(0)             # 1D complex: no shifts at all
            inv_off.append(0)

    fwd_scale, inv_scale = _scales(fft_norm, n_in, n_out)

    zero_imag = []
    if not complex_data:
        n_last = n_out[-1]
        zero_imag.append(0)
        if n_last % 2 == 0:
            zero_imag.append(n_last // 2)                     # the c2r transform reads only Re here
            if enforce_hermitian_symmetry:
                zero_imag.append(fft_size[-1] - 1)            # out_fft[..., -1].imag.zero_() (:555-556)
        zero_imag = sorted(set(zero_imag))

    return Geometry(order=order, complex_data=complex_data, n_in=n_in, n_out=n_out, kept=kept,
                    weight_slices=tuple(w_slices), fwd_off=fwd_off, inv_off=inv_off,
                    fwd_scale=fwd_scale, inv_scale=inv_scale, zero_imag_bins=zero_imag)


def adjoint_geometry(geo: Geometry) -> Geometry:
    """Geometry of the adjoint of one forward call (the input gradient is its forward on dL/dy).

    The forward is  y = inv_scale * c2r(pad(W . (fwd_scale * trunc(r2c(x)))));  its adjoint with respect
    to the real inner product is the same chain with the grids, the bin maps (fwd_off <-> inv_off) and the
    scales swapped and W replaced by its per-mode conjugate transpose: the c2r adjoint doubles interior
    last-axis bins and the r2c adjoint halves them, which cancel.  Only defined here for n_out == n_in
    (the Nyquist bin of one grid would otherwise be an interior bin of the other).
    """
    if list(geo.n_out) != list(geo.n_in):
        raise NotImplementedError("backward of a SpectralConv that resamples its output "
                                  f"({geo.n_in} -> {geo.n_out}) is not implemented")
    return Geometry(order=geo.order, complex_data=geo.complex_data, n_in=list(geo.n_out), n_out=list(geo.n_in),
                    kept=list(geo.kept), weight_slices=geo.weight_slices, fwd_off=list(geo.inv_off),
                    inv_off=list(geo.fwd_off), fwd_scale=geo.inv_scale, inv_scale=geo.fwd_scale,
                    zero_imag_bins=list(geo.zero_imag_bins))
