"""Direct-DFT formulation of the spectral block in float64 (TEST INFRASTRUCTURE).

The CUDA kernels do not shift, pad or slice spectra.  They evaluate, per axis, a
truncated DFT whose kept mode ``m`` is bin ``u = (m - off) mod N``, contract the kept
modes, and evaluate the inverse only at the kept bins.  This module writes that
formulation out with explicit DFT matrices in float64 so the tests can show it equals
the reference's fftshift/slice/ifftshift/irfft sequence
(neuralop/layers/spectral_convolution.py:417-570) on every golden case.

Inputs are the per-axis numbers the kernels receive: ``n_in``, ``n_out``, ``kept``,
``fwd_off``, ``inv_off``, the two scales and the last-axis bins forced real.
"""

from __future__ import annotations

import math

import torch


def _fwd_matrix(n: int, kept: int, off: int) -> torch.Tensor:
    """(kept, n) matrix  F[m, t] = exp(-2 pi i u(m) t / n),  u(m) = (m - off) mod n."""
    m = torch.arange(kept, dtype=torch.float64)
    u = torch.remainder(m - off, n)
    t = torch.arange(n, dtype=torch.float64)
    ang = -2.0 * math.pi * torch.remainder(torch.outer(u, t), n) / n
    return torch.polar(torch.ones_like(ang), ang)


def _inv_matrix(n_in: int, n_out: int, kept: int, off: int) -> torch.Tensor:
    """(n_out, kept) matrix for the complex inverse of an axis (ifftn with s=n_out).

    Mode m sits at index u(m) = (m - off) mod n_in of the un-shifted spectrum; ifftn with
    s=n_out keeps indices < n_out (truncate / zero-pad at the end) and treats index u
    as frequency u of an n_out-point transform.
    """
    m = torch.arange(kept, dtype=torch.float64)
    u = torch.remainder(m - off, n_in)
    t = torch.arange(n_out, dtype=torch.float64)
    ang = 2.0 * math.pi * torch.remainder(torch.outer(t, u), n_out) / n_out
    mat = torch.polar(torch.ones_like(ang), ang)
    mat[:, u >= n_out] = 0
    return mat


def _apply(mat: torch.Tensor, x: torch.Tensor, axis: int) -> torch.Tensor:
    x = x.movedim(axis, -1)
    y = x @ mat.transpose(0, 1)
    return y.movedim(-1, axis)


def forward_spectrum(x: torch.Tensor, n_in, kept, fwd_off, fwd_scale, complex_data: bool) -> torch.Tensor:
    """Kept modes of the (scaled) forward transform, layout (B, C, *kept)."""
    order = len(n_in)
    h = x.to(torch.complex128)
    for j in reversed(range(order)):          # last axis first, as the kernels do
        axis = 2 + j
        h = _apply(_fwd_matrix(n_in[j], kept[j], fwd_off[j]), h, axis)
    return h * fwd_scale


def inverse(spec: torch.Tensor, n_in, n_out, kept, inv_off, inv_scale, complex_data: bool,
            zero_imag_bins) -> torch.Tensor:
    """Inverse of the kept modes onto the output grid (real data: Hermitian c2r last axis)."""
    order = len(n_in)
    h = spec.to(torch.complex128)
    last_complex = order if complex_data else order - 1
    for j in range(last_complex):
        h = _apply(_inv_matrix(n_in[j], n_out[j], kept[j], inv_off[j]), h, 2 + j)
    if complex_data:
        return h * inv_scale
    # real last axis: bins k = m (offset 0), k <= n_out//2 used, weights 1 / 2 / 1
    n = n_out[-1]
    k_used = min(kept[-1], n // 2 + 1)
    h = h[..., :k_used].clone()
    for b in zero_imag_bins:
        if b < k_used:
            h[..., b] = h[..., b].real.to(h.dtype)
    k = torch.arange(k_used, dtype=torch.float64)
    wts = torch.full((k_used,), 2.0, dtype=torch.float64)
    wts[0] = 1.0
    if n % 2 == 0 and n // 2 < k_used:
        wts[n // 2] = 1.0
    t = torch.arange(n, dtype=torch.float64)
    ang = 2.0 * math.pi * torch.remainder(torch.outer(t, k), n) / n
    c, s = torch.cos(ang) * wts, torch.sin(ang) * wts
    y = h.real @ c.transpose(0, 1) - h.imag @ s.transpose(0, 1)
    return y * inv_scale


def spectral_conv_direct(x, w_dense, bias, *, n_in, n_out, kept, fwd_off, inv_off, fwd_scale, inv_scale,
                         complex_data, zero_imag_bins, separable=False):
    """Full forward in the kernels' formulation (float64); ``w_dense`` is the sliced weight."""
    xs = forward_spectrum(x, n_in, kept, fwd_off, fwd_scale, complex_data)
    w = w_dense.to(torch.complex128)
    if separable:
        ys = xs * w
    else:
        ys = torch.einsum("bi...,io...->bo...", xs, w)
    y = inverse(ys, n_in, n_out, kept, inv_off, inv_scale, complex_data, zero_imag_bins)
    if bias is not None:
        y = y + bias.to(torch.float64)
    return y


def mode_factors(kept, n_out, complex_data: bool) -> torch.Tensor:
    """Per-mode factor d_t of the weight gradient, shape ``kept`` (float64).

    torch's backward of the c2r inverse (irfft, neuralop/layers/spectral_convolution.py:547-559) is an
    r2c transform of dL/dy with the interior one-sided bins doubled (they stand for two bins of the full
    spectrum); bin 0 and, for even n_out, the Nyquist bin n_out/2 are not doubled.  Complex data: 1.
    """
    d = torch.ones(list(kept), dtype=torch.float64)
    if complex_data:
        return d
    n = n_out[-1]
    k = torch.arange(kept[-1])
    last = torch.where((k == 0) | ((n % 2 == 0) & (k == n // 2)), 1.0, 2.0).to(torch.float64)
    return d * last


def weight_grad_direct(xs: torch.Tensor, gs: torch.Tensor, kept, n_out, complex_data: bool,
                       separable: bool = False) -> torch.Tensor:
    """dL/dW of the sliced dense weight from the kept spectra of x (forward geometry) and of dL/dy
    (adjoint geometry: grids, bin maps and scales swapped), as torch autograd of the contraction einsum
    (spectral_convolution.py:21-52) gives it: d_t * sum_b conj(xs[b, i, t]) * gs[b, o, t]."""
    d = mode_factors(kept, n_out, complex_data)
    if separable:
        return torch.einsum("bi...,bi...->i...", xs.conj(), gs) * d
    return torch.einsum("bi...,bo...->io...", xs.conj(), gs) * d
