"""Host logic: the kernels' direct-DFT formulation, driven by the package's geometry, equals
the reference's fftshift/slice/ifftshift/irfft sequence on every golden case (float64)."""

import os

import pytest
import torch

import oracle
from oracle import dft_formulation as dft
from conftest import GOLDEN, rel_l2
from neuraloperator_b200.geometry import active_modes, compute_geometry, output_sizes

SPECTRAL = torch.load(os.path.join(GOLDEN, "spectral_cases.pt"), weights_only=False)
CONFIG = torch.load(os.path.join(GOLDEN, "config_layers.pt"), weights_only=False)


def case_geometry(case):
    kw = case["kwargs"]
    cplx = kw.get("complex_data", False)
    modes = active_modes(case["active_modes"] or case["n_modes"], cplx)
    mx = kw.get("max_n_modes")
    max_modes = active_modes(case["n_modes"], cplx) if mx is None else list(mx)
    r = kw.get("resolution_scaling_factor")
    order = case["order"]
    scaling = None if r is None else ([r] * order if isinstance(r, (int, float)) else list(r))
    sizes = list(case["x"].shape[2:])
    out = output_sizes(sizes, scaling, case["forward_kwargs"].get("output_shape"))
    return compute_geometry(sizes, modes, max_modes, complex_data=cplx,
                            enforce_hermitian_symmetry=kw.get("enforce_hermitian_symmetry", True),
                            fft_norm=kw.get("fft_norm", "forward"), out_sizes=out)


def sliced_dense_weight(case, geo):
    sep = case["kwargs"].get("separable", False)
    lead = (slice(None),) * (1 if sep else 2)
    w = case["weight"]
    kind = case["weight_kind"]
    if kind == "dense":
        return w[lead + geo.weight_slices]
    if kind == "tucker":
        full = oracle.tucker_to_dense(w["core"], w["factors"])
    elif kind == "cp":
        full = oracle.cp_to_dense(w["weights"], w["factors"])
    else:
        full = oracle.tt_to_dense(w["factors"])
    return full[lead + geo.weight_slices]


@pytest.mark.parametrize("case", SPECTRAL + CONFIG, ids=[c["name"] for c in SPECTRAL + CONFIG])
def test_direct_formulation_matches_reference(case):
    geo = case_geometry(case)
    w = sliced_dense_weight(case, geo)
    y = dft.spectral_conv_direct(
        case["x"], w, case["bias"], n_in=geo.n_in, n_out=geo.n_out, kept=geo.kept, fwd_off=geo.fwd_off,
        inv_off=geo.inv_off, fwd_scale=geo.fwd_scale, inv_scale=geo.inv_scale,
        complex_data=geo.complex_data, zero_imag_bins=geo.zero_imag_bins,
        separable=case["kwargs"].get("separable", False))
    assert tuple(y.shape) == tuple(case["y"].shape)
    assert rel_l2(y, case["y"]) <= 2e-6


def test_geometry_configs():
    """Kept bins of the five benchmark configurations (index table of the spectral block)."""
    g = compute_geometry([256, 256], active_modes((64, 64), False), active_modes((64, 64), False))
    assert g.kept == [64, 33] and g.fwd_off == [32, 0] and g.zero_imag_bins == [0, 128]
    g = compute_geometry([8192], active_modes(16, False), active_modes(16, False))
    assert g.kept == [9] and g.fwd_off == [0]
    g = compute_geometry([256] * 3, active_modes((32,) * 3, False), active_modes((32,) * 3, False))
    assert g.kept == [32, 32, 17] and g.fwd_off == [16, 16, 0]
    g = compute_geometry([128, 128], active_modes((16, 16), False), active_modes((16, 16), False))
    assert g.kept == [16, 9]
