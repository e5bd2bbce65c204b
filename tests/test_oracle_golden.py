"""The CPU oracle reproduces the reference's own outputs (golden vectors) — pins the oracle."""

import pytest
import torch

import oracle
from conftest import rel_l2

TOL_ORACLE = 2e-6   # float32 rounding differences only (same torch.fft / einsum sequence)


def _scaling(kw, order):
    r = kw.get("resolution_scaling_factor")
    if r is None:
        return None
    return [r] * order if isinstance(r, (int, float)) else list(r)


def run_oracle_case(case):
    kw = case["kwargs"]
    order = case["order"]
    complex_data = kw.get("complex_data", False)
    # constructor: max_n_modes defaults to the effective modes of the constructor n_modes
    max_n_modes = kw.get("max_n_modes")
    if max_n_modes is None:
        max_n_modes = oracle.effective_modes(case["n_modes"], complex_data)
    n_modes = case["active_modes"] or case["n_modes"]
    return oracle.spectral_conv(
        case["x"], case["weight"], case["bias"], n_modes, max_n_modes,
        weight_kind=case["weight_kind"], complex_data=complex_data,
        separable=kw.get("separable", False),
        enforce_hermitian_symmetry=kw.get("enforce_hermitian_symmetry", True),
        fft_norm=kw.get("fft_norm", "forward"),
        output_shape=case["forward_kwargs"].get("output_shape"),
        resolution_scaling_factor=_scaling(kw, order))


def _ids(cases):
    return [c["name"] for c in cases]


SPECTRAL = torch.load(__import__("os").path.join(__import__("conftest").GOLDEN, "spectral_cases.pt"),
                      weights_only=False)
CONFIG = torch.load(__import__("os").path.join(__import__("conftest").GOLDEN, "config_layers.pt"),
                    weights_only=False)
FNO = torch.load(__import__("os").path.join(__import__("conftest").GOLDEN, "fno_cases.pt"), weights_only=False)


@pytest.mark.parametrize("case", SPECTRAL, ids=_ids(SPECTRAL))
def test_spectral_conv_matches_reference(case):
    y = run_oracle_case(case)
    assert y.shape == case["y"].shape and y.dtype == case["y"].dtype
    assert rel_l2(y, case["y"]) <= TOL_ORACLE


@pytest.mark.parametrize("case", CONFIG, ids=_ids(CONFIG))
def test_config_layers_match_reference(case):
    y = run_oracle_case(case)
    assert y.shape == case["y"].shape
    assert rel_l2(y, case["y"]) <= TOL_ORACLE


def fno_cfg(case):
    kw = case["kwargs"]
    return dict(n_modes=kw["n_modes"], weight_kind=case["weight_kind"],
                fno_skip=kw.get("fno_skip", "linear"), channel_mlp_skip=kw.get("channel_mlp_skip", "soft-gating"),
                use_channel_mlp=kw.get("use_channel_mlp", True), preactivation=kw.get("preactivation", False))


@pytest.mark.parametrize("case", [c for c in FNO if c["model"] != "FNOBlocks"],
                         ids=[c["name"] for c in FNO if c["model"] != "FNOBlocks"])
def test_fno_matches_reference(case):
    y = oracle.fno_forward(case["x"], case["params"], fno_cfg(case))
    assert y.shape == case["y"].shape
    assert rel_l2(y, case["y"]) <= TOL_ORACLE


def test_fnoblocks_matches_reference():
    case = [c for c in FNO if c["model"] == "FNOBlocks"][0]
    cfg = fno_cfg(case)
    h = case["x"]
    for i, blk in enumerate(case["params"]["blocks"]):
        h = oracle.fno_block(h, blk, i, 2, cfg)
        assert rel_l2(h, case["y"][i]) <= TOL_ORACLE


def test_factorized_equals_reconstructed():
    """Known-answer property of the reference suite (test_spectral_convolution.py:53-65)."""
    for case in SPECTRAL:
        if case["weight_kind"] == "dense" or case["kwargs"].get("separable"):
            continue
        w = case["weight"]
        if case["weight_kind"] == "tucker":
            dense = oracle.tucker_to_dense(w["core"], w["factors"])
        elif case["weight_kind"] == "cp":
            dense = oracle.cp_to_dense(w["weights"], w["factors"])
        else:
            dense = oracle.tt_to_dense(w["factors"])
        d = dict(case, weight=dense, weight_kind="dense")
        assert rel_l2(run_oracle_case(d), case["y"]) <= 1e-5, case["name"]
