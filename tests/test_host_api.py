"""CPU checks of the host-side mirror of the reference API (no kernel launches)."""

import os

import pytest
import torch

import neuraloperator_b200 as nb
from conftest import GOLDEN
from helpers import build_fno, build_spectral_conv

FNO_CASES = torch.load(os.path.join(GOLDEN, "fno_cases.pt"), weights_only=False)
SPECTRAL = torch.load(os.path.join(GOLDEN, "spectral_cases.pt"), weights_only=False)


def test_n_modes_setter_semantics():
    """neuralop/layers/tests/test_fno_block.py:25-34: last axis keeps m//2+1 modes."""
    max_n_modes = [8, 8, 8, 8]
    n_modes = [4, 4, 4, 4]
    for dim in [1, 2, 3, 4]:
        block = nb.FNOBlocks(3, 4, max_n_modes[:dim], max_n_modes=max_n_modes[:dim], n_layers=1,
                             channel_mlp_skip="linear")
        assert block.convs[0].n_modes[:-1] == max_n_modes[: dim - 1]
        assert block.convs[0].n_modes[-1] == max_n_modes[dim - 1] // 2 + 1
        block.n_modes = n_modes[:dim]
        assert block.convs[0].n_modes[:-1] == n_modes[: dim - 1]
        assert block.convs[0].n_modes[-1] == n_modes[dim - 1] // 2 + 1


def test_weight_shapes_and_kinds():
    conv = nb.SpectralConv(3, 4, (10, 8))
    assert isinstance(conv.weight, nb.DenseTensor) and conv.weight.shape == (3, 4, 10, 5)
    assert torch.is_complex(conv.weight.to_tensor())
    t = nb.SpectralConv(64, 64, (64, 64), factorization="tucker", implementation="factorized", rank=0.1)
    assert t.weight.rank == [36, 36, 36, 19]
    sep = nb.SpectralConv(3, 3, (6, 6), separable=True)
    assert sep.weight.shape == (3, 6, 4)
    with pytest.raises(ValueError):
        nb.SpectralConv(3, 4, (6, 6), separable=True)


def test_forward_on_cpu_fails_loudly():
    conv = nb.SpectralConv(2, 2, (4, 4))
    with pytest.raises(RuntimeError, match="CUDA"):
        conv(torch.randn(1, 2, 8, 8))


def test_unsupported_precision_raises():
    conv = nb.SpectralConv(2, 2, (4, 4), fno_block_precision="half")
    with pytest.raises(NotImplementedError):
        conv(torch.randn(1, 2, 8, 8))


def test_state_dict_keys_match_reference_layout():
    m = nb.FNO(n_modes=(8, 8), in_channels=1, out_channels=1, hidden_channels=8, n_layers=2)
    keys = set(m.state_dict().keys())
    for k in ["fno_blocks.convs.0.weight.tensor", "fno_blocks.convs.1.bias", "fno_blocks.fno_skips.0.conv.weight",
              "fno_blocks.channel_mlp.1.fcs.1.bias", "fno_blocks.channel_mlp_skips.0.weight",
              "lifting.fcs.0.weight", "projection.fcs.1.bias"]:
        assert k in keys
    sd = dict(m.state_dict())
    sd["_metadata"] = {"n_modes": (8, 8)}
    m.load_state_dict(sd)  # reference checkpoints carry _metadata


@pytest.mark.parametrize("case", FNO_CASES[:-1], ids=[c["name"] for c in FNO_CASES[:-1]])
def test_golden_parameters_load(case):
    model = build_fno(case, device="cpu")
    assert model.fno_blocks.n_layers == len(case["params"]["blocks"])


@pytest.mark.parametrize("case", SPECTRAL, ids=[c["name"] for c in SPECTRAL])
def test_golden_spectral_weights_load(case):
    conv = build_spectral_conv(case, device="cpu")
    geo = conv.geometry(list(case["x"].shape[2:]), case["forward_kwargs"].get("output_shape"))
    kind, ws, ranks = conv.kernel_operands(geo)
    assert kind in ("dense", "tucker", "cp")
    assert tuple(geo.n_out) == tuple(case["y"].shape[2:])
