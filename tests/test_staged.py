"""FNOStaged (per-layer Fourier modes, neuralop/models/fno_staged.py): the oracle reproduces the
reference's outputs, and reference checkpoints load into neuraloperator_b200.FNOStaged."""

import os

import pytest
import torch

import neuraloperator_b200 as nb
import oracle
from conftest import GOLDEN, rel_l2

CASES = torch.load(os.path.join(GOLDEN, "staged_cases.pt"), weights_only=False)
TOL = 2e-6


def oracle_params(sd, n_layers):
    """The oracle's parameter payload from a reference FNOStaged state_dict."""
    def fcs(prefix):
        out, j = [], 0
        while f"{prefix}.fcs.{j}.weight" in sd:
            out.append((sd[f"{prefix}.fcs.{j}.weight"], sd[f"{prefix}.fcs.{j}.bias"]))
            j += 1
        return out
    blocks, kind = [], "dense"
    for i in range(n_layers):
        p = f"convs.{i}.weight."
        if p + "tensor" in sd:
            w = sd[p + "tensor"]
        else:
            kind = "tucker"
            nf = sum(1 for k in sd if k.startswith(p + "factors."))
            w = {"core": sd[p + "core"], "factors": [sd[f"{p}factors.{j}"] for j in range(nf)]}
        blocks.append({"weight": w, "bias": sd[f"convs.{i}.bias"], "fno_skip": sd[f"fno_skips.{i}.conv.weight"],
                       "mlp": fcs(f"channel_mlp.{i}"), "mlp_skip": sd[f"channel_mlp_skips.{i}.weight"]})
    return {"lifting": fcs("lifting"), "projection": fcs("projection"), "blocks": blocks}, kind


def oracle_cfg(case, kind):
    kw = case["kwargs"]
    # the reference passes the per-layer modes themselves as max_n_modes when none are given
    # (fno_staged.py:79-80, :168), so the last weight axis keeps n_modes entries, not n_modes // 2 + 1
    return dict(n_modes=kw["n_modes_per_layer"][0], n_modes_per_layer=kw["n_modes_per_layer"],
                max_n_modes_per_layer=kw.get("max_n_modes_per_layer") or kw["n_modes_per_layer"],
                weight_kind=kind)


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_oracle_matches_reference_fnostaged(case):
    params, kind = oracle_params(case["state_dict"], len(case["kwargs"]["n_modes_per_layer"]))
    y = oracle.fno_forward(case["x"], params, oracle_cfg(case, kind))
    assert rel_l2(y, case["y"]) <= TOL


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_reference_checkpoint_loads(case):
    model = nb.FNOStaged(**case["kwargs"])
    res = model.load_state_dict(dict(case["state_dict"], _metadata={"args": ()}))
    assert not res.missing_keys and not res.unexpected_keys
    assert model.n_modes_per_layer == [list(m) for m in case["kwargs"]["n_modes_per_layer"]]
    for conv, m in zip(model.fno_blocks.convs, case["kwargs"]["n_modes_per_layer"]):
        assert list(conv.n_modes)[:-1] == list(m)[:-1] and conv.n_modes[-1] == m[-1] // 2 + 1
    w0 = model.fno_blocks.convs[0].weight
    assert torch.equal(next(iter(w0.parameters())), next(v for k, v in case["state_dict"].items()
                                                          if k.startswith("convs.0.weight.")))


def test_fnostaged_argument_errors():
    with pytest.raises(ValueError):
        nb.FNOStaged([(8, 8), (4, 4)], 1, 1, 8, n_layers=3)
    with pytest.raises(ValueError):
        nb.FNOStaged([(8, 8), (4, 4)], 1, 1, 8, max_n_modes_per_layer=[(8, 8)])
    with pytest.raises(NotImplementedError):
        nb.FNOStaged([(8, 8)], 1, 1, 8, no_br=True)
    m = nb.FNOStaged([(8, 8), (6, 6)], 1, 1, 4)
    m.n_modes = [(6, 6), (4, 4)]
    assert m.n_modes == [[6, 4], [4, 3]]
