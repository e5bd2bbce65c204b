"""Shared helpers: build package modules from golden / oracle parameter payloads."""

from __future__ import annotations

import torch

import neuraloperator_b200 as nb


def build_spectral_conv(case, device="cuda", **extra):
    """A neuraloperator_b200.SpectralConv carrying the golden case's weights."""
    kw = dict(case["kwargs"])
    conv = nb.SpectralConv(case["in_channels"], case["out_channels"], tuple(case["n_modes"]), **kw, **extra)
    load_weight(conv, case["weight_kind"], case["weight"])
    if case["bias"] is not None:
        with torch.no_grad():
            conv.bias.copy_(case["bias"])
    if case.get("active_modes"):
        conv.n_modes = tuple(case["active_modes"])
    return conv.to(device)


def load_weight(conv, kind, payload):
    w = conv.weight
    with torch.no_grad():
        if kind == "dense":
            w.tensor.copy_(payload)
        elif kind == "tucker":
            w.core.copy_(payload["core"])
            for f, v in zip(w.factors, payload["factors"]):
                f.copy_(v)
        elif kind == "cp":
            w.weights.copy_(payload["weights"])
            for f, v in zip(w.factors, payload["factors"]):
                f.copy_(v)
        else:
            for f, v in zip(w.factors, payload["factors"]):
                f.copy_(v)


def load_block(fb, i, blk, kind):
    load_weight(fb.convs[i], kind, blk["weight"])
    with torch.no_grad():
        fb.convs[i].bias.copy_(blk["bias"])
        if fb.fno_skips is not None and blk.get("fno_skip") is not None:
            sk = fb.fno_skips[i]
            (sk.conv.weight if hasattr(sk, "conv") else sk.weight).copy_(blk["fno_skip"])
        if fb.use_channel_mlp:
            for fc, (W, b) in zip(fb.channel_mlp[i].fcs, blk["mlp"]):
                fc.weight.copy_(W)
                fc.bias.copy_(b)
            if fb.channel_mlp_skips is not None and blk.get("mlp_skip") is not None:
                sk = fb.channel_mlp_skips[i]
                (sk.conv.weight if hasattr(sk, "conv") else sk.weight).copy_(blk["mlp_skip"])


def build_fno(case, device="cuda", **extra):
    kw = dict(case["kwargs"])
    cls = nb.TFNO if case["model"] == "TFNO" else nb.FNO
    model = cls(**kw, **extra)
    P = case["params"]
    with torch.no_grad():
        for fc, (W, b) in zip(model.lifting.fcs, P["lifting"]):
            fc.weight.copy_(W)
            fc.bias.copy_(b)
        for fc, (W, b) in zip(model.projection.fcs, P["projection"]):
            fc.weight.copy_(W)
            fc.bias.copy_(b)
    for i, blk in enumerate(P["blocks"]):
        load_block(model.fno_blocks, i, blk, case["weight_kind"])
    return model.to(device)


def case_scaling(case):
    r = case["kwargs"].get("resolution_scaling_factor")
    if r is None:
        return None
    order = case["order"]
    return [r] * order if isinstance(r, (int, float)) else list(r)


def oracle_weight(conv):
    """(payload, kind) of a SpectralConv's weight in the oracle's format (CPU tensors)."""
    w = conv.weight
    if hasattr(w, "core"):
        return {"core": w.core.detach().cpu(), "factors": [f.detach().cpu() for f in w.factors]}, "tucker"
    if hasattr(w, "weights"):
        return {"weights": w.weights.detach().cpu(), "factors": [f.detach().cpu() for f in w.factors]}, "cp"
    return w.tensor.detach().cpu(), "dense"


def oracle_model(model):
    """(params, cfg) of an FNO / TFNO in the oracle's format: oracle.fno_forward(x, params, cfg)."""
    lin = lambda fcs: [(fc.weight.detach().cpu(), fc.bias.detach().cpu()) for fc in fcs]  # noqa: E731
    fb = model.fno_blocks
    blocks, kind = [], "dense"
    for i in range(fb.n_layers):
        wp, kind = oracle_weight(fb.convs[i])
        blocks.append({"weight": wp, "bias": fb.convs[i].bias.detach().cpu(),
                       "fno_skip": fb.fno_skips[i].conv.weight.detach().cpu(), "mlp": lin(fb.channel_mlp[i].fcs),
                       "mlp_skip": fb.channel_mlp_skips[i].weight.detach().cpu()})
    params = {"lifting": lin(model.lifting.fcs), "projection": lin(model.projection.fcs), "blocks": blocks}
    return params, {"n_modes": tuple(model.n_modes), "weight_kind": kind}
