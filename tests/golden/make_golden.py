"""Generate golden input/output vectors from the reference's own forward code.

Run in the build container (it needs the reference checkout; see ``ref_loader``):

    NOP_REFERENCE_ROOT=<reference checkout> python tests/golden/make_golden.py

Writes ``spectral_cases.pt`` (SpectralConv cases: dense, Tucker, CP, TT, separable,
complex data, odd sizes, Nyquist kept, incremental modes, output_shape, fft_norm),
``fno_cases.pt`` (FNOBlocks / FNO / TFNO end to end), ``config_layers.pt`` (single
SpectralConv layers with the modes and grids of the five benchmark configurations, at
reduced batch/channel counts) and ``grad_cases.pt`` (gradients: torch autograd through the
reference's forward for a seeded dL/dy, for SpectralConv layers and for small FNO / TFNO models)
and ``staged_cases.pt`` (FNOStaged with per-layer modes: the reference's state_dict, input and output).  Every tensor is generated from fixed seeds; the
reference modules compute the outputs.  The files are committed so the tests need no
reference checkout.
"""

from __future__ import annotations

import math
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import ref_loader  # noqa: E402

torch.set_default_dtype(torch.float32)


def _cn(gen, shape, std):
    """Complex normal with ``std`` per real and imaginary part."""
    re = torch.randn(shape, generator=gen) * std
    im = torch.randn(shape, generator=gen) * std
    return torch.complex(re, im)


def _weight_payload(w):
    """Plain-tensor copy of a stub weight container (the oracle's weight format)."""
    name = w.name.lower()
    if name.endswith("dense"):
        return "dense", w.tensor.detach().clone()
    if name.endswith("tucker"):
        return "tucker", {"core": w.core.detach().clone(), "factors": [f.detach().clone() for f in w.factors]}
    if name.endswith("cp"):
        return "cp", {"weights": w.weights.detach().clone(), "factors": [f.detach().clone() for f in w.factors]}
    return "tt", {"factors": [f.detach().clone() for f in w.factors]}


def _randomise_weight(w, gen, std):
    with torch.no_grad():
        for p in w.parameters():
            p.copy_(_cn(gen, p.shape, std))


def spectral_cases(mods):
    SC = mods["spectral_convolution"].SpectralConv
    cases = []

    def add(name, ci, co, n_modes, size, batch=2, seed=0, set_modes=None, fwd_kwargs=None, wstd=None, **kw):
        gen = torch.Generator().manual_seed(seed)
        conv = SC(ci, co, n_modes, **kw)
        order = len(size)
        std = wstd if wstd is not None else (2.0 / (ci + co)) ** 0.5
        if kw.get("factorization") not in (None, "Dense", "dense"):
            # factors scaled so the reconstructed weight has roughly ``std``
            nf = sum(1 for _ in conv.weight.parameters())
            _randomise_weight(conv.weight, gen, std ** (1.0 / max(nf - 1, 1)))
        else:
            _randomise_weight(conv.weight, gen, std)
        if conv.bias is not None:
            with torch.no_grad():
                conv.bias.copy_(torch.randn(conv.bias.shape, generator=gen) * std)
        if set_modes is not None:
            conv.n_modes = set_modes
        cplx = kw.get("complex_data", False)
        if cplx:
            x = _cn(gen, (batch, ci, *size), 1.0)
        else:
            x = torch.randn((batch, ci, *size), generator=gen)
        with torch.no_grad():
            y = conv(x, **(fwd_kwargs or {}))
        kind, payload = _weight_payload(conv.weight)
        cases.append(dict(
            name=name, in_channels=ci, out_channels=co, n_modes=list(n_modes),
            active_modes=list(set_modes) if set_modes is not None else None,
            kwargs={k: v for k, v in kw.items()}, forward_kwargs=fwd_kwargs or {},
            weight_kind=kind, weight=payload,
            bias=None if conv.bias is None else conv.bias.detach().clone(),
            x=x, y=y.detach().clone(), order=order))

    # dense, real data, 1D..4D, even / odd sizes, non-uniform modes
    add("d1_even", 3, 4, (8,), (16,))
    add("d1_odd", 3, 4, (5,), (9,))
    add("d1_allbins", 2, 3, (16,), (16,))                      # keeps the Nyquist bin
    add("d2_ref_modes", 3, 4, (10, 8), (12, 12))
    add("d2_odd", 3, 4, (4, 5), (9, 9))
    add("d2_nonsquare", 3, 2, (6, 6), (16, 12))
    add("d2_nyquist", 2, 3, (8, 8), (8, 8))                    # all y modes, last axis incl. Nyquist
    add("d2_nohermitian", 3, 4, (4, 4), (8, 8), enforce_hermitian_symmetry=False)
    add("d2_nobias", 3, 4, (6, 6), (12, 12), bias=False)
    add("d3_even", 3, 4, (4, 4, 4), (8, 8, 8))
    add("d3_odd", 3, 4, (4, 5, 7), (9, 9, 9))
    add("d4", 2, 3, (4, 4, 4, 4), (6, 6, 6, 6))
    # incremental modes: max_n_modes above the active n_modes (weight slicing)
    add("d2_incremental", 3, 4, (8, 8), (12, 12), max_n_modes=(8, 8), set_modes=(4, 6))
    add("d1_incremental", 3, 3, (12,), (16,), set_modes=(6,))
    # output resolution changes
    add("d2_out_up", 3, 4, (6, 6), (10, 10), resolution_scaling_factor=2)
    add("d2_out_down", 3, 4, (6, 6), (12, 12), resolution_scaling_factor=0.5)
    add("d1_out_shape", 3, 4, (6,), (12,), fwd_kwargs={"output_shape": (17,)})
    add("d3_out_up", 2, 3, (4, 4, 4), (6, 6, 6), resolution_scaling_factor=2)
    add("d2_out_odd", 2, 3, (4, 4), (8, 8), fwd_kwargs={"output_shape": (11, 9)})
    # fft normalisations
    add("d2_norm_backward", 3, 4, (6, 6), (12, 12), fft_norm="backward")
    add("d2_norm_ortho", 3, 4, (6, 6), (12, 12), fft_norm="ortho")
    # complex-valued data
    add("c1", 3, 4, (6,), (12,), complex_data=True)
    add("c2", 3, 4, (6, 4), (12, 10), complex_data=True)
    add("c2_allmodes", 2, 2, (8, 8), (8, 8), complex_data=True)
    # separable
    add("d2_separable", 3, 3, (6, 6), (12, 12), separable=True)
    add("d1_separable_tucker", 3, 3, (6,), (12,), separable=True, factorization="tucker",
        implementation="factorized", rank=0.5)
    # factorized weights
    add("tucker_d1", 3, 4, (8,), (16,), factorization="tucker", implementation="factorized", rank=0.5)
    add("tucker_d2", 3, 4, (10, 8), (12, 12), factorization="tucker", implementation="factorized", rank=0.4)
    add("tucker_d2_recon", 3, 4, (10, 8), (12, 12), factorization="tucker", implementation="reconstructed",
        rank=0.4)
    add("tucker_d3", 3, 4, (4, 4, 4), (8, 8, 8), factorization="tucker", implementation="factorized", rank=0.5)
    add("tucker_d2_incremental", 3, 4, (8, 8), (12, 12), factorization="tucker", implementation="factorized",
        rank=0.5, set_modes=(4, 6))
    add("cp_d2", 3, 4, (6, 6), (12, 12), factorization="cp", implementation="factorized", rank=0.5)
    add("tt_d2", 3, 4, (6, 6), (12, 12), factorization="tt", implementation="factorized", rank=0.5)
    return cases


def _block_payload(fb, i):
    kind, w = _weight_payload(fb.convs[i].weight)
    blk = {"weight": w, "bias": fb.convs[i].bias.detach().clone()}
    if fb.fno_skips is not None:
        sk = fb.fno_skips[i]
        blk["fno_skip"] = sk.conv.weight.detach().clone() if hasattr(sk, "conv") else (
            sk.weight.detach().clone() if hasattr(sk, "weight") else None)
    if fb.use_channel_mlp:
        blk["mlp"] = [(fc.weight.detach().clone(), fc.bias.detach().clone()) for fc in fb.channel_mlp[i].fcs]
        if fb.channel_mlp_skips is not None:
            sk = fb.channel_mlp_skips[i]
            blk["mlp_skip"] = sk.weight.detach().clone() if hasattr(sk, "weight") else (
                sk.conv.weight.detach().clone() if hasattr(sk, "conv") else None)
    return kind, blk


def _randomise_module(mod, gen):
    with torch.no_grad():
        for name, p in mod.named_parameters():
            if p.is_complex():
                p.copy_(_cn(gen, p.shape, 0.3))
            else:
                p.copy_(torch.randn(p.shape, generator=gen) * (0.5 if p.ndim > 1 else 0.1))


def fno_cases(mods):
    FNO = mods["fno"].FNO
    TFNO = mods["fno"].TFNO
    FNOBlocks = mods["fno_block"].FNOBlocks
    out = []

    def add_model(name, cls, size, batch, seed, **kw):
        gen = torch.Generator().manual_seed(seed)
        torch.manual_seed(seed)
        model = cls(**kw)
        _randomise_module(model, gen)
        x = torch.randn((batch, kw["in_channels"], *size), generator=gen)
        with torch.no_grad():
            y = model(x)
        fb = model.fno_blocks
        blocks, kind = [], None
        for i in range(fb.n_layers):
            kind, blk = _block_payload(fb, i)
            blocks.append(blk)
        params = {
            "lifting": [(fc.weight.detach().clone(), fc.bias.detach().clone()) for fc in model.lifting.fcs],
            "projection": [(fc.weight.detach().clone(), fc.bias.detach().clone()) for fc in model.projection.fcs],
            "blocks": blocks,
        }
        out.append(dict(name=name, model=cls.__name__, kwargs=kw, weight_kind=kind, params=params, x=x,
                        y=y.detach().clone()))

    add_model("fno1d_burgers_small", FNO, (64,), 2, 1, n_modes=(16,), in_channels=1, out_channels=1,
              hidden_channels=8, n_layers=4)
    add_model("fno2d_darcy_small", FNO, (32, 32), 2, 2, n_modes=(16, 16), in_channels=1, out_channels=1,
              hidden_channels=8, n_layers=4)
    add_model("tfno2d_ns_small", TFNO, (32, 32), 2, 3, n_modes=(12, 12), in_channels=1, out_channels=1,
              hidden_channels=8, n_layers=4)
    add_model("fno3d_small", FNO, (12, 12, 12), 1, 4, n_modes=(6, 6, 6), in_channels=3, out_channels=3,
              hidden_channels=6, n_layers=2)
    add_model("fno2d_preact_linear", FNO, (16, 16), 2, 5, n_modes=(8, 8), in_channels=2, out_channels=1,
              hidden_channels=6, n_layers=3, preactivation=True, channel_mlp_skip="linear")
    add_model("fno2d_identity_skip", FNO, (16, 16), 2, 6, n_modes=(8, 8), in_channels=1, out_channels=2,
              hidden_channels=6, n_layers=2, fno_skip="identity", use_channel_mlp=False)

    # a bare FNOBlocks stack (2 layers)
    gen = torch.Generator().manual_seed(7)
    fb = FNOBlocks(4, 4, (8, 6), n_layers=2)
    _randomise_module(fb, gen)
    x = torch.randn((2, 4, 12, 10), generator=gen)
    with torch.no_grad():
        y1 = fb(x, 0)
        y2 = fb(y1, 1)
    blocks = [_block_payload(fb, i)[1] for i in range(2)]
    out.append(dict(name="fnoblocks_2layer", model="FNOBlocks", kwargs=dict(in_channels=4, out_channels=4,
                    n_modes=(8, 6), n_layers=2), weight_kind="dense", params={"blocks": blocks}, x=x,
                    y=torch.stack([y1, y2])))
    return out


def config_layers(mods):
    """One SpectralConv per benchmark configuration: its grid and modes, small batch/channels."""
    SC = mods["spectral_convolution"].SpectralConv
    cases = []

    def add(name, ci, co, n_modes, size, batch, seed, **kw):
        gen = torch.Generator().manual_seed(seed)
        conv = SC(ci, co, n_modes, **kw)
        std = (2.0 / (ci + co)) ** 0.5
        if kw.get("factorization"):
            nf = sum(1 for _ in conv.weight.parameters())
            _randomise_weight(conv.weight, gen, std ** (1.0 / max(nf - 1, 1)))
        else:
            _randomise_weight(conv.weight, gen, std)
        with torch.no_grad():
            conv.bias.copy_(torch.randn(conv.bias.shape, generator=gen) * std)
        x = torch.randn((batch, ci, *size), generator=gen)
        with torch.no_grad():
            y = conv(x)
        kind, payload = _weight_payload(conv.weight)
        cases.append(dict(name=name, in_channels=ci, out_channels=co, n_modes=list(n_modes), active_modes=None,
                          kwargs=kw, forward_kwargs={}, weight_kind=kind, weight=payload,
                          bias=conv.bias.detach().clone(), x=x, y=y.detach().clone(), order=len(size)))

    add("cfg1_darcy_128", 4, 4, (16, 16), (128, 128), 1, 11)
    add("cfg2_micro_256", 2, 2, (64, 64), (256, 256), 1, 12)
    add("cfg3_burgers_8192", 2, 2, (16,), (8192,), 2, 13)
    add("cfg4_tfno_256", 2, 2, (64, 64), (256, 256), 1, 14, factorization="tucker", implementation="factorized",
        rank=0.1)
    add("cfg5_fno3d_48", 2, 2, (32, 32, 32), (48, 48, 48), 1, 15)
    return cases


def _grad_payload(w):
    """Gradients of a stub weight container, in the structure of ``_weight_payload``."""
    g = lambda p: None if p.grad is None else p.grad.detach().clone()
    name = w.name.lower()
    if name.endswith("dense"):
        return g(w.tensor)
    if name.endswith("tucker"):
        return {"core": g(w.core), "factors": [g(f) for f in w.factors]}
    if name.endswith("cp"):
        return {"weights": g(w.weights), "factors": [g(f) for f in w.factors]}
    return {"factors": [g(f) for f in w.factors]}


def grad_cases(mods):
    """Backward goldens: for y = module(x) and a seeded G = dL/dy (L = sum(y * G), real part for complex
    data), the reference's autograd gives dL/dx and dL/d every parameter."""
    SC = mods["spectral_convolution"].SpectralConv
    layers = []

    def add(name, ci, co, n_modes, size, batch=2, seed=100, set_modes=None, **kw):
        gen = torch.Generator().manual_seed(seed)
        conv = SC(ci, co, n_modes, **kw)
        std = (2.0 / (ci + co)) ** 0.5
        if kw.get("factorization") not in (None, "Dense", "dense"):
            nf = sum(1 for _ in conv.weight.parameters())
            _randomise_weight(conv.weight, gen, std ** (1.0 / max(nf - 1, 1)))
        else:
            _randomise_weight(conv.weight, gen, std)
        if conv.bias is not None:
            with torch.no_grad():
                conv.bias.copy_(torch.randn(conv.bias.shape, generator=gen) * std)
        if set_modes is not None:
            conv.n_modes = set_modes
        cplx = kw.get("complex_data", False)
        x = _cn(gen, (batch, ci, *size), 1.0) if cplx else torch.randn((batch, ci, *size), generator=gen)
        x.requires_grad_(True)
        y = conv(x)
        G = _cn(gen, y.shape, 1.0) if cplx else torch.randn(y.shape, generator=gen)
        y.backward(G)
        kind, payload = _weight_payload(conv.weight)
        layers.append(dict(
            name=name, in_channels=ci, out_channels=co, n_modes=list(n_modes),
            active_modes=list(set_modes) if set_modes is not None else None, kwargs=dict(kw), forward_kwargs={},
            weight_kind=kind, weight=payload, bias=None if conv.bias is None else conv.bias.detach().clone(),
            x=x.detach().clone(), order=len(size), grad_y=G,
            grad_x=x.grad.detach().clone(), grad_weight=_grad_payload(conv.weight),
            grad_bias=None if conv.bias is None else conv.bias.grad.detach().clone()))

    # generic-engine shapes
    add("g_d1_even", 3, 4, (8,), (16,))
    add("g_d1_odd", 3, 4, (5,), (9,))
    add("g_d1_allbins", 2, 3, (16,), (16,))
    add("g_d2_ref_modes", 3, 4, (10, 8), (12, 12))
    add("g_d2_odd", 3, 4, (4, 5), (9, 9))
    add("g_d2_nyquist", 2, 3, (8, 8), (8, 8))
    add("g_d2_nohermitian", 3, 4, (4, 4), (8, 8), enforce_hermitian_symmetry=False)
    add("g_d2_nobias", 3, 4, (6, 6), (12, 12), bias=False)
    add("g_d3_odd", 3, 4, (4, 5, 7), (9, 9, 9))
    add("g_d4", 2, 3, (4, 4, 4, 4), (6, 6, 6, 6))
    add("g_d2_incremental", 3, 4, (8, 8), (12, 12), max_n_modes=(8, 8), set_modes=(4, 6))
    add("g_d2_norm_backward", 3, 4, (6, 6), (12, 12), fft_norm="backward")
    add("g_d2_norm_ortho", 3, 4, (6, 6), (12, 12), fft_norm="ortho")
    add("g_c1", 3, 4, (6,), (12,), complex_data=True)
    add("g_c2", 3, 4, (6, 4), (12, 10), complex_data=True)
    add("g_d2_separable", 3, 3, (6, 6), (12, 12), separable=True)
    add("g_tucker_d2", 3, 4, (10, 8), (12, 12), factorization="tucker", implementation="factorized", rank=0.4)
    add("g_tucker_d2_recon", 3, 4, (10, 8), (12, 12), factorization="tucker", implementation="reconstructed",
        rank=0.4)
    add("g_tucker_sep_d1", 3, 3, (6,), (12,), separable=True, factorization="tucker",
        implementation="factorized", rank=0.5)
    add("g_cp_d2", 3, 4, (6, 6), (12, 12), factorization="cp", implementation="factorized", rank=0.5)
    add("g_tt_d2", 3, 4, (6, 6), (12, 12), factorization="tt", implementation="factorized", rank=0.5)
    # fused-engine shapes (plane kernels for 128 / 256, long 1D lines, Tucker core on 256); 512 x 512
    # planes are checked on the GPU through the adjoint identity instead (fixture size)
    add("g_fast_128", 2, 3, (16, 16), (128, 128), batch=1)
    add("g_fast_256", 1, 2, (64, 64), (256, 256), batch=1)
    add("g_fast_256_tucker", 1, 1, (64, 64), (256, 256), batch=1, factorization="tucker",
        implementation="factorized", rank=0.1)
    add("g_fast_1d", 2, 2, (16,), (8192,), batch=2)

    FNO, TFNO = mods["fno"].FNO, mods["fno"].TFNO
    models = []

    def add_model(name, cls, size, batch, seed, **kw):
        gen = torch.Generator().manual_seed(seed)
        torch.manual_seed(seed)
        model = cls(**kw)
        _randomise_module(model, gen)
        x = torch.randn((batch, kw["in_channels"], *size), generator=gen)
        x.requires_grad_(True)
        y = model(x)
        G = torch.randn(y.shape, generator=gen)
        y.backward(G)
        fb = model.fno_blocks
        blocks, gblocks, kind = [], [], None
        for i in range(fb.n_layers):
            kind, blk = _block_payload(fb, i)
            blocks.append(blk)
            gb = {"weight": _grad_payload(fb.convs[i].weight), "bias": fb.convs[i].bias.grad.detach().clone()}
            sk = fb.fno_skips[i]
            gb["fno_skip"] = (sk.conv.weight if hasattr(sk, "conv") else sk.weight).grad.detach().clone()
            gb["mlp"] = [(fc.weight.grad.detach().clone(), fc.bias.grad.detach().clone())
                         for fc in fb.channel_mlp[i].fcs]
            gb["mlp_skip"] = fb.channel_mlp_skips[i].weight.grad.detach().clone()
            gblocks.append(gb)
        lin = lambda fcs: [(fc.weight.detach().clone(), fc.bias.detach().clone()) for fc in fcs]
        glin = lambda fcs: [(fc.weight.grad.detach().clone(), fc.bias.grad.detach().clone()) for fc in fcs]
        params = {"lifting": lin(model.lifting.fcs), "projection": lin(model.projection.fcs), "blocks": blocks}
        grads = {"lifting": glin(model.lifting.fcs), "projection": glin(model.projection.fcs), "blocks": gblocks}
        n_params = sum(1 for _ in model.parameters())
        n_with_grad = sum(1 for p in model.parameters() if p.grad is not None)
        models.append(dict(name=name, model=cls.__name__, kwargs=kw, weight_kind=kind, params=params,
                           x=x.detach().clone(), y=y.detach().clone(), grad_y=G, grad_x=x.grad.detach().clone(),
                           grads=grads, n_params=n_params, n_params_with_grad=n_with_grad))

    add_model("fno2d_darcy_small", FNO, (32, 32), 2, 21, n_modes=(16, 16), in_channels=1, out_channels=1,
              hidden_channels=8, n_layers=4)
    add_model("tfno2d_small", TFNO, (32, 32), 2, 22, n_modes=(12, 12), in_channels=1, out_channels=1,
              hidden_channels=8, n_layers=2)
    add_model("fno1d_small", FNO, (64,), 2, 23, n_modes=(16,), in_channels=1, out_channels=1,
              hidden_channels=8, n_layers=2)
    return {"layers": layers, "models": models}


def staged_cases(mods):
    """FNOStaged (neuralop/models/fno_staged.py): per-layer modes, the reference's state_dict and output."""
    import importlib
    FS = importlib.import_module("neuralop.models.fno_staged").FNOStaged
    out = []

    def add(name, size, batch, seed, **kw):
        gen = torch.Generator().manual_seed(seed)
        torch.manual_seed(seed)
        model = FS(**kw)
        _randomise_module(model, gen)
        x = torch.randn((batch, kw["in_channels"], *size), generator=gen)
        with torch.no_grad():
            y = model(x)
        sd = {k: v.detach().clone() for k, v in model.state_dict().items() if torch.is_tensor(v)}
        out.append(dict(name=name, kwargs=kw, state_dict=sd, x=x, y=y.detach().clone()))

    add("staged2d", (32, 32), 2, 31, n_modes_per_layer=[(12, 12), (8, 8), (6, 6)], in_channels=1,
        out_channels=1, hidden_channels=8)
    add("staged2d_max_modes", (24, 24), 2, 32, n_modes_per_layer=[(8, 8), (6, 6)],
        max_n_modes_per_layer=[(10, 10), (8, 8)], in_channels=2, out_channels=1, hidden_channels=6)
    add("staged1d_tucker", (64,), 2, 33, n_modes_per_layer=[(16,), (8,), (4,)], in_channels=1, out_channels=1,
        hidden_channels=8, factorization="tucker", rank=0.5)
    return out


def main():
    mods = ref_loader.install()
    torch.save(spectral_cases(mods), os.path.join(HERE, "spectral_cases.pt"))
    torch.save(fno_cases(mods), os.path.join(HERE, "fno_cases.pt"))
    torch.save(config_layers(mods), os.path.join(HERE, "config_layers.pt"))
    torch.save(grad_cases(mods), os.path.join(HERE, "grad_cases.pt"))
    torch.save(staged_cases(mods), os.path.join(HERE, "staged_cases.pt"))
    for f in ("spectral_cases.pt", "fno_cases.pt", "config_layers.pt", "grad_cases.pt", "staged_cases.pt"):
        print(f, os.path.getsize(os.path.join(HERE, f)) // 1024, "KiB")


if __name__ == "__main__":
    main()
