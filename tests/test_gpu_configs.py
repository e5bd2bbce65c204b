"""Parity at the benchmark configurations' own sizes: the CUDA path against the oracle.

The golden vectors (test_gpu_parity.py) pin the CUDA path to the reference's own outputs on small
shapes; here every benchmark configuration (C1-C5) runs at its full batch, channel count and grid, so
the kernel instantiations the benchmark times (the C2 contraction at 64 x 64 channels, the Tucker
chain at C4's ranks on 512^2, the 3D plane kernels at 256^3, the per-pixel chain kernel at hidden
widths 32 and 64) are the ones checked.  Batch rows are independent, so the oracle -- the reference's
forward restated on the CPU (oracle/spectral_oracle.py) -- runs on the first few samples and the
CUDA output's rows for them are compared.  Tolerances (the benchmark's stated bars): relative L2 <= 1e-5 with
the fp32 contraction, <= 2e-2 with the bf16 contraction.
"""

import pytest
import torch

import neuraloperator_b200 as nb
import oracle
from conftest import rel_l2
from helpers import oracle_model, oracle_weight
from neuraloperator_b200 import _lib

pytestmark = pytest.mark.gpu

TOL = {"fp32": 1e-5, "bf16": 2e-2}


@pytest.fixture(autouse=True, scope="module")
def _fp32_torch():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    torch.set_num_threads(max(1, torch.get_num_threads()))
    yield


def _layer(ci, co, modes, fact, seed, precision):
    g = torch.Generator().manual_seed(seed)
    kw = dict(factorization=fact, implementation="factorized", rank=0.1) if fact else {}
    conv = nb.SpectralConv(ci, co, modes, contraction_precision=precision, **kw)
    std = (2.0 / (ci + co)) ** 0.5
    with torch.no_grad():
        for p in conv.weight.parameters():
            p.copy_(torch.complex(torch.randn(p.shape, generator=g), torch.randn(p.shape, generator=g)) *
                    (std if not fact else 0.5))
        conv.bias.copy_(torch.randn(conv.bias.shape, generator=g) * std)
    return conv, g


# name, batch, channels, grid, n_modes, factorization, precision, samples checked against the oracle
LAYERS = [
    ("c1_darcy_layer", 16, 32, (128, 128), (16, 16), None, "fp32", 4),
    ("c2_micro", 64, 64, (256, 256), (64, 64), None, "fp32", 2),
    ("c2_micro_bf16", 64, 64, (256, 256), (64, 64), None, "bf16", 2),
    ("c3_burgers_layer", 256, 64, (8192,), (16,), None, "fp32", 8),
    ("c4_tfno_layer", 32, 64, (512, 512), (64, 64), "tucker", "fp32", 1),
    ("c4_tfno_layer_bf16", 32, 64, (512, 512), (64, 64), "tucker", "bf16", 1),
    ("c5_fno3d_layer", 8, 32, (256, 256, 256), (32, 32, 32), None, "fp32", 1),
]


@pytest.mark.parametrize("case", LAYERS, ids=[c[0] for c in LAYERS])
def test_spectral_layer_at_config_size(case):
    name, batch, ch, grid, modes, fact, precision, k = case
    conv, _ = _layer(ch, ch, modes, fact, 11, precision)
    gen = torch.Generator(device="cuda").manual_seed(12)
    x = torch.randn((batch, ch, *grid), generator=gen, device="cuda")  # 17 GB at C5: drawn on the device
    with torch.no_grad():
        y = conv.cuda()(x)
        torch.cuda.synchronize()
        y_k, x_k = y[:k].cpu(), x[:k].cpu()
        del y, x
        w, kind = oracle_weight(conv)
        ref = oracle.spectral_conv(x_k, w, conv.bias.detach().cpu(), modes, weight_kind=kind)
    assert rel_l2(y_k, ref) <= TOL[precision], name
    assert _lib.device_status() == 0


# name, class, n_modes, hidden, in, out, grid, batch, kwargs, samples checked
MODELS = [
    ("c1_fno2d_darcy", "FNO", (16, 16), 32, 1, 1, (128, 128), 16, {}, 2),
    ("c3_fno1d_burgers", "FNO", (16,), 64, 1, 1, (8192,), 256, {}, 4),
    ("c4_tfno2d_ns", "TFNO", (64, 64), 64, 1, 1, (512, 512), 32,
     dict(factorization="tucker", implementation="factorized", rank=0.1), 1),
    ("c4_tfno2d_ns_bf16", "TFNO", (64, 64), 64, 1, 1, (512, 512), 32,
     dict(factorization="tucker", implementation="factorized", rank=0.1, contraction_precision="bf16"), 1),
    ("c5_fno3d", "FNO", (32, 32, 32), 32, 3, 3, (256, 256, 256), 8, {}, 1),
]


@pytest.mark.parametrize("case", MODELS, ids=[c[0] for c in MODELS])
def test_fno_forward_at_config_size(case):
    """The FNO / TFNO forward through the fused path (chain kernels for lifting, blocks and projection,
    the spectral kernels in between) on the configuration's full batch and grid, against the oracle's
    FNO forward (fno.py:342-408) on the first samples."""
    name, cls, modes, hidden, cin, cout, grid, batch, kw, k = case
    torch.manual_seed(5)
    model = getattr(nb, cls)(n_modes=modes, in_channels=cin, out_channels=cout, hidden_channels=hidden,
                             n_layers=4, **kw)
    gen = torch.Generator(device="cuda").manual_seed(6)
    x = torch.randn((batch, cin, *grid), generator=gen, device="cuda")
    precision = kw.get("contraction_precision", "fp32")
    model = model.cuda().eval()
    with torch.no_grad():
        assert model.fused_plan(x) is not None, "the configuration must take the fused path"
        y = model(x)
        torch.cuda.synchronize()
        y_k, x_k = y[:k].cpu(), x[:k].cpu()
        del y, x
        params, cfg = oracle_model(model)
        ref = oracle.fno_forward(x_k, params, cfg)
    assert rel_l2(y_k, ref) <= TOL[precision], name
    assert _lib.device_status() == 0
