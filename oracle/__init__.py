"""CPU oracle for the FNO spectral block (TEST INFRASTRUCTURE ONLY).

This package restates, in plain PyTorch on the CPU, the reference forward path of
``neuralop.layers.spectral_convolution.SpectralConv`` inside ``FNOBlocks`` / ``FNO``
(AnirudhG07/neuraloperator, v2.0.0).  It is the checker the CUDA path is compared
against; it is never the thing measured or shipped.  Only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may import it.

Parity pinning: the restatement is checked against golden vectors produced by the
reference's own ``spectral_convolution.py`` / ``fno_block.py`` / ``fno.py`` run
in the build container under small stand-ins for the absent third-party modules
(tensorly 0.9.0, tensorly-torch 0.5.0, opt-einsum 3.4.0); see
``tests/golden/make_golden.py`` and ``tests/test_oracle_golden.py``.
"""

from .spectral_oracle import (  # noqa: F401
    effective_modes,
    spectral_conv,
    contract_dense,
    contract_tucker,
    contract_cp,
    contract_tt,
    tucker_to_dense,
    cp_to_dense,
    tt_to_dense,
    channel_mlp,
    fno_block,
    fno_forward,
    grid_embedding,
    resample,
)
