"""B200-native FNO spectral block: a drop-in for neuralop's SpectralConv inside FNOBlocks.

Public API mirrors the reference (neuralop.layers.spectral_convolution.SpectralConv,
neuralop.layers.fno_block.FNOBlocks, neuralop.models.FNO / TFNO).  The compute path is
libnop_b200.so (hand-written sm_100a CUDA, C ABI in include/nop_spectral.h).
"""

from .factorized import CPTensor, DenseTensor, FactorizedTensor, TTTensor, TuckerTensor  # noqa: F401
from .fno import FNO, TFNO  # noqa: F401
from .fno_block import FNOBlocks  # noqa: F401
from .fno_staged import FNOStaged  # noqa: F401
from .layers import ChannelMLP, GridEmbeddingND, SoftGating, skip_connection  # noqa: F401
from .spectral_convolution import BaseSpectralConv, SpectralConv  # noqa: F401
from .utils import count_model_params  # noqa: F401
