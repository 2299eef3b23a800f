"""B200-native (sm_100a) NVFP4 / FP8 transformer-FFN path of FlashVSR v1.1.

Drop-in for the reference's ``ffn_quantization`` module: ``install_ffn``,
``QuantLinear``, ``global_scale``; the fused ``NVFP4FFN``; and the raw
operators in :mod:`.ops`.  The compute runs in ``libfvq.so`` (C ABI in
``include/fvq.h``), hand-written CUDA for sm_100a; there is no CPU fallback.
"""
from ._lib import FvqError, LIB_PATH, load as load_library
from .ffn_quantization import (FP8FFN, NVFP4FFN, NVFP4FFNStack, GraphedFFNStack, QuantLinear, global_scale,
                               install_ffn, row_quant)
from . import ops

__all__ = ["install_ffn", "QuantLinear", "NVFP4FFN", "NVFP4FFNStack", "GraphedFFNStack", "FP8FFN", "global_scale", "row_quant", "ops",
           "FvqError",
           "LIB_PATH", "load_library"]
