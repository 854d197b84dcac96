"""polarflash_b200: B200-native (sm_100a) compressed-linear hot path of POLAR-FLASH.

y = W x computed straight from packed low-bit weights (INT4/INT3/INT2, E8 root
residual VQ, recursive polar blocks) with the inverse block RWHT folded in,
behind mirrors of the reference operator API:

* ``UnifiedQuantizer``      -- polarflash_quant/unified_quantizer.py
* ``PolarLinearLayer``      -- polarflash_rt/cpu/engine.py
* ``PFlashCUDAEngine``      -- polarflash_rt/cuda/engine.py
* ``NativeLowBitCUDAEngine``-- polarflash_rt/cuda/native_kernels.py
* ``PFlashReader/Writer``   -- polarflash_core/formats/pflash_format.py
* ``BlockHadamardTransform``-- polarflash_quant/transforms/hadamard.py

The compute path is the CUDA library ``lib/libpolarflash_b200.so`` (C ABI in
include/polarflash_b200.h); there is no CPU fallback.
"""
from . import _lib, encoders
from ._lib import PolarFlashError, version
from .engine import PFlashCUDAEngine
from .hadamard import BlockHadamardTransform
from .linear import PolarLinearLayer
from .native import NativeLowBitCUDAEngine
from .pflash import PFlashReader, PFlashWriter
from .qweight import QWeight, dequantize, qlinear, qweight_from_payload, unpack_codes
from .quantizer import UnifiedQuantizer

__all__ = [
    "BlockHadamardTransform", "NativeLowBitCUDAEngine", "PFlashCUDAEngine", "PFlashReader", "PFlashWriter",
    "PolarFlashError", "PolarLinearLayer", "QWeight", "UnifiedQuantizer", "dequantize", "encoders", "qlinear",
    "qweight_from_payload", "unpack_codes", "version",
]
