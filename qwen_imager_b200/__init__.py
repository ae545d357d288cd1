"""B200-native MLX affine group-quantized linear (the quantized DiT linear of
image-forger / vincenthz/qwen-imager), behind the reference's operator API.

Public API:
  Linear, linear, Affine   -- src/quant.rs `quant::Linear` mirror (quant.py)
  VarBuilder               -- weight supply (weights.py)
  QmmError                 -- non-OK status of the C ABI (include/qmm.h)
"""
from ._lib import QmmError
from .quant import Affine, Linear, device_error, linear
from .weights import VarBuilder, WeightError

__all__ = ["Affine", "Linear", "QmmError", "VarBuilder", "WeightError", "device_error", "linear"]
