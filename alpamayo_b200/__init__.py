"""alpamayo_b200 — B200-native (sm_100a) ParoQuant W4A8 rotated linear.

A drop-in for the reference's quantised-linear path: the module API of
``alpamayo_r1.utils.quantization`` (``RotateLinearInt4``, ``WQLinear``,
``MarlinW4A8Linear``, ``BF16RotateLinearWrapper``, the loaders) over a C-ABI
library of hand-written CUDA kernels (``include/paro_b200.h``).  The public
loader entry points match ``alpamayo_r1.utils`` (reference
src/alpamayo_r1/utils/__init__.py:2,9-10).
"""
from . import ops  # noqa: F401  (loads the native operators; raises if not built)
from .quantization import (  # noqa: F401
    BF16RotateLinearWrapper, MarlinW4A8Linear, Rotation, RotateLinearInt4, WQLinear, convert_model_to_marlin_w4a8,
    load_paroquant_model)

__all__ = ["ops", "BF16RotateLinearWrapper", "MarlinW4A8Linear", "Rotation", "RotateLinearInt4", "WQLinear",
           "convert_model_to_marlin_w4a8", "load_paroquant_model"]
