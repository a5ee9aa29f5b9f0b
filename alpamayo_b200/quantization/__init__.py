"""Drop-in mirror of the reference's ``alpamayo_r1.utils.quantization``
package, backed by the paro_b200 sm_100a kernels."""
from .qmodule import WQLinear, calculate_zeros_width, make_divisible, pack_intweight
from .rotation_linear import Rotation, RotateLinearGroup, RotateLinearInt4
from .rotation_utils import apply_rotation_step, rotate_tensor, quantizer
from .quantization_utils import pseudo_quantize_tensor, set_op_by_name
from .paroquant_marlin_w4a8 import (
    AWQBuffers, BF16RotateLinearWrapper, MarlinW4A8Linear, convert_model_to_marlin_w4a8, convert_wqlinear_layer,
    dequant_awq, dequant_wqlinear, load_paroquant_model, pack_awq_int32, replace_linears_with_rotate_linear,
    unpack_wqlinear_qweight, wqlinear_to_awq)

__all__ = [
    "WQLinear", "calculate_zeros_width", "make_divisible", "pack_intweight", "Rotation", "RotateLinearInt4", "RotateLinearGroup",
    "apply_rotation_step", "rotate_tensor", "quantizer", "pseudo_quantize_tensor", "set_op_by_name", "AWQBuffers",
    "BF16RotateLinearWrapper", "MarlinW4A8Linear", "convert_model_to_marlin_w4a8", "convert_wqlinear_layer",
    "dequant_awq", "dequant_wqlinear", "load_paroquant_model", "pack_awq_int32",
    "replace_linears_with_rotate_linear", "unpack_wqlinear_qweight", "wqlinear_to_awq",
]
