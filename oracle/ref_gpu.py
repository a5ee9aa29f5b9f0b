"""The reference's own GPU path for the W4A8 linear (test infrastructure).

TEST / BENCH INFRASTRUCTURE ONLY: imported by tests/ and by bench.py's
reference-GPU leg as the checker and the baseline, never by the product
package.

The reference runs one rotated linear as (paths relative to the reference
project):

  BF16RotateLinearWrapper.forward   src/alpamayo_r1/utils/quantization/paroquant_marlin_w4a8.py:59-65
    x.to(float16)
    rotation::rotate                kernels/paroquant_kernels/src/rotation.cu:456-493
    MarlinW4A8Linear.forward        paroquant_marlin_w4a8.py:314-333
      apply_awq_marlin_linear       vllm/model_executor/layers/quantization/utils/marlin_utils.py:577
        per_token_quant_int8 (Triton) and ops.marlin_gemm (compiled vLLM)
    out.to(bfloat16)

Here the rotation is the reference's own kernel, compiled from its source
by ``oracle/build_ref.py`` into ``oracle/_ref/librotation_ref.so``, and the
quantiser and GEMM are vLLM's installed ops, called in the order of
``MarlinW4A8Linear.load_from_awq`` (paroquant_marlin_w4a8.py:274-312) and
``forward`` (:314-333).  Nothing under the reference checkout is read at run
time.  ``available()`` reports why a piece cannot run.
"""
from __future__ import annotations

import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF_SO = os.path.join(HERE, "_ref", "librotation_ref.so")

_rot_loaded = None


def load_rotate():
    """torch.ops.rotation.rotate from the reference's compiled kernel."""
    global _rot_loaded
    if _rot_loaded is None:
        if not os.path.exists(REF_SO):
            raise FileNotFoundError(f"{REF_SO} missing: run python oracle/build_ref.py")
        torch.ops.load_library(REF_SO)
        _rot_loaded = torch.ops.rotation.rotate
    return _rot_loaded


def vllm_ops():
    """vLLM's custom ops and Marlin helpers (the reference's GEMM path)."""
    from vllm import _custom_ops as ops
    from vllm.model_executor.layers.quantization.utils import marlin_utils as mu
    from vllm.model_executor.layers.quantization.utils.int8_utils import per_token_quant_int8
    from vllm.scalar_type import scalar_types
    return ops, mu, per_token_quant_int8, scalar_types


def available():
    """(rotate_ok, marlin_ok, reason) on this machine."""
    reasons = []
    rot_ok = marlin_ok = False
    try:
        load_rotate()
        rot_ok = True
    except Exception as e:  # noqa: BLE001 (report any load failure)
        reasons.append(f"rotate: {type(e).__name__}: {str(e).splitlines()[0][:200]}")
    try:
        vllm_ops()
        marlin_ok = hasattr(torch.ops._C, "marlin_gemm")
        if not marlin_ok:
            reasons.append("marlin: torch.ops._C.marlin_gemm not registered")
    except Exception as e:  # noqa: BLE001
        reasons.append(f"marlin: {type(e).__name__}: {str(e).splitlines()[0][:200]}")
    return rot_ok, marlin_ok, "; ".join(reasons)


class MarlinW4A8:
    """The reference's MarlinW4A8Linear state built from AWQ int32 buffers
    with vLLM's helpers (paroquant_marlin_w4a8.py:274-312): repack with the
    8-bit-activation tile layout, permute the scales, requantise them to
    int16 with a global factor when there is more than one group, convert
    the zero points."""

    def __init__(self, awq_qweight, awq_scales, awq_qzeros, K, N, group_size=128, bias=None):
        ops, mu, _, scalar_types = vllm_ops()
        dev = awq_qweight.device
        self.K, self.N = K, N
        self.quant_type = scalar_types.uint4
        self.workspace = mu.marlin_make_workspace_new(dev)
        self.g_idx = mu.marlin_make_empty_g_idx(dev)
        self.g_idx_sort_indices = mu.marlin_make_empty_g_idx(dev)
        self.qweight = ops.awq_marlin_repack(awq_qweight, size_k=K, size_n=N, num_bits=4, is_a_8bit=True)
        s = mu.marlin_permute_scales(awq_scales, size_k=K, size_n=N, group_size=group_size, is_a_8bit=True)
        if K // group_size > 1:
            s, gs = mu.marlin_act_int8_process_scales(s)
        else:
            gs = torch.ones(1, dtype=torch.float32, device=dev)
        self.scales = s
        self.input_global_scale = gs
        self.qzeros = mu.awq_to_marlin_zero_points(awq_qzeros, size_k=K // group_size, size_n=N, num_bits=4,
                                                   is_a_8bit=True)
        self.bias = bias

    @torch.no_grad()
    def __call__(self, x_fp16):
        """MarlinW4A8Linear.forward (paroquant_marlin_w4a8.py:314-333)."""
        _, mu, _, _ = vllm_ops()
        return mu.apply_awq_marlin_linear(
            input=x_fp16, weight=self.qweight, weight_scale=self.scales, weight_zp=self.qzeros,
            g_idx=self.g_idx, g_idx_sort_indices=self.g_idx_sort_indices, workspace=self.workspace,
            quant_type=self.quant_type, output_size_per_partition=self.N, input_size_per_partition=self.K,
            input_global_scale=self.input_global_scale, bias=self.bias, input_dtype=torch.int8)


class ReferenceLinear:
    """One rotated W4A8 linear run the reference's way on the GPU:
    bf16 -> fp16, the reference's rotate kernel, vLLM per-token int8 +
    Marlin W4A8, fp16 -> bf16 (BF16RotateLinearWrapper + RotateLinearInt4 +
    MarlinW4A8Linear)."""

    def __init__(self, pairs, theta, channel_scales, awq_qweight, awq_scales, awq_qzeros, K, N, bias=None):
        self.rotate = load_rotate()
        self.pairs = pairs.contiguous()
        self.theta = theta.to(torch.float16).contiguous()
        self.cs = channel_scales.to(torch.float16).contiguous()
        self.marlin = MarlinW4A8(awq_qweight, awq_scales, awq_qzeros, K, N, bias=bias)

    def rotated(self, x):
        return self.rotate(x.to(torch.float16), self.pairs, self.theta, self.cs, 128)

    @torch.no_grad()
    def __call__(self, x):
        in_dtype = x.dtype
        return self.marlin(self.rotated(x)).to(in_dtype)

    def quantised(self, x):
        """The int8 codes and token scales vLLM's quantiser makes from the
        rotated rows (marlin_utils.py:500-506 -> int8_utils.py:131-156)."""
        _, _, ptq, _ = vllm_ops()
        r = self.rotated(x)
        return ptq(r.reshape(-1, r.shape[-1]))
