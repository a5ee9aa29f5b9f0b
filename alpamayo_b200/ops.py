"""Python entry points for the ``torch.ops.paro_b200`` operators.

Each function is a direct call into the native operator (CUDA only).  Fake
(meta) kernels are registered so the operators trace under
``torch.compile(fullgraph=True)`` and CUDA-graph capture, the way the
reference registers ``rotation::rotate`` (kernels/paroquant_kernels/
__init__.py:7-28).
"""
from __future__ import annotations

import torch

from ._native import load_ops

load_ops()

_ops = torch.ops.paro_b200


@torch.library.register_fake("paro_b200::rotate")
def _rotate_fake(x, idx_ij, theta, scales, group_size):
    return torch.empty_like(x)


@torch.library.register_fake("paro_b200::prepare_rotation")
def _prepare_rotation_fake(pairs, theta, group_size):
    return torch.empty(pairs.shape, dtype=torch.int32, device=pairs.device)


@torch.library.register_fake("paro_b200::prepare_rotation_matrices")
def _prepare_rotation_matrices_fake(rot_table):
    return torch.empty((136, rot_table.shape[1]), dtype=torch.int32, device=rot_table.device)


@torch.library.register_fake("paro_b200::rotq_int8")
def _rotq_fake(x, rot_table, scales, group_size, fp16_round):
    q = torch.empty(x.shape, dtype=torch.int8, device=x.device)
    s = torch.empty(tuple(x.shape[:-1]) + (1,), dtype=torch.float32, device=x.device)
    return q, s


@torch.library.register_fake("paro_b200::quant_int8")
def _quant_fake(x):
    q = torch.empty(x.shape, dtype=torch.int8, device=x.device)
    s = torch.empty(tuple(x.shape[:-1]) + (1,), dtype=torch.float32, device=x.device)
    return q, s


def packed_weight_bytes(N: int, K: int) -> int:
    """Bytes of the tile-record weight buffer (16-row x 128-channel records of
    1072 bytes)."""
    if N % 16 or K % 128:
        raise ValueError("N must be a multiple of 16 and K a multiple of 128")
    return (N // 16) * (K // 128) * 1072


@torch.library.register_fake("paro_b200::prepare_weights")
def _prep_fake(qweight, scales, scaled_zeros, N, K):
    return torch.empty(packed_weight_bytes(N, K), dtype=torch.uint8, device=qweight.device)


@torch.library.register_fake("paro_b200::prepare_weights_awq")
def _prep_awq_fake(qweight, scales, qzeros, N, K):
    return torch.empty(packed_weight_bytes(N, K), dtype=torch.uint8, device=qweight.device)


@torch.library.register_fake("paro_b200::w4a8_gemm")
def _gemm_fake(xq, xscale, packed, N, bias, out_dtype):
    return torch.empty(tuple(xq.shape[:-1]) + (N,), dtype=out_dtype, device=xq.device)


@torch.library.register_fake("paro_b200::linear_w4a8")
def _linear_fake(x, rot_table, channel_scales, packed, N, bias, fp16_round, out_dtype):
    return torch.empty(tuple(x.shape[:-1]) + (N,), dtype=out_dtype, device=x.device)


def rotate(x, idx_ij, theta, scales=None, group_size=128):
    """Drop-in for ``torch.ops.rotation.rotate`` (rotation.cu:576-584)."""
    return _ops.rotate(x, idx_ij, theta, scales, group_size)


def prepare_rotation(pairs, theta, group_size=128, matrices=False):
    """Validate the pair table (each layer-group a permutation of 0..127) and
    build the per-channel rotation table (int32 [krot, K]: partner channel,
    role bit, exchange slot, fp16 angle bits) the fused kernels read.

    ``matrices=True`` (krot 8 only) also builds each 128-channel group's
    rotation matrix once, into rows 8-135 of an int32 [136, K] table: the
    prefill rotation then loads it instead of building it in every CTA
    (bit-identical results; 512 bytes per channel of device memory)."""
    table = _ops.prepare_rotation(pairs, theta.to(torch.float16).contiguous(), group_size)
    if matrices:
        table = _ops.prepare_rotation_matrices(table)
    return table


def rotq_int8(x, rot_table, scales=None, group_size=128, fp16_round=True):
    """Fused channel scale + Givens rotation + per-token int8 quantisation."""
    return _ops.rotq_int8(x, rot_table, scales, group_size, fp16_round)


def per_token_quant_int8(x):
    """Drop-in for vLLM ``per_token_quant_int8`` (int8_utils.py:131-156)."""
    return _ops.quant_int8(x)


def prepare_weights(qweight, scales, scaled_zeros, N, K):
    return _ops.prepare_weights(qweight, scales, scaled_zeros, N, K)


def prepare_weights_awq(qweight, scales, qzeros, N, K):
    return _ops.prepare_weights_awq(qweight, scales, qzeros, N, K)


def w4a8_gemm(xq, xscale, packed, N, bias=None, out_dtype=torch.bfloat16):
    return _ops.w4a8_gemm(xq, xscale, packed, N, bias, out_dtype)


def linear_w4a8(x, rot_table, channel_scales, packed, N, bias=None, fp16_round=True, out_dtype=None):
    """One W4A8 rotated linear: fused activation kernel + GEMM."""
    return _ops.linear_w4a8(x, rot_table, channel_scales, packed, N, bias, fp16_round,
                            out_dtype if out_dtype is not None else x.dtype)


@torch.library.register_fake("paro_b200::add_rmsnorm")
def _add_rmsnorm_fake(x, residual, weight, eps):
    return torch.empty_like(x), torch.empty_like(x)


@torch.library.register_fake("paro_b200::silu_mul")
def _silu_mul_fake(x):
    return x.new_empty((*x.shape[:-1], x.shape[-1] // 2))


@torch.library.register_fake("paro_b200::linear_w4a8_rmsnorm")
def _linear_rmsnorm_fake(x, residual, norm_weight, eps, rot_table, channel_scales, packed, N, bias, fp16_round,
                         out_dtype):
    return x.new_empty((*x.shape[:-1], N), dtype=out_dtype), torch.empty_like(x)


@torch.library.register_fake("paro_b200::linear_w4a8_silu")
def _linear_silu_fake(gate_up, rot_table, channel_scales, packed, N, bias, fp16_round, out_dtype):
    return gate_up.new_empty((*gate_up.shape[:-1], N), dtype=out_dtype)


def linear_w4a8_rmsnorm(x, residual, norm_weight, rot_table, channel_scales, packed, N, bias=None, eps=1e-6,
                        fp16_round=True, out_dtype=torch.bfloat16):
    """Residual add + RMSNorm fused into the rotated linear that follows it
    (decoder layer: input_layernorm -> qkv, post_attention_layernorm ->
    gate_up): returns (y, new residual stream)."""
    return _ops.linear_w4a8_rmsnorm(x, residual, norm_weight, eps, rot_table, channel_scales, packed, N, bias,
                                    fp16_round, out_dtype)


def linear_w4a8_silu(gate_up, rot_table, channel_scales, packed, N, bias=None, fp16_round=True,
                     out_dtype=torch.bfloat16):
    """SiLU(gate) * up fused into the rotated down projection: gate_up is the
    fused [..., 2K] output, gate columns first."""
    return _ops.linear_w4a8_silu(gate_up, rot_table, channel_scales, packed, N, bias, fp16_round, out_dtype)


@torch.library.register_fake("paro_b200::linear_w4a8_group")
def _linear_group_fake(x, residual, norm_weight, eps, prologue, rot_tables, channel_scales, packed, n_per_table, bias,
                       fp16_round, out_dtype):
    return x.new_empty((*x.shape[:-1], sum(n_per_table)), dtype=out_dtype), torch.empty_like(x)


PROLOGUE = {"none": 0, "add_rmsnorm": 1, "silu_mul": 2}


def linear_w4a8_group(x, rot_tables, channel_scales, packed, n_per_table, bias=None, prologue="none", residual=None,
                      norm_weight=None, eps=1e-6, fp16_round=True, out_dtype=torch.bfloat16):
    """A group of rotated linears that share x, one rotation table each
    (q / k / v, gate / up of a real checkpoint), weights concatenated along
    N: returns ([..., sum(n_per_table)], new residual stream or x)."""
    return _ops.linear_w4a8_group(x, residual, norm_weight, eps, PROLOGUE[prologue], list(rot_tables),
                                  list(channel_scales), packed, list(n_per_table), bias, fp16_round, out_dtype)


def add_rmsnorm(x, residual, weight, eps=1e-6):
    """Residual add + Qwen3VLTextRMSNorm (bf16): returns (normalised, new
    residual stream)."""
    return _ops.add_rmsnorm(x, residual, weight, eps)


def silu_mul(x):
    """SiLU(gate) * up of a fused gate_up output [..., 2I] -> [..., I] (bf16)."""
    return _ops.silu_mul(x)


def device_error_word(clear=True):
    """Error bits the kernels raised instead of hanging (1 = a bounded
    pipeline wait ran out, 2 = tensor-memory allocation failed, 4 = a wait
    for the other CTAs of the same launch ran out); 0 when all
    is well, -1 if the word could not be read.  Synchronises the device.

    A non-zero word means the outputs of the calls since the last clean read
    are invalid and a GEMM workspace may hold the partial sums or counters
    of an unfinished cross-CTA fix-up, so this also zero-fills every
    workspace the operators own before returning; the next call then starts
    from a clean workspace.  (Callers of the C ABI with their own workspaces
    must zero-fill those themselves.)"""
    from . import _native
    w = _native.capi().paro_device_error_word(1 if clear else 0)
    if w != 0:
        if _native.shim().paro_torch_reset_workspaces() < 0:
            raise RuntimeError("paro_b200: could not reset the operator workspaces after a device error")
    return w
