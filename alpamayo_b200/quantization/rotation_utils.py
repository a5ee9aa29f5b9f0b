"""Weight-side rotation helpers (offline quantisation), mirroring
src/alpamayo_r1/utils/quantization/rotation_utils.py (reference).

``apply_rotation_step`` and ``rotate_tensor`` run on the GPU through the
paro_b200 rotate kernel (one launch for all layers); they need CUDA tensors.
"""
from __future__ import annotations

import gc

import torch
import torch.nn as nn

from .. import ops
from .quantization_utils import pseudo_quantize_tensor
from .qmodule import WQLinear


def apply_rotation_step(t: torch.Tensor, idx_ij: torch.Tensor, theta: torch.Tensor, group_size: int):
    """One Givens layer (rotation_utils.py:8-29) on the GPU."""
    t2 = t.reshape(-1, t.size(-1)).contiguous()
    return ops.rotate(t2, idx_ij.reshape(1, -1).to(torch.int16).contiguous(), theta.reshape(1, -1).contiguous(),
                      None, group_size)


def rotate_tensor(tensor, rotation_angles, rotation_pairs, channel_scales, permu=None, divide_scale=True):
    """Weight-side transform (rotation_utils.py:32-77): optional channel
    permutation, divide (or multiply) by the channel scales, then every
    Givens layer, in float32 on the GPU; returns the input dtype/shape."""
    if tensor is None:
        return tensor
    assert rotation_pairs is None or tensor.size(-1) == rotation_pairs.size(-1)
    assert rotation_angles is None or tensor.size(-1) // 2 == rotation_angles.size(-1)
    assert tensor.size(-1) == channel_scales.size(-1)
    shape, dtype = tensor.shape, tensor.dtype
    t = tensor.cuda().float().reshape(-1, tensor.size(-1))
    if permu is not None:
        t = t.index_select(-1, permu.to(torch.int64).cuda())
    if channel_scales is not None:
        cs = channel_scales.to(torch.float32).cuda().reshape(1, -1)
        t = t / cs if divide_scale else t * cs
    if rotation_pairs is not None and rotation_angles is not None:
        t = ops.rotate(t.contiguous(), rotation_pairs.to(torch.int16).cuda().contiguous(),
                       rotation_angles.to(torch.float32).cuda().contiguous(), None, 128)
    return t.to(dtype).view(shape)


@torch.no_grad()
def quantizer(linear: nn.Linear, w_bit, q_grpsize, qscales=None, qzeros=None):
    """nn.Linear -> WQLinear (rotation_utils.py:80-97)."""
    dev = linear.weight.device
    orig = linear.weight.data.detach().clone()
    assert (qscales is None) == (qzeros is None)
    if qscales is None:
        wq, qscales, qzeros = pseudo_quantize_tensor(linear.weight.data, n_bit=w_bit, get_scale_zp=True,
                                                     q_group_size=q_grpsize)
        linear.weight.copy_(wq)
    q = WQLinear.from_linear(linear, w_bit, q_grpsize, False, qscales, qzeros)
    linear.weight.copy_(orig)
    linear.to(dev)
    gc.collect()
    return q
