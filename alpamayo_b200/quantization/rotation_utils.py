"""Weight-side rotation helpers (offline quantisation), mirroring
src/alpamayo_r1/utils/quantization/rotation_utils.py (reference).

These run once per layer when a checkpoint is made, not per token, so they
are plain torch on whatever device the tensor is on.  The arithmetic is the
reference's, operation for operation: sin / cos of the float32 angles by
torch, then per pair ``c*a + s*b`` and ``-s*a + c*b`` with every product and
sum rounded separately, so a weight transformed here equals the reference's
bit for bit on the same device.  (The reference moves the tensor to CUDA
unconditionally, rotation_utils.py:49; here the caller's device is kept, so
a checkpoint can also be converted on a machine without a GPU.)
"""
from __future__ import annotations

import gc

import torch
import torch.nn as nn

from .quantization_utils import pseudo_quantize_tensor
from .qmodule import WQLinear


def _pair_columns(idx_ij: torch.Tensor, hidden: int, group_size: int):
    """Absolute column indices of the first and second element of every
    pair, all groups at once: entries 2p and 2p+1 of a group form pair p."""
    idx = idx_ij.reshape(-1).to(torch.int64)
    base = torch.arange(0, hidden, group_size, device=idx.device).repeat_interleave(group_size // 2)
    return idx[0::2] + base, idx[1::2] + base


def apply_rotation_step(t: torch.Tensor, idx_ij: torch.Tensor, theta: torch.Tensor, group_size: int):
    """One Givens layer (rotation_utils.py:8-29): every group's 64 disjoint
    pairs (i, j) with angle th become (c*a_i + s*a_j, -s*a_i + c*a_j); the
    groups are done together (the reference loops over them; the pairs are
    disjoint, so the order does not matter)."""
    t = t.reshape(-1, t.size(-1)).clone()
    di, dj = _pair_columns(idx_ij.to(t.device), t.size(-1), group_size)
    th = theta.reshape(-1).to(t.device)
    s = torch.sin(th).to(t.dtype).unsqueeze(0)
    c = torch.cos(th).to(t.dtype).unsqueeze(0)
    a, b = t[:, di], t[:, dj]
    t[:, di] = c * a + s * b
    t[:, dj] = -s * a + c * b
    return t


def rotate_tensor(tensor, rotation_angles, rotation_pairs, channel_scales, permu=None, divide_scale=True):
    """Weight-side transform (rotation_utils.py:32-77): optional channel
    permutation, divide (or multiply) by the channel scales, then every
    Givens layer, in float32; returns the input dtype / shape on the
    input's device."""
    if tensor is None:
        return tensor
    assert rotation_pairs is None or tensor.size(-1) == rotation_pairs.size(-1)
    assert rotation_angles is None or tensor.size(-1) // 2 == rotation_angles.size(-1)
    assert tensor.size(-1) == channel_scales.size(-1)
    assert permu is None or tensor.size(-1) == permu.size(-1)
    shape, dtype, dev = tensor.shape, tensor.dtype, tensor.device
    t = tensor.float().reshape(-1, tensor.size(-1))
    if permu is not None:
        t = t.index_select(-1, permu.to(device=dev, dtype=torch.int64))
    if channel_scales is not None:
        cs = channel_scales.to(device=dev, dtype=torch.float32)
        t = t / cs if divide_scale else t * cs
    if rotation_pairs is not None and rotation_angles is not None:
        pairs = rotation_pairs.to(dev)
        angles = rotation_angles.to(device=dev, dtype=torch.float32)
        for r in range(pairs.size(0)):
            t = apply_rotation_step(t, pairs[r], angles[r], 128)
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
