"""Rotation and RotateLinearInt4 — the ParoQuant rotated int4 linear.

Mirrors src/alpamayo_r1/utils/quantization/rotation_linear.py (reference):
same constructors, buffers (``rotation.theta`` fp16 [8, K/2],
``rotation.pairs`` int16 [8, K], ``rotation.channel_scales`` fp16 [1, K]) and
``buffer_name`` accessor, so state dicts load unchanged.

Forward paths (all CUDA, through torch.ops.paro_b200):
  * ``Rotation.forward`` is ``rotation::rotate`` (rotation.cu:456-493).
  * ``RotateLinearInt4.forward`` with a W4A8 ``qlinear`` runs the fused
    activation kernel (channel scale + 8 Givens layers + per-token int8, the
    rotated value rounded to fp16 first as the reference's rotate kernel
    stores it) and the int4 x int8 GEMM: two launches instead of the
    reference's six (paroquant_marlin_w4a8.py:59-65 + rotation.cu + vLLM).
"""
from __future__ import annotations

import torch
import torch.nn as nn

from .. import ops
from .qmodule import WQLinear
from .rotation_utils import quantizer, rotate_tensor
from .quantization_utils import pseudo_quantize_tensor


def _default_device():
    """Device of the default buffers ``Rotation`` creates when no tables are
    given.  The reference hard-codes "cuda" (rotation_linear.py:25-29); here
    it is "cuda" when a GPU is present and "cpu" otherwise, so modules can
    be built and checkpoints loaded or converted on a machine without a GPU
    (the forward still needs CUDA tensors)."""
    return "cuda" if torch.cuda.is_available() else "cpu"


class Rotation(nn.Module):
    def __init__(self, dim, krot=8, group_size=128, rotation_angles=None, rotation_pairs=None,
                 channel_scales=None):
        super().__init__()
        if krot != 8 or group_size != 128:
            raise NotImplementedError()
        assert dim % group_size == 0
        num_groups = dim // group_size
        device = _default_device()
        if rotation_angles is None:
            rotation_angles = torch.zeros(krot, dim // 2, device=device, dtype=torch.float16)
        if rotation_pairs is None:
            one = torch.randperm(group_size, dtype=torch.int, device=device)
            rotation_pairs = one.repeat(num_groups).unsqueeze(0).expand(krot, -1)
        if channel_scales is None:
            channel_scales = torch.ones(1, dim, dtype=torch.half)
        self.register_buffer("theta", rotation_angles.clone().contiguous())
        self.register_buffer("pairs", rotation_pairs.clone().short().contiguous())
        self.register_buffer("channel_scales", channel_scales.clone().contiguous())
        self._rot_table = None
        self._rot_key = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return ops.rotate(x, self.pairs, self.theta, self.channel_scales, 128)

    def rot_table(self) -> torch.Tensor:
        """Per-channel rotation table (partner, role, fp16 angle) built from
        ``pairs`` / ``theta`` after checking that every layer's pairs are
        disjoint, with each group's rotation matrix for the prefill path
        (int32 [136, K]); derived and cached, rebuilt if the buffers change."""
        key = (self.pairs.data_ptr(), self.pairs._version, self.theta.data_ptr(), self.theta._version,
               self.pairs.device)
        if self._rot_table is None or self._rot_key != key:
            self._rot_table = ops.prepare_rotation(self.pairs.contiguous(), self.theta, 128, matrices=True)
            self._rot_key = key
        return self._rot_table

    def quantize_activations(self, x: torch.Tensor, fp16_round: bool = True):
        """x -> (int8 codes, float32 per-token scales) in one kernel."""
        cs = self.channel_scales.reshape(-1).to(torch.float16)
        return ops.rotq_int8(x, self.rot_table(), cs, 128, fp16_round)


class RotateLinearInt4(nn.Module):
    def __init__(self, in_feat, out_feat, bias, dtype, rotation_angles=None, rotation_pairs=None,
                 channel_scales=None):
        super().__init__()
        self.in_features = in_feat
        self.out_features = out_feat
        self.rotation = Rotation(in_feat, rotation_angles=rotation_angles, rotation_pairs=rotation_pairs,
                                 channel_scales=channel_scales)
        self.qlinear = WQLinear(4, 128, self.in_features, self.out_features, bias, dtype=dtype)

    @classmethod
    def from_linear(cls, linear, rotation_angles=None, rotation_pairs=None, channel_scales=None, qscales=None,
                    qzeros=None, rotate_weight=False, init_only=True):
        rl = cls(linear.in_features, linear.out_features, linear.bias is not None, linear.weight.dtype,
                 rotation_angles, rotation_pairs, channel_scales)
        if rotate_weight:
            with torch.no_grad():
                w = linear.weight.data.detach().clone()
                w = rotate_tensor(w, rotation_angles, rotation_pairs, channel_scales)
                if qscales is not None:
                    w = pseudo_quantize_tensor(w, 4, q_group_size=128, qzeros=qzeros, qscales=qscales)
                    qzeros = qzeros.view(w.size(0), -1)
                    qscales = qscales.view(w.size(0), -1)
                linear.weight.copy_(w)
        if init_only:
            return rl
        linear.to(torch.half)
        assert (qscales is None) == (qzeros is None)
        rl.qlinear = quantizer(linear, 4, 128, qscales=qscales, qzeros=qzeros)
        return rl

    def _packed_and_bias(self):
        q = self.qlinear
        if hasattr(q, "packed_weight"):
            return q.packed_weight(), q.bias
        return q.packed(), q.bias

    @torch.no_grad()
    def forward(self, x, out_dtype=None):
        packed, bias = self._packed_and_bias()
        cs = self.rotation.channel_scales.reshape(-1).to(torch.float16)
        return ops.linear_w4a8(x, self.rotation.rot_table(), cs, packed, self.out_features, bias, True,
                               out_dtype if out_dtype is not None else x.dtype)

    def buffer_name(self, buffer_name: str):
        if buffer_name == "qlinear.qweight":
            return self.qlinear.qweight
        elif buffer_name == "qlinear.scaled_zeros":
            return self.qlinear.scaled_zeros
        elif buffer_name == "qlinear.scales":
            return self.qlinear.scales
        elif buffer_name == "rotation.theta":
            return self.rotation.theta
        elif buffer_name == "rotation.pairs":
            return self.rotation.pairs
        elif buffer_name == "rotation.channel_scales":
            return self.rotation.channel_scales
        raise ValueError(f"Invalid buffer name: {buffer_name}")


class RotateLinearGroup(nn.Module):
    """Several RotateLinearInt4 that read the same input, each keeping its own
    rotation (the q / k / v or gate / up projections of a real ParoQuant
    checkpoint, which the reference loads as separate modules with separate
    tables: paroquant_marlin_w4a8.py:455-460), run as one group: one rotation
    and one quantisation launch over all tables and one GEMM over the
    concatenated weights at decode sizes.  ``forward(x)`` returns
    ``[..., sum(out_features)]``, the members' outputs side by side; the
    members stay usable on their own and keep their state-dict keys."""

    def __init__(self, linears):
        super().__init__()
        mods = [getattr(m, "rotate_linear", m) for m in linears]
        if not 1 <= len(mods) <= 4:
            raise ValueError("a group holds 1 to 4 rotated linears")
        if len({m.in_features for m in mods}) != 1:
            raise ValueError("the linears of a group must share in_features")
        self.members = nn.ModuleList(mods)
        self.in_features = mods[0].in_features
        self.out_features = sum(m.out_features for m in mods)
        self._packed = None
        self._key = None

    def _parts(self):
        packs, biases = zip(*(m._packed_and_bias() for m in self.members))
        key = tuple(p.data_ptr() for p in packs)
        if self._packed is None or self._key != key:
            self._packed = torch.cat([p.reshape(-1) for p in packs]).contiguous()
            self._key = key
        bias = None
        if any(b is not None for b in biases):
            ref = next(b for b in biases if b is not None)
            bias = torch.cat([b.reshape(-1) if b is not None else ref.new_zeros(m.out_features)
                              for b, m in zip(biases, self.members)])
        return self._packed, bias

    @torch.no_grad()
    def forward(self, x, out_dtype=None, prologue="none", residual=None, norm_weight=None, eps=1e-6):
        packed, bias = self._parts()
        tabs = [m.rotation.rot_table() for m in self.members]
        css = [m.rotation.channel_scales.reshape(-1).to(torch.float16) for m in self.members]
        y, res = ops.linear_w4a8_group(x, tabs, css, packed, [m.out_features for m in self.members], bias,
                                       prologue=prologue, residual=residual, norm_weight=norm_weight, eps=eps,
                                       out_dtype=out_dtype if out_dtype is not None else x.dtype)
        return (y, res) if prologue == "add_rmsnorm" else y
