"""ParoQuant W4A8 loading and the W4A8 linear, B200-native.

Mirrors the public surface of
src/alpamayo_r1/utils/quantization/paroquant_marlin_w4a8.py (reference):

  BF16RotateLinearWrapper, MarlinW4A8Linear (load_from_awq / forward),
  unpack_wqlinear_qweight, pack_awq_int32, AWQBuffers, wqlinear_to_awq,
  dequant_wqlinear, dequant_awq, convert_wqlinear_layer,
  replace_linears_with_rotate_linear, load_paroquant_model,
  convert_model_to_marlin_w4a8

with the vLLM Marlin kernels, the Triton per-token quantiser and the separate
rotation kernel replaced by the paro_b200 CUDA kernels.  ``MarlinW4A8Linear``
keeps its name so callers do not change; it stores the weights as
tile records and its group scales as the checkpoint's fp16 values (no int16
re-quantisation of the scales, which Marlin needs and this kernel does not).
"""
from __future__ import annotations

import logging
from typing import NamedTuple

import torch
import torch.nn as nn

from .. import ops
from .qmodule import WQLinear
from .rotation_linear import RotateLinearInt4

logger = logging.getLogger(__name__)


class BF16RotateLinearWrapper(nn.Module):
    """Lets a RotateLinearInt4 take and return bfloat16 (reference :47-71).

    The reference casts bf16 -> fp16, runs the fp16 rotation + Marlin path and
    casts the fp16 result back.  The B200 kernels take bf16 directly and
    write bf16 directly; the fp16 rounding of the rotated activation that the
    reference's rotate kernel performs is kept inside the fused kernel.
    """

    def __init__(self, rotate_linear: nn.Module):
        super().__init__()
        self.rotate_linear = rotate_linear

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if isinstance(self.rotate_linear, RotateLinearInt4):
            return self.rotate_linear(x, out_dtype=x.dtype)
        with torch.amp.autocast("cuda", enabled=False):
            out = self.rotate_linear(x.to(torch.float16))
        return out.to(x.dtype)

    def __getattr__(self, name: str):
        try:
            return super().__getattr__(name)
        except AttributeError:
            return getattr(self.rotate_linear, name)


def _get_alpamayo_layers(model, target="vlm"):
    """Transformer layer list of a component (reference :74-80)."""
    if target == "expert":
        return model.expert.layers
    return model.vlm.model.language_model.layers


def _iter_linears(module, prefix=""):
    for name, child in module.named_children():
        full = f"{prefix}.{name}" if prefix else name
        if isinstance(child, nn.Linear):
            yield full, module, name, child
        yield from _iter_linears(child, full)


# ---------------------------------------------------------------------------
# WQLinear <-> raw int4 <-> AWQ int32 (load-time, torch index arithmetic)
# ---------------------------------------------------------------------------

def _wq_index(N, K, device):
    from .qmodule import wq_code_position
    import numpy as np
    nn_, kk_ = np.meshgrid(np.arange(N), np.arange(K), indexing="ij")
    r, c, v = wq_code_position(nn_, kk_, K)
    flat = torch.from_numpy((r * K + c).astype(np.int64)).to(device)
    nib = torch.from_numpy(v.astype(np.int64)).to(device)
    return flat, nib


def unpack_wqlinear_qweight(qweight: torch.Tensor, out_features: int, in_features: int, interleave: int = 4,
                            kstride: int = 64) -> torch.Tensor:
    """WQLinear int16 [N/4, K] -> int4 codes [N, K] int32 (reference :95-142)."""
    N, K = out_features, in_features
    flat, nib = _wq_index(N, K, qweight.device)
    w = qweight.reshape(-1).view(torch.int16).to(torch.int32) & 0xFFFF
    return ((w[flat] >> (4 * nib)) & 0xF).to(torch.int32)


_AWQ_ORDER = [0, 2, 4, 6, 1, 3, 5, 7]


def pack_awq_int32(values: torch.Tensor) -> torch.Tensor:
    """(rows, cols) int4 values -> (rows, cols/8) int32, AWQ nibble order
    [0,2,4,6,1,3,5,7] (reference :149-164)."""
    assert values.shape[1] % 8 == 0, f"cols={values.shape[1]} must be divisible by 8"
    return _to_i32(_pack8(values))


def _to_i32(u):
    return torch.where(u >= (1 << 31), u - (1 << 32), u).to(torch.int32)


class AWQBuffers(NamedTuple):
    qweight: torch.Tensor      # (K, N//8) int32
    scales: torch.Tensor       # (num_groups, N) float16
    qzeros: torch.Tensor       # (num_groups, N//8) int32
    int4_values: torch.Tensor  # (N, K) int32
    zeros: torch.Tensor        # (num_groups, N) int32


def wqlinear_to_awq(qweight_i16, scales, scaled_zeros, out_features, in_features, group_size) -> AWQBuffers:
    """WQLinear buffers -> AWQ int32 buffers (reference :179-209); zero points
    recovered as clamp(round(-sz / s), 0, 15)."""
    N, K = out_features, in_features
    G = K // group_size
    codes = unpack_wqlinear_qweight(qweight_i16, N, K)
    awq_q = _to_i32(_pack8(codes.t().contiguous()))
    awq_s = scales[:G, :N].contiguous().to(torch.float16)
    safe = awq_s.float().clone()
    safe[safe.abs() < 1e-10] = 1.0
    zeros = (-scaled_zeros[:G, :N].float() / safe).round().clamp(0, 15).to(torch.int32)
    return AWQBuffers(awq_q, awq_s, _to_i32(_pack8(zeros)), codes, zeros)


def _pack8(values):
    rows, cols = values.shape
    v = values.to(torch.int64).reshape(rows, cols // 8, 8)[:, :, _AWQ_ORDER] & 0xF
    shifts = 4 * torch.arange(8, device=values.device, dtype=torch.int64)
    return (v << shifts).sum(dim=-1)


def dequant_wqlinear(int4_NK, scales, scaled_zeros, group_size):
    """w = q * s + sz (reference :216-224)."""
    N, K = int4_NK.shape
    G = K // group_size
    sc = scales[:G, :N].float().repeat_interleave(group_size, dim=0).t()
    sz = scaled_zeros[:G, :N].float().repeat_interleave(group_size, dim=0).t()
    return int4_NK.float() * sc + sz


def dequant_awq(int4_NK, zeros, scales, group_size):
    """w = (q - z) * s (reference :227-235)."""
    N, K = int4_NK.shape
    G = K // group_size
    sc = scales[:G, :N].float().repeat_interleave(group_size, dim=0).t()
    zp = zeros[:G, :N].float().repeat_interleave(group_size, dim=0).t()
    return (int4_NK.float() - zp) * sc


# ---------------------------------------------------------------------------
# the W4A8 linear
# ---------------------------------------------------------------------------

class MarlinW4A8Linear(nn.Module):
    """int4 weight x per-token int8 activation linear (reference :242-333),
    computed by the paro_b200 GEMM.

    Lifecycle as in the reference: construct, ``load_from_awq`` (or
    ``load_from_wqlinear``), then ``forward``.  ``forward(x)`` quantises x per
    token to int8 and returns ``x.dtype`` (fp16 for fp16 input, as the
    reference's Marlin path; bf16 for bf16).
    """

    def __init__(self, in_features: int, out_features: int, group_size: int = 128):
        super().__init__()
        if group_size != 128:
            raise NotImplementedError("the W4A8 kernels use 128-channel groups")
        self.in_features = in_features
        self.out_features = out_features
        self.group_size = group_size
        self.register_buffer("qweight", torch.empty(0, dtype=torch.uint8))    # tile records
        self.register_buffer("scales", torch.empty(0, dtype=torch.float16))   # [G, N] fp16
        self.register_buffer("qzeros", torch.empty(0, dtype=torch.int32))     # AWQ-packed zero points
        self.register_buffer("workspace", torch.empty(0, dtype=torch.int32))
        self.register_buffer("g_idx", torch.empty(0, dtype=torch.int32))
        self.register_buffer("g_idx_sort_indices", torch.empty(0, dtype=torch.int32))
        self.register_buffer("input_global_scale", torch.ones(1, dtype=torch.float32))
        # registered up front so a bias tensor can be assigned later (the
        # reference sets a plain attribute and then registers over it, which
        # torch rejects for layers that do have a bias)
        self.register_buffer("bias", None)

    def load_from_awq(self, awq_qweight, awq_scales, awq_qzeros, bias=None):
        K, N = self.in_features, self.out_features
        self.qweight = ops.prepare_weights_awq(awq_qweight.contiguous(), awq_scales.to(torch.float16).contiguous(),
                                               awq_qzeros.contiguous(), N, K)
        self.scales = awq_scales.to(torch.float16).contiguous()
        self.qzeros = awq_qzeros.contiguous()
        self.workspace = torch.empty(0, dtype=torch.int32, device=awq_qweight.device)
        self.input_global_scale = torch.ones(1, dtype=torch.float32, device=awq_qweight.device)
        self.bias = bias

    def load_from_wqlinear(self, qweight_i16, scales, scaled_zeros, bias=None):
        """Direct WQLinear -> tile records (same codes and zero points as the
        AWQ route, without materialising the AWQ buffers)."""
        K, N = self.in_features, self.out_features
        G = K // self.group_size
        self.qweight = ops.prepare_weights(qweight_i16.contiguous(), scales.to(torch.float16).contiguous(),
                                           scaled_zeros.to(torch.float16).contiguous(), N, K)
        self.scales = scales[:G, :N].to(torch.float16).contiguous()
        self.bias = bias

    def packed_weight(self):
        return self.qweight

    @torch.no_grad()
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        xq, xs = ops.per_token_quant_int8(x)
        return ops.w4a8_gemm(xq, xs, self.qweight, self.out_features, self.bias,
                             x.dtype if x.dtype in (torch.float16, torch.bfloat16) else torch.float16)


def convert_wqlinear_layer(qweight_i16, scales, scaled_zeros, out_features, in_features, group_size, bias=None,
                           device="cuda"):
    """WQLinear buffers -> MarlinW4A8Linear on ``device`` (reference :340-353)."""
    awq = wqlinear_to_awq(qweight_i16, scales, scaled_zeros, out_features, in_features, group_size)
    mod = MarlinW4A8Linear(in_features, out_features, group_size)
    mod.load_from_awq(awq.qweight.to(device), awq.scales.to(device), awq.qzeros.to(device),
                      bias=bias.to(device) if bias is not None else None)
    return mod, awq


def _wrap_rotate_linears(model, target="vlm"):
    for layer in _get_alpamayo_layers(model, target):
        for _, child in layer.named_children():
            for sub_name, sub_child in child.named_children():
                if isinstance(sub_child, RotateLinearInt4):
                    setattr(child, sub_name, BF16RotateLinearWrapper(sub_child))


def replace_linears_with_rotate_linear(model, target="vlm", init_only: bool = True,
                                       ignore_suffix: tuple = ("lm_head",)):
    """Swap nn.Linear modules of the target layers for empty RotateLinearInt4
    shells, to be filled by load_state_dict (reference :366-387)."""
    for layer in _get_alpamayo_layers(model, target):
        for _, parent, child_name, linear in list(_iter_linears(layer)):
            if child_name in ignore_suffix:
                continue
            setattr(parent, child_name, RotateLinearInt4(in_feat=linear.in_features, out_feat=linear.out_features,
                                                         bias=linear.bias is not None, dtype=torch.float16))


def _sanitise_channel_scales(model):
    """Clamp INF / NaN / overflowing channel scales to +-65504/128
    (reference :390-423)."""
    safe = 65504.0 / 128.0
    n_fixed = 0
    for name, mod in model.named_modules():
        if not isinstance(mod, RotateLinearInt4):
            continue
        cs = mod.rotation.channel_scales
        bad = torch.isinf(cs) | torch.isnan(cs) | (cs.abs() > safe)
        n_bad = int(bad.sum().item())
        if n_bad:
            with torch.no_grad():
                cs.nan_to_num_(nan=safe, posinf=safe, neginf=-safe).clamp_(-safe, safe)
            n_fixed += 1
            logger.warning(f"  Clamped {n_bad}/{cs.numel()} channel_scales in {name} (had INF/NaN/overflow values)")
    if n_fixed:
        logger.warning(f"Sanitised channel_scales in {n_fixed} RotateLinearInt4 modules")
    return n_fixed


def load_paroquant_model(model_path: str, paro_checkpoint, *, mode: str = "streaming",
                         dtype: torch.dtype = torch.bfloat16, device: str = "cuda", model_factory=None):
    """Load a model with ParoQuant int4 weights (reference :426-510).

    ``model_factory(model_path, dtype)`` builds the base model; by default the
    Alpamayo-R1 class is imported as in the reference.  ``paro_checkpoint`` is
    a path or an already-loaded state dict.
    """
    if model_factory is None:
        from alpamayo_r1.models.alpamayo_r1_unified import AlpamayoR1FlashDrive  # noqa: F401  (caller's package)

        def model_factory(p, dt):
            m = AlpamayoR1FlashDrive.from_pretrained(p, dtype=dt)
            m.setup_patch_for_torch_compile(torch_compile="max-autotune", mode=mode, fuse_qkv=False,
                                            fuse_gate_up=False)
            return m
    model = model_factory(model_path, dtype)
    replace_linears_with_rotate_linear(model, target="vlm", init_only=True)
    sd = paro_checkpoint if isinstance(paro_checkpoint, dict) else torch.load(paro_checkpoint, map_location="cpu",
                                                                             weights_only=True)
    missing, unexpected = model.load_state_dict(sd, strict=False)
    quant_missing = [k for k in missing if any(s in k for s in ("qlinear", "rotation", "qweight", "scales",
                                                               "scaled_zeros"))]
    if quant_missing:
        logger.warning(f"  CRITICAL quant missing: {quant_missing[:10]}")
    if unexpected:
        logger.warning(f"Unexpected keys ({len(unexpected)}): {unexpected[:20]}")
    n_zero = sum(1 for name, b in model.named_buffers() if "scales" in name and b.numel() > 0 and torch.all(b == 0))
    if n_zero:
        logger.error(f"CRITICAL: {n_zero} layers have zero scales — checkpoint keys likely mismatched!")
    _sanitise_channel_scales(model)
    _wrap_rotate_linears(model, target="vlm")
    model = model.to(device)
    model.eval()
    return model


def convert_model_to_marlin_w4a8(model):
    """Replace every RotateLinearInt4's WQLinear by a MarlinW4A8Linear backed
    by the paro_b200 kernels (reference :513-529)."""
    n = 0
    for _, mod in model.named_modules():
        if not isinstance(mod, RotateLinearInt4):
            continue
        wq = mod.qlinear
        if not isinstance(wq, WQLinear):
            continue
        m = MarlinW4A8Linear(wq.in_features, wq.out_features, wq.group_size)
        m.load_from_wqlinear(wq.qweight.data, wq.scales.data, wq.scaled_zeros.data, bias=wq.bias)
        mod.qlinear = m
        n += 1
    logger.info(f"Converted {n} WQLinear -> MarlinW4A8Linear (paro_b200 W4A8)")
    return n
