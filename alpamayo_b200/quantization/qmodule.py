"""WQLinear: the ParoQuant int4 checkpoint container.

Mirrors src/alpamayo_r1/utils/quantization/qmodule.py (reference): same
constructor, buffer names, shapes and dtypes, so ParoQuant state dicts load
unchanged:

  qweight       int16 [N/4, K]        four int4 codes per element
  scales        fp16  [G_pad, N]      group scales, rows >= K/128 zero
  scaled_zeros  fp16  [G_pad, N]      -scale * zero_point
  bias          fp16  [N] (optional)

The reference forwards through AWQ W4A16 kernels of the absent
``inference_engine`` package (qmodule.py:207-232).  Here the forward runs the
B200 W4A8 path (per-token int8 activations, the tcgen05 / streaming GEMM) on
a derived tile-record buffer built from these checkpoint tensors on first
use; the checkpoint tensors stay the source of truth.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn as nn

from .. import ops


def make_divisible(c, divisor):
    """Ceiling division (qmodule.py:20-21)."""
    return (c + divisor - 1) // divisor


def calculate_zeros_width(in_features, group_size=128, pack_num=8):
    """Number of 8-group blocks of scale rows (qmodule.py:24-36)."""
    if group_size >= 128:
        mult = 1
    elif group_size == 64:
        mult = 2
    elif group_size == 32:
        mult = 4
    else:
        raise NotImplementedError
    base = make_divisible(in_features // group_size, pack_num)
    return make_divisible(base, mult) * mult


def wq_code_position(n, k, K):
    """Where code (n, k) lives in WQLinear.qweight: (row, column, nibble).

    The checkpoint format (qmodule.py:39-78) shuffles each 32-channel block
    (positions a*8+b*2+c -> b*8+a*2+c, then d*8+e*2+f -> d*8+f*4+e),
    interleaves 4 output rows over 64-channel strips and stores four nibbles
    per int16.  Vectorised over numpy integer arrays.
    """
    n = np.asarray(n)
    k = np.asarray(k)
    kb, w = k >> 5, k & 31
    p1 = ((w & 7) >> 1) * 8 + (w >> 3) * 2 + (w & 1)
    p2 = (p1 >> 3) * 8 + (p1 & 1) * 4 + ((p1 & 7) >> 1)
    kk = kb * 32 + p2
    flat = (n & 3) * 64 + (kk & 63)
    return n >> 2, (kk >> 6) * 64 + (flat >> 2), flat & 3


def pack_intweight(unpacked_qweight, interleave=4, kstride=64):
    """int4 codes [N, K] (values 0..15) -> int16 [N/4, K] checkpoint layout."""
    assert interleave == 4 and kstride == 64, "the checkpoint format uses interleave 4, kstride 64"
    codes = unpacked_qweight.detach().cpu().numpy().astype(np.int64)
    N, K = codes.shape
    nn_, kk_ = np.meshgrid(np.arange(N), np.arange(K), indexing="ij")
    r, c, v = wq_code_position(nn_, kk_, K)
    out = np.zeros((N // 4, K), dtype=np.int64)
    np.add.at(out, (r, c), (codes & 0xF) << (4 * v))
    q = torch.from_numpy(out.astype(np.uint16).view(np.int16).copy())
    return q.to(unpacked_qweight.device).contiguous()


class WQLinear(nn.Module):
    def __init__(self, w_bit, group_size, in_features, out_features, bias, dtype=torch.float16):
        super().__init__()
        if w_bit not in [4]:
            raise NotImplementedError("Only 4-bit are supported for now.")
        self.in_features = in_features
        self.out_features = out_features
        self.w_bit = w_bit
        self.group_size = group_size if group_size != -1 else in_features
        self.split_k_iters = 8
        self.interleave = 4
        assert self.in_features % self.group_size == 0
        assert out_features % (32 // self.w_bit) == 0
        gp = calculate_zeros_width(in_features, self.group_size) * (32 // self.w_bit)
        self.register_buffer("qweight", torch.zeros(
            (out_features // self.interleave, in_features // (16 // self.w_bit) * self.interleave),
            dtype=torch.int16))
        self.register_buffer("scales", torch.zeros((gp, out_features), dtype=dtype))
        self.register_buffer("scaled_zeros", torch.zeros((gp, out_features), dtype=dtype))
        if bias:
            self.register_buffer("bias", torch.zeros((out_features), dtype=dtype))
        else:
            self.bias = None
        self._packed = None
        self._packed_key = None

    @classmethod
    def from_linear(cls, linear, w_bit, group_size, init_only=False, scales=None, zeros=None):
        """Quantised container from a linear whose weight already lies on the
        (scale, zero) grid (qmodule.py:149-205).  Codes are clamped to
        [0, 15] (the reference does not clamp; out-of-range codes would
        corrupt neighbouring nibbles)."""
        q = cls(w_bit, group_size, linear.in_features, linear.out_features, linear.bias is not None,
                dtype=linear.weight.data.dtype)
        if init_only:
            return q
        assert scales is not None and zeros is not None
        N, K = linear.out_features, linear.in_features
        G = K // group_size
        dtype = scales.dtype
        gp = calculate_zeros_width(K, group_size) * 8
        qscales = torch.zeros((N, gp), dtype=dtype, device=scales.device)
        qscales[:, :G] = scales
        q.scales = qscales.transpose(1, 0).contiguous()
        if linear.bias is not None:
            q.bias = linear.bias.detach().clone().to(dtype)
        sz = (zeros * scales)
        w = linear.weight.data
        gi = torch.arange(K, device=w.device) // group_size
        codes = torch.round((w + sz[:, gi].to(w.device)) / qscales[:, gi].to(w.device))
        codes = codes.clamp(0, 15).to(torch.int32)
        q.qweight = pack_intweight(codes)
        szeros = torch.zeros_like(qscales)
        szeros[:, :G] = -(qscales[:, :G] * zeros.to(torch.int32).to(torch.float32)).to(dtype)
        q.scaled_zeros = szeros.transpose(1, 0).contiguous()
        return q

    def packed(self):
        """Tile-record buffer derived from the checkpoint tensors (rebuilt if
        they change)."""
        key = (self.qweight.data_ptr(), self.qweight._version, self.scales._version,
               self.scaled_zeros._version, self.qweight.device)
        if self._packed is None or self._packed_key != key:
            self._packed = ops.prepare_weights(self.qweight, self.scales.to(torch.float16).contiguous(),
                                               self.scaled_zeros.to(torch.float16).contiguous(),
                                               self.out_features, self.in_features)
            self._packed_key = key
        return self._packed

    @torch.no_grad()
    def forward(self, inputs):
        xq, xs = ops.per_token_quant_int8(inputs)
        out = ops.w4a8_gemm(xq, xs, self.packed(), self.out_features, self.bias, inputs.dtype)
        return out

    def extra_repr(self) -> str:
        return "in_features={}, out_features={}, bias={}, w_bit={}, group_size={}".format(
            self.in_features, self.out_features, self.bias is not None, self.w_bit, self.group_size)
