"""Seeded synthetic ParoQuant layers on the GPU (bench / smoke inputs).

Follows the recipe the reference's path is benchmarked on (no checkpoint or
dataset is available): W ~ N(0, 0.02^2), channel scales ~ U(0.5, 2) fp16,
per layer and group a random permutation of 128 channels (consecutive
entries form the 64 disjoint Givens pairs), angles ~ U(-pi, pi) fp16, the
weight-side transform R(W / s), int4 asymmetric group-128 quantisation with
fp16 scales, packed into the WQLinear checkpoint layout and then into tile
records.  Activations are N(0, 1) with a seeded 1% of channels x 20.
"""
from __future__ import annotations

import math

import torch

from . import ops
from .quantization.qmodule import calculate_zeros_width, wq_code_position

GROUP = 128
KROT = 8


def _gen(seed, device):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def make_rotation(K, seed, device="cuda"):
    g = _gen(seed, device)
    G = K // GROUP
    keys = torch.rand(KROT, G, GROUP, generator=g, device=device)
    pairs = keys.argsort(dim=-1).reshape(KROT, K).to(torch.int16)
    theta = ((torch.rand(KROT, K // 2, generator=g, device=device) * 2 - 1) * math.pi).to(torch.float16)
    cs = (0.5 + 1.5 * torch.rand(1, K, generator=g, device=device)).to(torch.float16)
    return pairs.contiguous(), theta.contiguous(), cs.contiguous()


def make_activations(M, K, seed, dtype=torch.bfloat16, device="cuda"):
    g = _gen(seed, device)
    x = torch.randn(M, K, generator=g, device=device)
    ch = torch.randperm(K, generator=g, device=device)[: max(1, K // 100)]
    x[:, ch] *= 20.0
    return x.to(dtype)


_AWQ_ORDER = [0, 2, 4, 6, 1, 3, 5, 7]


def pack_awq_gpu(values):
    """(rows, cols) int4 values -> (rows, cols/8) int32 in AWQ nibble order."""
    rows, cols = values.shape
    v = values.to(torch.int64).reshape(rows, cols // 8, 8)[:, :, _AWQ_ORDER] & 0xF
    shifts = 4 * torch.arange(8, device=values.device, dtype=torch.int64)
    u = (v << shifts).sum(dim=-1)
    return torch.where(u >= (1 << 31), u - (1 << 32), u).to(torch.int32).contiguous()


def pack_wqlinear_gpu(codes):
    """int4 codes [N, K] -> WQLinear int16 [N/4, K] on the GPU."""
    import numpy as np
    N, K = codes.shape
    dev = codes.device
    out = torch.zeros((N // 4) * K, dtype=torch.int32, device=dev)
    step = max(1, (1 << 24) // K)
    for n0 in range(0, N, step):
        n1 = min(N, n0 + step)
        nn_, kk_ = np.meshgrid(np.arange(n0, n1), np.arange(K), indexing="ij")
        r, c, v = wq_code_position(nn_, kk_, K)
        idx = torch.from_numpy((r * K + c).reshape(-1)).to(dev)
        sh = torch.from_numpy(4 * v.reshape(-1)).to(dev)
        out.index_add_(0, idx, (codes[n0:n1].reshape(-1).to(torch.int32) & 0xF) << sh.to(torch.int32))
    return torch.where(out >= 32768, out - 65536, out).to(torch.int16).reshape(N // 4, K)


@torch.no_grad()
def make_layer(N, K, seed, device="cuda", checkpoint=True, keep_awq=False):
    """A quantised layer: rotation buffers, WQLinear buffers (if
    ``checkpoint``) and the derived tile records / uint8 pairs; with
    ``keep_awq`` (AWQ route only) also the AWQ int32 buffers
    ``awq_qweight`` [K, N/8], ``awq_scales`` [G, N], ``awq_qzeros`` [G, N/8]."""
    pairs, theta, cs = make_rotation(K, seed, device)
    g = _gen(seed + 1, device)
    W = torch.randn(N, K, generator=g, device=device) * 0.02
    Wr = ops.rotate((W / cs.float()).contiguous(), pairs, theta.float(), None, GROUP)
    del W
    G = K // GROUP
    w = Wr.reshape(-1, GROUP)
    mx, mn = w.amax(dim=1, keepdim=True), w.amin(dim=1, keepdim=True)
    s = ((mx - mn).clamp(min=1e-5) / 15)
    z = (-torch.round(mn / s)).clamp(0, 15)
    codes = (torch.round(w / s) + z).clamp(0, 15).to(torch.uint8).reshape(N, K)
    del Wr, w
    s16 = s.reshape(N, G).to(torch.float16)
    zf = z.reshape(N, G)
    Gp = calculate_zeros_width(K, GROUP) * 8
    scales = torch.zeros(Gp, N, dtype=torch.float16, device=device)
    scales[:G] = s16.t()
    szeros = torch.zeros(Gp, N, dtype=torch.float16, device=device)
    szeros[:G] = (-(s16.float() * zf)).to(torch.float16).t()
    layer = dict(N=N, K=K, pairs=pairs, theta=theta, channel_scales=cs, scales=scales.contiguous(),
                 scaled_zeros=szeros.contiguous())
    if checkpoint:
        qweight = pack_wqlinear_gpu(codes)
        layer["packed"] = ops.prepare_weights(qweight, layer["scales"], layer["scaled_zeros"], N, K)
        layer["qweight"] = qweight
    else:
        # AWQ int32 route: same codes / zero points, vectorised on the GPU
        zq = torch.clamp(torch.round(-szeros[:G].float() / scales[:G].float()), 0, 15)
        awq = (pack_awq_gpu(codes.t().contiguous()), scales[:G].contiguous(), pack_awq_gpu(zq.to(torch.uint8)))
        layer["packed"] = ops.prepare_weights_awq(awq[0], awq[1], awq[2], N, K)
        if keep_awq:
            layer["awq_qweight"], layer["awq_scales"], layer["awq_qzeros"] = awq
        del awq
    del codes
    layer["rot_table"] = ops.prepare_rotation(pairs, theta, GROUP, matrices=True)
    layer["cs_vec"] = cs.reshape(-1).contiguous()
    return layer


def weight_stream_bytes(N, K):
    """Algorithmic weight bytes of one GEMM: int4 codes + fp16 scales + int4
    zero points."""
    G = K // GROUP
    return N * K // 2 + G * N * 2 + G * N // 2
