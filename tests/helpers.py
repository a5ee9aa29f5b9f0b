"""Seeded synthetic layers for the tests (numpy, via the CPU oracle)."""
from __future__ import annotations

import math

import numpy as np

from oracle import paro_oracle as O

GROUP = 128
KROT = 8


def make_rotation(K, seed):
    rng = np.random.default_rng(seed)
    G = K // GROUP
    pairs = np.stack([np.concatenate([rng.permutation(GROUP) for _ in range(G)]) for _ in range(KROT)])
    theta = ((rng.random((KROT, K // 2)) * 2 - 1) * math.pi).astype(np.float16)
    cs = (0.5 + 1.5 * rng.random((1, K))).astype(np.float16)
    return pairs.astype(np.int16), theta, cs


def make_activations(M, K, seed, outlier_frac=0.01):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, K)).astype(np.float32)
    ch = rng.permutation(K)[:max(1, int(K * outlier_frac))]
    x[:, ch] *= 20.0
    return x


def make_codes(N, K, seed):
    """Random int4 codes, fp16 group scales ~ N(0,0.02)-recipe magnitudes and
    zero points in 0..15, plus the WQLinear checkpoint buffers."""
    rng = np.random.default_rng(seed)
    G = K // GROUP
    codes = rng.integers(0, 16, size=(N, K))
    scales_ng = (0.004 + 0.006 * rng.random((N, G))).astype(np.float16).astype(np.float32)
    zeros_ng = rng.integers(0, 16, size=(N, G)).astype(np.float32)
    qweight, wq_s, wq_sz = O.make_wqlinear_buffers(codes, scales_ng, zeros_ng)
    zeros_gn = O.recover_zeros(wq_s, wq_sz, N, K)
    return dict(codes=codes, scales_gn=wq_s[:G].astype(np.float32), zeros_gn=zeros_gn, qweight=qweight,
                wq_scales=wq_s, wq_scaled_zeros=wq_sz)


def make_quantized_layer(N, K, seed):
    """The BASELINE recipe: W ~ N(0, 0.02^2), weight-side transform R(W/s),
    int4 asymmetric group-128 quantisation, WQLinear buffers."""
    rng = np.random.default_rng(seed)
    pairs, theta, cs = make_rotation(K, seed + 1)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    w_rot = O.rotate_tensor_weight(W, pairs, theta.astype(np.float32), cs.astype(np.float32))
    _, s, z, codes = O.pseudo_quantize_tensor(w_rot)
    qweight, wq_s, wq_sz = O.make_wqlinear_buffers(codes, s, z)
    G = K // GROUP
    return dict(W=W, pairs=pairs, theta=theta, channel_scales=cs, codes=codes, qweight=qweight,
                wq_scales=wq_s, wq_scaled_zeros=wq_sz, scales_gn=wq_s[:G].astype(np.float32),
                zeros_gn=O.recover_zeros(wq_s, wq_sz, N, K))


def rel_l2(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def expected_records(codes, scales_gn, zeros_gn):
    """The tile-record layout, restated independently of the kernel: per
    16-row block nb and group g, 1072 bytes = codes (row r at r*64; word
    t*4+j byte b = code k | code (k+64) << 4 with k = 32*(j>>1) + 16*(j&1) +
    4t + b), 16 fp16 scales, 16 uint8 zero points."""
    codes = np.asarray(codes)
    N, K = codes.shape
    G = K // GROUP
    out = np.zeros(((N // 16) * G, 1072), dtype=np.uint8)
    # k = 64h + 32s + 16half + 4t + b, word j = 2s + half
    c = codes.reshape(N // 16, 16, G, 2, 2, 2, 4, 4)  # nb, r, g, h, s, half, t, b
    lo = c[:, :, :, 0]
    hi = c[:, :, :, 1]
    byte = (lo | (hi << 4)).astype(np.uint8)            # nb, r, g, s, half, t, b
    byte = byte.reshape(N // 16, 16, G, 4, 4, 4)        # nb, r, g, j, t, b
    byte = byte.transpose(0, 2, 1, 4, 3, 5)             # nb, g, r, t, j, b
    out[:, :1024] = byte.reshape((N // 16) * G, 1024)
    s16 = np.asarray(scales_gn, dtype=np.float32).astype(np.float16)  # [G, N]
    out[:, 1024:1056] = s16.T.reshape(N // 16, 16, G).transpose(0, 2, 1).reshape(-1, 16).view(np.uint8).reshape(-1, 32)
    out[:, 1056:1072] = np.asarray(zeros_gn).astype(np.uint8).T.reshape(N // 16, 16, G).transpose(0, 2, 1).reshape(-1, 16)
    return out.reshape(-1)


_AWQ_ORDER = [0, 2, 4, 6, 1, 3, 5, 7]


def awq_columns(layer, cols):
    """Codes [len(cols), K], zero points [G, len(cols)] and fp32 group scales
    [G, len(cols)] of the given output columns, read back from a synthetic
    layer's AWQ int32 buffers (alpamayo_b200.synthetic.make_layer with
    keep_awq=True): column c = 8 j + AWQ_ORDER[i] sits in nibble i of word j."""
    import torch
    cols = np.asarray(cols)
    c_t = torch.from_numpy(cols).to(layer["awq_qweight"].device)
    nib = torch.tensor([_AWQ_ORDER.index(o) for o in range(8)], device=c_t.device)[c_t % 8]
    w = layer["awq_qweight"][:, c_t // 8].to(torch.int64) & 0xFFFFFFFF        # [K, n]
    codes = ((w >> (4 * nib)[None, :]) & 0xF).t().contiguous().cpu().numpy()
    zw = layer["awq_qzeros"][:, c_t // 8].to(torch.int64) & 0xFFFFFFFF        # [G, n]
    zeros = ((zw >> (4 * nib)[None, :]) & 0xF).cpu().numpy()
    scales = layer["awq_scales"][:, c_t].float().cpu().numpy()
    return codes, zeros, scales
