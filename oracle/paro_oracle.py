"""CPU oracle for the ParoQuant W4A8 rotated-linear path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this file;
only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference arm may use it, and only as the checker or as the timed CPU
restatement of the reference.  It is never the thing measured as the GPU
product and never a fallback.

Every function restates one reference function (path relative to the
reference project root; ``vllm/...`` is the installed vLLM 0.22 package the
reference calls into).  Arithmetic is numpy: integer work in int64, float
work in float32 where the reference computes in float32, float64 where the
reference's exact accumulation order is not observable (the compiled Marlin
GEMM), so the oracle gives the mathematically exact value for those sums.

Parity is pinned by ``tests/golden/`` fixtures produced by importing the
reference's own Python functions (``tests/golden/gen_golden.py``).
"""
from __future__ import annotations

import numpy as np

GROUP = 128
KROT = 8


# ---------------------------------------------------------------------------
# float helpers
# ---------------------------------------------------------------------------

def f32(a):
    return np.asarray(a, dtype=np.float32)


def round_to_fp16(a):
    """IEEE round-to-nearest-even to binary16, returned as float32."""
    return f32(a).astype(np.float16).astype(np.float32)


def round_to_bf16(a):
    """IEEE round-to-nearest-even float32 -> bfloat16, returned as float32."""
    u = f32(a).view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16) << 16
    out = r.astype(np.uint32).view(np.float32)
    nan = np.isnan(f32(a))
    if nan.any():
        out = out.copy()
        out[nan] = np.nan
    return out


def bf16_bits_to_f32(u16):
    return (np.asarray(u16, dtype=np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(a):
    return (round_to_bf16(a).view(np.uint32) >> 16).astype(np.uint16)


def round_half_away(v):
    """Round half away from zero, exact for float32 inputs (computed in f64).

    libdevice ``round`` semantics used by vLLM's Triton quant kernel
    (vllm/model_executor/layers/quantization/utils/int8_utils.py:101-102).
    """
    v64 = np.asarray(v, dtype=np.float64)
    return np.sign(v64) * np.floor(np.abs(v64) + 0.5)


# ---------------------------------------------------------------------------
# rotation
# ---------------------------------------------------------------------------

def _sin_cos_f32(th):
    """float32 sin/cos exactly as the reference evaluates them on CPU
    (``torch.sin(theta)`` on a float32 tensor, rotation_utils.py:14-15), so
    the oracle's rotation is bit-identical to the reference's CPU path."""
    import torch
    t = torch.from_numpy(np.ascontiguousarray(f32(th)))
    return torch.sin(t).numpy(), torch.cos(t).numpy()


def apply_rotation_step(t, idx_ij, theta, group_size=GROUP):
    """One Givens layer, restating
    src/alpamayo_r1/utils/quantization/rotation_utils.py:8-29.

    t: [rows, K] float32; idx_ij: [K] group-local indices (consecutive
    entries (i, j) form a pair); theta: [K/2].  For pair p of group g:
    xi' = c*xi + s*xj, xj' = -s*xi + c*xj with c = cos(theta), s = sin(theta)
    computed in float32 like torch.sin/torch.cos on a float32 tensor.
    """
    t = f32(t).reshape(-1, np.shape(t)[-1]).copy()
    hidden = t.shape[-1]
    n_groups = hidden // group_size
    half = group_size // 2
    th = f32(theta).reshape(n_groups, half)
    s, c = _sin_cos_f32(th)
    idx = np.asarray(idx_ij).astype(np.int64).reshape(n_groups, group_size)
    starts = (np.arange(n_groups) * group_size)[:, None]
    di = (idx[:, 0::2] + starts).reshape(-1)
    dj = (idx[:, 1::2] + starts).reshape(-1)
    cg = c.reshape(-1)[None, :]
    sg = s.reshape(-1)[None, :]
    a = t[:, di]
    b = t[:, dj]
    # torch evaluates c*a + s*b as two float32 products and one float32 add
    t[:, di] = (cg * a) + (sg * b)
    t[:, dj] = (-sg * a) + (cg * b)
    return t


def rotate_activations(x, pairs, theta, channel_scales, group_size=GROUP):
    """Forward of ``rotation::rotate`` (kernels/paroquant_kernels/src/
    rotation.cu:15-60 with RotateAccess<__half>, rotation.cuh:248-337):
    x * channel_scale in float32, then every Givens layer in order.
    Returns the float32 result BEFORE the kernel's store rounding.
    """
    x = f32(x)
    K = x.shape[-1]
    t = x.reshape(-1, K)
    if channel_scales is not None:
        t = t * f32(channel_scales).reshape(1, K)
    for r in range(np.shape(pairs)[0]):
        t = apply_rotation_step(t, pairs[r], theta[r], group_size)
    return t.reshape(x.shape)


def rotate_tensor_weight(w, pairs, theta, channel_scales, group_size=GROUP):
    """Weight-side transform of rotation_utils.py:32-77 (divide_scale=True):
    W / s then the same Givens layers, float32."""
    w = f32(w)
    t = w / f32(channel_scales).reshape(1, -1)
    for r in range(np.shape(pairs)[0]):
        t = apply_rotation_step(t, pairs[r], theta[r], group_size)
    return t


def validate_pairs(pairs, group_size=GROUP):
    """True when every layer-group of ``pairs`` is a permutation of
    0..group_size-1 (the disjointness invariant ``rotate`` relies on,
    rotation.cuh:299-316; Rotation defaults to a randperm,
    rotation_linear.py:32-37)."""
    p = np.asarray(pairs).astype(np.int64)
    L, K = p.shape
    g = p.reshape(L, K // group_size, group_size)
    srt = np.sort(g, axis=-1)
    return bool((srt == np.arange(group_size)[None, None, :]).all())


# ---------------------------------------------------------------------------
# per-token int8 activation quantisation (vLLM)
# ---------------------------------------------------------------------------

def per_token_quant_int8(x):
    """Restates vllm/model_executor/layers/quantization/utils/int8_utils.py
    :106-128 (``_per_token_quant_int8``): absmax = max(max|x|, 1e-10),
    scale = absmax / 127, q = round(x * (127 / absmax)) with round half away
    from zero; all float32.  Returns (int8 [M,K], float32 [M])."""
    x = f32(x)
    K = x.shape[-1]
    t = x.reshape(-1, K)
    absmax = np.maximum(np.abs(t).max(axis=1), np.float32(1e-10)).astype(np.float32)
    scale = (absmax / np.float32(127.0)).astype(np.float32)
    inv = (np.float32(127.0) / absmax).astype(np.float32)
    v = (t * inv[:, None]).astype(np.float32)
    q = np.clip(round_half_away(v), -128, 127).astype(np.int8)
    return q, scale


# ---------------------------------------------------------------------------
# int4 weight quantisation and the WQLinear checkpoint layout
# ---------------------------------------------------------------------------

def pseudo_quantize_tensor(w, n_bit=4, q_group_size=GROUP):
    """Asymmetric group quantisation, restating
    src/alpamayo_r1/utils/quantization/quantization_utils.py:18-73
    (zero_point=True branch): s = (max-min).clamp(1e-5)/15,
    z = clamp(-round(min/s), 0, 15), q = clamp(round(w/s) + z, 0, 15).
    ``torch.round`` is round-half-to-even, as is ``np.rint``.
    Returns (w_dq [N,K] f32, scales [N,G] f32, zeros [N,G] f32, codes [N,K] i64).
    """
    w = f32(w)
    N, K = w.shape
    t = w.reshape(-1, q_group_size)
    max_val = t.max(axis=1, keepdims=True)
    min_val = t.min(axis=1, keepdims=True)
    max_int = 2 ** n_bit - 1
    scales = (np.maximum(max_val - min_val, np.float32(1e-5)) / np.float32(max_int)).astype(np.float32)
    zeros = np.clip(-np.rint(min_val / scales), 0, max_int).astype(np.float32)
    codes = np.clip(np.rint(t / scales) + zeros, 0, max_int)
    w_dq = ((codes - zeros) * scales).astype(np.float32)
    G = K // q_group_size
    return (w_dq.reshape(N, K), scales.reshape(N, G), zeros.reshape(N, G),
            codes.astype(np.int64).reshape(N, K))


def calculate_zeros_width(in_features, group_size=GROUP, pack_num=8):
    """qmodule.py:24-36."""
    def make_divisible(c, divisor):
        return (c + divisor - 1) // divisor
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


def padded_groups(in_features, group_size=GROUP):
    """Rows of WQLinear.scales / scaled_zeros (qmodule.py:123-142)."""
    return calculate_zeros_width(in_features, group_size) * 8


def pack_intweight(codes, interleave=4, kstride=64):
    """qmodule.py:39-78: 32-K shuffle, pair swap, 4-row x 64-K interleave,
    four nibbles per int16.  codes: [N, K] ints in [0, 15]."""
    c = np.asarray(codes).astype(np.int64)
    N, K = c.shape
    p = c.reshape(N, K // 32, 4, 4, 2).transpose(0, 1, 3, 2, 4).reshape(N, K // 32, 32)
    p = p.reshape(N, K // 32, 4, 4, 2).transpose(0, 1, 2, 4, 3).reshape(N, K)
    p = p.reshape(N // interleave, interleave, K // kstride, kstride).transpose(0, 2, 1, 3)
    p = p.reshape(N // interleave, K // kstride, kstride, interleave)
    p = p[..., 0] | (p[..., 1] << 4) | (p[..., 2] << 8) | (p[..., 3] << 12)
    return p.reshape(N // interleave, K).astype(np.int64).astype(np.uint16).view(np.int16)


def unpack_wqlinear_qweight(qweight, N, K, interleave=4, kstride=64):
    """Inverse of pack_intweight, restating
    src/alpamayo_r1/utils/quantization/paroquant_marlin_w4a8.py:95-142."""
    pw = np.asarray(qweight).view(np.uint16).astype(np.int64)
    x = np.stack([pw & 0xF, (pw >> 4) & 0xF, (pw >> 8) & 0xF, (pw >> 12) & 0xF], axis=-1)
    x = x.reshape(N // interleave, K // kstride, kstride, interleave)
    x = x.reshape(N // interleave, K // kstride, interleave, kstride)
    x = x.transpose(0, 2, 1, 3).reshape(N, K)
    x = x.reshape(N, K // 32, 4, 2, 4).transpose(0, 1, 2, 4, 3).reshape(N, K)
    x = x.reshape(N, K // 32, 4, 4, 2).transpose(0, 1, 3, 2, 4).reshape(N, K)
    return x


def make_wqlinear_buffers(codes, scales_ng, zeros_ng, group_size=GROUP):
    """Checkpoint buffers written by WQLinear.from_linear (qmodule.py:149-205):
    qweight int16 [N/4, K]; scales fp16 [G_pad, N]; scaled_zeros fp16
    [G_pad, N] = -(fp16 s * z) rounded to fp16, rows beyond G zero.
    ``codes`` are the clamped codes (the reference does not clamp; the
    fixture generator always produces codes in range).
    """
    N, K = np.shape(codes)
    G = K // group_size
    Gp = padded_groups(K, group_size)
    s16 = np.asarray(scales_ng, dtype=np.float32).astype(np.float16)  # [N, G]
    scales = np.zeros((Gp, N), dtype=np.float16)
    scales[:G, :] = s16.T
    sz = np.zeros((Gp, N), dtype=np.float16)
    sz[:G, :] = (-(s16.astype(np.float32) * np.asarray(zeros_ng, np.float32))).astype(np.float16).T
    return pack_intweight(codes), scales, sz


def recover_zeros(scales, scaled_zeros, N, K, group_size=GROUP):
    """paroquant_marlin_w4a8.py:197-204: z = clamp(round(-sz / s), 0, 15)
    with |s| < 1e-10 replaced by 1; float32, round half to even."""
    G = K // group_size
    sc = np.asarray(scales)[:G, :N].astype(np.float32).copy()
    sc[np.abs(sc) < 1e-10] = 1.0
    sz = np.asarray(scaled_zeros)[:G, :N].astype(np.float32)
    return np.clip(np.rint(-sz / sc), 0, 15).astype(np.int64)  # [G, N]


def dequant_wqlinear(codes, scales, scaled_zeros, group_size=GROUP):
    """paroquant_marlin_w4a8.py:216-224: w = q * s + sz (float32)."""
    N, K = np.shape(codes)
    G = K // group_size
    sc = np.repeat(np.asarray(scales)[:G, :N].astype(np.float32), group_size, axis=0).T
    sz = np.repeat(np.asarray(scaled_zeros)[:G, :N].astype(np.float32), group_size, axis=0).T
    return np.asarray(codes).astype(np.float32) * sc + sz


def dequant_awq(codes, zeros_gn, scales, group_size=GROUP):
    """paroquant_marlin_w4a8.py:227-235: w = (q - z) * s (float32)."""
    N, K = np.shape(codes)
    G = K // group_size
    sc = np.repeat(np.asarray(scales)[:G, :N].astype(np.float32), group_size, axis=0).T
    zp = np.repeat(np.asarray(zeros_gn)[:G, :N].astype(np.float32), group_size, axis=0).T
    return (np.asarray(codes).astype(np.float32) - zp) * sc


def marlin_act_int8_process_scales(s_fp16):
    """vllm/model_executor/layers/quantization/utils/marlin_utils.py:326-330:
    in float16 arithmetic, s_i16 = round(s / max(s) * 4096) and a float32
    global factor max(s) / 4096 folded into the activation scale."""
    s = np.asarray(s_fp16, dtype=np.float16)
    smax = s.max()
    glob = np.float32(1.0 / 4096.0) * np.float32(smax)
    t = (s / smax).astype(np.float16)
    t = (t * np.float16(4096)).astype(np.float16)
    return np.rint(t.astype(np.float32)).astype(np.int64), np.float32(glob)


# ---------------------------------------------------------------------------
# the int4 x int8 GEMM (Marlin contract, apply_awq_marlin_linear)
# ---------------------------------------------------------------------------

def group_partials(xq, codes, zeros_gn, group_size=GROUP):
    """Exact int32 per-group partials P[m, n, g] = sum_{k in g} (q[n,k] -
    z[g,n]) * xq[m,k] (int64 here; |P| <= 128*15*127 fits int32)."""
    # float64 products and sums of these integers are exact (|P| < 2^18), and
    # let the matmul use BLAS
    xq = np.asarray(xq).astype(np.float64)
    c = np.asarray(codes).astype(np.float64)
    M, K = xq.shape
    N = c.shape[0]
    G = K // group_size
    z = np.asarray(zeros_gn).astype(np.float64)[:G, :N]  # [G, N]
    P = np.empty((M, N, G), dtype=np.int64)
    for g in range(G):
        sl = slice(g * group_size, (g + 1) * group_size)
        wg = c[:, sl] - z[g][:, None]          # [N, 128]
        P[:, :, g] = np.rint(xq[:, sl] @ wg.T).astype(np.int64)
    return P


def w4a8_linear(xq, xscale, codes, zeros_gn, scales_gn, bias=None,
                group_size=GROUP, variant="fp16"):
    """y[m,n] = xscale[m] * sum_g s[g,n] * P[m,n,g] (+ bias), float64.

    variant "fp16": the checkpoint's fp16 group scales (the build's
    semantics).  variant "marlin": the scales as Marlin consumes them after
    marlin_act_int8_process_scales (int16 codes times a global factor folded
    into the activation scale; vllm/.../marlin_utils.py:326-330, 605-611),
    applied only when G > 1 (paroquant_marlin_w4a8.py:296-302).
    """
    P = group_partials(xq, codes, zeros_gn, group_size).astype(np.float64)
    M, N, G = P.shape
    s = np.asarray(scales_gn)[:G, :N]
    a = np.asarray(xscale, dtype=np.float32).astype(np.float64).reshape(M, 1)
    if variant == "marlin" and G > 1:
        s_i16, glob = marlin_act_int8_process_scales(s)
        a = (np.asarray(xscale, np.float32) * glob).astype(np.float32).astype(np.float64).reshape(M, 1)
        sf = s_i16.astype(np.float64)
    else:
        sf = s.astype(np.float32).astype(np.float64)
    y = np.einsum("mng,gn->mn", P, sf) * a
    if bias is not None:
        y = y + np.asarray(bias, dtype=np.float32).astype(np.float64)[None, :]
    return y


def rmsnorm(x, weight, eps=1e-6):
    """Qwen3VLTextRMSNorm, src/alpamayo_r1/models/qwen3_vl/modeling_qwen3_vl.py
    :340-357: float32 math, normalised value cast to the input dtype (bf16)
    before the weight multiply (weight bf16; product rounded to bf16)."""
    x32 = f32(x)
    var = (x32.astype(np.float32) ** 2).mean(axis=-1, keepdims=True, dtype=np.float32)
    h = x32 * (1.0 / np.sqrt(var + np.float32(eps))).astype(np.float32)
    h = round_to_bf16(h)
    return round_to_bf16(f32(weight) * h)


def silu_mul(x, eps_unused=None):
    """act_fn(gate_proj(x)) * up_proj(x) of the decoder MLP on a fused
    gate_up output [..., 2I] (gate first): SiLU in float32 rounded to bf16,
    times up, rounded to bf16 (bf16 torch semantics)."""
    x32 = f32(x)
    I = x32.shape[-1] // 2
    g, u = x32[..., :I], x32[..., I:]
    s = round_to_bf16(g / (np.float32(1.0) + np.exp(-g, dtype=np.float32)))
    return round_to_bf16(s * u)


def add_rmsnorm(x, residual, weight, eps=1e-6):
    """Residual add in bf16 (s = bf16(x + residual)) followed by rmsnorm;
    returns (normalised, s)."""
    s = round_to_bf16(f32(x) + f32(residual)) if residual is not None else round_to_bf16(x)
    return rmsnorm(s, weight, eps), s


def rot_quant_reference(x, pairs, theta, channel_scales, group_size=GROUP,
                        fp16_intermediate=True):
    """The reference activation chain of one W4A8 linear: x (already fp16
    representable) -> rotate (float32) -> fp16 store (rotation.cuh:333-334)
    -> per-token int8 (int8_utils.py:106-128).  Returns (q, scale, rotated)."""
    r = rotate_activations(x, pairs, theta, channel_scales, group_size)
    if fp16_intermediate:
        r = round_to_fp16(r)
    q, s = per_token_quant_int8(r)
    return q, s, r


def fake_quant_linear(x, pairs, theta, channel_scales, w_dq, group_size=GROUP):
    """The reference's PyTorch CPU fake-quant pipeline used as the CPU
    baseline: x*s -> Givens layers -> per-token int8 quant/dequant -> fp32
    matmul with the dequantised int4 weight -> bf16."""
    r = rotate_activations(x, pairs, theta, channel_scales, group_size)
    q, s = per_token_quant_int8(r)
    xdq = q.astype(np.float32) * s[:, None]
    y = xdq @ f32(w_dq).T
    return round_to_bf16(y)
