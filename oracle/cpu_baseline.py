"""CPU port of the reference's PyTorch fake-quant path, used ONLY as the
timed CPU baseline (bench.py ``cpu_baseline`` leg and ``--impl reference``).

TEST / BASELINE INFRASTRUCTURE: never imported by the product package.

The pipeline restates, with torch CPU tensors and all host threads:
  x * channel_scales                      rotation_utils.py:58-63 (multiply side)
  8 x apply_rotation_step                 src/alpamayo_r1/utils/quantization/rotation_utils.py:8-29
  per-token int8 quantise / dequantise    vllm/.../int8_utils.py:106-128
  x_dq @ W_dq.T in float32                W_dq = dequant_awq (paroquant_marlin_w4a8.py:227-235)
  cast to bfloat16
The reference's own Python cannot travel to the GPU host, so this port is
what runs there (``kind: "port"``).
"""
from __future__ import annotations

import math
import os
import time

import torch

GROUP = 128
KROT = 8


def apply_rotation_step(t, idx_ij, theta, group_size=GROUP):
    n_groups = t.size(-1) // group_size
    half = group_size // 2
    s = torch.sin(theta).view(n_groups, half)
    c = torch.cos(theta).view(n_groups, half)
    idx = idx_ij.to(torch.int64).view(n_groups, group_size)
    starts = (torch.arange(n_groups) * group_size).unsqueeze(1)
    di = (idx[:, 0::2] + starts).reshape(-1)
    dj = (idx[:, 1::2] + starts).reshape(-1)
    cg = c.reshape(1, -1)
    sg = s.reshape(1, -1)
    a = t[:, di]
    b = t[:, dj]
    out = t.clone()
    out[:, di] = cg * a + sg * b
    out[:, dj] = -sg * a + cg * b
    return out


def per_token_quant_dequant(x):
    absmax = x.abs().amax(dim=-1, keepdim=True).clamp_min(1e-10)
    scale = absmax / 127.0
    v = x * (127.0 / absmax)
    q = torch.sign(v) * torch.floor(v.abs() + 0.5)
    return q * scale


def fake_quant_linear(x, pairs, theta, channel_scales, w_dq):
    t = x * channel_scales
    for r in range(pairs.shape[0]):
        t = apply_rotation_step(t, pairs[r], theta[r])
    y = per_token_quant_dequant(t) @ w_dq.t()
    return y.to(torch.bfloat16)


def make_case(N, K, M, seed):
    """Seeded synthetic layer (same recipe as the GPU bench, dequantised int4
    weights held as float32) and activations."""
    g = torch.Generator().manual_seed(seed)
    G = K // GROUP
    pairs = torch.stack([torch.cat([torch.randperm(GROUP, generator=g) for _ in range(G)]) for _ in range(KROT)])
    theta = (torch.rand(KROT, K // 2, generator=g) * 2 - 1) * math.pi
    theta = theta.to(torch.float16).float()
    cs = (0.5 + 1.5 * torch.rand(1, K, generator=g)).to(torch.float16).float()
    codes = torch.randint(0, 16, (N, K), generator=g, dtype=torch.uint8)
    s = (0.004 + 0.006 * torch.rand(G, N, generator=g)).to(torch.float16).float()
    z = torch.randint(0, 16, (G, N), generator=g).float()
    w_dq = (codes.float().view(N, G, GROUP) - z.t().unsqueeze(-1)) * s.t().unsqueeze(-1)
    x = torch.randn(M, K, generator=g)
    ch = torch.randperm(K, generator=g)[: max(1, K // 100)]
    x[:, ch] *= 20.0
    return dict(x=x, pairs=pairs, theta=theta, cs=cs, w_dq=w_dq.reshape(N, K).contiguous())


def time_cases(cases, budget_s=10.0, min_reps=1):
    """Run the fake-quant linear over ``cases`` repeatedly for about
    ``budget_s`` seconds; returns (calls, seconds, threads)."""
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    for c in cases:  # warm-up
        fake_quant_linear(c["x"], c["pairs"], c["theta"], c["cs"], c["w_dq"])
    calls, t0 = 0, time.perf_counter()
    reps = 0
    while True:
        for c in cases:
            fake_quant_linear(c["x"], c["pairs"], c["theta"], c["cs"], c["w_dq"])
            calls += 1
        reps += 1
        el = time.perf_counter() - t0
        if reps >= min_reps and el >= budget_s:
            break
    return calls, time.perf_counter() - t0, threads
