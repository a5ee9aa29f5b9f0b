"""Generate the golden fixtures for the W4A8 rotated-linear path by running
the REFERENCE's own Python functions (imported from a checkout of the
reference project) on seeded synthetic inputs.

Usage:  python tests/golden/gen_golden.py <reference-project-root>

It needs the reference sources and vLLM (for its CPU-only scale helper); it
runs on CPU only.  The fixtures it writes (``*.npz`` beside this file) are
committed; tests never need the reference itself.

Functions called from the reference (paths relative to its root):
  src/alpamayo_r1/utils/quantization/rotation_linear.py:78-118 RotateLinearInt4.from_linear
      (rotate_weight=True, init_only=False: rotate_tensor -> quantizer ->
      pseudo_quantize_tensor -> WQLinear.from_linear); the reference moves
      tensors to CUDA there (rotation_utils.py:49,83), so while it runs
      Tensor.cuda / Module.cuda are no-ops and everything stays on the CPU
  src/alpamayo_r1/utils/quantization/rotation_utils.py:8-29   apply_rotation_step
  src/alpamayo_r1/utils/quantization/quantization_utils.py:18-73 pseudo_quantize_tensor
  src/alpamayo_r1/utils/quantization/qmodule.py:39-78,149-205  pack_intweight, WQLinear.from_linear
  src/alpamayo_r1/utils/quantization/paroquant_marlin_w4a8.py:95-142,152-164,179-235
      unpack_wqlinear_qweight, pack_awq_int32, wqlinear_to_awq, dequant_wqlinear, dequant_awq
  vllm/model_executor/layers/quantization/utils/marlin_utils.py:326-330
      marlin_act_int8_process_scales
"""
from __future__ import annotations

import importlib.util
import math
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
GROUP = 128
KROT = 8


def import_reference(root):
    qdir = os.path.join(root, "src", "alpamayo_r1", "utils", "quantization")
    spec = importlib.util.spec_from_loader("refq", loader=None, is_package=True)
    pkg = importlib.util.module_from_spec(spec)
    pkg.__path__ = [qdir]
    sys.modules["refq"] = pkg
    import refq.rotation_utils as ru
    import refq.quantization_utils as qu
    import refq.qmodule as qm
    import refq.rotation_linear as rl
    # The Marlin adapter imports its module classes from the absent
    # ParoQuant ``inference_engine`` package; point those names at the
    # reference's own local copies.
    for name in ("inference_engine", "inference_engine.model_executor",
                 "inference_engine.model_executor.modules"):
        sys.modules.setdefault(name, types.ModuleType(name))
    sys.modules["inference_engine.model_executor.modules.rotation_linear"] = rl
    sys.modules["inference_engine.model_executor.modules.qmodule"] = qm
    import refq.paroquant_marlin_w4a8 as pm
    from vllm.model_executor.layers.quantization.utils import marlin_utils as mu
    return ru, qu, qm, rl, pm, mu


def gen(seed):
    return torch.Generator().manual_seed(seed)


def make_rotation(K, seed):
    """pairs: per layer and group a randperm(128) (consecutive entries form
    the 64 disjoint pairs); theta ~ U(-pi, pi) stored fp16; channel scales
    ~ U(0.5, 2) fp16."""
    G = K // GROUP
    g = gen(seed)
    pairs = torch.stack([
        torch.cat([torch.randperm(GROUP, generator=g) for _ in range(G)])
        for _ in range(KROT)]).to(torch.int16)
    theta = ((torch.rand(KROT, K // 2, generator=g) * 2 - 1) * math.pi).to(torch.float16)
    cs = (0.5 + 1.5 * torch.rand(1, K, generator=g)).to(torch.float16)
    return pairs, theta, cs


def make_activations(M, K, seed):
    """x ~ N(0,1) fp32 with a seeded 1% of channels multiplied by 20."""
    g = gen(seed)
    x = torch.randn(M, K, generator=g)
    n_out = max(1, K // 100)
    ch = torch.randperm(K, generator=g)[:n_out]
    x[:, ch] *= 20.0
    return x


def ref_rotate(ru, t, pairs, theta, cs, divide):
    t = t.float()
    t = t / cs.float() if divide else t * cs.float()
    for r in range(KROT):
        t = ru.apply_rotation_step(t, pairs[r].to(torch.int32), theta[r].float(), GROUP)
    return t


def sha256(a):
    import hashlib
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def reference_from_linear(rl, qm, W, pairs, theta, cs, bias=None):
    """The reference's offline path, RotateLinearInt4.from_linear(linear,
    theta, pairs, cs, rotate_weight=True, init_only=False), on the CPU; also
    returns the raw int codes its WQLinear.from_linear hands to
    pack_intweight (before any packing, so out-of-range codes are seen)."""
    N, K = W.shape
    lin = torch.nn.Linear(K, N, bias=bias is not None)
    with torch.no_grad():
        lin.weight.copy_(W)
        if bias is not None:
            lin.bias.copy_(bias)
    seen = {}
    orig_pack = qm.pack_intweight

    def recording_pack(intweight, *a, **k):
        seen["codes"] = intweight.clone()
        return orig_pack(intweight, *a, **k)

    saved = (torch.Tensor.cuda, torch.nn.Module.cuda)
    torch.Tensor.cuda = lambda self, *a, **k: self
    torch.nn.Module.cuda = lambda self, *a, **k: self
    qm.pack_intweight = recording_pack
    try:
        m = rl.RotateLinearInt4.from_linear(lin, theta, pairs, cs, rotate_weight=True, init_only=False)
    finally:
        torch.Tensor.cuda, torch.nn.Module.cuda = saved
        qm.pack_intweight = orig_pack
    q = m.qlinear
    return q.qweight.clone(), q.scales.clone(), q.scaled_zeros.clone(), seen["codes"].to(torch.int32)


def per_token_int8(v):
    """vLLM per_token_quant_int8 (int8_utils.py:106-128), restated: absmax
    clamped at 1e-10, scale absmax / 127, codes round-half-away of
    v * (127 / absmax)."""
    absmax = v.abs().amax(dim=-1, keepdim=True).clamp_min(1e-10)
    t = v * (127.0 / absmax)
    q = torch.sign(t) * torch.floor(t.abs() + 0.5)
    return q.clamp(-127, 127), absmax / 127.0


def main(root):
    ru, qu, qm, rl, pm, mu = import_reference(root)
    torch.set_num_threads(max(1, os.cpu_count() or 1))

    # ---- the reference's offline from_linear on a small layer --------------
    N, K = 128, 1024
    pairs, theta, cs = make_rotation(K, 41)
    W = torch.randn(N, K, generator=gen(42)) * 0.02
    qweight, scales, szeros, raw = reference_from_linear(rl, qm, W, pairs, theta, cs)
    np.savez_compressed(os.path.join(HERE, f"fromlinear_n{N}_k{K}.npz"), W=W.numpy(), pairs=pairs.numpy(),
                        theta=theta.numpy(), channel_scales=cs.numpy(), qweight=qweight.numpy(),
                        scales=scales.numpy(), scaled_zeros=szeros.numpy(), raw_codes=raw.numpy().astype(np.int8))

    # ---- M=16, K=N=3584, fp32 activations ----------------------
    # weights through the reference's from_linear; the activation half and
    # the fake-quant matmul of the reference's CPU path: x * s, 8 x
    # apply_rotation_step, per-token int8 quantise / dequantise, x_dq @ W_dq^T
    # with W_dq = dequant_wqlinear of the WQLinear buffers, output bf16
    N = K = 3584
    M = 16
    pairs, theta, cs = make_rotation(K, 31)
    W = torch.randn(N, K, generator=gen(32)) * 0.02
    qweight, scales, szeros, raw = reference_from_linear(rl, qm, W, pairs, theta, cs)
    codes = raw.clamp(0, 15)
    x = make_activations(M, K, 33)
    rot_x = ref_rotate(ru, x, pairs, theta, cs, divide=False)
    xq, xs = per_token_int8(rot_x)
    w_dq = pm.dequant_wqlinear(codes, scales, szeros, GROUP)
    y = (xq * xs) @ w_dq.t()
    np.savez_compressed(
        os.path.join(HERE, "cfg0_m16_k3584.npz"),
        W_sha256=sha256(W.numpy()), pairs=pairs.numpy(), theta=theta.numpy(), channel_scales=cs.numpy(),
        qweight_sha256=sha256(qweight.numpy()), codes_sha256=sha256(codes.numpy().astype(np.uint8)),
        out_of_range_codes=np.int64(((raw < 0) | (raw > 15)).sum().item()),
        scales=scales.numpy(), scaled_zeros=szeros.numpy(), x=x.numpy(), x_rotated=rot_x.numpy(),
        xq=xq.numpy().astype(np.int8), xscale=xs.numpy().reshape(-1), y=y.numpy(),
        y_bf16=y.to(torch.bfloat16).float().numpy())

    # ---- rotation fixtures (activation side) ------------------------------
    for (M, K, seed) in [(16, 1024, 11), (4, 3584, 12)]:
        pairs, theta, cs = make_rotation(K, seed)
        x = make_activations(M, K, seed + 100)
        rot = ref_rotate(ru, x, pairs, theta, cs, divide=False)
        # inverse check trick of interface.py:43-52: rotating back by -theta
        # in reverse layer order restores x*s
        back = rot.clone()
        for r in reversed(range(KROT)):
            back = ru.apply_rotation_step(back, pairs[r].to(torch.int32), -theta[r].float(), GROUP)
        np.savez_compressed(
            os.path.join(HERE, f"rot_m{M}_k{K}.npz"),
            x=x.numpy(), pairs=pairs.numpy(), theta=theta.numpy(),
            channel_scales=cs.numpy(), rotated=rot.numpy(),
            unrotated=back.numpy())

    # ---- weight fixtures ---------------------------------------------------
    N, K, M = 128, 1024, 16
    G = K // GROUP
    pairs, theta, cs = make_rotation(K, 21)
    W = torch.randn(N, K, generator=gen(22)) * 0.02
    w_rot = ref_rotate(ru, W, pairs, theta, cs, divide=True)
    w_dq, s_ng, z_ng = qu.pseudo_quantize_tensor(
        w_rot.clone(), n_bit=4, q_group_size=GROUP, get_scale_zp=True)
    s16 = s_ng.to(torch.float16)
    # fake-quant weight on the fp16 scale grid so that WQLinear.from_linear
    # recovers exactly the clamped codes
    wg = w_rot.reshape(-1, GROUP)
    codes = torch.clamp(torch.round(wg / s_ng.reshape(-1, 1)) + z_ng.reshape(-1, 1), 0, 15)
    codes = codes.reshape(N, K).to(torch.int32)
    w_grid = ((codes.float().reshape(-1, GROUP) - z_ng.reshape(-1, 1))
              * s16.float().reshape(-1, 1)).reshape(N, K)
    lin = torch.nn.Linear(K, N, bias=True)
    with torch.no_grad():
        lin.weight.copy_(w_grid)
        lin.bias.copy_((torch.randn(N, generator=gen(23)) * 0.1))
    wq = qm.WQLinear.from_linear(lin, 4, GROUP, False, s16, z_ng.to(torch.float16))
    qweight = wq.qweight.clone()
    unpacked = pm.unpack_wqlinear_qweight(qweight, N, K)
    assert torch.equal(unpacked, codes), "pack/unpack round trip must be exact"
    awq = pm.wqlinear_to_awq(qweight, wq.scales, wq.scaled_zeros, N, K, GROUP)
    deq_wq = pm.dequant_wqlinear(unpacked, wq.scales, wq.scaled_zeros, GROUP)
    deq_awq = pm.dequant_awq(unpacked, awq.zeros, awq.scales, GROUP)
    s_i16, glob = mu.marlin_act_int8_process_scales(awq.scales.clone())
    x = make_activations(M, K, 24)
    rot_x = ref_rotate(ru, x, pairs, theta, cs, divide=False)
    np.savez_compressed(
        os.path.join(HERE, f"wq_n{N}_k{K}.npz"),
        W=W.numpy(), pairs=pairs.numpy(), theta=theta.numpy(),
        channel_scales=cs.numpy(), w_rot=w_rot.numpy(), w_dq=w_dq.numpy(),
        pq_scales=s_ng.numpy(), pq_zeros=z_ng.numpy(), codes=codes.numpy(),
        qweight=qweight.numpy(), wq_scales=wq.scales.numpy(),
        wq_scaled_zeros=wq.scaled_zeros.numpy(), bias=wq.bias.detach().numpy(),
        unpacked=unpacked.numpy(), awq_qweight=awq.qweight.numpy(),
        awq_qzeros=awq.qzeros.numpy(), awq_zeros=awq.zeros.numpy(),
        awq_scales=awq.scales.numpy(), dequant_wqlinear=deq_wq[:32].numpy(),
        dequant_awq=deq_awq[:32].numpy(),
        marlin_s_i16=s_i16.view(torch.int16).numpy(),
        marlin_global=np.float32(glob.item()),
        x=x.numpy(), x_rotated=rot_x.numpy())
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit(__doc__)
    main(sys.argv[1])
