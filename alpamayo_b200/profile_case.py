"""Run one W4A8 linear case a few times, for profilers.

    python -m alpamayo_b200.profile_case --shape gate_up --M 8 --iters 4

Builds one seeded synthetic layer of the named projection shape (the
7B-class decoder shapes the benchmark uses), then runs the fused activation
kernel and the GEMM ``--iters`` times on the current GPU and prints the
CUDA-event time of the last pair.  M <= 64 runs the streaming decode GEMM
(except gate_up above 24 tokens), larger M the tcgen05 kernel.  Meant to be launched under ``ncu -k <kernel>``
with a small launch count; it holds at most a few hundred MB on the device.
"""
from __future__ import annotations

import argparse

import torch

SHAPES = {"qkv": (4608, 3584), "o_proj": (3584, 3584), "gate_up": (37888, 3584), "down": (3584, 18944)}


def main() -> int:
    p = argparse.ArgumentParser()
    p.add_argument("--shape", choices=sorted(SHAPES), default="gate_up")
    p.add_argument("--M", type=int, default=8)
    p.add_argument("--iters", type=int, default=4)
    p.add_argument("--linear", action="store_true", help="run torch.ops.paro_b200.linear_w4a8 (the op's own route)")
    a = p.parse_args()

    import alpamayo_b200.ops as ops
    from alpamayo_b200 import _native
    from alpamayo_b200 import synthetic as syn

    N, K = SHAPES[a.shape]
    L = syn.make_layer(N, K, seed=1, checkpoint=False)
    x = syn.make_activations(a.M, K, seed=2)
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    for _ in range(a.iters):
        ev[0].record()
        if a.linear:
            ops.linear_w4a8(x, L["rot_table"], L["cs_vec"], L["packed"], N, None, True, torch.bfloat16)
            ev[1].record()
        else:
            q, s = ops.rotq_int8(x, L["rot_table"], L["cs_vec"], 128, True)
            ev[1].record()
            ops.w4a8_gemm(q, s, L["packed"], N, None, torch.bfloat16)
        ev[2].record()
    torch.cuda.synchronize()
    err = _native.capi().paro_device_error_word(1)
    print(f"{a.shape} M={a.M}: activation {ev[0].elapsed_time(ev[1]) * 1e3:.1f} us, "
          f"gemm {ev[1].elapsed_time(ev[2]) * 1e3:.1f} us, device error word {err}")
    return 1 if err else 0


if __name__ == "__main__":
    raise SystemExit(main())
