#!/usr/bin/env python
"""Benchmark of the B200 W4A8 rotated-linear path (one JSON line on rank 0).

Headline workload ("decode sweep"): the four
projection shapes of one 7B-class decoder layer (qkv 3584->4608, o 3584->3584,
gate_up 3584->37888, down 18944->3584) at M = 1, 4 and 8 tokens; each linear
runs through torch.ops.paro_b200.linear_w4a8: the activation (channel
scale, 8 Givens layers, per-token int8) and the persistent W4A8 GEMM,
chained by programmatic dependent launch (at these sizes the activation is
a rotation kernel and a quantiser, so three kernels per linear).  One step
= STEP_SWEEPS passes over the 12 (shape, M) cases.  Three
weight replicas (one per M) make the per-pass weight working set 363 MB
(> 126 MB L2), so every GEMM streams its weights from HBM.  The metric value
is weight-stream GB/s (algorithmic int4 code + fp16 scale + int4 zero bytes
per second), whole job.

Timing: CUDA graph of one step, replayed; CUDA events around the timed
replays, barrier + synchronize on both sides, max over ranks.  Roofline of
the dominant kernel (the decode GEMM): its average launch duration over the
step's own 192 GEMM launches (16 sweeps x 12 cases on the same three weight
replicas, working set > L2), replayed back to back as a CUDA graph of the
int8-input paro_w4a8_gemm and timed with CUDA events on the launching
stream.  Beside it, each case's single launch after an L2 flush (a 512 MiB
write, then a 256 MiB read so that the lines left in the L2 are clean and
the timed kernel pays for no write-backs), which adds a cold launch's fixed
start-up to every figure.

reference_gpu: the reference's own GPU path on the same B200 (its rotate
kernel compiled from its source, vLLM's per-token int8 quantiser and Marlin
W4A8 GEMM, bf16 <-> fp16 casts), timed the same way on the same cases.

Prefill (configs[2], the "prefill" object): the same four projections at
M = 2048, 4096, 8192 through the tcgen05 GEMM, TOPS against the dense int8
peak measured in the same run (torch._int_mm on 8192^3), plus the
activation kernel's share of each linear's time.

--impl reference: the reference's CPU fake-quant path (oracle/cpu_baseline.py,
a port, since the reference's own Python cannot run here) on the host cores,
same metric.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

SHAPES = [("qkv", 4608, 3584), ("o_proj", 3584, 3584), ("gate_up", 37888, 3584), ("down", 3584, 18944)]
DECODE_M = [1, 4, 8]
STEP_SWEEPS = 16
L2_BYTES = 126 * 2 ** 20
METRIC = "W4A8 rot-GEMM decode weight GB/s & prefill int8 TOPS vs roofline, 1-8 B200"


def args_():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-prefill", action="store_true")
    p.add_argument("--no-stack", action="store_true")
    p.add_argument("--no-sharded", action="store_true")
    p.add_argument("--no-verify", action="store_true", help="skip the DFlash verify / decode-loop section")
    p.add_argument("--no-reference-gpu", action="store_true",
                   help="skip timing the reference's own GPU path (its rotate kernel + vLLM Marlin)")
    p.add_argument("--case", default=None, metavar="SHAPE:M",
                   help="profiling mode: run one case (e.g. gate_up:8) --case-iters times and exit")
    p.add_argument("--case-iters", type=int, default=4)
    p.add_argument("--case-linear", action="store_true",
                   help="with --case: run the whole linear op (linear_w4a8) instead of activation kernel + GEMM")
    return p.parse_args()


def weight_bytes(N, K):
    G = K // 128
    return N * K // 2 + G * N * 2 + G * N // 2


def gemm_alg_bytes(M, N, K):
    """Algorithmic bytes of one decode GEMM launch: weights + int8 activations
    + fp32 token scales + bf16 output."""
    return weight_bytes(N, K) + M * K + 4 * M + 2 * M * N


def linear_alg_bytes(M, N, K):
    """Algorithmic bytes of one fused decode linear: int4 weights + fp16
    scales + int4 zeros, bf16 activations, the reference's rotation tables,
    bf16 output."""
    L = 8
    return weight_bytes(N, K) + 2 * M * K + 2 * L * K + L * K + 2 * K + 2 * M * N


def act_alg_bytes(M, K):
    """Activation kernel: bf16 in, int8 + fp32 scale out, and the reference's
    rotation tables (int16 pairs, fp16 angles, fp16 channel scales)."""
    L = 8
    return 2 * M * K + M * K + 4 * M + 2 * L * K + L * K + 2 * K


FLUSH_BYTES = 512 * 2 ** 20
CLEAN_BYTES = 256 * 2 ** 20


class L2Flush:
    """Evicts the L2 between timed launches: a 512 MiB write (larger than the
    126 MiB L2), then a 256 MiB read of another buffer, so that the L2 ends
    up holding clean lines of neither the inputs nor the outputs and the
    timed kernel's misses cause no write-backs of the flush's dirty lines."""

    def __init__(self, torch, dev):
        self.w = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
        self.r = torch.zeros(CLEAN_BYTES // 4, dtype=torch.float32, device=dev)
        self.o = torch.empty((), dtype=torch.float32, device=dev)
        self.torch = torch

    def __call__(self):
        self.w.zero_()
        self.torch.sum(self.r, dim=0, out=self.o)
PAIR_REPS = 5
PREFILL_M = [2048, 4096, 8192]


def kernel_pair_times(torch, flush, act_fn, gemm_fn, reps):
    """Device time of the activation kernel and of the GEMM that consumes its
    output, each bracketed by CUDA events on the current stream, with the L2
    flushed (L2Flush) before every pair."""
    ta, tg = [], []
    gemm_fn(act_fn())   # untimed: first launches load the kernels
    for _ in range(reps):
        flush()
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record()
        q = act_fn()
        e1.record()
        gemm_fn(q)
        e2.record()
        torch.cuda.synchronize()
        ta.append(e0.elapsed_time(e1) * 1e-3)
        tg.append(e1.elapsed_time(e2) * 1e-3)
    return ta, tg


def kernel_times(torch, flush, fn, reps):
    """Device time of one launch of fn, with the L2 flushed (L2Flush) before
    every launch, CUDA events on the current stream."""
    ts = []
    fn()   # untimed: first launches load the kernels
    for _ in range(reps):
        flush()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1) * 1e-3)
    return ts


def int8_peak_tops(torch):
    """Dense int8 tensor throughput of this GPU, measured as torch._int_mm
    (cuBLASLt) on 8192^3, best of 5 after warm-up."""
    n = 8192
    a = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda")
    b = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda").t()
    for _ in range(3):
        torch._int_mm(a, b)
    best = None
    for _ in range(5):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch._int_mm(a, b)
        e1.record()
        torch.cuda.synchronize()
        t = e0.elapsed_time(e1) * 1e-3
        best = t if best is None or t < best else best
    del a, b
    return 2 * n ** 3 / best / 1e12


def prefill_section(torch, ops, syn, layers, flush, rank):
    """the four projections at M = 2048, 4096, 8192, activation
    kernel + tcgen05 GEMM per linear, L2 flushed before each pair."""
    peak = int8_peak_tops(torch)
    out, ops_sum, t_sum, act_sum = {}, 0.0, 0.0, 0.0
    for M in PREFILL_M:
        xk = {K: syn.make_activations(M, K, seed=31 * M + K + rank) for K in {3584, 18944}}
        for (name, N, K) in SHAPES:
            L = layers[name]
            ta_l, tg_l = kernel_pair_times(
                torch, flush, lambda: ops.rotq_int8(xk[K], L["rot_table"], L["cs_vec"], 128, True),
                lambda q: ops.w4a8_gemm(q[0], q[1], L["packed"], N, None, torch.bfloat16), 3)
            tg, ta = statistics.median(tg_l), statistics.median(ta_l)
            tops = 2 * M * N * K / tg / 1e12
            ops_sum += 2 * M * N * K
            t_sum += tg
            act_sum += ta
            out[f"{name}_m{M}"] = {"gemm_us": round(tg * 1e6, 1), "tops": round(tops, 1),
                                   "frac": round(tops / peak, 4), "act_us": round(ta * 1e6, 1),
                                   "act_share": round(ta / (ta + tg), 4),
                                   "act_GBps": round(act_alg_bytes(M, K) / ta / 1e9, 1)}
        del xk
    agg = ops_sum / t_sum / 1e12
    return {"workload": "configs[2]: qkv/o/gate_up/down at M=2048,4096,8192, bf16 activations",
            "kernel": "gemm_tc (tcgen05 kind::i8, TMEM accumulators)", "tops": round(agg, 1),
            "int8_peak_tops": round(peak, 1), "peak_kind": "measured in this run: torch._int_mm 8192^3",
            "frac": round(agg / peak, 4), "act_share": round(act_sum / (act_sum + t_sum), 4), "cases": out}


STACK_CLIPS = 64
STACK_LAYERS = 28
SHARD_M, SHARD_N, SHARD_K = 16384, 37888, 3584


def stack_section(torch, world, rank, per_projection=False):
    """28 rotated W4A8 decoder layers at decode, 64 independent
    clips x 1 token split across the ranks (no collective); tokens/s of the
    whole job and weight-stream GB/s per GPU, CUDA-graph timed, max over
    ranks.  per_projection: q / k / v and gate / up with their own rotation
    tables (a real checkpoint's layout), run as projection groups."""
    from alpamayo_b200 import synthetic as syn
    from alpamayo_b200.stack import DecoderStack
    if STACK_CLIPS % world:
        return {"skipped": f"{STACK_CLIPS} clips do not split over {world} ranks"}
    M = STACK_CLIPS // world
    st = DecoderStack(layers=STACK_LAYERS, seed=0, per_projection=per_projection)
    x = syn.make_activations(M, 3584, seed=500 + rank)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        st.forward(x)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        y = st.forward(x)
    for _ in range(3):
        g.replay()
    reps = 10
    barrier_sync(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    barrier_sync(world)
    t = max_over_ranks(e0.elapsed_time(e1) * 1e-3 / reps, world)
    finite = bool(torch.isfinite(y).all().item())
    wb = st.weight_bytes()
    del g, st
    torch.cuda.empty_cache()
    return {"workload": "configs[3]: 28-layer decode stack (RMSNorm -> qkv, identity attention -> o, RMSNorm -> "
                        "gate_up -> SiLU*up -> down), 64 clips x 1 token split over the ranks, no collective"
                        + ("; q/k/v and gate/up with per-projection rotation tables" if per_projection else "")
                        + "; RMSNorm and SiLU*up fused into the following linear's rotation kernel",
            "tokens_per_rank": M, "ms_per_forward": round(t * 1e3, 3),
            "tokens_per_s": round(STACK_CLIPS / t, 1),
            "weight_GBps_per_gpu": round(wb / t / 1e9, 1), "weight_bytes_per_forward": wb,
            "outputs_finite": finite}


VERIFY_M = [8, 16, 48, 96]
LOOP_TOKENS = 32


def verify_section(torch, world, rank):
    """Next consumers of the linear (the scope table's next rows): DFlash's
    verify step runs the target model on a draft block (block_size 8, or 16
    for the b16 draft model: src/alpamayo_r1/utils/dflash/
    dflash_integration.py:144,276), times the trajectory samples (1 or 6);
    the streaming rollout's decode loop replays the language model's CUDA
    graph once per token with a host check of the stop condition in between
    (src/alpamayo_r1/models/alpamayo_r1_unified.py:585-640,1677-1700).  Here
    the 28-layer decode stack stands in for the language model: one forward
    per verify block at M = 8, 16, 48, 96 (graph replays, CUDA events), and a
    32-token loop at M = 1 and 6 with a host synchronisation after every
    replay (host wall clock per token).  Per rank, no collective."""
    from alpamayo_b200 import synthetic as syn
    from alpamayo_b200.stack import DecoderStack
    st = DecoderStack(layers=STACK_LAYERS, seed=0)
    wb = st.weight_bytes()

    def graph_of(x):
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            st.forward(x)
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            y = st.forward(x)
        return g, y

    blocks = {}
    for M in VERIFY_M:
        x = syn.make_activations(M, 3584, seed=600 + M + rank)
        g, _ = graph_of(x)
        for _ in range(3):
            g.replay()
        reps = 5
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        t = e0.elapsed_time(e1) * 1e-3 / reps
        blocks[f"m{M}"] = {"ms_per_forward": round(t * 1e3, 3), "tokens_per_s": round(M / t, 1),
                           "weight_GBps": round(wb / t / 1e9, 1)}
        del g
    loop = {}
    for M in (1, 6):
        x = syn.make_activations(M, 3584, seed=700 + M + rank)
        g, y = graph_of(x)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(LOOP_TOKENS):
            g.replay()
            bool(torch.isfinite(y[0, 0]).item())   # the loop's per-token host check
        el = (time.perf_counter() - t0) / LOOP_TOKENS
        loop[f"m{M}"] = {"ms_per_token": round(el * 1e3, 3), "tokens_per_s": round(M / el, 1),
                         "weight_GBps": round(wb / el / 1e9, 1)}
        del g
    del st
    torch.cuda.empty_cache()
    return {"workload": "28-layer decode stack as the target model: DFlash verify blocks and the per-token "
                        "graph-replay decode loop", "verify_blocks": blocks, "decode_loop": loop}


def sharded_section(torch, world, rank):
    """gate_up (K=3584, N=37888) at M=16384, output columns split
    over the ranks, the bf16 blocks gathered on every rank; end-to-end time,
    the exposed gather time and int8 TOPS of the whole job, max over ranks.
    Four gathers: NCCL all_gather_into_tensor after the linear, the same in
    row blocks overlapped with the linear, copy-engine peer copies
    (cudaMemcpyAsync into every peer's IPC-mapped buffer) overlapped with the
    next row block's GEMM, and none at all: the GEMM's epilogue stores
    through an NVLink multicast address; the headline is the fastest whose
    result equals the NCCL gather."""
    from alpamayo_b200 import synthetic as syn
    from alpamayo_b200.stack import ColumnShardedLinear, column_shard, linear, serving_layer
    c0, c1 = column_shard(SHARD_N, rank, world)
    L = serving_layer(c1 - c0, SHARD_K, seed=700 + rank)
    x = syn.make_activations(SHARD_M, SHARD_K, seed=701)
    csl = ColumnShardedLinear(lambda v: linear(L, v))
    for _ in range(2):
        csl(x)
    reps = 5
    tl, tt = [], []
    for _ in range(reps):
        barrier_sync(world)
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record()
        y = csl.local_fn(x)
        e1.record()
        blocks = csl.gather(y)
        e2.record()
        torch.cuda.synchronize()
        tl.append(e0.elapsed_time(e1) * 1e-3)
        tt.append(e0.elapsed_time(e2) * 1e-3)
    t_lin = max_over_ranks(min(tl), world)
    t_tot = max_over_ranks(min(tt), world)
    # the same with the all-gather overlapped: 4 row blocks, block i gathered
    # while block i + 1 is computed
    CH = 4
    for _ in range(2):
        csl.overlapped(x, CH)
    to = []
    for _ in range(reps):
        barrier_sync(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        ob = csl.overlapped(x, CH)
        e1.record()
        torch.cuda.synchronize()
        to.append(e0.elapsed_time(e1) * 1e-3)
    del ob
    t_ov = max_over_ranks(min(to), world)
    # the gather by copy engines over NVLink into every peer's mapped
    # buffer, overlapped with the GEMM of the next row block
    p2p = {}
    if world > 1:
        from alpamayo_b200.stack import linear_into
        csl2 = ColumnShardedLinear(None, block_columns=c1 - c0)
        into = lambda v, dst: linear_into(L, v.contiguous(), dst)
        try:
            for ch in (4, 8, 16):
                for _ in range(2):
                    csl2.peer_gathered(x, into, ch)
                tp = []
                for _ in range(reps):
                    barrier_sync(world)
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record()
                    csl2.peer_gathered(x, into, ch)
                    e1.record()
                    torch.cuda.synchronize()
                    tp.append(e0.elapsed_time(e1) * 1e-3)
                t_p = max_over_ranks(min(tp), world)
                pg = csl2.peer_gathered(x, into, ch)
                same = torch.tensor([1 if torch.equal(pg, blocks) else 0], dtype=torch.int32, device="cuda")
                torch.distributed.all_reduce(same, op=torch.distributed.ReduceOp.MIN)
                del pg
                p2p[ch] = {"row_blocks": ch, "matches_nccl_gather": bool(same.item()),
                           "ms_end_to_end": round(t_p * 1e3, 3), "ms_exposed_gather": round((t_p - t_lin) * 1e3, 3),
                           "int8_tops_end_to_end": round(2.0 * SHARD_M * SHARD_N * SHARD_K / t_p / 1e12, 1),
                           "_t": t_p}
        except Exception as e:  # peer mappings unavailable: report, keep the NCCL numbers
            p2p = {"unavailable": str(e).splitlines()[0][:200]}
        csl2.close_peer_buffers()
        del csl2
    # the gather done by the GEMM's epilogue: multimem stores through the
    # NVLink multicast address of a symmetric-memory buffer every rank holds
    mcast = None
    if world > 1:
        import alpamayo_b200.ops as ops_
        csl3 = ColumnShardedLinear(None, block_columns=c1 - c0)
        quant = lambda v: ops_.rotq_int8(v, L["rot_table"], L["cs_vec"], 128, True)
        try:
            for _ in range(2):
                csl3.multicast_gathered(x, quant, L["packed"], SHARD_K)
            tm = []
            for _ in range(reps):
                barrier_sync(world)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                csl3.multicast_gathered(x, quant, L["packed"], SHARD_K)
                e1.record()
                torch.cuda.synchronize()
                tm.append(e0.elapsed_time(e1) * 1e-3)
            t_m = max_over_ranks(min(tm), world)
            mg = csl3.multicast_gathered(x, quant, L["packed"], SHARD_K)
            same = torch.tensor([1 if torch.equal(mg, blocks) else 0], dtype=torch.int32, device="cuda")
            torch.distributed.all_reduce(same, op=torch.distributed.ReduceOp.MIN)
            mcast = {"matches_nccl_gather": bool(same.item()), "ms_end_to_end": round(t_m * 1e3, 3),
                     "ms_exposed_gather": round((t_m - t_lin) * 1e3, 3),
                     "int8_tops_end_to_end": round(2.0 * SHARD_M * SHARD_N * SHARD_K / t_m / 1e12, 1), "_t": t_m}
        except Exception as e:  # no multicast on this box: report, keep the other numbers
            mcast = {"unavailable": str(e).splitlines()[0][:200]}
        csl3.close_multicast_buffers()
        del csl3
    ops_total = 2.0 * SHARD_M * SHARD_N * SHARD_K
    shape = list(blocks.shape)
    del L, x, y, blocks
    torch.cuda.empty_cache()
    nccl = {"ms_end_to_end": round(t_tot * 1e3, 3), "ms_exposed_gather": round((t_tot - t_lin) * 1e3, 3),
            "int8_tops_end_to_end": round(ops_total / t_tot / 1e12, 1)}
    nccl_ov = {"row_blocks": CH, "ms_end_to_end": round(t_ov * 1e3, 3),
               "ms_exposed_gather": round((t_ov - t_lin) * 1e3, 3),
               "int8_tops_end_to_end": round(ops_total / t_ov / 1e12, 1)}
    ce = [v for k, v in p2p.items() if k != "unavailable"]
    # the headline is the fastest of every gather measured
    variants = [("NCCL all_gather_into_tensor after the linear", t_tot, nccl),
                (f"NCCL all_gather in {CH} row blocks overlapped with the linear", t_ov, nccl_ov)]
    variants += [(f"copy-engine peer copies in {v['row_blocks']} row blocks overlapped with the next block's GEMM",
                  v["_t"], v) for v in ce]
    for v in ce:
        v.pop("_t")
    if mcast and "_t" in mcast and mcast["matches_nccl_gather"]:
        variants.append(("GEMM epilogue stores through the NVLink multicast address (multimem), no separate gather",
                         mcast.pop("_t"), mcast))
    elif mcast:
        mcast.pop("_t", None)
    name, t_best, head = min(variants, key=lambda z: z[1])
    return {"workload": "configs[4]: gate_up K=3584 N=37888 at M=16384, N split over the ranks, bf16 output "
                        "blocks gathered on every rank", "world": world, "block_columns": c1 - c0,
            "gathered_shape": shape, "gather": name if world > 1 else "none (one rank)",
            "ms_end_to_end": head["ms_end_to_end"], "ms_linear": round(t_lin * 1e3, 3),
            "ms_exposed_gather": head.get("ms_exposed_gather", 0.0),
            "int8_tops_end_to_end": head.get("int8_tops_end_to_end", round(ops_total / t_lin / 1e12, 1)),
            "gather_GBps_per_rank": (round((world - 1) / world * SHARD_M * SHARD_N * 2 /
                                           max(t_best - t_lin, 1e-9) / 1e9, 1) if world > 1 else None),
            "nccl_all_gather": nccl, "nccl_all_gather_overlapped": nccl_ov,
            "copy_engine_gather": (p2p.get("unavailable") and p2p) or ce or None,
            "multicast_epilogue": mcast}


def reference_gpu_section(torch, syn, flush, steps, warmup):
    """The reference's own GPU path on this B200, timed like ours: its rotate
    kernel (compiled from the reference's source by oracle/build_ref.py) and
    vLLM's per-token int8 quantiser + Marlin W4A8 GEMM, called as
    BF16RotateLinearWrapper -> RotateLinearInt4 -> MarlinW4A8Linear do
    (oracle/ref_gpu.py).  Decode sweep: the same 12 (shape, M)
    linears, 16 sweeps per step over three weight replicas, CUDA graph,
    weight-stream GB/s.  Prefill: each shape at M = 2048, 4096,
    8192, one call after an L2 flush, CUDA events, int8 TOPS."""
    from oracle import ref_gpu as R
    rot_ok, marlin_ok, why = R.available()
    if not (rot_ok and marlin_ok):
        return {"unavailable": why}
    reps = []
    for ri, M in enumerate(DECODE_M):
        layer = {}
        for si, (name, N, K) in enumerate(SHAPES):
            L = syn.make_layer(N, K, seed=5000 + 100 * ri + si, checkpoint=False, keep_awq=True)
            layer[name] = R.ReferenceLinear(L["pairs"], L["theta"], L["channel_scales"], L["awq_qweight"],
                                            L["awq_scales"], L["awq_qzeros"], K, N)
            del L
        reps.append(layer)
    xs = {(M, K): syn.make_activations(M, K, seed=7 * M + K) for M in DECODE_M for K in {3584, 18944}}

    def step():
        for _ in range(STEP_SWEEPS):
            for ri, M in enumerate(DECODE_M):
                for (name, N, K) in SHAPES:
                    reps[ri][name](xs[(M, K)])

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream().wait_stream(s)
    mode = "CUDA graph of one step"
    try:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            step()
        run = g.replay
    except Exception as e:  # the reference's ops not capturable: time eager launches
        g, run, mode = None, step, f"eager launches ({type(e).__name__} under capture)"
    for _ in range(warmup):
        run()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        run()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    wset = sum(weight_bytes(N, K) for (_, N, K) in SHAPES) * len(DECODE_M)
    dec = {"weight_GBps": round(STEP_SWEEPS * wset / (ms * 1e-3) / 1e9, 1), "ms_per_step": round(ms, 4),
           "timing": mode}
    cases = {}
    for (name, N, K) in SHAPES:
        lin = reps[0][name]
        for M in (1, 8):
            x = xs[(M, K)]
            ts = kernel_times(torch, flush, lambda: lin(x), PAIR_REPS)
            cases[f"{name}_m{M}"] = {"linear_us": round(1e6 * statistics.median(ts), 2)}
    del g, reps
    torch.cuda.empty_cache()
    pre, ops_sum, t_sum = {}, 0.0, 0.0
    for (name, N, K) in SHAPES:
        L = syn.make_layer(N, K, seed=6000 + N, checkpoint=False, keep_awq=True)
        lin = R.ReferenceLinear(L["pairs"], L["theta"], L["channel_scales"], L["awq_qweight"], L["awq_scales"],
                                L["awq_qzeros"], K, N)
        del L
        for M in PREFILL_M:
            x = syn.make_activations(M, K, seed=M + K)
            t = statistics.median(kernel_times(torch, flush, lambda: lin(x), 3))
            ops_sum += 2 * M * N * K
            t_sum += t
            pre[f"{name}_m{M}"] = {"linear_us": round(t * 1e6, 1), "tops": round(2 * M * N * K / t / 1e12, 1)}
            del x
        del lin
        torch.cuda.empty_cache()
    return {"path": "reference rotate kernel (sm_100a build of kernels/paroquant_kernels/src/rotation.cu) + "
                    "vLLM per_token_quant_int8 + marlin_gemm (uint4 x int8), bf16 <-> fp16 casts",
            "decode_sweep": dec, "decode_cases": cases,
            "prefill": {"tops": round(ops_sum / t_sum / 1e12, 1), "cases": pre,
                        "timing": "one whole linear per call after an L2 flush, CUDA events, median of 3"}}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profile_traffic(name):
    """dram bytes per launch recorded from an ncu capture (profiles/*.md line
    'traffic_bytes_per_launch: <n>'), or None."""
    p = os.path.join(ROOT, "profiles", name)
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.strip().startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


class Clocks:
    """nvidia-smi clock / throttle-reason sampling while the timed region runs."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_uuid=None):
        self.uuid = device_uuid
        self.proc = None
        self.f = None

    def start(self):
        try:
            self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            cmd = ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits", "-lms", "20"]
            if self.uuid:
                cmd += ["-i", self.uuid]
            self.proc = subprocess.Popen(cmd, stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.flush()
        rows = [l.split(",") for l in open(self.f.name).read().strip().splitlines() if l.count(",") >= 8]
        os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def dist_setup(n):
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier_sync(world):
    import torch
    import torch.distributed as dist
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(v, world):
    import torch
    import torch.distributed as dist
    if world == 1:
        return v
    t = torch.tensor([v], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def cpu_baseline_sample(budget_s=10.0):
    """The reference's CPU fake-quant path on config 0 (M=16, K=N=3584)."""
    from oracle.cpu_baseline import make_case, time_cases
    case = make_case(3584, 3584, 16, seed=0)
    calls, sec, threads = time_cases([case], budget_s=budget_s)
    gbs = calls * weight_bytes(3584, 3584) / sec / 1e9
    return {"value": gbs, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"config 0 (M=16, K=N=3584) fake-quant linear x{calls} in {sec:.1f} s, torch CPU, "
                      f"{threads} threads"}


def run_reference(a):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import torch
    from oracle.cpu_baseline import make_case, time_cases
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cases = {(name, M): make_case(N, K, M, seed=i * 10 + M)
             for i, (name, N, K) in enumerate(SHAPES) for M in DECODE_M}
    keys = list(cases)

    def step(i):
        # bounded sample: one M value's four shapes per step, cycling M
        M = DECODE_M[i % len(DECODE_M)]
        sel = [cases[k] for k in keys if k[1] == M]
        t0 = time.perf_counter()
        from oracle.cpu_baseline import fake_quant_linear
        for c in sel:
            fake_quant_linear(c["x"], c["pairs"], c["theta"], c["cs"], c["w_dq"])
        return time.perf_counter() - t0, sum(weight_bytes(N, K) for (_, N, K) in SHAPES)

    for i in range(a.warmup):
        step(i)
    tot_t, tot_b = 0.0, 0
    for i in range(a.steps):
        t, b = step(i)
        tot_t += t
        tot_b += b
    val = tot_b / tot_t / 1e9
    line = {"metric": METRIC, "value": val, "unit": "GB/s", "impl": "reference", "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": 1e3 * tot_t / a.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "decode sweep (configs[1]): qkv/o/gate_up/down x M in {1,4,8}; one M per step",
                       "parallelism": "cpu"},
            "cpu_baseline": {"value": val, "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": "per step the four shapes at one M (cycling 1, 4, 8), torch CPU fake-quant"},
            "e2e": {"value": val, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def run_case(a):
    """Profiling mode (--case SHAPE:M): one seeded synthetic layer of the
    named projection shape, then the activation kernel and the GEMM (or,
    with --case-linear, the whole linear op) --case-iters times on the
    current GPU; prints the CUDA-event time of the last iteration and the
    device error word.  Meant to be launched under ``ncu -k <kernel>`` with a
    small launch count: it holds at most a few hundred MB on the device."""
    import torch
    import alpamayo_b200.ops as ops
    from alpamayo_b200 import _native
    from alpamayo_b200 import synthetic as syn
    shape, m = a.case.split(":")
    N, K = {name: (n, k) for (name, n, k) in SHAPES}[shape]
    M = int(m)
    L = syn.make_layer(N, K, seed=1, checkpoint=False)
    x = syn.make_activations(M, K, seed=2)
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    for _ in range(a.case_iters):
        ev[0].record()
        if a.case_linear:
            ops.linear_w4a8(x, L["rot_table"], L["cs_vec"], L["packed"], N, None, True, torch.bfloat16)
            ev[1].record()
        else:
            q, s = ops.rotq_int8(x, L["rot_table"], L["cs_vec"], 128, True)
            ev[1].record()
            ops.w4a8_gemm(q, s, L["packed"], N, None, torch.bfloat16)
        ev[2].record()
    torch.cuda.synchronize()
    err = _native.capi().paro_device_error_word(1)
    print(f"{shape} M={M}: activation {ev[0].elapsed_time(ev[1]) * 1e3:.1f} us, "
          f"gemm {ev[1].elapsed_time(ev[2]) * 1e3:.1f} us, device error word {err}")
    return 1 if err else 0


def main():
    a = args_()
    if a.impl == "reference":
        return run_reference(a)
    if a.case:
        return run_case(a)
    import torch
    world, rank, local = dist_setup(a.gpus)
    import alpamayo_b200.ops as ops
    from alpamayo_b200 import synthetic as syn

    dev = torch.device("cuda", torch.cuda.current_device())
    # --- inputs: three weight replicas (one per M), activations per (M, K)
    reps = []
    for ri, M in enumerate(DECODE_M):
        reps.append({name: syn.make_layer(N, K, seed=1000 * rank + 100 * ri + si, checkpoint=False)
                     for si, (name, N, K) in enumerate(SHAPES)})
    xs = {(M, K): syn.make_activations(M, K, seed=7 * M + K + rank) for M in DECODE_M for K in {3584, 18944}}
    torch.cuda.synchronize()
    wset = sum(weight_bytes(N, K) for (_, N, K) in SHAPES) * len(DECODE_M)

    def linear(L, x, M):
        # the whole rotated linear through the public op: the activation
        # kernel and the decode GEMM chained with programmatic dependent
        # launch
        return ops.linear_w4a8(x, L["rot_table"], L["cs_vec"], L["packed"], L["N"], None, True, torch.bfloat16)

    def sweep():
        for ri, M in enumerate(DECODE_M):
            for (name, N, K) in SHAPES:
                linear(reps[ri][name], xs[(M, K)], M)

    def step():
        for _ in range(STEP_SWEEPS):
            sweep()

    bytes_per_step = STEP_SWEEPS * wset
    # rotation kernel + quantiser + GEMM per linear (every decode shape takes
    # the three-kernel route: all of them stream on the mma.sync kernel)
    launches_per_step = STEP_SWEEPS * 3 * len(DECODE_M) * len(SHAPES)

    # --- capture one step as a CUDA graph
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    for _ in range(a.warmup):
        g.replay()
    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        pass
    clocks = Clocks(uuid)
    clocks.start()
    time.sleep(0.2)
    barrier_sync(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.steps):
        g.replay()
    e1.record()
    barrier_sync(world)
    ms = e0.elapsed_time(e1) / a.steps
    clk = clocks.stop()
    ms = max_over_ranks(ms, world)
    value = world * bytes_per_step / (ms * 1e-3) / 1e9

    # --- per-kernel launch durations for the roofline: the decode GEMM (the
    # dominant kernel) and the activation kernel of each case, L2 flushed
    # before every pair, CUDA events on the launching stream around each
    # kernel; and the whole linear through the op, timed the same way
    flush = L2Flush(torch, dev)
    gemm_t, gemm_b, act_t, act_b, cases = 0.0, 0, 0.0, 0, {}
    for ri, M in enumerate(DECODE_M):
        for (name, N, K) in SHAPES:
            L = reps[ri][name]
            ta_l, tg_l = kernel_pair_times(
                torch, flush, lambda: ops.rotq_int8(xs[(M, K)], L["rot_table"], L["cs_vec"], 128, True),
                lambda q: ops.w4a8_gemm(q[0], q[1], L["packed"], N, None, torch.bfloat16), PAIR_REPS)
            tl = kernel_times(torch, flush, lambda: linear(L, xs[(M, K)], M), PAIR_REPS)
            act_t += sum(ta_l)
            act_b += act_alg_bytes(M, K) * len(ta_l)
            gemm_t += sum(tg_l)
            gemm_b += gemm_alg_bytes(M, N, K) * len(tg_l)
            cases[f"{name}_m{M}"] = {"gemm_us": round(1e6 * statistics.median(tg_l), 2),
                                     "act_us": round(1e6 * statistics.median(ta_l), 2),
                                     "linear_us": round(1e6 * statistics.median(tl), 2),
                                     "weight_GBps": round(weight_bytes(N, K) / statistics.median(tg_l) / 1e9, 1)}
    hbm, peak_kind = peaks()
    cold_gbs = gemm_b / gemm_t / 1e9
    case_out = cases

    # --- the decode GEMM's average launch duration over the step's own
    # launches: the benchmark step's 16 sweeps x 12 GEMMs (same cases, same
    # three weight replicas, same order; 346 MiB of weights per sweep > L2),
    # int8 rows already quantised, captured back to back as a CUDA graph and
    # timed with CUDA events on the launching stream
    qx = {}
    for ri, M in enumerate(DECODE_M):
        for (name, N, K) in SHAPES:
            L = reps[ri][name]
            qx[(ri, name)] = ops.rotq_int8(xs[(M, K)], L["rot_table"], L["cs_vec"], 128, True)
    gy = {k: None for k in qx}

    def gemm_step():
        for _ in range(STEP_SWEEPS):
            for ri, M in enumerate(DECODE_M):
                for (name, N, K) in SHAPES:
                    q = qx[(ri, name)]
                    gy[(ri, name)] = ops.w4a8_gemm(q[0], q[1], reps[ri][name]["packed"], N, None, torch.bfloat16)

    sg = torch.cuda.Stream()
    sg.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(sg):
        gemm_step()
    torch.cuda.current_stream().wait_stream(sg)
    gg = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gg):
        gemm_step()
    for _ in range(a.warmup):
        gg.replay()
    torch.cuda.synchronize()
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g0.record()
    for _ in range(a.steps):
        gg.replay()
    g1.record()
    torch.cuda.synchronize()
    gemm_launches = STEP_SWEEPS * len(DECODE_M) * len(SHAPES)
    gemm_step_s = g0.elapsed_time(g1) * 1e-3 / a.steps
    gemm_step_bytes = STEP_SWEEPS * sum(gemm_alg_bytes(M, N, K) for M in DECODE_M for (_, N, K) in SHAPES)
    gemm_gbs = gemm_step_bytes / gemm_step_s / 1e9
    del gg, qx, gy
    traffic = profile_traffic("gemm_decode_sweep_traffic.md")

    # --- prefill: tcgen05 GEMM and activation kernel per shape
    stack = None if a.no_stack else stack_section(torch, world, rank)
    if stack is not None and "skipped" not in stack:
        stack["per_projection_tables"] = stack_section(torch, world, rank, per_projection=True)
    verify = None if a.no_verify else verify_section(torch, world, rank)
    sharded = None if a.no_sharded else sharded_section(torch, world, rank)
    prefill = None
    if not a.no_prefill:
        prefill = prefill_section(torch, ops, syn, reps[0], flush, rank)
    ref_gpu = None
    if rank == 0 and world == 1 and not a.no_reference_gpu:
        try:
            ref_gpu = reference_gpu_section(torch, syn, flush, a.steps, a.warmup)
        except Exception as e:  # report why, keep the rest of the line
            ref_gpu = {"unavailable": f"{type(e).__name__}: {str(e).splitlines()[0][:200]}"}
            torch.cuda.empty_cache()
    del flush

    # --- end to end through the public op with host buffers (graph of the step)
    e2e = None
    if not a.no_e2e:
        hx = {k: v.cpu().pin_memory() for k, v in xs.items()}
        dxs = [{k: torch.empty_like(v) for k, v in xs.items()} for _ in range(2)]
        hy = {(ri, name): torch.empty((M, N), dtype=torch.bfloat16).pin_memory()
              for ri, M in enumerate(DECODE_M) for (name, N, K) in SHAPES}
        h2d = sum(v.numel() * 2 for v in xs.values())
        d2h = sum(v.numel() * 2 for v in hy.values())
        copy_stream = torch.cuda.Stream()

        def e2e_step(par):
            # the benchmark step (STEP_SWEEPS sweeps) as a serving loop runs
            # it: its inputs were copied in from pinned host memory during
            # the step before (double-buffered device inputs); the next
            # step's inputs are copied in on a side stream while this one
            # computes, and the last sweep's outputs are copied out on that
            # stream as soon as each is produced; the step ends when every
            # copy has landed
            main = torch.cuda.current_stream()
            cur, nxt = dxs[par], dxs[1 - par]
            copy_stream.wait_stream(main)
            with torch.cuda.stream(copy_stream):
                for k in nxt:
                    nxt[k].copy_(hx[k], non_blocking=True)
            for sw in range(STEP_SWEEPS):
                for ri, M in enumerate(DECODE_M):
                    for (name, N, K) in SHAPES:
                        L = reps[ri][name]
                        y = ops.linear_w4a8(cur[(M, K)], L["rot_table"], L["cs_vec"], L["packed"], N, None, True,
                                            torch.bfloat16)
                        if sw == STEP_SWEEPS - 1:
                            copy_stream.wait_stream(main)
                            with torch.cuda.stream(copy_stream):
                                hy[(ri, name)].copy_(y, non_blocking=True)
            main.wait_stream(copy_stream)

        for k in dxs[0]:
            dxs[0][k].copy_(hx[k])
        graphs = []
        for par in range(2):
            s2 = torch.cuda.Stream()
            s2.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s2):
                e2e_step(par)
            torch.cuda.current_stream().wait_stream(s2)
            g2 = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g2):
                e2e_step(par)
            graphs.append(g2)
        for i in range(2 * a.warmup):
            graphs[i % 2].replay()
        torch.cuda.synchronize()
        barrier_sync(world)
        t0 = time.perf_counter()
        for i in range(a.steps):
            graphs[i % 2].replay()
            torch.cuda.synchronize()  # the step's results are read on the host
        barrier_sync(world)
        el = max_over_ranks((time.perf_counter() - t0) / a.steps, world)
        e2e = {"value": world * STEP_SWEEPS * wset / el / 1e9, "unit": "GB/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "ms_per_step": el * 1e3,
               "path": f"torch.ops.paro_b200.linear_w4a8 per linear, the benchmark step ({STEP_SWEEPS} sweeps) "
                       "with pinned host inputs copied in (double-buffered: the next step's during this one) and "
                       "the outputs copied out as they are produced, CUDA graph replay + host sync per step, host "
                       "wall clock"}
        del graphs

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        cpu = cpu_baseline_sample()

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world,
            "value_per_gpu": round(value / world, 1), "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int4xint8->int32 (bf16 act/out)", "data": "synthetic",
            "config": {"workload": "decode sweep, BASELINE configs[1]: qkv 3584->4608, o 3584->3584, "
                                   "gate_up 3584->37888, down 18944->3584 at M=1,4,8; per linear the op "
                                   "linear_w4a8: activation kernel (channel scale + 8 Givens layers + per-token "
                                   "int8) and W4A8 GEMM chained by programmatic dependent launch",
                       "step": f"{STEP_SWEEPS} sweeps of the 12 (shape, M) linears, CUDA graph",
                       "l2": f"weight working set {wset / 2**20:.0f} MiB per sweep > L2 {L2_BYTES / 2**20:.0f} MiB "
                             "(3 replicas, one per M); inputs not flushed",
                       "parallelism": f"dp{world} (independent replicas, no collective)"},
            "roofline": {"kernel": "decode W4A8 GEMM (gemm_stream_kernel: TMA bulk weight stream, mma.sync "
                                   "int4 x int8, stream-K)", "bound": "hbm",
                         "achieved": round(gemm_gbs, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(gemm_gbs / hbm, 4), "peak_kind": peak_kind,
                         "traffic": traffic,
                         "traffic_source": "mean DRAM bytes per launch of the sweep's 12 GEMM launches, one ncu "
                                           "capture (profiles/gemm_decode_sweep_traffic.md)",
                         "alg_bytes": "N*K/2 + G*N*2 + G*N/2 + M*K + 4M + 2*M*N per launch",
                         "avg_launch_us": round(gemm_step_s / gemm_launches * 1e6, 3),
                         "timing": f"the step's {gemm_launches} GEMM launches (16 sweeps x 12 cases, 3 weight "
                                   "replicas > L2) back to back in a CUDA graph, CUDA events on the launching "
                                   "stream; achieved = algorithmic bytes / time",
                         "cold_launch": {"achieved": round(cold_gbs, 1), "frac": round(cold_gbs / hbm, 4),
                                         "timing": "one launch after an L2 flush (512 MiB write, then 256 MiB "
                                                   "read), CUDA events, median of 5 per case"}},
            "activation_kernel": {"achieved_GBps": round(act_b / act_t / 1e9, 1),
                                  "frac": round(act_b / act_t / 1e9 / hbm, 4),
                                  "alg_bytes": "2MK + MK + 4M + tables 2LK + LK + 2K (L = 8) per launch"},
            "prefill": prefill,
            "stack": stack,
            "verify_and_decode_loop": verify,
            "sharded_prefill": sharded,
            "cases": case_out,
            "gpu_launches": launches_per_step * a.steps,
            "clocks": clk,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "reference_gpu": ref_gpu,
        }
        print(json.dumps(line), flush=True)
    del g
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
