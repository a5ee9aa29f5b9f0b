"""The column-sharded linear gathered by the GEMM's own epilogue (multimem
stores through an NVLink multicast address, ColumnShardedLinear.
multicast_gathered) against the NCCL all-gather of the same blocks: equal
bit for bit on every rank, on both of the alternating buffers.  Two ranks,
one GPU each, NCCL with a short timeout; skipped with fewer than two GPUs
or where the GPUs have no multicast support."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, result):
    import datetime

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        import alpamayo_b200.ops as ops
        from alpamayo_b200 import synthetic as syn
        from alpamayo_b200.stack import ColumnShardedLinear, column_shard, linear, serving_layer
        N, K, M = 4608 * world, 3584, 640
        c0, c1 = column_shard(N, rank, world)
        L = serving_layer(c1 - c0, K, seed=50 + rank)
        nccl = ColumnShardedLinear(lambda v: linear(L, v))
        mc = ColumnShardedLinear(None, block_columns=c1 - c0)
        quant = lambda v: ops.rotq_int8(v, L["rot_table"], L["cs_vec"], 128, True)  # noqa: E731
        ok = True
        try:
            for seed in (1, 2, 3):
                x = syn.make_activations(M, K, seed=seed)
                ref = nccl(x)
                got = mc.multicast_gathered(x, quant, L["packed"], K)
                ok &= bool(torch.equal(got, ref))
        except RuntimeError as e:
            if "multicast" in str(e):
                result[rank] = "skip: " + str(e)
                return
            raise
        mc.close_multicast_buffers()
        flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device="cuda")
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        result[rank] = "ok" if flag.item() == 1 else "mismatch"
    finally:
        dist.destroy_process_group()


def _worker(rank, world, port, q):
    res = {}
    try:
        _rank(rank, world, port, res)
    except Exception as e:  # reported to the parent
        res[rank] = f"error: {e}"
    q.put((rank, res.get(rank, "error: no result")))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_multicast_epilogue_gather_equals_nccl_gather():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    for _ in procs:
        r, v = q.get(timeout=300)
        out[r] = v
    for p in procs:
        p.join(timeout=60)
    if all(v.startswith("skip") for v in out.values()):
        pytest.skip(out[0])
    assert out == {0: "ok", 1: "ok"}, out
