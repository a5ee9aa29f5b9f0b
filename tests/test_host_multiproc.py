"""Multi-process host logic on CPU (gloo, world size 2): the column split of
the sharded-prefill linear and the all-gather that reassembles it, with a
CPU matmul standing in for the GPU linear (the kernels themselves are
covered by the GPU tests)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from alpamayo_b200.stack import ColumnShardedLinear, column_shard


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, M, N, K, ret):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        x = torch.randn(M, K, generator=g)
        w = torch.randn(N, K, generator=g)
        c0, c1 = column_shard(N, rank, world)
        csl = ColumnShardedLinear(lambda v: v @ w[c0:c1].t())
        blocks = csl(x)
        full = ColumnShardedLinear.assemble(blocks)
        chunked = ColumnShardedLinear.assemble_chunks(csl.overlapped(x, chunks=3))
        ret[rank] = max(float((full - x @ w.t()).abs().max()), float((chunked - x @ w.t()).abs().max()))
    finally:
        dist.destroy_process_group()


def test_column_sharded_gather_reassembles_the_full_output():
    world, M, N, K = 2, 6, 64, 32
    ret = mp.Manager().dict()
    mp.spawn(_worker, args=(world, _free_port(), M, N, K, ret), nprocs=world, join=True)
    assert len(ret) == world and max(ret.values()) == 0.0


def test_column_shard_bounds():
    assert column_shard(37888, 0, 2) == (0, 18944)
    assert column_shard(37888, 7, 8) == (33152, 37888)
    with pytest.raises(ValueError):
        column_shard(100, 0, 3)
    with pytest.raises(ValueError):
        column_shard(37888, 0, 5)
