"""Decoder stacks and column-sharded linears built from the W4A8 ops.

* DecoderStack — the decode-stack workload: L rotated
  W4A8 decoder layers of a 7B-class model (hidden 3584, 28 heads of 128, 4 KV
  heads, intermediate 18944).  Per layer: residual add + RMSNorm -> qkv;
  attention replaced by identity (the query heads pass through) -> o_proj;
  residual add + RMSNorm -> gate_up -> SiLU * up -> down_proj.  Seeded
  random-init weights, quantised with the reference's recipe.  Independent
  clips shard across GPUs with no collective: every rank holds the whole
  stack and runs its share of the tokens.
* ColumnShardedLinear — the sharded-prefill workload:
  one rotated linear whose output columns are split across the ranks of a
  process group; each rank computes its [M, N / world] block and an
  all-gather assembles [world, M, N / world] (rank-major blocks).
"""
from __future__ import annotations

import torch

from . import ops
from . import synthetic as syn

HIDDEN, HEADS, KV_HEADS, HEAD_DIM, INTER = 3584, 28, 4, 128, 18944


def serving_layer(N, K, seed, device="cuda"):
    """A seeded quantised linear reduced to what the forward reads: tile
    records, rotation table, channel scales."""
    L = syn.make_layer(N, K, seed=seed, device=device, checkpoint=False)
    return {"N": N, "K": K, "packed": L["packed"], "rot_table": L["rot_table"], "cs_vec": L["cs_vec"]}


def linear(L, x, out_dtype=torch.bfloat16):
    return ops.linear_w4a8(x, L["rot_table"], L["cs_vec"], L["packed"], L["N"], None, True, out_dtype)


class DecoderStack:
    def __init__(self, layers=28, seed=0, device="cuda", eps=1e-6):
        qkv_n = (HEADS + 2 * KV_HEADS) * HEAD_DIM
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        self.eps = eps
        self.layers = []
        for i in range(layers):
            s = seed * 1000 + 10 * i
            norm = lambda: (0.9 + 0.2 * torch.rand(HIDDEN, generator=g, device=device)).to(torch.bfloat16)
            self.layers.append({
                "in_norm": norm(), "post_norm": norm(),
                "qkv": serving_layer(qkv_n, HIDDEN, s + 1, device),
                "o": serving_layer(HIDDEN, HEADS * HEAD_DIM, s + 2, device),
                "gate_up": serving_layer(2 * INTER, HIDDEN, s + 3, device),
                "down": serving_layer(HIDDEN, INTER, s + 4, device),
            })
        self.final_norm = (0.9 + 0.2 * torch.rand(HIDDEN, generator=g, device=device)).to(torch.bfloat16)

    def weight_bytes(self):
        """Algorithmic weight-stream bytes of one forward (all four
        projections of every layer)."""
        return sum(syn.weight_stream_bytes(L[k]["N"], L[k]["K"]) for L in self.layers
                   for k in ("qkv", "o", "gate_up", "down"))

    def forward(self, x):
        """x: bf16 [M, 3584] (one token per clip) -> bf16 [M, 3584]."""
        res = None
        mlp_out = x
        for L in self.layers:
            h, res = ops.add_rmsnorm(mlp_out, res, L["in_norm"], self.eps)
            qkv = linear(L["qkv"], h)
            attn = qkv[:, :HEADS * HEAD_DIM].contiguous()   # identity attention
            o = linear(L["o"], attn)
            h, res = ops.add_rmsnorm(o, res, L["post_norm"], self.eps)
            a = ops.silu_mul(linear(L["gate_up"], h))
            mlp_out = linear(L["down"], a)
        out, _ = ops.add_rmsnorm(mlp_out, res, self.final_norm, self.eps)
        return out


def column_shard(N, rank, world, align=16):
    """The [start, stop) output columns of `rank` when N columns are split
    across `world` ranks in equal blocks (N / world a multiple of `align`)."""
    if N % world or (N // world) % align:
        raise ValueError(f"N={N} does not split into {world} blocks of a multiple of {align}")
    w = N // world
    return rank * w, (rank + 1) * w


class ColumnShardedLinear:
    """One rank's column block of an N x K rotated linear plus the gather.

    `local_fn(x)` computes this rank's [M, N / world] block (the W4A8 linear
    on the GPU; any callable in tests).  `gather(y_local)` all-gathers the
    blocks over the process group into a [world, M, N / world] tensor."""

    def __init__(self, local_fn, group=None):
        import torch.distributed as dist
        self.local_fn = local_fn
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1

    def gather(self, y_local):
        import torch.distributed as dist
        if self.world == 1:
            return y_local.unsqueeze(0)
        y = y_local.contiguous()
        out = y.new_empty((self.world * y.shape[0], *y.shape[1:]))   # rank blocks concatenated on dim 0
        dist.all_gather_into_tensor(out, y, group=self.group)
        return out.view(self.world, *y.shape)

    def __call__(self, x):
        return self.gather(self.local_fn(x))

    def overlapped(self, x, chunks=4):
        """The same result computed in `chunks` row blocks: the all-gather
        of block i (asynchronous, on the collective's own stream) runs while
        block i + 1 is computed.  Returns [chunks, world, M / chunks, N /
        world] (see assemble_chunks)."""
        import torch.distributed as dist
        M = x.shape[0]
        if self.world == 1 or chunks <= 1 or M % chunks:
            return self(x).unsqueeze(0)
        mc = M // chunks
        outs, works = [], []
        for c in range(chunks):
            y = self.local_fn(x[c * mc:(c + 1) * mc].contiguous()).contiguous()
            out = y.new_empty((self.world * mc, *y.shape[1:]))
            works.append(dist.all_gather_into_tensor(out, y, group=self.group, async_op=True))
            outs.append(out.view(self.world, mc, *y.shape[1:]))
        for w in works:
            w.wait()
        return torch.stack(outs)

    @staticmethod
    def assemble(blocks):
        """[world, M, N / world] -> [M, N] (columns in rank order)."""
        w, M, n = blocks.shape
        return blocks.permute(1, 0, 2).reshape(M, w * n)

    @staticmethod
    def assemble_chunks(blocks):
        """[chunks, world, M / chunks, N / world] -> [M, N]."""
        c, w, mc, n = blocks.shape
        return blocks.permute(0, 2, 1, 3).reshape(c * mc, w * n)
