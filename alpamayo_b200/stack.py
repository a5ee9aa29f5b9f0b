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
  process group; each rank computes its [M, N / world] block and a gather
  assembles [world, M, N / world] (rank-major blocks) on every rank: an
  NCCL all-gather, or copy-engine copies into buffers every peer has mapped
  (peer_gathered), which overlap the GEMM because they use no SM.
"""
from __future__ import annotations

import torch

from . import ops
from . import synthetic as syn

HIDDEN, HEADS, KV_HEADS, HEAD_DIM, INTER = 3584, 28, 4, 128, 18944


def serving_layer(N, K, seed, device="cuda", keep=False):
    """A seeded quantised linear reduced to what the forward reads: tile
    records, rotation table, channel scales (with ``keep``, also the
    rotation buffers and AWQ int32 weights it was built from, for checks)."""
    L = syn.make_layer(N, K, seed=seed, device=device, checkpoint=False, keep_awq=keep)
    out = {"N": N, "K": K, "packed": L["packed"], "rot_table": L["rot_table"], "cs_vec": L["cs_vec"]}
    if keep:
        for k in ("pairs", "theta", "channel_scales", "awq_qweight", "awq_scales", "awq_qzeros"):
            out[k] = L[k]
    return out


def linear(L, x, out_dtype=torch.bfloat16):
    return ops.linear_w4a8(x, L["rot_table"], L["cs_vec"], L["packed"], L["N"], None, True, out_dtype)


def linear_rmsnorm(L, x, residual, norm_weight, eps, out_dtype=torch.bfloat16):
    """Residual add + RMSNorm fused into the rotated linear L: (y, new residual)."""
    return ops.linear_w4a8_rmsnorm(x, residual, norm_weight, L["rot_table"], L["cs_vec"], L["packed"], L["N"], None,
                                   eps, True, out_dtype)


def linear_silu(L, gate_up, out_dtype=torch.bfloat16):
    """SiLU(gate) * up fused into the rotated linear L."""
    return ops.linear_w4a8_silu(gate_up, L["rot_table"], L["cs_vec"], L["packed"], L["N"], None, True, out_dtype)


def group_rmsnorm(G, x, residual, norm_weight, eps, fused=True, out_dtype=torch.bfloat16):
    """Residual add + RMSNorm, then a projection group (fused into the
    group's rotation kernel, or as a separate kernel): (y, new residual)."""
    if fused:
        return ops.linear_w4a8_group(x, G["rot_tables"], G["channel_scales"], G["packed"], G["n_per_table"],
                                     prologue="add_rmsnorm", residual=residual, norm_weight=norm_weight, eps=eps,
                                     out_dtype=out_dtype)
    h, res = ops.add_rmsnorm(x, residual, norm_weight, eps)
    y, _ = ops.linear_w4a8_group(h, G["rot_tables"], G["channel_scales"], G["packed"], G["n_per_table"],
                                 out_dtype=out_dtype)
    return y, res


_ws_cache = {}


def linear_into(L, x, out):
    """linear() writing into a given bf16 [M, N] tensor (through the C ABI's
    paro_w4a8_linear, whose output is any device pointer)."""
    import ctypes
    from ._native import capi
    Lc = capi()
    M, K = x.shape
    N = L["N"]
    wsb = Lc.paro_w4a8_linear_workspace_size(M, N, K)
    scb = Lc.paro_w4a8_linear_scratch_size(M, N, K, 1)
    key = (x.device, torch.cuda.current_stream().cuda_stream)
    ws = _ws_cache.get(key)
    if ws is None or ws.numel() < wsb + 256:
        ws = torch.zeros(max(wsb, 16 << 20) + 256, dtype=torch.uint8, device=x.device)
        _ws_cache[key] = ws
    sc = torch.empty(scb + 256, dtype=torch.uint8, device=x.device)
    al = lambda t: (t.data_ptr() + 255) & ~255
    st = Lc.paro_w4a8_linear(x.data_ptr(), 2, M, K, N, L["cs_vec"].data_ptr(), L["rot_table"].data_ptr(), 1,
                             L["packed"].data_ptr(), None, 0, out.data_ptr(), 2, al(ws), wsb, al(sc), scb,
                             ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    if st:
        raise RuntimeError(f"paro_w4a8_linear: {Lc.paro_status_string(st).decode()}")
    return out


def projection_group(parts):
    """Layers that share their input, each with its own rotation, as one
    group for ops.linear_w4a8_group: concatenated tile records, per-part
    tables and channel scales, output widths."""
    return {"N": sum(L["N"] for L in parts), "K": parts[0]["K"], "parts": parts,
            "packed": torch.cat([L["packed"] for L in parts]),
            "rot_tables": [L["rot_table"] for L in parts], "channel_scales": [L["cs_vec"] for L in parts],
            "n_per_table": [L["N"] for L in parts]}


class DecoderStack:
    """per_projection: q / k / v and gate / up as separate linears with their
    own rotation tables (the layout of a real ParoQuant checkpoint), run as
    groups (one rotation + quantisation launch over the tables, one GEMM over
    the concatenated weights); otherwise fused qkv and gate_up with one table
    each (the synthetic BASELINE shapes)."""

    def __init__(self, layers=28, seed=0, device="cuda", eps=1e-6, keep=False, per_projection=False):
        qkv_n = (HEADS + 2 * KV_HEADS) * HEAD_DIM
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        self.eps = eps
        self.per_projection = per_projection
        self.layers = []
        for i in range(layers):
            s = seed * 1000 + 10 * i
            norm = lambda: (0.9 + 0.2 * torch.rand(HIDDEN, generator=g, device=device)).to(torch.bfloat16)
            L = {"in_norm": norm(), "post_norm": norm(),
                 "o": serving_layer(HIDDEN, HEADS * HEAD_DIM, s + 2, device, keep),
                 "down": serving_layer(HIDDEN, INTER, s + 4, device, keep)}
            if per_projection:
                L["qkv"] = projection_group([serving_layer(n, HIDDEN, s + 100 + j, device, keep)
                                             for j, n in enumerate((HEADS * HEAD_DIM, KV_HEADS * HEAD_DIM,
                                                                    KV_HEADS * HEAD_DIM))])
                L["gate_up"] = projection_group([serving_layer(INTER, HIDDEN, s + 110 + j, device, keep)
                                                 for j in range(2)])
            else:
                L["qkv"] = serving_layer(qkv_n, HIDDEN, s + 1, device, keep)
                L["gate_up"] = serving_layer(2 * INTER, HIDDEN, s + 3, device, keep)
            self.layers.append(L)
        self.final_norm = (0.9 + 0.2 * torch.rand(HIDDEN, generator=g, device=device)).to(torch.bfloat16)

    def weight_bytes(self):
        """Algorithmic weight-stream bytes of one forward (all four
        projections of every layer)."""
        return sum(syn.weight_stream_bytes(L[k]["N"], L[k]["K"]) for L in self.layers
                   for k in ("qkv", "o", "gate_up", "down"))

    def forward(self, x, fused=True):
        """x: bf16 [M, 3584] (one token per clip) -> bf16 [M, 3584].

        fused: the residual add + RMSNorm before qkv and gate_up and the
        SiLU * up before down run inside those linears' activation kernels
        (linear_w4a8_rmsnorm / linear_w4a8_silu); otherwise as separate
        kernels (add_rmsnorm, silu_mul).  Both give the same bits."""
        res = None
        mlp_out = x
        for L in self.layers:
            if self.per_projection:
                qkv, res = group_rmsnorm(L["qkv"], mlp_out, res, L["in_norm"], self.eps, fused)
            elif fused:
                qkv, res = linear_rmsnorm(L["qkv"], mlp_out, res, L["in_norm"], self.eps)
            else:
                h, res = ops.add_rmsnorm(mlp_out, res, L["in_norm"], self.eps)
                qkv = linear(L["qkv"], h)
            attn = qkv[:, :HEADS * HEAD_DIM].contiguous()   # identity attention
            o = linear(L["o"], attn)
            if self.per_projection:
                gu, res = group_rmsnorm(L["gate_up"], o, res, L["post_norm"], self.eps, fused)
                mlp_out = linear_silu(L["down"], gu) if fused else linear(L["down"], ops.silu_mul(gu))
            elif fused:
                gu, res = linear_rmsnorm(L["gate_up"], o, res, L["post_norm"], self.eps)
                mlp_out = linear_silu(L["down"], gu)
            else:
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

    def __init__(self, local_fn, group=None, block_columns=None):
        import torch.distributed as dist
        self.local_fn = local_fn
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self._n = block_columns

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

    def peer_gathered(self, x, into_fn, chunks=4):
        """The gather done by the copy engines over NVLink instead of a
        collective kernel, so that it overlaps the GEMM (which holds every
        SM).  The result lives in one of two [world, M, N / world] buffers
        that every peer has mapped (CUDA IPC, plain peer mappings).  For each
        of `chunks` row blocks, `into_fn(x_rows, dst)` writes this rank's
        block straight into its own slot; a side stream then copies the slot
        into every peer's buffer with cudaMemcpyAsync (DMA; no kernel reads
        or writes peer memory) while the next block is computed (one stream
        for all peers measured faster at 4 ranks than one per peer).  A
        one-word
        all-reduce after the copies tells every rank that all blocks have
        landed.  The two buffers alternate, so the result of a call stays
        valid until the call after next; the closing all-reduce of the next
        call also orders a peer's writes after this rank's use of the
        buffer.  Returns [world, M, N / world]; close_peer_buffers() frees
        the buffers (collective)."""
        import torch.distributed as dist
        from cuda.bindings import runtime as cudart
        M = x.shape[0]
        if self.world == 1:
            out = torch.empty((1, M, self._n), dtype=torch.bfloat16, device=x.device)
            into_fn(x, out[0])
            return out
        key = (M, self._n, x.device)
        if getattr(self, "_peer", None) is None or self._peer.key != key:
            self.close_peer_buffers()
            self._peer = _PeerBuffers(self.world, (self.world, M, self._n), x.device, self.group, key)
            self._comm = torch.cuda.Stream(device=x.device)
            self._flag = torch.zeros(1, dtype=torch.int32, device=x.device)
        pb = self._peer
        b = pb.flip()
        out = pb.tensor(b)
        rank = pb.rank
        mc = M // chunks if chunks > 1 and M % chunks == 0 else M
        blk = mc * self._n * 2
        cur = torch.cuda.current_stream()
        for r0 in range(0, M, mc):
            mine = out[rank, r0:r0 + mc]
            into_fn(x[r0:r0 + mc], mine)
            ev = torch.cuda.Event()
            ev.record(cur)
            self._comm.wait_event(ev)
            off = (rank * M + r0) * self._n * 2
            for j in range(self.world):
                if j != rank:
                    err, = cudart.cudaMemcpyAsync(pb.ptrs[b][j] + off, pb.ptrs[b][rank] + off, blk,
                                                  cudart.cudaMemcpyKind.cudaMemcpyDeviceToDevice,
                                                  self._comm.cuda_stream)
                    if err != cudart.cudaError_t.cudaSuccess:
                        raise RuntimeError(f"peer copy failed: {err}")
        cur.wait_stream(self._comm)
        dist.all_reduce(self._flag, group=self.group)
        return out

    def multicast_gathered(self, x, quantise, packed, K):
        """The gather done by the GEMM's own epilogue: every rank's copy of a
        [world, M, N / world] bf16 buffer in torch symmetric memory is bound
        to one NVLink multicast object, and this rank's W4A8 GEMM
        (paro_w4a8_gemm_multicast) stores its block through the multicast
        address, so the NVSwitch delivers it to every rank while the GEMM
        runs; a one-word all-reduce then makes the whole buffer valid.
        `quantise(x)` returns the int8 activations and token scales of x
        (the rotation + quantiser of the linear); `packed` is this rank's
        column block of tile records.  Two buffers alternate, so the result
        of a call stays valid until the call after next (the closing
        all-reduce of the next call orders a peer's writes after this rank's
        use).
        Raises RuntimeError where the GPUs have no multicast support.
        close_multicast_buffers() frees the buffers (collective)."""
        import ctypes
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem
        from ._native import capi
        M = x.shape[0]
        if self.world == 1:
            raise RuntimeError("multicast gather needs more than one rank")
        key = (M, self._n, x.device)
        if getattr(self, "_mc", None) is None or self._mc["key"] != key:
            self.close_multicast_buffers()
            group = self.group if self.group is not None else dist.group.WORLD
            bufs, hdls = [], []
            for _ in range(2):
                buf = symm_mem.empty((self.world, M, self._n), dtype=torch.bfloat16, device=x.device)
                hdl = symm_mem.rendezvous(buf, group)
                if not hdl.has_multicast_support or not hdl.multicast_ptr:
                    raise RuntimeError("no NVLink multicast support for this group")
                bufs.append(buf)
                hdls.append(hdl)
            self._mc = {"key": key, "bufs": bufs, "hdls": hdls, "next": 0,
                        "flag": torch.zeros(1, dtype=torch.int32, device=x.device)}
        mc = self._mc
        b = mc["next"]
        mc["next"] ^= 1
        hdl = mc["hdls"][b]
        xq, xs = quantise(x)
        dst = hdl.multicast_ptr + hdl.rank * M * self._n * 2
        st = capi().paro_w4a8_gemm_multicast(xq.data_ptr(), xs.data_ptr(), M, self._n, K, packed.data_ptr(), None, 0,
                                             ctypes.c_void_p(dst),
                                             ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        if st:
            raise RuntimeError(f"paro_w4a8_gemm_multicast: {capi().paro_status_string(st).decode()}")
        # a one-word all-reduce as the cross-rank barrier (the process
        # group's timeout bounds it on the host): a peer's contribution
        # arrives only after its GEMM's multicast stores, which the kernel
        # orders at system scope
        dist.all_reduce(mc["flag"], group=self.group)
        return mc["bufs"][b]

    def close_multicast_buffers(self):
        """Drop the multicast_gathered buffers (every rank calls it, after a
        barrier, so that no peer still writes into them)."""
        mc = getattr(self, "_mc", None)
        if mc is not None:
            import torch.distributed as dist
            torch.cuda.synchronize()
            dist.barrier(group=self.group)
            self._mc = None
            del mc

    def close_peer_buffers(self):
        """Unmap and free the peer_gathered buffers (every rank calls it)."""
        pb = getattr(self, "_peer", None)
        if pb is not None:
            pb.close()
            self._peer = None

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


class _PeerBuffers:
    """Two bf16 buffers of `shape` on every rank, each from its own
    cudaMalloc, exported with cudaIpcGetMemHandle and opened by every peer
    (cudaIpcOpenMemHandle with lazy peer access): ptrs[b][j] is rank j's
    buffer b as this rank addresses it.  Setup and close are collective; a
    failure on any rank raises on every rank."""

    def __init__(self, world, shape, device, group, key):
        import torch.distributed as dist
        from cuda.bindings import runtime as cudart
        self.world, self.shape, self.device, self.group, self.key = world, shape, device, group, key
        self.rank = dist.get_rank(group)
        self.nbytes = 2
        for d in shape:
            self.nbytes *= d
        self.own, self.opened, self.ptrs, self._b = [], [], [], 1
        ok = True
        cudart.cudaSetDevice(device.index)
        for _ in range(2):
            h = b""
            if ok:
                err, p = cudart.cudaMalloc(self.nbytes)
                ok = err == cudart.cudaError_t.cudaSuccess
                if ok:
                    self.own.append(p)
                    err, hd = cudart.cudaIpcGetMemHandle(p)
                    ok = err == cudart.cudaError_t.cudaSuccess
                    h = bytes(hd.reserved) if ok else b""
            handles = [None] * world
            dist.all_gather_object(handles, h, group=group)
            row = []
            for j in range(world):
                if j == self.rank:
                    row.append(self.own[-1] if ok else 0)
                elif ok and handles[j]:
                    hh = cudart.cudaIpcMemHandle_t()
                    hh.reserved = handles[j]
                    err, q = cudart.cudaIpcOpenMemHandle(hh, cudart.cudaIpcMemLazyEnablePeerAccess)
                    ok = err == cudart.cudaError_t.cudaSuccess
                    if ok:
                        self.opened.append(q)
                    row.append(q if ok else 0)
                else:
                    ok = False
                    row.append(0)
            self.ptrs.append(row)
        flag = torch.tensor([0 if ok else 1], dtype=torch.int32, device=device)
        dist.all_reduce(flag, group=group)
        if flag.item():
            self.close()
            raise RuntimeError("peer buffer setup failed on at least one rank")
        self._views = [self._wrap(self.own[b]) for b in range(2)]

    def _wrap(self, ptr):
        class _Mem:
            __cuda_array_interface__ = {"shape": tuple(self.shape), "typestr": "<i2", "data": (ptr, False),
                                        "version": 3, "strides": None}
        return torch.as_tensor(_Mem(), device=self.device).view(torch.bfloat16)

    def flip(self):
        self._b ^= 1
        return self._b

    def tensor(self, b):
        return self._views[b]

    def close(self):
        import torch.distributed as dist
        from cuda.bindings import runtime as cudart
        torch.cuda.synchronize(self.device)
        for q in self.opened:
            cudart.cudaIpcCloseMemHandle(q)
        self.opened = []
        dist.barrier(group=self.group)
        for p in self.own:
            cudart.cudaFree(p)
        self.own = []
        self._views = []
