"""The decoder-stack and column-sharded workloads built from the W4A8 ops
(BASELINE configs[3] and [4]) on one GPU."""
import numpy as np
import pytest
import torch

from tests.helpers import rel_l2

pytestmark = pytest.mark.gpu


def test_decoder_stack_forward_rows_are_independent():
    """Clips are independent: a batch of 4 tokens gives each token what it
    gets alone (up to the bf16 rounding of float32 sums added in a different
    order), and the forward is deterministic."""
    from alpamayo_b200 import synthetic as syn
    from alpamayo_b200.stack import DecoderStack
    st = DecoderStack(layers=2, seed=3)
    x = syn.make_activations(4, 3584, seed=4)
    y = st.forward(x)
    assert y.shape == (4, 3584) and y.dtype == torch.bfloat16 and torch.isfinite(y).all()
    assert torch.equal(st.forward(x), y)
    for r in range(4):
        yr = st.forward(x[r:r + 1].contiguous())
        assert rel_l2(yr.float().cpu().numpy(), y[r:r + 1].float().cpu().numpy()) <= 2e-2
    assert st.weight_bytes() == 2 * sum(syn.weight_stream_bytes(n, k) for (n, k) in
                                        [(4608, 3584), (3584, 3584), (37888, 3584), (3584, 18944)])


def test_column_sharded_linear_single_rank_is_the_full_linear():
    from alpamayo_b200 import synthetic as syn
    from alpamayo_b200.stack import ColumnShardedLinear, linear, serving_layer
    L = serving_layer(1024, 2048, seed=5)
    x = syn.make_activations(300, 2048, seed=6)
    csl = ColumnShardedLinear(lambda v: linear(L, v, torch.float32))
    blocks = csl(x)
    assert blocks.shape == (1, 300, 1024)
    full = linear(L, x, torch.float32)
    assert torch.equal(ColumnShardedLinear.assemble(blocks), full)


@pytest.mark.parametrize("M", [1, 64, 300, 2048])
def test_linear_into_writes_the_linear_into_a_slice(M):
    """linear_into (the C ABI with an explicit output pointer) writes the
    op's bf16 values into a row slice of a larger buffer and leaves the rest
    of the buffer alone; the single-rank peer_gathered path returns the full
    linear.  (Up to 64 tokens the stream-K GEMM adds float32 partial sums in
    a run-dependent order, so bf16 outputs may differ in the last place:
    1e-3 relative L2.)"""
    from alpamayo_b200 import synthetic as syn
    from alpamayo_b200.stack import ColumnShardedLinear, linear, linear_into, serving_layer
    L = serving_layer(1024, 2048, seed=7)
    x = syn.make_activations(M, 2048, seed=8)
    buf = torch.full((2, M, 1024), 3.0, dtype=torch.bfloat16, device="cuda")
    linear_into(L, x, buf[1])
    ref = linear(L, x)
    assert rel_l2(buf[1].float().cpu().numpy(), ref.float().cpu().numpy()) <= 1e-3
    assert torch.all(buf[0] == 3.0)
    csl = ColumnShardedLinear(None, block_columns=1024)
    out = csl.peer_gathered(x, lambda v, dst: linear_into(L, v.contiguous(), dst), chunks=4)
    assert out.shape == (1, M, 1024)
    assert rel_l2(out[0].float().cpu().numpy(), ref.float().cpu().numpy()) <= 1e-3


@pytest.mark.parametrize("M", [1, 8, 33, 64, 100])
def test_fused_prologues_give_the_separate_kernels_bits(M):
    """Residual add + RMSNorm fused into the next linear's rotation kernel
    (and SiLU * up into down's) against the separate kernels followed by the
    linear: the same bits, for decode sizes (fused in the rotation kernel:
    streaming GEMM at 1 / 8 tokens, tensor-core GEMM behind the chain at 33
    and 64 on gate_up and down) and prefill sizes (separate kernel inside the
    entry point), with and without an incoming residual."""
    import alpamayo_b200.ops as ops
    from alpamayo_b200 import synthetic as syn
    from alpamayo_b200.stack import linear, linear_rmsnorm, linear_silu, serving_layer
    qkv = serving_layer(4608, 3584, seed=11)
    gate_up = serving_layer(37888, 3584, seed=12)
    down = serving_layer(3584, 18944, seed=13)
    w = (0.9 + 0.2 * torch.rand(3584, device="cuda")).to(torch.bfloat16)
    x = syn.make_activations(M, 3584, seed=M)
    r = syn.make_activations(M, 3584, seed=M + 1)
    for res in (None, r):
        y, res_out = linear_rmsnorm(qkv, x, res, w, 1e-6)
        h, res_ref = ops.add_rmsnorm(x, res, w, 1e-6)
        assert torch.equal(res_out, res_ref)
        assert torch.equal(y, linear(qkv, h))
        assert res is None or torch.equal(r, syn.make_activations(M, 3584, seed=M + 1))   # input untouched
    gu, _ = linear_rmsnorm(gate_up, x, r, w, 1e-6)
    assert torch.equal(gu, linear(gate_up, ops.add_rmsnorm(x, r, w, 1e-6)[0]))
    assert torch.equal(linear_silu(down, gu), linear(down, ops.silu_mul(gu)))


def test_decoder_stack_fused_equals_unfused():
    from alpamayo_b200 import synthetic as syn
    from alpamayo_b200.stack import DecoderStack
    st = DecoderStack(layers=2, seed=3)
    for M in (4, 64):
        x = syn.make_activations(M, 3584, seed=9)
        assert torch.equal(st.forward(x, fused=True), st.forward(x, fused=False))


def test_decoder_stack_per_projection_tables():
    """q / k / v and gate / up with their own rotation tables, run as groups:
    the fused and unfused prologues agree bit for bit, and each group's
    output is its members' outputs side by side."""
    import alpamayo_b200.ops as ops
    from alpamayo_b200 import synthetic as syn
    from alpamayo_b200.stack import DecoderStack, linear
    st = DecoderStack(layers=2, seed=4, per_projection=True)
    for M in (3, 64):
        x = syn.make_activations(M, 3584, seed=M)
        y = st.forward(x)
        assert y.shape == (M, 3584) and torch.isfinite(y).all()
        assert torch.equal(y, st.forward(x, fused=False))
    G = st.layers[0]["qkv"]
    h = syn.make_activations(8, 3584, seed=1)
    yg, _ = ops.linear_w4a8_group(h, G["rot_tables"], G["channel_scales"], G["packed"], G["n_per_table"],
                                  out_dtype=torch.float32)
    ref = torch.cat([linear(L, h, torch.float32) for L in G["parts"]], dim=1)
    assert rel_l2(yg.cpu().numpy(), ref.cpu().numpy()) <= 1e-6
