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
