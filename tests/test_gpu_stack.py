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
