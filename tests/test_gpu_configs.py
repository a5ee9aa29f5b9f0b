"""Parity on the exact BASELINE configurations.

  configs[0]  M = 16, K = N = 3584, fp32 activations: the module built by the
              product's from_linear from the reference's seed (checked by the
              reference's hashes), against the reference pipeline's outputs
              (tests/golden/cfg0_m16_k3584.npz).
  configs[2]  prefill, the four projections at M = 8192 through linear_w4a8.
  configs[3]  two decoder layers of the stack at 8 and 64 tokens, step by step
              against the composed oracle (add + RMSNorm, rotated linear,
              SiLU * up), and the step-by-step result equals the stack's own
              forward.
  configs[4]  gate_up at M = 16384: the column shards of 2 and 8 ranks,
              computed on one GPU and reassembled, equal the unsharded linear.

Tolerances (north_star): activation codes within 1 LSB on at most 0.1 % of
elements; given the kernel's codes, outputs within 1e-3 relative L2 of the
oracle rounded to the output dtype (1e-6 in fp32).  At prefill and shard
sizes the oracle runs on sampled rows and columns (rows are independent;
columns are independent)."""
import os

import numpy as np
import pytest
import torch

from oracle import paro_oracle as O
from tests.helpers import awq_columns, rel_l2

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
SHAPES = {"qkv": (4608, 3584), "o_proj": (3584, 3584), "gate_up": (37888, 3584), "down": (3584, 18944)}


@pytest.fixture(scope="module")
def ops():
    import alpamayo_b200.ops as ops
    return ops


def _code_check(qk, q_ref):
    dq = np.abs(qk.astype(np.int32) - q_ref.astype(np.int32))
    assert dq.max() <= 1 and (dq > 0).mean() <= 1e-3, (int(dq.max()), float((dq > 0).mean()))


def _sampled_parity(ops, L, x, y, rows, cols):
    """Codes of the sampled rows against the oracle's; the sampled outputs
    against the oracle's GEMM on the kernel's own codes, rounded to y's
    dtype."""
    qk, sk = ops.rotq_int8(x, L["rot_table"], L["cs_vec"], 128, True)
    r_t = torch.from_numpy(rows).to(x.device)
    qk = qk[r_t].cpu().numpy()
    sk = sk.reshape(-1)[r_t].cpu().numpy()
    xr = x[r_t].float().cpu().numpy()
    q_ref, _, _ = O.rot_quant_reference(xr, L["pairs"].cpu().numpy(), L["theta"].float().cpu().numpy(),
                                        L["channel_scales"].float().cpu().numpy())
    _code_check(qk, q_ref)
    codes, zeros, scales = awq_columns(L, cols)
    ref = O.w4a8_linear(qk, sk, codes, zeros, scales)
    got = y[r_t][:, torch.from_numpy(cols).to(y.device)].float().cpu().numpy()
    if y.dtype == torch.float32:
        assert rel_l2(got, ref) <= 1e-6
    else:
        assert rel_l2(got, O.round_to_bf16(ref)) <= 1e-3


def test_config0_against_reference_golden(ops):
    import hashlib
    from alpamayo_b200.quantization import RotateLinearInt4
    d = np.load(os.path.join(GOLD, "cfg0_m16_k3584.npz"))
    W = torch.randn(3584, 3584, generator=torch.Generator().manual_seed(32)) * 0.02
    assert hashlib.sha256(W.numpy().tobytes()).hexdigest() == str(d["W_sha256"])
    lin = torch.nn.Linear(3584, 3584, bias=False)
    with torch.no_grad():
        lin.weight.copy_(W)
    m = RotateLinearInt4.from_linear(lin, torch.from_numpy(d["theta"]), torch.from_numpy(d["pairs"]),
                                     torch.from_numpy(d["channel_scales"]), rotate_weight=True, init_only=False)
    assert hashlib.sha256(m.qlinear.qweight.numpy().tobytes()).hexdigest() == str(d["qweight_sha256"])
    m = m.cuda()
    x = torch.from_numpy(d["x"]).cuda()
    y = m(x)
    assert y.dtype == torch.float32 and y.shape == (16, 3584)
    # codes: the reference's CPU path quantises the float32 rotation (the
    # golden's codes), its GPU path the rotation rounded to fp16 as its
    # rotate kernel stores it (what the module's forward does)
    q32, _ = m.rotation.quantize_activations(x, fp16_round=False)
    _code_check(q32.cpu().numpy(), d["xq"])
    q, s = m.rotation.quantize_activations(x)
    q16_ref, _ = O.per_token_quant_int8(O.round_to_fp16(d["x_rotated"]))
    _code_check(q.cpu().numpy(), q16_ref)
    yy = y.cpu().numpy()
    # against the golden output, the like-for-like route: quantise the
    # float32 rotation, as the reference's CPU path does (the fp16-rounded
    # route quantises differently, so its int8 noise differs by ~3e-3)
    y_cpu_route = ops.linear_w4a8(x, m.rotation.rot_table(), m.rotation.channel_scales.reshape(-1).half(),
                                  m.qlinear.packed(), 3584, None, False, torch.float32)
    assert rel_l2(y_cpu_route.cpu().numpy(), d["y"]) <= 1e-3
    # given the kernel's codes, the exact GEMM
    codes = O.unpack_wqlinear_qweight(m.qlinear.qweight.cpu().numpy(), 3584, 3584)
    zeros = O.recover_zeros(d["scales"], d["scaled_zeros"], 3584, 3584)
    ref = O.w4a8_linear(q.cpu().numpy(), s.cpu().numpy().reshape(-1), codes, zeros, d["scales"][:28].astype(np.float32))
    assert rel_l2(yy, ref) <= 1e-6


@pytest.mark.parametrize("name", list(SHAPES))
def test_config2_prefill_m8192(ops, name):
    from alpamayo_b200 import synthetic as syn
    N, K = SHAPES[name]
    M = 8192
    L = syn.make_layer(N, K, seed=90 + K + N, checkpoint=False, keep_awq=True)
    x = syn.make_activations(M, K, seed=91 + N)
    y = ops.linear_w4a8(x, L["rot_table"], L["cs_vec"], L["packed"], N, None, True, torch.bfloat16)
    rng = np.random.default_rng(N + K)
    rows = np.sort(rng.choice(M, size=64, replace=False))
    cols = np.sort(rng.choice(N, size=256, replace=False))
    _sampled_parity(ops, L, x, y, rows, cols)
    del y, x, L
    torch.cuda.empty_cache()


def test_config4_column_shards_reassemble_to_the_full_linear(ops):
    from alpamayo_b200 import synthetic as syn
    from alpamayo_b200.ops import packed_weight_bytes
    from alpamayo_b200.stack import ColumnShardedLinear, column_shard
    M, N, K = 16384, 37888, 3584
    L = syn.make_layer(N, K, seed=700, checkpoint=False, keep_awq=True)
    x = syn.make_activations(M, K, seed=701)
    full = ops.linear_w4a8(x, L["rot_table"], L["cs_vec"], L["packed"], N, None, True, torch.bfloat16)
    per_block = packed_weight_bytes(16, K)   # bytes of one 16-row block's records
    for world in (2, 8):
        blocks = []
        for rank in range(world):
            c0, c1 = column_shard(N, rank, world)
            shard = L["packed"][c0 // 16 * per_block:c1 // 16 * per_block]
            blocks.append(ops.linear_w4a8(x, L["rot_table"], L["cs_vec"], shard, c1 - c0, None, True,
                                          torch.bfloat16))
        got = ColumnShardedLinear.assemble(torch.stack(blocks))
        assert torch.equal(got, full), world
        del blocks, got
    rng = np.random.default_rng(4)
    rows = np.sort(rng.choice(M, size=64, replace=False))
    cols = np.sort(rng.choice(N, size=256, replace=False))
    _sampled_parity(ops, L, x, full, rows, cols)
    del full, x, L
    torch.cuda.empty_cache()


@pytest.mark.parametrize("M", [8, 64])
def test_config3_two_layers_against_composed_oracle(ops, M):
    """Each step of two decoder layers against the oracle on the same input
    (per-step parity; a free-running comparison would compound the allowed
    1-LSB code flips), and the step-by-step output equals DecoderStack's."""
    from alpamayo_b200 import synthetic as syn
    from alpamayo_b200.stack import HEAD_DIM, HEADS, DecoderStack, linear
    st = DecoderStack(layers=2, seed=3, keep=True)
    x = syn.make_activations(M, 3584, seed=5)
    rng = np.random.default_rng(M)
    rows = np.arange(M)
    f = lambda t: t.float().cpu().numpy()  # noqa: E731

    def lin(L, a):
        y = linear(L, a)
        cols = np.sort(rng.choice(L["N"], size=256, replace=False))
        _sampled_parity(ops, L, a, y, rows, cols)
        return y

    res, mlp_out = None, x
    for L in st.layers:
        h, res_new = ops.add_rmsnorm(mlp_out, res, L["in_norm"], st.eps)
        h_ref, s_ref = O.add_rmsnorm(f(mlp_out), None if res is None else f(res), f(L["in_norm"]), st.eps)
        assert np.array_equal(f(res_new), s_ref)
        assert rel_l2(f(h), h_ref) <= 2e-3
        res = res_new
        qkv = lin(L["qkv"], h)
        attn = qkv[:, :HEADS * HEAD_DIM].contiguous()
        o = lin(L["o"], attn)
        h, res_new = ops.add_rmsnorm(o, res, L["post_norm"], st.eps)
        h_ref, s_ref = O.add_rmsnorm(f(o), f(res), f(L["post_norm"]), st.eps)
        assert np.array_equal(f(res_new), s_ref)
        assert rel_l2(f(h), h_ref) <= 2e-3
        res = res_new
        gu = lin(L["gate_up"], h)
        a = ops.silu_mul(gu)
        assert rel_l2(f(a), O.silu_mul(f(gu))) <= 2e-3
        mlp_out = lin(L["down"], a)
    out, _ = ops.add_rmsnorm(mlp_out, res, st.final_norm, st.eps)
    assert torch.equal(out, st.forward(x))
