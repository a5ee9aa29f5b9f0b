"""Activation-side kernels against the CPU oracle (which is pinned bit-exact
to the reference's own rotation in test_oracle.py).

Tolerances (north_star): int8 activation codes may differ from the
reference's by at most 1 LSB on at most 0.1% of elements; per-token scales
follow from the same absolute maximum.
"""
import os

import numpy as np
import pytest
import torch

from oracle import paro_oracle as O
from tests.helpers import make_activations, make_rotation

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
CODE_LSB_FRAC = 1e-3


@pytest.fixture(scope="module")
def ops():
    import alpamayo_b200.ops as ops
    return ops


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t.to(dtype) if dtype is not None else t


def check_codes(q, q_ref, s, s_ref):
    q = q.astype(np.int32)
    d = np.abs(q - q_ref.astype(np.int32))
    assert d.max() <= 1, f"code difference {d.max()} LSB"
    frac = (d > 0).mean()
    assert frac <= CODE_LSB_FRAC, f"{frac:.2e} of codes differ"
    assert np.allclose(s, s_ref, rtol=2 ** -10, atol=0)
    return frac


@pytest.mark.parametrize("name", ["rot_m16_k1024.npz", "rot_m4_k3584.npz"])
def test_rotate_matches_reference_golden_fp32(ops, name):
    d = np.load(os.path.join(GOLD, name))
    out = ops.rotate(dev(d["x"]), dev(d["pairs"]), dev(d["theta"]), dev(d["channel_scales"]), 128)
    out = out.cpu().numpy()
    ref = d["rotated"]
    # float32 chain; the device uses __sincosf like the reference's kernel
    assert np.abs(out - ref).max() <= 2e-5 * np.abs(ref).max()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_rotate_half_types_round_like_reference(ops, dtype):
    d = np.load(os.path.join(GOLD, "rot_m16_k1024.npz"))
    x = torch.from_numpy(d["x"]).to(dtype)
    theta = torch.from_numpy(d["theta"]).to(dtype)
    cs = torch.from_numpy(d["channel_scales"]).to(dtype)
    out = ops.rotate(x.cuda(), dev(d["pairs"]), theta.cuda(), cs.cuda(), 128).float().cpu().numpy()
    ref = O.rotate_activations(x.float().numpy(), d["pairs"], theta.float().numpy(), cs.float().numpy())
    ref = torch.from_numpy(ref).to(dtype).float().numpy()
    ulp = 2 ** -10 if dtype == torch.float16 else 2 ** -7
    diff = np.abs(out - ref)
    assert (diff > 0).mean() < 0.01
    # one ulp of the element, or float32-chain noise relative to the row
    assert (diff <= ulp * np.abs(ref) + 1e-5 * np.abs(ref).max(axis=1, keepdims=True)).all()


@pytest.mark.parametrize("krot,group", [(1, 128), (2, 128), (4, 128), (16, 128), (8, 64), (2, 64)])
def test_rotate_krot_group_variants(ops, krot, group):
    rng = np.random.default_rng(krot * 10 + group)
    K, M = 512, 7
    G = K // group
    pairs = np.stack([np.concatenate([rng.permutation(group) for _ in range(G)]) for _ in range(krot)]).astype(np.int16)
    theta = ((rng.random((krot, K // 2)) * 2 - 1) * np.pi).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    out = ops.rotate(dev(x), dev(pairs), dev(theta), None, group).cpu().numpy()
    ref = O.rotate_activations(x, pairs, theta, None, group_size=group)
    assert np.abs(out - ref).max() <= 2e-5 * np.abs(ref).max()


@pytest.mark.parametrize("M,K,xdt", [(1, 3584, torch.bfloat16), (4, 3584, torch.bfloat16),
                                     (8, 18944, torch.bfloat16), (37, 1024, torch.float16),
                                     (64, 3584, torch.bfloat16), (16, 2048, torch.float32),
                                     (300, 3584, torch.bfloat16)])
def test_rotq_int8_matches_reference_chain(ops, M, K, xdt):
    pairs, theta, cs = make_rotation(K, seed=M + K)
    x = make_activations(M, K, seed=7 * M + K)
    xt = torch.from_numpy(x).to(xdt)
    pu8 = ops.prepare_rotation(dev(pairs), dev(theta), 128)
    q, s = ops.rotq_int8(xt.cuda(), pu8, dev(cs.reshape(-1)), 128, True)
    q_ref, s_ref, _ = O.rot_quant_reference(xt.float().numpy(), pairs, theta.astype(np.float32),
                                            cs.astype(np.float32))
    assert tuple(q.shape) == (M, K) and tuple(s.shape) == (M, 1)
    check_codes(q.cpu().numpy(), q_ref, s.cpu().numpy().reshape(-1), s_ref)


def test_rotq_int8_golden_fixture(ops):
    d = np.load(os.path.join(GOLD, "rot_m4_k3584.npz"))
    pu8 = ops.prepare_rotation(dev(d["pairs"]), dev(d["theta"]), 128)
    q, s = ops.rotq_int8(dev(d["x"]), pu8, dev(d["channel_scales"].reshape(-1)), 128, True)
    # reference chain: its rotation (fixture), fp16 store, vLLM int8 quant
    q_ref, s_ref = O.per_token_quant_int8(O.round_to_fp16(d["rotated"]))
    check_codes(q.cpu().numpy(), q_ref, s.cpu().numpy().reshape(-1), s_ref)


def test_rotq_int8_without_fp16_rounding(ops):
    M, K = 16, 1024
    pairs, theta, cs = make_rotation(K, seed=3)
    x = make_activations(M, K, seed=4)
    pu8 = ops.prepare_rotation(dev(pairs), dev(theta), 128)
    q, s = ops.rotq_int8(dev(x), pu8, dev(cs.reshape(-1)), 128, False)
    q_ref, s_ref, _ = O.rot_quant_reference(x, pairs, theta.astype(np.float32), cs.astype(np.float32),
                                            fp16_intermediate=False)
    check_codes(q.cpu().numpy(), q_ref, s.cpu().numpy().reshape(-1), s_ref)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_quant_int8_bit_exact(ops, dtype):
    x = make_activations(33, 3584, seed=9)
    x[3] = 0.0  # all-zero row: absmax clamps to 1e-10
    x[5, :8] = np.array([127, 0.5, -0.5, 1.5, -2.5, 63.25, -126.5, 0], dtype=np.float32)
    x[5, 8:] = 0
    xt = torch.from_numpy(x).to(dtype)
    q, s = ops.per_token_quant_int8(xt.cuda())
    q_ref, s_ref = O.per_token_quant_int8(xt.float().numpy())
    assert np.array_equal(q.cpu().numpy(), q_ref)
    assert np.array_equal(s.cpu().numpy().reshape(-1), s_ref)
    assert q[5, :8].tolist() == [127, 1, -1, 2, -3, 63, -127, 0]


def expected_rot_table(pairs, theta):
    """Per-channel table restated from the pair list: partner channel, role
    bit (second element of its pair), fp16 angle bits of the pair."""
    L, K = pairs.shape
    out = np.zeros((L, K), dtype=np.uint32)
    tb = theta.view(np.uint16).astype(np.uint32)
    for l in range(L):
        for g in range(K // 128):
            blk = pairs[l, g * 128:(g + 1) * 128].astype(np.int64)
            for t in range(128):
                v, w = blk[t], blk[t ^ 1]
                out[l, g * 128 + v] = w | ((t & 1) << 7) | (tb[l, g * 64 + t // 2] << 16)
    return out.view(np.int32)


def check_exchange_slots(table):
    """Bits 8-14 of each (layer, group) block: a permutation of the 128 slots
    in which warp w's channels (32w .. 32w+31) write 32 different banks
    (slot % 32) and the partners of warp w's channels, which warp w reads,
    also sit in 32 different banks."""
    u = table.view(np.uint32)
    L, K = u.shape
    for l in range(L):
        for g in range(K // 128):
            blk = u[l, g * 128:(g + 1) * 128]
            slot = ((blk >> 8) & 0x7F).astype(np.int64)
            partner = (blk & 0x7F).astype(np.int64)
            assert sorted(slot) == list(range(128)), (l, g)
            for w in range(4):
                chans = np.arange(32 * w, 32 * w + 32)
                assert len(set(slot[chans] % 32)) == 32, (l, g, w)
                assert len(set(slot[partner[chans]] % 32)) == 32, (l, g, w)


def test_prepare_rotation_table_and_rejects_overlapping_pairs(ops):
    pairs, theta, _ = make_rotation(256, seed=1)
    ok = ops.prepare_rotation(dev(pairs), dev(theta), 128).cpu().numpy()
    # partner, role and angle bits as restated from the pair list; the
    # exchange slots (bits 8-14) by their defining property
    assert np.array_equal(ok.view(np.uint32) & 0xFFFF80FF, expected_rot_table(pairs, theta).view(np.uint32))
    check_exchange_slots(ok)
    pairs[2, 130] = pairs[2, 131]
    with pytest.raises(RuntimeError, match="not permutations"):
        ops.prepare_rotation(dev(pairs), dev(theta), 128)


def test_exchange_slots_for_checkpoint_like_pairings(ops):
    """Slots for several random pairings, including ones that pair channels
    only within a warp and only across warps."""
    for seed in range(4):
        pairs, theta, _ = make_rotation(512, seed=10 + seed)
        check_exchange_slots(ops.prepare_rotation(dev(pairs), dev(theta), 128).cpu().numpy())
    pairs, theta, _ = make_rotation(128, seed=3)
    ident = np.tile(np.arange(128, dtype=pairs.dtype), (pairs.shape[0], 1))   # pairs (2i, 2i+1): same warp
    check_exchange_slots(ops.prepare_rotation(dev(ident), dev(theta), 128).cpu().numpy())
    cross = np.tile(np.stack([np.arange(64), np.arange(64) + 64], 1).reshape(-1).astype(pairs.dtype),
                    (pairs.shape[0], 1))   # pairs (i, i + 64): always another warp
    check_exchange_slots(ops.prepare_rotation(dev(cross), dev(theta), 128).cpu().numpy())


def test_empty_batch(ops):
    pairs, theta, cs = make_rotation(256, seed=1)
    pu8 = ops.prepare_rotation(dev(pairs), dev(theta), 128)
    q, s = ops.rotq_int8(torch.zeros(0, 256, device="cuda", dtype=torch.bfloat16), pu8, dev(cs.reshape(-1)), 128,
                         True)
    assert q.shape == (0, 256) and s.shape == (0, 1)


def test_leading_batch_dims(ops):
    pairs, theta, cs = make_rotation(512, seed=2)
    x = make_activations(6, 512, seed=3).reshape(2, 3, 512)
    pu8 = ops.prepare_rotation(dev(pairs), dev(theta), 128)
    q, s = ops.rotq_int8(dev(x, torch.bfloat16), pu8, dev(cs.reshape(-1)), 128, True)
    assert q.shape == (2, 3, 512) and s.shape == (2, 3, 1)
    q2, s2 = ops.rotq_int8(dev(x.reshape(6, 512), torch.bfloat16), pu8, dev(cs.reshape(-1)), 128, True)
    assert torch.equal(q.reshape(6, 512), q2) and torch.equal(s.reshape(6, 1), s2)


@pytest.mark.parametrize("M", [1, 2, 3, 5, 8, 9, 17])
def test_rotq_ragged_rows_and_large_k(ops, M):
    """Row counts that do not fill a cluster's row block, at the down_proj K
    (several groups per thread)."""
    K = 18944
    pairs, theta, cs = make_rotation(K, seed=M)
    x = make_activations(M, K, seed=M + 1)
    xt = torch.from_numpy(x).to(torch.bfloat16)
    table = ops.prepare_rotation(dev(pairs), dev(theta), 128)
    q, s = ops.rotq_int8(xt.cuda(), table, dev(cs.reshape(-1)), 128, True)
    q_ref, s_ref, _ = O.rot_quant_reference(xt.float().numpy(), pairs, theta.astype(np.float32),
                                            cs.astype(np.float32))
    check_codes(q.cpu().numpy(), q_ref, s.cpu().numpy().reshape(-1), s_ref)


@pytest.mark.parametrize("M,K,xdt", [(512, 1024, torch.bfloat16), (700, 3584, torch.bfloat16),
                                     (1030, 18944, torch.bfloat16), (600, 640, torch.float16),
                                     (520, 256, torch.float32)])
def test_rotq_two_pass_path_matches_fused_kernel_and_oracle(ops, M, K, xdt):
    """Prefill sizes run the two-pass path (rotation into an fp16 workspace,
    then quantisation).  For fp16 / fp32 rows the rotation does the cluster
    kernel's arithmetic on packed row pairs, so its codes match the
    single-pass kernel's (C ABI without workspace) up to a handful of 1-LSB
    flips per million.  bf16 rows are rotated on the tensor cores as one
    matrix per group (bf16 hi + lo split of the composed rotation), whose
    rounding differs from the layer-by-layer chain by about 2^-16 relative:
    their codes are held to the code tolerance.  Both are checked against
    the oracle on sampled rows within the code tolerance."""
    from alpamayo_b200 import _native
    L = _native.capi()
    assert L.paro_rotq_int8_workspace_size(M, K, 1) > 0
    pairs, theta, cs = make_rotation(K, seed=M + K)
    x = make_activations(M, K, seed=M)
    xt = torch.from_numpy(x).to(xdt).cuda()
    table = ops.prepare_rotation(dev(pairs), dev(theta), 128)
    csd = dev(cs.reshape(-1))
    q, s = ops.rotq_int8(xt, table, csd, 128, True)          # two-pass path
    q1 = torch.empty_like(q)
    s1 = torch.empty_like(s)
    code = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}[xdt]
    st = L.paro_rotq_int8(xt.data_ptr(), code, M, K, csd.data_ptr(), table.data_ptr(), 8, 128, 1,
                          q1.data_ptr(), s1.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert st == 0
    torch.cuda.synchronize()
    check_codes(q.cpu().numpy(), q1.cpu().numpy(), s.cpu().numpy().reshape(-1), s1.cpu().numpy().reshape(-1))
    if xdt != torch.bfloat16:
        assert (q.int() - q1.int()).abs().gt(0).float().mean().item() <= 1e-5
    rows = np.sort(np.random.default_rng(M).choice(M, size=48, replace=False))
    q_ref, s_ref, _ = O.rot_quant_reference(xt.float().cpu().numpy()[rows], pairs, theta.astype(np.float32),
                                            cs.astype(np.float32))
    check_codes(q.cpu().numpy()[rows], q_ref, s.cpu().numpy().reshape(-1)[rows], s_ref)


@pytest.mark.parametrize("M,K,with_res", [(1, 3584, True), (64, 3584, False), (7, 18944, True)])
def test_add_rmsnorm_against_oracle(ops, M, K, with_res):
    rng = np.random.default_rng(M + K)
    x = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).to(torch.bfloat16)
    r = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).to(torch.bfloat16) if with_res else None
    w = torch.from_numpy((0.9 + 0.2 * rng.random(K)).astype(np.float32)).to(torch.bfloat16)
    y, s = ops.add_rmsnorm(x.cuda(), None if r is None else r.cuda(), w.cuda(), 1e-6)
    y_ref, s_ref = O.add_rmsnorm(x.float().numpy(), None if r is None else r.float().numpy(), w.float().numpy())
    assert np.array_equal(s.float().cpu().numpy(), s_ref)
    d = np.abs(y.float().cpu().numpy() - y_ref)
    # summation order and rsqrt may move a value across a bf16 rounding boundary
    assert (d > 0).mean() <= 1e-2 and d.max() <= 2 ** -6 * np.abs(y_ref).max()


@pytest.mark.parametrize("M,I", [(1, 18944), (37, 1024)])
def test_silu_mul_against_oracle(ops, M, I):
    rng = np.random.default_rng(M)
    x = torch.from_numpy((3 * rng.standard_normal((M, 2 * I))).astype(np.float32)).to(torch.bfloat16)
    y = ops.silu_mul(x.cuda()).float().cpu().numpy()
    ref = O.silu_mul(x.float().numpy())
    d = np.abs(y - ref)
    assert (d > 0).mean() <= 1e-3 and d.max() <= 2 ** -7 * np.abs(ref).max()
