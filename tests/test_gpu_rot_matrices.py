"""Rotation tables carrying each group's rotation matrix (built once at load
time, paro_prepare_rotation_matrices) against tables without them.

The prefill rotation (tensor-core path for bf16 rows, from
paro_rotq_int8_workspace_size tokens on) loads the matrix instead of
building it in every CTA.  The load-time kernel runs the same build code,
so every output must be bit-identical with and without the matrices; the
matrices themselves are the composed Givens layers of the oracle (float32
chain; the kernels take sin / cos from the fast hardware approximation, so
entries agree to 1e-5)."""
import numpy as np
import pytest
import torch

from oracle import paro_oracle as O
from tests.helpers import make_activations, make_rotation

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    import alpamayo_b200.ops as ops
    return ops


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def tables(ops, K, seed):
    pairs, theta, cs = make_rotation(K, seed=seed)
    plain = ops.prepare_rotation(dev(pairs), dev(theta), 128)
    full = ops.prepare_rotation(dev(pairs), dev(theta), 128, matrices=True)
    return pairs, theta, cs, plain, full


@pytest.mark.parametrize("K", [256, 3584])
def test_table_layout_and_matrices(ops, K):
    pairs, theta, cs, plain, full = tables(ops, K, seed=K)
    assert tuple(full.shape) == (136, K) and full.dtype == torch.int32
    p = plain.cpu().numpy().view(np.uint32)
    f = full.cpu().numpy().view(np.uint32)
    # rows 0-7: the table's words, with the matrices flag (bit 15) in word 0
    assert p[0, 0] & 0x8000 == 0 and f[0, 0] & 0x8000
    f8 = f[:8].copy()
    f8[0, 0] &= ~np.uint32(0x8000)
    assert np.array_equal(f8, p)
    # rows 8-135: R_g, element (n, k) at g*16384 + ((k/8)*128 + n)*8 + k%8
    G = K // 128
    m = f[8:].reshape(-1).view(np.float32).reshape(G, 16, 128, 8)   # [g][k/8][n][k%8]
    R = m.transpose(0, 2, 1, 3).reshape(G, 128, 128)                 # [g][n][k]
    eye = np.zeros((128, K), np.float32)
    for g in range(G):
        eye[np.arange(128), g * 128 + np.arange(128)] = 1.0
    cols = O.rotate_activations(eye, pairs, theta.astype(np.float32), None)   # [k][g*128 + n] = R_g[n][k]
    R_ref = cols.reshape(128, G, 128).transpose(1, 2, 0)
    assert np.abs(R - R_ref).max() <= 1e-5
    # orthogonal to float32 accuracy
    for g in range(G):
        assert np.abs(R[g] @ R[g].T - np.eye(128)).max() <= 1e-5


@pytest.mark.parametrize("M,K,scaled", [(512, 1024, True), (1000, 3584, True), (777, 3584, False),
                                        (2048, 18944, True), (8192, 3584, True)])
def test_prefill_codes_bit_identical_with_matrices(ops, M, K, scaled):
    pairs, theta, cs, plain, full = tables(ops, K, seed=M + K)
    x = torch.from_numpy(make_activations(M, K, seed=M)).to(torch.bfloat16).cuda()
    csd = dev(cs.reshape(-1)) if scaled else None
    q0, s0 = ops.rotq_int8(x, plain, csd, 128, True)
    q1, s1 = ops.rotq_int8(x, full, csd, 128, True)
    assert torch.equal(q0, q1) and torch.equal(s0, s1)
    # and within the code tolerance of the oracle on sampled rows
    rows = np.sort(np.random.default_rng(M).choice(M, size=24, replace=False))
    q_ref, s_ref, _ = O.rot_quant_reference(x.float().cpu().numpy()[rows], pairs, theta.astype(np.float32),
                                            (cs if scaled else np.ones_like(cs)).astype(np.float32))
    d = np.abs(q1.cpu().numpy()[rows].astype(np.int32) - q_ref.astype(np.int32))
    assert d.max() <= 1 and (d > 0).mean() <= 1e-3


@pytest.mark.parametrize("M", [1, 8, 64, 600])
def test_linear_bit_identical_with_matrices(ops, M):
    """Decode sizes ignore the matrices; prefill sizes load them."""
    from alpamayo_b200 import synthetic as syn
    from alpamayo_b200.stack import serving_layer
    L = serving_layer(4608, 3584, seed=11)
    assert L["rot_table"].shape[0] == 136
    plain = L["rot_table"][:8].clone()
    plain[0, 0] = plain[0, 0] & ~0x8000
    x = syn.make_activations(M, 3584, seed=M)
    y0 = ops.linear_w4a8(x, plain, L["cs_vec"], L["packed"], 4608, None, True, torch.bfloat16)
    y1 = ops.linear_w4a8(x, L["rot_table"], L["cs_vec"], L["packed"], 4608, None, True, torch.bfloat16)
    assert torch.equal(y0, y1)


def test_prepare_rotation_matrices_rejects(ops):
    with pytest.raises(RuntimeError):
        ops._ops.prepare_rotation_matrices(torch.zeros(4, 256, dtype=torch.int32, device="cuda"))
    with pytest.raises(RuntimeError):
        ops._ops.prepare_rotation_matrices(torch.zeros(8, 200, dtype=torch.int32, device="cuda"))


@pytest.mark.parametrize("M,K", [(512, 1024), (1000, 3584), (2047, 3584), (4100, 18944), (8192, 3584)])
def test_single_pass_quantiser_equals_two_pass(ops, M, K):
    """bf16 prefill rows: where every group's CTA fits the GPU at once the
    quantiser runs inside the tensor-core rotation kernel (row maxima
    exchanged between the groups' CTAs per 128-row tile); with int8 rows
    that are not 16-byte aligned the fp16 rows go through the workspace and
    a second kernel.  Same fp16 values, same quantiser arithmetic: the
    codes and scales must be equal bit for bit."""
    from alpamayo_b200 import _native
    L = _native.capi()
    pairs, theta, cs, plain, full = tables(ops, K, seed=3 * M + K)
    x = torch.from_numpy(make_activations(M, K, seed=M)).to(torch.bfloat16).cuda()
    x[3] = 0   # an all-zero row: absmax clamps to 1e-10
    csd = dev(cs.reshape(-1))
    wsb = L.paro_rotq_int8_workspace_size(M, K, 1)
    assert wsb > 0
    ws = torch.empty(wsb + 256, dtype=torch.uint8, device="cuda")
    wsp = (ws.data_ptr() + 255) // 256 * 256
    stream = torch.cuda.current_stream().cuda_stream
    outs = []
    for off in (0, 8):
        qb = torch.empty(M * K + 16, dtype=torch.int8, device="cuda")
        s = torch.empty(M, dtype=torch.float32, device="cuda")
        st = L.paro_rotq_int8_ws(x.data_ptr(), 2, M, K, csd.data_ptr(), full.data_ptr(), 8, 128, 1,
                                 qb.data_ptr() + off, s.data_ptr(), wsp, wsb, stream)
        assert st == 0
        torch.cuda.synchronize()
        outs.append((qb[off:off + M * K].view(M, K).clone(), s.clone()))
    assert ops.device_error_word() == 0
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
    assert outs[0][0][3].abs().max().item() == 0
    # the torch operator takes the single-pass mode
    q, s = ops.rotq_int8(x, full, csd, 128, True)
    assert torch.equal(q, outs[0][0]) and torch.equal(s.reshape(-1), outs[0][1])


def test_single_pass_quantiser_ties_round_half_away(ops):
    """Zero angles (R = I) and unit channel scales: the rotated rows are the
    inputs, so rows built from half-integers put exact ties under the
    quantiser (row maxima 127 and 63.5: 127/a = 1 and 2).  Codes must be the
    oracle's round-half-away codes bit for bit, in both the single-pass and
    the two-pass mode."""
    from alpamayo_b200 import _native
    L = _native.capi()
    M, K = 512, 1024
    pairs, theta, _ = make_rotation(K, seed=5)
    theta = np.zeros_like(theta)
    table = ops.prepare_rotation(dev(pairs), dev(theta), 128, matrices=True)
    x = make_activations(M, K, seed=6)
    ties = np.array([127, 2.5, -3.5, 0.5, -0.5, 1.5, 126.5, -126.5, 4.5, -0.0, 63.5, -62.5], np.float32)
    x[0, :] = 0
    x[0, :len(ties)] = ties
    x[1, :] = 0
    x[1, :len(ties)] = ties / 2          # a = 63.5: inv = 2, ties again
    x[2, 700:712] = ties                 # in another group
    xt = torch.from_numpy(x).to(torch.bfloat16)
    assert torch.equal(xt[:2].float(), torch.from_numpy(x[:2]))   # exact in bf16
    assert torch.equal(xt[2, 700:712].float(), torch.from_numpy(ties))
    q_ref, s_ref = O.per_token_quant_int8(O.round_to_fp16(xt.float().numpy()))
    assert q_ref[0, :8].tolist() == [127, 3, -4, 1, -1, 2, 127, -127]
    wsb = L.paro_rotq_int8_workspace_size(M, K, 1)
    ws = torch.empty(wsb + 256, dtype=torch.uint8, device="cuda")
    wsp = (ws.data_ptr() + 255) // 256 * 256
    xd = xt.cuda()
    for off in (0, 8):
        qb = torch.empty(M * K + 16, dtype=torch.int8, device="cuda")
        s = torch.empty(M, dtype=torch.float32, device="cuda")
        st = L.paro_rotq_int8_ws(xd.data_ptr(), 2, M, K, None, table.data_ptr(), 8, 128, 1, qb.data_ptr() + off,
                                 s.data_ptr(), wsp, wsb, torch.cuda.current_stream().cuda_stream)
        assert st == 0
        torch.cuda.synchronize()
        q = qb[off:off + M * K].view(M, K).cpu().numpy()
        assert np.array_equal(q, q_ref), f"offset {off}: {np.argwhere(q != q_ref)[:5]}"
        assert np.array_equal(s.cpu().numpy(), s_ref.reshape(-1))


def test_wide_layer_takes_the_two_pass_path(ops):
    """K = 20480: 160 groups, more than the GPU has SMs, so the single-pass
    kernel cannot have every group's CTA resident and the fp16 rows go
    through the workspace and a second kernel.  Codes bit-identical with and
    without the matrices, within the code tolerance of the oracle."""
    M, K = 600, 20480
    pairs, theta, cs, plain, full = tables(ops, K, seed=9)
    x = torch.from_numpy(make_activations(M, K, seed=10)).to(torch.bfloat16).cuda()
    csd = dev(cs.reshape(-1))
    q0, s0 = ops.rotq_int8(x, plain, csd, 128, True)
    q1, s1 = ops.rotq_int8(x, full, csd, 128, True)
    assert ops.device_error_word() == 0
    assert torch.equal(q0, q1) and torch.equal(s0, s1)
    rows = np.sort(np.random.default_rng(K).choice(M, size=16, replace=False))
    q_ref, s_ref, _ = O.rot_quant_reference(x.float().cpu().numpy()[rows], pairs, theta.astype(np.float32),
                                            cs.astype(np.float32))
    d = np.abs(q1.cpu().numpy()[rows].astype(np.int32) - q_ref.astype(np.int32))
    assert d.max() <= 1 and (d > 0).mean() <= 1e-3
    assert np.allclose(s1.cpu().numpy().reshape(-1)[rows], s_ref, rtol=2 ** -10, atol=0)
