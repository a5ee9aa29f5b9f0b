"""The CPU oracle pinned against the reference's own outputs (golden
fixtures made by tests/golden/gen_golden.py from the reference's Python
functions) and against hand-checked known answers."""
import os

import numpy as np
import pytest

from oracle import paro_oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    return np.load(os.path.join(GOLD, name))


@pytest.mark.parametrize("name", ["rot_m16_k1024.npz", "rot_m4_k3584.npz"])
def test_rotation_matches_reference_bit_exact(name):
    d = load(name)
    r = O.rotate_activations(d["x"], d["pairs"], d["theta"].astype(np.float32),
                             d["channel_scales"].astype(np.float32))
    assert np.array_equal(r, d["rotated"])


@pytest.mark.parametrize("name", ["rot_m16_k1024.npz", "rot_m4_k3584.npz"])
def test_rotation_inverse_restores_scaled_input(name):
    d = load(name)
    xs = d["x"] * d["channel_scales"].astype(np.float32)
    # the reference's inverse (reverse layers, -theta) restores x*s
    assert np.allclose(d["unrotated"], xs, rtol=0, atol=2e-4 * np.abs(xs).max())
    back = d["rotated"].copy()
    th = d["theta"].astype(np.float32)
    for r in reversed(range(th.shape[0])):
        back = O.apply_rotation_step(back, d["pairs"][r], -th[r])
    assert np.array_equal(back, d["unrotated"])


def test_rotation_is_norm_preserving():
    d = load("rot_m16_k1024.npz")
    xs = d["x"] * d["channel_scales"].astype(np.float32)
    n0 = np.linalg.norm(xs.reshape(16, -1, 128), axis=-1)
    n1 = np.linalg.norm(d["rotated"].reshape(16, -1, 128), axis=-1)
    assert np.allclose(n0, n1, rtol=1e-5)


def test_weight_side_rotation_matches_reference():
    w = load("wq_n128_k1024.npz")
    wr = O.rotate_tensor_weight(w["W"], w["pairs"], w["theta"].astype(np.float32),
                                w["channel_scales"].astype(np.float32))
    assert np.array_equal(wr, w["w_rot"])


def test_rotation_identity_weight_times_activation():
    """<R(W/s), R(s*x)> = W.x : the transform the quantised path relies on."""
    w = load("wq_n128_k1024.npz")
    lhs = w["x_rotated"] @ w["w_rot"].T
    rhs = w["x"] @ w["W"].T
    assert np.allclose(lhs, rhs, rtol=1e-3, atol=1e-3 * np.abs(rhs).max())


def test_pseudo_quantize_matches_reference():
    w = load("wq_n128_k1024.npz")
    wdq, s, z, c = O.pseudo_quantize_tensor(w["w_rot"])
    assert np.array_equal(wdq, w["w_dq"])
    assert np.array_equal(s, w["pq_scales"]) and np.array_equal(z, w["pq_zeros"])
    assert np.array_equal(c, w["codes"])


def test_wqlinear_buffers_match_reference():
    w = load("wq_n128_k1024.npz")
    q, s, sz = O.make_wqlinear_buffers(w["codes"], w["pq_scales"], w["pq_zeros"])
    assert np.array_equal(q, w["qweight"])
    assert np.array_equal(s, w["wq_scales"]) and np.array_equal(sz, w["wq_scaled_zeros"])


def test_unpack_and_zero_recovery_match_reference():
    w = load("wq_n128_k1024.npz")
    assert np.array_equal(O.unpack_wqlinear_qweight(w["qweight"], 128, 1024), w["unpacked"])
    assert np.array_equal(O.recover_zeros(w["wq_scales"], w["wq_scaled_zeros"], 128, 1024), w["awq_zeros"])


def test_pack_unpack_round_trip_exact():
    rng = np.random.default_rng(5)
    for N, K in [(4, 128), (64, 256), (256, 3584)]:
        c = rng.integers(0, 16, (N, K))
        assert np.array_equal(O.unpack_wqlinear_qweight(O.pack_intweight(c), N, K), c)


def test_dequant_helpers_match_reference():
    w = load("wq_n128_k1024.npz")
    a = O.dequant_wqlinear(w["unpacked"], w["wq_scales"], w["wq_scaled_zeros"])[:32]
    b = O.dequant_awq(w["unpacked"], w["awq_zeros"], w["wq_scales"])[:32]
    assert np.array_equal(a, w["dequant_wqlinear"]) and np.array_equal(b, w["dequant_awq"])
    # the two dequantisations agree to fp16 rounding of -s*z
    assert np.abs(a - b).max() <= 1e-4


def test_marlin_scale_requantisation_matches_vllm():
    w = load("wq_n128_k1024.npz")
    s_i16, g = O.marlin_act_int8_process_scales(w["awq_scales"])
    assert np.array_equal(s_i16, w["marlin_s_i16"].astype(np.int64))
    assert np.float32(g) == w["marlin_global"]


def test_per_token_quant_known_answers():
    # absmax 127 -> unit multiplier; ties round away from zero
    x = np.array([[127.0, 0.5, -0.5, 1.5, -2.5, 63.49, -126.5, 0.0]], dtype=np.float32)
    q, s = O.per_token_quant_int8(x)
    assert q.tolist() == [[127, 1, -1, 2, -3, 63, -127, 0]]
    assert s[0] == np.float32(1.0)
    # all-zero row: absmax clamps to 1e-10, codes 0
    q, s = O.per_token_quant_int8(np.zeros((1, 16), np.float32))
    assert (q == 0).all() and s[0] == np.float32(1e-10) / np.float32(127)


def test_round_half_away_exact_near_half():
    # 0.49999997 + 0.5 rounds to 1.0 in float32; the oracle must not
    v = np.array([0.49999997, -0.49999997, 0.5, 2.5, -3.5, 126.5], dtype=np.float32)
    assert O.round_half_away(v).tolist() == [0.0, -0.0, 1.0, 3.0, -4.0, 127.0]


def test_group_partials_bounds_and_linearity():
    rng = np.random.default_rng(3)
    xq = rng.integers(-127, 128, (4, 256))
    codes = np.full((16, 256), 15)
    zeros = np.zeros((2, 16))
    P = O.group_partials(np.full((4, 256), 127), codes, zeros)
    assert P.max() == 128 * 15 * 127  # the int32 bound the kernels rely on
    P1 = O.group_partials(xq, codes, zeros)
    P2 = O.group_partials(2 * xq, codes, zeros)
    assert np.array_equal(P2, 2 * P1)


def test_validate_pairs():
    rng = np.random.default_rng(0)
    p = np.stack([rng.permutation(128) for _ in range(8)])
    assert O.validate_pairs(p)
    p[3, 5] = p[3, 6]
    assert not O.validate_pairs(p)


def test_bf16_rounding_matches_torch():
    import torch
    rng = np.random.default_rng(1)
    v = (rng.standard_normal(10000) * 100).astype(np.float32)
    t = torch.from_numpy(v).to(torch.bfloat16).float().numpy()
    assert np.array_equal(O.round_to_bf16(v), t)


def test_fake_quant_path_close_to_exact_linear():
    w = load("wq_n128_k1024.npz")
    wdq = O.dequant_awq(w["unpacked"], w["awq_zeros"], w["wq_scales"])
    y = O.fake_quant_linear(w["x"], w["pairs"], w["theta"].astype(np.float32),
                            w["channel_scales"].astype(np.float32), wdq)
    ref = w["x"] @ w["W"].T
    # int4 weights + int8 activations: a few percent of error against the
    # unquantised product
    assert np.linalg.norm(y - ref) / np.linalg.norm(ref) < 0.15


# ---------------------------------------------------------------------------
# configs[0] (M=16, K=N=3584) against the reference's own pipeline
# ---------------------------------------------------------------------------

def test_config0_activation_chain_matches_reference():
    """x * s -> 8 Givens layers -> per-token int8, at config-0 size, bit for
    bit against the reference's functions (cfg0_m16_k3584.npz)."""
    d = load("cfg0_m16_k3584.npz")
    th = d["theta"].astype(np.float32)
    cs = d["channel_scales"].astype(np.float32)
    r = O.rotate_activations(d["x"], d["pairs"], th, cs)
    assert np.array_equal(r, d["x_rotated"])
    q, s = O.per_token_quant_int8(r)
    assert np.array_equal(q, d["xq"])
    assert np.array_equal(s, d["xscale"])


def test_config0_fake_quant_output_matches_reference():
    """The fake-quant linear of the oracle and of the timed CPU port
    (oracle/cpu_baseline.py, the bench's CPU baseline and reference arm) on
    config 0 against the reference pipeline's output: both restate the same
    float32 arithmetic (the matmul's summation order is the BLAS's), so
    1e-6 relative L2 in float32, and the same bf16 values but for ties."""
    import torch
    from oracle import cpu_baseline as C
    from tests.helpers import rel_l2
    d = load("cfg0_m16_k3584.npz")
    th = d["theta"].astype(np.float32)
    cs = d["channel_scales"].astype(np.float32)
    codes, sc, sz = _cfg0_codes(d)
    w_dq = (codes.astype(np.float32) * np.repeat(sc, 128, axis=0).T.astype(np.float32)
            + np.repeat(sz, 128, axis=0).T.astype(np.float32))
    y_or = O.fake_quant_linear(d["x"], d["pairs"], th, cs, w_dq)
    assert rel_l2(y_or, d["y_bf16"]) <= 1e-3
    assert np.mean(y_or != d["y_bf16"]) <= 0.01
    y_cpu = C.fake_quant_linear(torch.from_numpy(d["x"]), torch.from_numpy(d["pairs"]), torch.from_numpy(th),
                                torch.from_numpy(cs), torch.from_numpy(w_dq)).float().numpy()
    assert rel_l2(y_cpu, d["y_bf16"]) <= 1e-3
    assert np.mean(y_cpu != d["y_bf16"]) <= 0.01
    # the port's activation half alone is the reference's bit for bit
    t = torch.from_numpy(d["x"]) * torch.from_numpy(cs)
    for r in range(8):
        t = C.apply_rotation_step(t, torch.from_numpy(d["pairs"][r]), torch.from_numpy(th[r]))
    assert np.array_equal(t.numpy(), d["x_rotated"])


def _cfg0_codes(d):
    """Config-0 weights regenerated by the oracle from the reference's seed
    (torch.randn, as gen_golden.py draws them), checked against the
    reference's hashes: W, then the int4 codes of the weight-side transform
    + pseudo-quantisation (clamped, as WQLinear.from_linear computes them
    from the fp16 weight)."""
    import hashlib
    import torch
    W = (torch.randn(3584, 3584, generator=torch.Generator().manual_seed(32)) * 0.02).numpy()
    assert hashlib.sha256(W.tobytes()).hexdigest() == str(d["W_sha256"])
    G = 28
    sc = d["scales"][:G].astype(np.float32)
    sz = d["scaled_zeros"][:G].astype(np.float32)
    from alpamayo_b200.quantization import RotateLinearInt4
    lin = torch.nn.Linear(3584, 3584, bias=False)
    with torch.no_grad():
        lin.weight.copy_(torch.from_numpy(W))
    m = RotateLinearInt4.from_linear(lin, torch.from_numpy(d["theta"]), torch.from_numpy(d["pairs"]),
                                     torch.from_numpy(d["channel_scales"]), rotate_weight=True, init_only=False)
    q = m.qlinear
    assert np.array_equal(q.scales.numpy(), d["scales"]) and np.array_equal(q.scaled_zeros.numpy(), d["scaled_zeros"])
    codes = O.unpack_wqlinear_qweight(q.qweight.numpy(), 3584, 3584)
    assert hashlib.sha256(np.ascontiguousarray(codes.astype(np.uint8)).tobytes()).hexdigest() == str(d["codes_sha256"])
    assert hashlib.sha256(q.qweight.numpy().tobytes()).hexdigest() == str(d["qweight_sha256"])
    return codes, sc, sz
