"""The int4 x int8 GEMM and the weight preparation against the CPU oracle.

Tolerances (north_star): int32 per-group accumulation bit-exact given
identical codes; final bf16 / fp16 outputs within 1e-3 relative L2 of the
oracle's output rounded to the same dtype.
"""
import numpy as np
import pytest
import torch

from oracle import paro_oracle as O
from tests.helpers import expected_records, make_codes, rel_l2

pytestmark = pytest.mark.gpu
OUT_REL_L2 = 1e-3


@pytest.fixture(scope="module")
def ops():
    import alpamayo_b200.ops as ops
    return ops


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def prepared(ops, layer, N, K):
    return ops.prepare_weights(dev(layer["qweight"]), dev(layer["wq_scales"]), dev(layer["wq_scaled_zeros"]), N, K)


@pytest.mark.parametrize("N,K", [(16, 128), (64, 256), (256, 1024), (4608, 3584)])
def test_prepare_weights_bit_exact(ops, N, K):
    L = make_codes(N, K, seed=N + K)
    packed = prepared(ops, L, N, K).cpu().numpy()
    assert np.array_equal(packed, expected_records(L["codes"], L["scales_gn"], L["zeros_gn"]))


def test_prepare_weights_awq_matches_wqlinear_route(ops):
    from alpamayo_b200.quantization import wqlinear_to_awq
    N, K = 512, 1024
    L = make_codes(N, K, seed=5)
    awq = wqlinear_to_awq(torch.from_numpy(L["qweight"]), torch.from_numpy(L["wq_scales"]),
                          torch.from_numpy(L["wq_scaled_zeros"]), N, K, 128)
    a = ops.prepare_weights_awq(awq.qweight.cuda(), awq.scales.cuda(), awq.qzeros.cuda(), N, K)
    b = prepared(ops, L, N, K)
    assert torch.equal(a, b)


def _run(ops, xq, xs, packed, N, bias=None, out_dtype=torch.float32):
    return ops.w4a8_gemm(dev(xq), dev(xs.astype(np.float32)), packed, N,
                         None if bias is None else dev(bias), out_dtype)


@pytest.mark.parametrize("M", [1, 5, 8, 16, 64, 130])
def test_single_group_int32_exact(ops, M):
    """K = 128 (one group), scale 1, token scale 1: the fp32 output IS the
    int32 group partial sum."""
    N, K = 256, 128
    rng = np.random.default_rng(M)
    codes = rng.integers(0, 16, (N, K))
    zeros = rng.integers(0, 16, (N, 1)).astype(np.float32)
    ones = np.ones((N, 1), np.float32)
    qw, s, sz = O.make_wqlinear_buffers(codes, ones, zeros)
    packed = ops.prepare_weights(dev(qw), dev(s), dev(sz), N, K)
    xq = rng.integers(-127, 128, (M, K)).astype(np.int8)
    y = _run(ops, xq, np.ones(M), packed, N).cpu().numpy().astype(np.int64)
    P = O.group_partials(xq, codes, zeros.T)[:, :, 0]
    assert np.array_equal(y, P)


@pytest.mark.parametrize("M", [3, 8, 12, 256])
def test_multi_group_int32_exact_with_power_of_two_scales(ops, M):
    """Scales 2^-g keep every product and sum exact in fp32, so the output
    must equal the exact per-group partials combined (M <= 16: decode
    kernels, M = 256: prefill tensor-core kernel)."""
    N, K = 128, 512   # 18-bit partials x 2^-3 stay within fp32's 24 bits
    G = K // 128
    rng = np.random.default_rng(1)
    codes = rng.integers(0, 16, (N, K))
    zeros = rng.integers(0, 16, (N, G)).astype(np.float32)
    scales = np.tile(2.0 ** -np.arange(G), (N, 1)).astype(np.float32)
    qw, s, sz = O.make_wqlinear_buffers(codes, scales, zeros)
    packed = ops.prepare_weights(dev(qw), dev(s), dev(sz), N, K)
    xq = rng.integers(-127, 128, (M, K)).astype(np.int8)
    y = _run(ops, xq, np.ones(M), packed, N).cpu().numpy().astype(np.float64)
    P = O.group_partials(xq, codes, zeros.T).astype(np.float64)
    ref = (P * (2.0 ** -np.arange(G))[None, None, :]).sum(-1)
    assert np.array_equal(y, ref)


@pytest.mark.parametrize("M", [1, 3, 4, 8, 16, 33, 64, 100, 300])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16])
def test_gemm_matches_oracle(ops, M, out_dtype):
    N, K = 512, 2048
    L = make_codes(N, K, seed=M)
    packed = prepared(ops, L, N, K)
    rng = np.random.default_rng(M + 100)
    xq = rng.integers(-127, 128, (M, K)).astype(np.int8)
    xs = (rng.random(M) * 0.1 + 0.01).astype(np.float32)
    bias = (rng.standard_normal(N) * 0.1).astype(np.float16)
    y = _run(ops, xq, xs, packed, N, bias, out_dtype).float().cpu().numpy()
    ref = O.w4a8_linear(xq, xs, L["codes"], L["zeros_gn"], L["scales_gn"], bias=bias.astype(np.float32))
    ref_r = O.round_to_bf16(ref) if out_dtype == torch.bfloat16 else O.round_to_fp16(ref)
    assert rel_l2(y, ref_r) <= OUT_REL_L2
    # and fp32 output against the exact value
    y32 = _run(ops, xq, xs, packed, N, bias, torch.float32).cpu().numpy()
    assert rel_l2(y32, ref) <= 1e-6


def test_gemm_fp16_output_within_tolerance_of_marlin_semantics(ops):
    """Against the reference's Marlin contract (int16-requantised group scales
    with the global factor folded into the token scale, fp16 output)."""
    N, K, M = 1024, 3584, 8
    L = make_codes(N, K, seed=11)
    packed = prepared(ops, L, N, K)
    rng = np.random.default_rng(12)
    xq = rng.integers(-127, 128, (M, K)).astype(np.int8)
    xs = (rng.random(M) * 0.1 + 0.01).astype(np.float32)
    y = _run(ops, xq, xs, packed, N, None, torch.float16).float().cpu().numpy()
    ref_m = O.round_to_fp16(O.w4a8_linear(xq, xs, L["codes"], L["zeros_gn"], L["scales_gn"], variant="marlin"))
    assert rel_l2(y, ref_m) <= OUT_REL_L2


def records_layer(N, K, seed):
    """Random codes / fp16 scales / zero points written straight into the
    tile-record layout (the prepare kernel is checked separately)."""
    rng = np.random.default_rng(seed)
    G = K // 128
    codes = rng.integers(0, 16, (N, K), dtype=np.uint8)
    scales = (0.004 + 0.006 * rng.random((G, N))).astype(np.float16).astype(np.float32)
    zeros = rng.integers(0, 16, (G, N), dtype=np.uint8)
    return codes, scales, zeros, dev(expected_records(codes, scales, zeros))


@pytest.mark.parametrize("N,K", [(4608, 3584), (3584, 3584), (37888, 3584), (3584, 18944)])
@pytest.mark.parametrize("M", [1, 8])
def test_gemm_baseline_shapes(ops, N, K, M):
    codes, scales, zeros, packed = records_layer(N, K, seed=N // 16 + M)
    rng = np.random.default_rng(N + M)
    xq = rng.integers(-127, 128, (M, K)).astype(np.int8)
    xs = (rng.random(M) * 0.1 + 0.01).astype(np.float32)
    y = _run(ops, xq, xs, packed, N, None, torch.bfloat16).float().cpu().numpy()
    cols = np.sort(rng.choice(N, size=min(N, 768), replace=False))
    ref = O.round_to_bf16(O.w4a8_linear(xq, xs, codes[cols], zeros[:, cols], scales[:, cols]))
    assert rel_l2(y[:, cols], ref) <= OUT_REL_L2


def test_gemm_linearity_in_token_scale(ops):
    """Size-independent property: doubling a token's scale doubles its row."""
    N, K, M = 37888, 3584, 4
    _, _, _, packed = records_layer(N, K, seed=3)
    rng = np.random.default_rng(4)
    xq = rng.integers(-127, 128, (M, K)).astype(np.int8)
    xs = np.full(M, 0.01, np.float32)
    y1 = _run(ops, xq, xs, packed, N).cpu().numpy()
    y2 = _run(ops, xq, 2 * xs, packed, N).cpu().numpy()
    assert np.array_equal(2 * y1, y2)


@pytest.mark.parametrize("N,K,M", [(272, 256, 65), (512, 128, 129), (768, 1024, 300), (4608, 3584, 2048),
                                   (3584, 18944, 256), (37888, 3584, 160), (37888, 3584, 40), (4608, 3584, 65),
                                   (3584, 3584, 100), (3584, 18944, 16), (4608, 3584, 24), (37888, 3584, 17)])
def test_tensor_core_gemm_tiles_match_oracle(ops, N, K, M):
    """The tcgen05 kernel on the shapes paro_w4a8_gemm_path sends to it:
    full and partial 64- and 256-token x 256-row tiles, split-K and not,
    against the oracle on sampled rows and columns."""
    from alpamayo_b200 import _native
    assert _native.capi().paro_w4a8_gemm_path(M, N, K) == 1
    codes, scales, zeros, packed = records_layer(N, K, seed=N // 16 + K + M)
    rng = np.random.default_rng(N + K + M)
    xq = rng.integers(-127, 128, (M, K)).astype(np.int8)
    xs = (rng.random(M) * 0.1 + 0.01).astype(np.float32)
    bias = (rng.standard_normal(N) * 0.1).astype(np.float32)
    bias_bf = dev(bias).to(torch.bfloat16)
    rows = np.sort(rng.choice(M, size=min(M, 192), replace=False))
    cols = np.sort(rng.choice(N, size=min(N, 512), replace=False))
    ref = O.w4a8_linear(xq[rows], xs[rows], codes[cols], zeros[:, cols], scales[:, cols],
                        bias=bias_bf.float().cpu().numpy()[cols])
    y = ops.w4a8_gemm(dev(xq), dev(xs), packed, N, bias_bf, torch.bfloat16).float().cpu().numpy()
    assert rel_l2(y[rows][:, cols], O.round_to_bf16(ref)) <= OUT_REL_L2
    y32 = ops.w4a8_gemm(dev(xq), dev(xs), packed, N, bias_bf, torch.float32).cpu().numpy()
    assert rel_l2(y32[rows][:, cols], ref) <= 1e-6
    assert _native.capi().paro_device_error_word(1) == 0


@pytest.mark.parametrize("M,N,K", [(8, 1024, 18944), (65, 4608, 3584), (64, 256, 18944)])
def test_gemm_repeats_bit_for_bit(ops, M, N, K):
    """Partial sums that several CTAs add for one output (the streaming
    kernel's shared row blocks: 1024 x 18944 at 8 tokens spreads a row block
    over about three CTAs; the tensor-core kernel's split-K at 65 tokens and
    on a single tile) go through fixed-point integer adds, so the result does
    not depend on the order the CTAs finish in: two calls agree bit for bit."""
    codes, scales, zeros, packed = records_layer(N, K, seed=N // 16 + K + M)
    rng = np.random.default_rng(N + K + M)
    xq = rng.integers(-127, 128, (M, K)).astype(np.int8)
    xs = (rng.random(M) * 0.1 + 0.01).astype(np.float32)
    y1 = _run(ops, xq, xs, packed, N, None, torch.float32)
    y2 = _run(ops, xq, xs, packed, N, None, torch.float32)
    assert torch.equal(y1, y2)
    cols = np.sort(rng.choice(N, size=min(N, 256), replace=False))
    ref = O.w4a8_linear(xq, xs, codes[cols], zeros[:, cols], scales[:, cols])
    assert rel_l2(y1.cpu().numpy()[:, cols], ref) <= 1e-6
