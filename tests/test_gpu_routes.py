"""The GEMM kernels held to the oracle and to one another through the
explicit-route entry point (paro_w4a8_gemm_route): the streaming decode
kernel, and the tensor-core kernel with 256- and 64-token tiles.

Tolerances (north_star): int32 group sums bit-exact on every route (single
group with unit scales, and power-of-two scales, make the fp32 output the
exact sum); fp32 outputs within 1e-6 relative L2 of the oracle's exact GEMM
on the same codes; bf16 / fp16 outputs within 1e-3 of the oracle rounded to
the dtype; the two tensor-core tiles bit-identical where neither splits K."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import paro_oracle as O
from tests.helpers import awq_columns, rel_l2

pytestmark = pytest.mark.gpu
STREAM, TC256, TC64 = 1, 2, 3
DT = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}   # paro_dtype


@pytest.fixture(scope="module")
def L():
    from alpamayo_b200._native import capi
    return capi()


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def gemm_route(L, route, xq, xs, packed, N, out_dtype=torch.float32, bias=None, check_ws=True):
    M, K = xq.shape
    out = torch.empty(M, N, dtype=out_dtype, device="cuda")
    wsb = L.paro_w4a8_gemm_route_workspace_size(route, M, N, K)
    ws = torch.zeros(max(wsb, 256), dtype=torch.uint8, device="cuda")
    st = L.paro_w4a8_gemm_route(route, xq.data_ptr(), xs.data_ptr(), M, N, K, packed.data_ptr(),
                                None if bias is None else bias.data_ptr(), DT[bias.dtype] if bias is not None else 0,
                                out.data_ptr(), DT[out_dtype], ws.data_ptr(), ws.numel(),
                                ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0, st
    torch.cuda.synchronize()
    if check_ws:
        assert int(ws.count_nonzero()) == 0, "workspace left non-zero"
    return out


def _unit_layer(ops, N, K, rng, pow2=False):
    codes = rng.integers(0, 16, (N, K))
    G = K // 128
    zeros = rng.integers(0, 16, (N, G)).astype(np.float32)
    scales = (np.tile(2.0 ** -np.arange(G, dtype=np.float32), (N, 1)) if pow2 else np.ones((N, G), np.float32))
    qw, s, sz = O.make_wqlinear_buffers(codes, scales, zeros)
    return codes, zeros, scales, ops.prepare_weights(dev(qw), dev(s), dev(sz), N, K)


@pytest.fixture(scope="module")
def ops():
    import alpamayo_b200.ops as ops
    return ops


@pytest.mark.parametrize("route,M", [(STREAM, 1), (STREAM, 33), (STREAM, 64), (TC256, 17), (TC256, 130),
                                     (TC64, 1), (TC64, 17), (TC64, 64), (TC64, 65), (TC64, 129), (TC64, 200)])
def test_single_group_sums_exact(L, ops, route, M):
    N, K = 512, 128
    rng = np.random.default_rng(M + 10 * route)
    codes, zeros, _, packed = _unit_layer(ops, N, K, rng)
    xq = rng.integers(-127, 128, (M, K)).astype(np.int8)
    y = gemm_route(L, route, dev(xq), dev(np.ones(M, np.float32)), packed, N).cpu().numpy().astype(np.int64)
    assert np.array_equal(y, O.group_partials(xq, codes, zeros.T)[:, :, 0])


@pytest.mark.parametrize("route,M", [(STREAM, 24), (TC256, 48), (TC64, 5), (TC64, 48), (TC64, 100)])
def test_power_of_two_scales_exact(L, ops, route, M):
    N, K = 768, 512
    rng = np.random.default_rng(7 * M + route)
    codes, zeros, scales, packed = _unit_layer(ops, N, K, rng, pow2=True)
    xq = rng.integers(-127, 128, (M, K)).astype(np.int8)
    y = gemm_route(L, route, dev(xq), dev(np.ones(M, np.float32)), packed, N).cpu().numpy()
    P = O.group_partials(xq, codes, zeros.T).astype(np.float64)      # [M, N, G]
    ref = (P * scales[None, :, :].astype(np.float64)).sum(-1)
    assert np.array_equal(y.astype(np.float64), ref)


SHAPES = {"qkv": (4608, 3584), "o_proj": (3584, 3584), "gate_up": (37888, 3584), "down": (3584, 18944)}


@pytest.mark.parametrize("name", list(SHAPES))
@pytest.mark.parametrize("M", [25, 48, 64, 96])
def test_tc64_against_oracle_on_baseline_shapes(L, ops, name, M):
    from alpamayo_b200 import synthetic as syn
    N, K = SHAPES[name]
    lay = syn.make_layer(N, K, seed=N + M, checkpoint=False, keep_awq=True)
    rng = np.random.default_rng(M)
    xq = rng.integers(-127, 128, (M, K)).astype(np.int8)
    xs = (rng.random(M).astype(np.float32) + 0.5) / 127
    y = gemm_route(L, TC64, dev(xq), dev(xs), lay["packed"], N)
    cols = np.sort(rng.choice(N, size=384, replace=False))
    codes, zeros, scales = awq_columns(lay, cols)
    ref = O.w4a8_linear(xq, xs, codes, zeros, scales)
    assert rel_l2(y[:, torch.from_numpy(cols).cuda()].cpu().numpy(), ref) <= 1e-6
    # bf16 with a bias, the dtype the model runs in
    bias = torch.randn(N, device="cuda").to(torch.bfloat16)
    yb = gemm_route(L, TC64, dev(xq), dev(xs), lay["packed"], N, torch.bfloat16, bias)
    refb = ref + bias.float().cpu().numpy()[cols]
    assert rel_l2(yb[:, torch.from_numpy(cols).cuda()].float().cpu().numpy(), O.round_to_bf16(refb)) <= 1e-3


@pytest.mark.parametrize("M", [33, 64, 128])
def test_tensor_core_tiles_bit_identical_when_unsplit(L, ops, M):
    """gate_up has 148 tiles of 256 rows, as many as CTA pairs on a B200 and
    more: neither tile splits K, and every output row folds the same group
    sums in the same order."""
    from alpamayo_b200 import synthetic as syn
    N, K = SHAPES["gate_up"]
    lay = syn.make_layer(N, K, seed=3, checkpoint=False)
    rng = np.random.default_rng(M)
    xq = dev(rng.integers(-127, 128, (M, K)).astype(np.int8))
    xs = dev((rng.random(M).astype(np.float32) + 0.5) / 127)
    if L.paro_w4a8_gemm_route_workspace_size(TC64, M, N, K) or L.paro_w4a8_gemm_route_workspace_size(TC256, M, N, K):
        pytest.skip("this GPU has more CTA pairs than gate_up tiles")
    for dt in (torch.float32, torch.bfloat16):
        a = gemm_route(L, TC64, xq, xs, lay["packed"], N, dt)
        b = gemm_route(L, TC256, xq, xs, lay["packed"], N, dt)
        assert torch.equal(a, b), dt


@pytest.mark.parametrize("M", [1, 31, 63, 97, 127])
def test_tc64_split_k_repeatable_and_ragged(L, ops, M):
    """Split-K partial sums meet in 64-bit fixed point, so two calls agree bit
    for bit; ragged token counts leave the rows past M untouched."""
    from alpamayo_b200 import synthetic as syn
    N, K = SHAPES["qkv"]
    lay = syn.make_layer(N, K, seed=11, checkpoint=False, keep_awq=True)
    assert L.paro_w4a8_gemm_route_workspace_size(TC64, M, N, K) > 0   # qkv: 18 tiles per 64 tokens, split-K
    rng = np.random.default_rng(M)
    xq = rng.integers(-127, 128, (M, K)).astype(np.int8)
    xs = (rng.random(M).astype(np.float32) + 0.5) / 127
    a = gemm_route(L, TC64, dev(xq), dev(xs), lay["packed"], N, torch.float16)
    b = gemm_route(L, TC64, dev(xq), dev(xs), lay["packed"], N, torch.float16)
    assert torch.equal(a, b)
    cols = np.sort(rng.choice(N, size=256, replace=False))
    codes, zeros, scales = awq_columns(lay, cols)
    ref = O.w4a8_linear(xq, xs, codes, zeros, scales)
    got = a[:, torch.from_numpy(cols).cuda()].float().cpu().numpy()
    assert rel_l2(got, O.round_to_fp16(ref)) <= 1e-3


def test_route_errors(L, ops):
    N, K, M = 256, 128, 65
    xq = torch.zeros(M, K, dtype=torch.int8, device="cuda")
    xs = torch.ones(M, device="cuda")
    packed = torch.zeros(ops.packed_weight_bytes(N, K), dtype=torch.uint8, device="cuda")
    out = torch.empty(M, N, device="cuda")
    ws = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    args = (xq.data_ptr(), xs.data_ptr(), M, N, K, packed.data_ptr(), None, 0, out.data_ptr(), 0, ws.data_ptr(),
            ws.numel(), s)
    assert L.paro_w4a8_gemm_route(9, *args) == 1           # PARO_ERR_INVALID_ARGUMENT
    assert L.paro_w4a8_gemm_route(STREAM, *args) == 8      # PARO_ERR_TOO_LARGE: M > 64
    assert L.paro_w4a8_gemm_route_workspace_size(STREAM, M, N, K) == 0
