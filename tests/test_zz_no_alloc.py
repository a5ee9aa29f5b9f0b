"""paro_w4a8_gemm_noalloc (the allocation-free GEMM entry point) against
paro_w4a8_gemm, both called through the C ABI.

Kept in its own file, collected last, so it runs after every other test has
used the library as well as on its own.  Tolerance: the two entry points
run the same kernel with the same work split, and partial sums that cross
CTAs are added as 64-bit fixed point (order-independent), so the outputs
agree bit for bit, in every dtype, in both kernels' ranges.  The one
exception is a tensor-core shape whose split-K partial sums do not fit the
fixed array: it runs unsplit (the whole K range folded in float32
registers), so it agrees to float32 rounding (1e-5 relative L2 in fp32).
"""
import ctypes

import numpy as np
import pytest
import torch

from tests.helpers import expected_records, rel_l2

pytestmark = pytest.mark.gpu

PARO_OK = 0
PARO_ERR_TOO_LARGE = 8
SCRATCH_BYTES = 8 << 20
DT = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


@pytest.fixture(scope="module")
def L():
    from alpamayo_b200 import _native
    L = _native.capi()
    vp, i32, i64, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t
    L.paro_w4a8_gemm_noalloc.restype = i32
    L.paro_w4a8_gemm_noalloc.argtypes = [vp, vp, i64, i32, i32, vp, vp, i32, vp, i32, vp]
    return L


def _layer(N, K, M, seed):
    rng = np.random.default_rng(seed)
    G = K // 128
    codes = rng.integers(0, 16, (N, K), dtype=np.uint8)
    scales = (0.004 + 0.006 * rng.random((G, N))).astype(np.float16).astype(np.float32)
    zeros = rng.integers(0, 16, (G, N), dtype=np.uint8)
    packed = torch.from_numpy(expected_records(codes, scales, zeros)).cuda()
    xq = torch.from_numpy(rng.integers(-127, 128, (M, K)).astype(np.int8)).cuda()
    xs = torch.from_numpy((rng.random(M) * 0.1 + 0.01).astype(np.float32)).cuda()
    bias = torch.from_numpy((rng.standard_normal(N) * 0.1).astype(np.float16)).cuda()
    return dict(N=N, K=K, M=M, packed=packed, xq=xq, xs=xs, bias=bias)


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _with_workspace(L, c, out_dtype):
    M, N, K = c["M"], c["N"], c["K"]
    out = torch.empty(M, N, dtype=out_dtype, device="cuda")
    nbytes = L.paro_w4a8_gemm_workspace_size(M, N, K)
    ws = torch.zeros(max(nbytes, 1), dtype=torch.uint8, device="cuda")
    st = L.paro_w4a8_gemm(c["xq"].data_ptr(), c["xs"].data_ptr(), M, N, K, c["packed"].data_ptr(),
                          c["bias"].data_ptr(), DT[torch.float16], out.data_ptr(), DT[out_dtype], ws.data_ptr(),
                          nbytes, _stream())
    assert st == PARO_OK, L.paro_status_string(st)
    return out


def _noalloc(L, c, out_dtype):
    M, N, K = c["M"], c["N"], c["K"]
    out = torch.full((M, N), float("nan"), dtype=out_dtype, device="cuda")
    st = L.paro_w4a8_gemm_noalloc(c["xq"].data_ptr(), c["xs"].data_ptr(), M, N, K, c["packed"].data_ptr(),
                                  c["bias"].data_ptr(), DT[torch.float16], out.data_ptr(), DT[out_dtype], _stream())
    assert st == PARO_OK, L.paro_status_string(st)
    return out


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_noalloc_matches_workspace_entry_two_calls_in_a_row(L, out_dtype):
    # shapes alternating, so each call starts from the previous one's
    # leftovers in the shared array: two streaming-kernel shapes (one with
    # cross-CTA partial sums), a tensor-core shape with split-K through the
    # array (qkv at 65 tokens) and gate_up at 40 tokens (64-token tiles)
    cases = [_layer(3584, 3584, 8, seed=1), _layer(4608, 3584, 3, seed=2), _layer(4608, 3584, 65, seed=4),
             _layer(37888, 3584, 40, seed=5)]
    assert [L.paro_w4a8_gemm_path(c["M"], c["N"], c["K"]) for c in cases] == [0, 0, 1, 1]
    assert L.paro_w4a8_gemm_workspace_size(65, 4608, 3584) > 0   # split-K on that shape
    refs = [_with_workspace(L, c, out_dtype) for c in cases]
    for rep in range(2):
        for c, ref in zip(cases, refs):
            y = _noalloc(L, c, out_dtype)
            torch.cuda.synchronize()
            assert torch.isfinite(y).all()
            assert torch.equal(y, ref), (rep, c["M"], c["N"])
    assert L.paro_device_error_word(1) == 0


def test_noalloc_tensor_core_shape_beyond_the_array_runs_unsplit(L):
    # down at 400 tokens (256-token tiles, two splits): split-K would need
    # ~11.5 MB of partial sums
    M, N, K = 400, 3584, 18944
    assert L.paro_w4a8_gemm_path(M, N, K) == 1
    assert L.paro_w4a8_gemm_workspace_size(M, N, K) > SCRATCH_BYTES
    c = _layer(N, K, M, seed=6)
    ref = _with_workspace(L, c, torch.float32).cpu().numpy()
    for _ in range(2):
        y = _noalloc(L, c, torch.float32)
        torch.cuda.synchronize()
        y = y.cpu().numpy()
        assert np.isfinite(y).all()
        assert rel_l2(y, ref) <= 1e-5
    assert L.paro_device_error_word(1) == 0


def test_noalloc_rejects_shapes_beyond_its_scratch(L):
    M, N, K = 16, 98304, 256   # streaming-kernel range, needs ~12.6 MB > 8 MiB
    assert L.paro_w4a8_gemm_path(M, N, K) == 0
    assert L.paro_w4a8_gemm_workspace_size(M, N, K) > SCRATCH_BYTES
    c = _layer(N, K, M, seed=3)
    out = torch.zeros(M, N, dtype=torch.float32, device="cuda")
    st = L.paro_w4a8_gemm_noalloc(c["xq"].data_ptr(), c["xs"].data_ptr(), M, N, K, c["packed"].data_ptr(), None, 0,
                                  out.data_ptr(), DT[torch.float32], _stream())
    assert st == PARO_ERR_TOO_LARGE
    assert b"limit" in L.paro_status_string(st)
    torch.cuda.synchronize()
    assert torch.count_nonzero(out).item() == 0   # nothing was launched
