"""The decode GEMM with one row block per consumer warp (gemm_rows_kernel,
up to 16 tokens; through PARO_ROUTE_ROWS, since no automatic choice uses it
by default) on the shapes that exercise each part of its schedule:
whole row blocks cut into pieces across warps (qkv-like: two row blocks per
CTA), stream-K segments shared with neighbouring CTAs and fixed up through
the workspace (down-like, and an odd group count), exactly one row block per
warp (gate_up-like), several rounds of 16 segments (short rows, many row
blocks), single-record CTAs with idle warps (K = 128), and one row block
for the whole layer.

Tolerances: against the oracle's exact value, fp32 outputs to 1e-6
relative L2 (float32 sums in a different order); two calls agree bit for
bit (shared partial sums are added as 64-bit fixed point); the workspace is
left zero-filled."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import paro_oracle as O
from tests.helpers import expected_records, rel_l2

pytestmark = pytest.mark.gpu

SHAPES = [(4608, 3584), (3584, 18944), (37888, 3584), (98304, 256), (592, 128), (16, 128), (1040, 2304)]


def _layer(N, K, seed):
    rng = np.random.default_rng(seed)
    G = K // 128
    codes = rng.integers(0, 16, (N, K), dtype=np.uint8)
    scales = (0.004 + 0.006 * rng.random((G, N))).astype(np.float16).astype(np.float32)
    zeros = rng.integers(0, 16, (G, N), dtype=np.uint8)
    packed = torch.from_numpy(expected_records(codes, scales, zeros)).cuda()
    return codes, scales, zeros, packed


@pytest.mark.parametrize("N,K", SHAPES)
@pytest.mark.parametrize("M", [1, 3, 8, 9, 16])
def test_rows_kernel_matches_oracle_and_repeats(N, K, M):
    from alpamayo_b200 import _native
    L = _native.capi()
    ROWS = 4   # PARO_ROUTE_ROWS: this kernel on every shape it handles
    codes, scales, zeros, packed = _layer(N, K, seed=N + K + M)
    rng = np.random.default_rng(N * 7 + M)
    xq = rng.integers(-127, 128, (M, K)).astype(np.int8)
    xs = (rng.random(M) * 0.1 + 0.01).astype(np.float32)
    bias = (rng.standard_normal(N) * 0.1).astype(np.float32)
    dq, ds, db = (torch.from_numpy(a).cuda() for a in (xq, xs, bias))
    wsb = L.paro_w4a8_gemm_route_workspace_size(ROWS, M, N, K)
    ws = torch.zeros(wsb, dtype=torch.uint8, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    outs = []
    for _ in range(2):
        y = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
        st = L.paro_w4a8_gemm_route(ROWS, dq.data_ptr(), ds.data_ptr(), M, N, K, packed.data_ptr(),
                                    db.data_ptr(), 0, y.data_ptr(), 0, ws.data_ptr(), wsb, stream)
        if st == 3:   # PARO_ERR_UNSUPPORTED: the staged token rows leave too few ring stages
            assert M > 8 or K > 4096, "one token tile of rows up to K = 4096 always fits"
            pytest.skip("token rows beyond the kernel's shared-memory plan")
        assert st == 0, L.paro_status_string(st)
        outs.append(y)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])
    assert torch.count_nonzero(ws).item() == 0
    assert L.paro_device_error_word(1) == 0
    cols = np.sort(rng.choice(N, size=min(N, 512), replace=False))
    ref = O.w4a8_linear(xq, xs, codes[cols], zeros[:, cols], scales[:, cols], bias=bias[cols])
    assert rel_l2(outs[0].cpu().numpy()[:, cols], ref) <= 1e-6
