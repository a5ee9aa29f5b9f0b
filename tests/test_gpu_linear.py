"""paro_w4a8_linear (torch.ops.paro_b200.linear_w4a8): the whole rotated
linear.  Up to 64 tokens it is three chained kernels: a rotation kernel
(fp16 rows + row maxima), a quantiser (int8 codes in the GEMM's fragment
order + code sums + token scales) and the GEMM; the tests hold it to the
activation-kernel route (paro_rotq_int8 + paro_w4a8_gemm) and to the
oracle.

Tolerances: the two routes compute the same int8 codes and int32 group sums;
only the order of float32 additions across CTAs may differ, so float32
outputs agree to 1e-6 relative L2.  Against the oracle: activation codes
within 1 LSB on at most 0.1 % of elements, and, given the codes, bf16
outputs within 1e-3 relative L2 (north_star).  (One flipped code of a short
row moves that row's outputs by about 1e-3 by itself, so the output bound
is checked on the kernels' own codes.)
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import paro_oracle as O
from tests.helpers import make_activations, make_quantized_layer, rel_l2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    import alpamayo_b200.ops as ops
    return ops


def synthetic_layer(N, K, seed):
    from alpamayo_b200 import synthetic as syn
    return syn.make_layer(N, K, seed=seed, checkpoint=False)


def two_kernel(ops, x, L, N, out_dtype):
    q, s = ops.rotq_int8(x, L["rot_table"], L["cs_vec"], 128, True)
    return ops.w4a8_gemm(q, s, L["packed"], N, None, out_dtype)


@pytest.mark.parametrize("M", [1, 3, 8, 9, 16, 37, 64])
@pytest.mark.parametrize("N,K", [(512, 1024), (4608, 3584)])
def test_linear_matches_two_kernel_route(ops, M, N, K):
    L = synthetic_layer(N, K, seed=M + N)
    from alpamayo_b200 import synthetic as syn
    x = syn.make_activations(M, K, seed=M)
    y = ops.linear_w4a8(x, L["rot_table"], L["cs_vec"], L["packed"], N, None, True, torch.float32)
    y2 = two_kernel(ops, x, L, N, torch.float32)
    assert rel_l2(y.cpu().numpy(), y2.cpu().numpy()) <= 1e-6


@pytest.mark.parametrize("M,N,K", [(1, 3584, 18944), (3, 3584, 18944), (8, 3584, 18944), (4, 37888, 3584),
                                   (16, 37888, 3584), (20, 37888, 3584), (64, 256, 18944), (40, 37888, 3584),
                                   (48, 3584, 18944)])
def test_linear_large_shapes(ops, M, N, K):
    """down_proj / gate_up decode shapes: quantised rows staged in shared
    memory (down at 1 and 3 tokens; gate_up at 4, 16 and 20 tokens: one, two
    and four token tiles), read from L2 where they do not fit (down at 8
    tokens), and the tensor-core GEMM behind the same rotation + quantiser
    chain below 65 tokens: gate_up at 40 tokens, down at 48, and K = 18944
    at 64 tokens on one tile (split-K)."""
    L = synthetic_layer(N, K, seed=K + M)
    from alpamayo_b200 import synthetic as syn
    x = syn.make_activations(M, K, seed=M + 1)
    y = ops.linear_w4a8(x, L["rot_table"], L["cs_vec"], L["packed"], N, None, True, torch.float32)
    y2 = two_kernel(ops, x, L, N, torch.float32)
    assert rel_l2(y.cpu().numpy(), y2.cpu().numpy()) <= 1e-6


@pytest.mark.parametrize("M", [2, 8, 40])
def test_linear_against_oracle(ops, M):
    from alpamayo_b200.quantization import RotateLinearInt4
    N, K = 256, 2048
    d = make_quantized_layer(N, K, seed=M)
    m = RotateLinearInt4(K, N, False, torch.float16)
    m.load_state_dict({"rotation.theta": torch.from_numpy(d["theta"]), "rotation.pairs": torch.from_numpy(d["pairs"]),
                       "rotation.channel_scales": torch.from_numpy(d["channel_scales"]),
                       "qlinear.qweight": torch.from_numpy(d["qweight"]),
                       "qlinear.scales": torch.from_numpy(d["wq_scales"]),
                       "qlinear.scaled_zeros": torch.from_numpy(d["wq_scaled_zeros"])})
    m = m.cuda()
    x = torch.from_numpy(make_activations(M, K, seed=M + 5)).to(torch.bfloat16)
    y = m(x.cuda()).float().cpu().numpy()
    # the activation codes the kernels compute (the linear's rotation and
    # quantisation are the activation kernel's, operation for operation)
    # against the oracle's: the code tolerance
    qk, sk = ops.rotq_int8(x.cuda(), m.rotation.rot_table(), m.rotation.channel_scales.reshape(-1).cuda(), 128, True)
    qk, sk = qk.cpu().numpy(), sk.cpu().numpy().reshape(-1)
    q, s, _ = O.rot_quant_reference(x.float().numpy(), d["pairs"], d["theta"].astype(np.float32),
                                    d["channel_scales"].astype(np.float32))
    dq = np.abs(qk.astype(np.int32) - q.astype(np.int32))
    assert dq.max() <= 1 and (dq > 0).mean() <= 1e-3
    # given those codes, the output is the oracle's GEMM rounded to bf16
    ref = O.w4a8_linear(qk, sk, d["codes"], d["zeros_gn"], d["scales_gn"])
    assert rel_l2(y, O.round_to_bf16(ref)) <= 1e-3


def test_linear_c_abi_leaves_workspace_zero(ops):
    """Through the C ABI with an explicit zero-filled workspace: several
    calls of different shapes and routes in a row (streaming GEMM; the
    tensor-core GEMM behind the decode chain, with and without split-K; the
    two-kernel path with split-K), the workspace is all zero after each, and
    repeated calls give the same output bit for bit."""
    from alpamayo_b200 import _native
    from alpamayo_b200 import synthetic as syn
    Lc = _native.capi()
    shapes = [(8, 4608, 3584), (1, 512, 1024), (37, 4608, 3584), (48, 3584, 18944), (40, 37888, 3584),
              (100, 4608, 3584), (8, 4608, 3584), (48, 3584, 18944), (100, 4608, 3584)]
    layers = {(N, K): synthetic_layer(N, K, seed=N + K) for (_, N, K) in shapes}
    wsb = max(Lc.paro_w4a8_linear_workspace_size(M, N, K) for (M, N, K) in shapes)
    scb = max(Lc.paro_w4a8_linear_scratch_size(M, N, K, 1) for (M, N, K) in shapes)
    ws = torch.zeros(wsb, dtype=torch.uint8, device="cuda")
    sc = torch.empty(scb, dtype=torch.uint8, device="cuda")
    first = {}
    for (M, N, K) in shapes:
        L = layers[(N, K)]
        x = syn.make_activations(M, K, seed=M + K)
        y = torch.empty(M, N, dtype=torch.float32, device="cuda")
        st = Lc.paro_w4a8_linear(x.data_ptr(), 2, M, K, N, L["cs_vec"].data_ptr(), L["rot_table"].data_ptr(), 1,
                                 L["packed"].data_ptr(), None, 0, y.data_ptr(), 0, ws.data_ptr(), wsb,
                                 sc.data_ptr(), scb, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        assert st == 0, Lc.paro_status_string(st)
        torch.cuda.synchronize()
        assert torch.count_nonzero(ws).item() == 0
        if (M, N, K) in first:
            assert np.array_equal(y.cpu().numpy(), first[(M, N, K)])
        first[(M, N, K)] = y.cpu().numpy()
    assert Lc.paro_device_error_word(1) == 0


def test_linear_empty_batch(ops):
    L = synthetic_layer(256, 1024, seed=1)
    x = torch.empty(0, 1024, dtype=torch.bfloat16, device="cuda")
    y = ops.linear_w4a8(x, L["rot_table"], L["cs_vec"], L["packed"], 256, None, True, torch.bfloat16)
    assert y.shape == (0, 256)
