"""This build against the reference's own GPU path on the same B200.

The reference's rotate kernel is compiled from its source for sm_100a
(oracle/build_ref.py -> oracle/_ref/librotation_ref.so); its quantiser and
GEMM are vLLM's per_token_quant_int8 and marlin_gemm, driven as the
reference's MarlinW4A8Linear drives them (oracle/ref_gpu.py).  Skipped, with
the reason, where the prebuilt reference kernel or vLLM's ops are not
available.

Tolerances:
  * rotation::rotate (fp16 and fp32 in/out): bit-identical to the
    reference's kernel (same fast-math angle functions, same rounding of
    both products and the sum);
  * int8 activation codes: within 1 LSB on at most 0.1 % of elements; token
    scales within 1e-3 relative (one fp16 step of the row's maximum);
  * outputs: this build's float32 output against Marlin's fp16 output (its
    group scales requantised to int16 with a global factor, about 1e-4
    relative, then fp16 rounding) within 1e-3 relative L2.  The two bf16
    outputs are not compared to that bound: rounding nearly equal values
    to bf16 independently already moves them by about 1e-3.
"""
import numpy as np
import pytest
import torch

from tests.helpers import rel_l2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def R():
    from oracle import ref_gpu
    rot_ok, marlin_ok, why = ref_gpu.available()
    if not rot_ok:
        pytest.skip(f"reference rotate kernel unavailable: {why}")
    return ref_gpu


@pytest.fixture(scope="module")
def ops():
    import alpamayo_b200.ops as ops
    return ops


@pytest.mark.parametrize("M,K", [(1, 3584), (8, 3584), (300, 3584), (8, 18944), (2048, 1024)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_rotate_bit_identical_to_reference_kernel(R, ops, M, K, dtype):
    from alpamayo_b200 import synthetic as syn
    pairs, theta, cs = syn.make_rotation(K, seed=K + M)
    x = syn.make_activations(M, K, seed=M, dtype=dtype)
    rot = R.load_rotate()
    th = theta.to(dtype)
    c = cs.to(dtype)
    y_ref = rot(x, pairs, th, c, 128)
    y = ops.rotate(x, pairs, th, c, 128)
    assert torch.equal(y, y_ref)
    # without channel scales
    assert torch.equal(ops.rotate(x, pairs, th, None, 128), rot(x, pairs, th, None, 128))


@pytest.mark.parametrize("name,N,K", [("qkv", 4608, 3584), ("down", 3584, 18944)])
@pytest.mark.parametrize("M", [1, 8, 64, 2048])
def test_linear_against_reference_marlin_path(R, ops, name, N, K, M):
    _, marlin_ok, why = R.available()
    if not marlin_ok:
        pytest.skip(f"vLLM Marlin unavailable: {why}")
    from alpamayo_b200 import synthetic as syn
    L = syn.make_layer(N, K, seed=5 + N, checkpoint=False, keep_awq=True)
    ref = R.ReferenceLinear(L["pairs"], L["theta"], L["channel_scales"], L["awq_qweight"], L["awq_scales"],
                            L["awq_qzeros"], K, N)
    x = syn.make_activations(M, K, seed=M + 3)
    # activation codes: vLLM's quantiser on the reference's fp16 rotation
    qr, sr = ref.quantised(x)
    qo, so = ops.rotq_int8(x, L["rot_table"], L["cs_vec"], 128, True)
    dq = (qr.int() - qo.int()).abs()
    assert dq.max().item() <= 1 and (dq > 0).float().mean().item() <= 1e-3
    # token scales: a row's scale follows its largest fp16 value, which the
    # tensor-core rotation of prefill sizes can round one step apart
    so_, sr_ = so.reshape(-1).cpu().numpy(), sr.reshape(-1).cpu().numpy()
    assert np.max(np.abs(so_ - sr_) / sr_) <= 1e-3
    # outputs: Marlin's fp16 result against this build's float32 result
    y_marlin = ref.marlin(ref.rotated(x)).float().cpu().numpy()
    y32 = ops.linear_w4a8(x, L["rot_table"], L["cs_vec"], L["packed"], N, None, True, torch.float32)
    assert rel_l2(y32.cpu().numpy(), y_marlin) <= 1e-3
    # the whole reference chain (bf16 in and out) stays at bf16 rounding
    y_ref = ref(x).float().cpu().numpy()
    y = ops.linear_w4a8(x, L["rot_table"], L["cs_vec"], L["packed"], N, None, True, torch.bfloat16)
    assert rel_l2(y.float().cpu().numpy(), y_ref) <= 3e-3
    assert np.isfinite(y_ref).all()
