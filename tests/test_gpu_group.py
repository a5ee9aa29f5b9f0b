"""Per-projection rotation tables for fused projections: a group of rotated
linears that read the same input, each with its own rotation (q / k / v,
gate / up as a real checkpoint holds them), run as one group
(paro_w4a8_linear_group, RotateLinearGroup) against the members run one by
one and concatenated.

Tolerances: each member's activation codes are its own table's, so the
group computes the same int32 group sums; the GEMM over the concatenated
weights splits the work differently across CTAs, so float32 outputs agree to
1e-6 relative L2 (bf16 to 1e-3); the fused residual output is bit-exact."""
import numpy as np
import pytest
import torch

from tests.helpers import rel_l2

pytestmark = pytest.mark.gpu


def _layers(ns, K, seed):
    from alpamayo_b200.stack import serving_layer
    return [serving_layer(n, K, seed=seed + i) for i, n in enumerate(ns)]


@pytest.mark.parametrize("ns", [(3584, 512, 512), (18944, 18944), (256, 4608)])
@pytest.mark.parametrize("M", [1, 8, 33, 64, 100])
def test_group_equals_members_concatenated(ns, M):
    import alpamayo_b200.ops as ops
    from alpamayo_b200 import synthetic as syn
    from alpamayo_b200.stack import linear
    K = 3584
    Ls = _layers(ns, K, seed=20 + M)
    packed = torch.cat([L["packed"] for L in Ls])
    x = syn.make_activations(M, K, seed=M)
    y, res = ops.linear_w4a8_group(x, [L["rot_table"] for L in Ls], [L["cs_vec"] for L in Ls], packed, ns,
                                   out_dtype=torch.float32)
    ref = torch.cat([linear(L, x, torch.float32) for L in Ls], dim=1)
    assert y.shape == (M, sum(ns)) and res is x
    assert rel_l2(y.cpu().numpy(), ref.cpu().numpy()) <= 1e-6
    # with the residual add + RMSNorm fused in front
    r = syn.make_activations(M, K, seed=M + 1)
    w = (0.9 + 0.2 * torch.rand(K, device="cuda")).to(torch.bfloat16)
    y2, res2 = ops.linear_w4a8_group(x, [L["rot_table"] for L in Ls], [L["cs_vec"] for L in Ls], packed, ns,
                                     prologue="add_rmsnorm", residual=r, norm_weight=w, out_dtype=torch.float32)
    h, res_ref = ops.add_rmsnorm(x, r, w, 1e-6)
    assert torch.equal(res2, res_ref)
    ref2 = torch.cat([linear(L, h, torch.float32) for L in Ls], dim=1)
    assert rel_l2(y2.cpu().numpy(), ref2.cpu().numpy()) <= 1e-6


def test_rotate_linear_group_module():
    """RotateLinearGroup over RotateLinearInt4 modules built by from_linear
    (own tables each), bf16 in and out, against the members' own forwards."""
    from alpamayo_b200.quantization import RotateLinearGroup, RotateLinearInt4
    g = torch.Generator().manual_seed(0)
    K = 1024
    mods = []
    for n in (512, 256, 256):
        pairs = torch.stack([torch.cat([torch.randperm(128, generator=g) for _ in range(K // 128)])
                             for _ in range(8)]).to(torch.int16)
        theta = ((torch.rand(8, K // 2, generator=g) * 2 - 1) * np.pi).to(torch.float16)
        cs = (0.5 + 1.5 * torch.rand(1, K, generator=g)).to(torch.float16)
        lin = torch.nn.Linear(K, n, bias=True)
        with torch.no_grad():
            lin.weight.copy_(torch.randn(n, K, generator=g) * 0.02)
            lin.bias.copy_(torch.randn(n, generator=g) * 0.1)
        mods.append(RotateLinearInt4.from_linear(lin, theta, pairs, cs, rotate_weight=True, init_only=False).cuda())
    grp = RotateLinearGroup(mods)
    assert grp.out_features == 1024 and grp.in_features == K
    for M in (1, 6, 200):
        x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
        y = grp(x, out_dtype=torch.float32)
        ref = torch.cat([m(x, out_dtype=torch.float32) for m in mods], dim=1)
        assert rel_l2(y.cpu().numpy(), ref.cpu().numpy()) <= 1e-6
        yb = grp(x)
        refb = torch.cat([m(x) for m in mods], dim=1)
        assert yb.dtype == torch.bfloat16 and rel_l2(yb.float().cpu().numpy(), refb.float().cpu().numpy()) <= 1e-3


def test_group_rejects_bad_arguments_on_the_host():
    import ctypes
    from alpamayo_b200 import _native
    L = _native.capi()
    n = (ctypes.c_int * 3)(512, 100, 512)   # 100 is not a multiple of 16
    assert L.paro_w4a8_linear_group_workspace_size(8, 3, n, 1024) == 0
    n5 = (ctypes.c_int * 5)(16, 16, 16, 16, 16)
    assert L.paro_w4a8_linear_group_workspace_size(8, 5, n5, 1024) == 0
