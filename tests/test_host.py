"""Host-side checks that need no GPU: the C-ABI library exports every entry
point declared in include/paro_b200.h, argument validation returns status
codes before any launch, and the Python API mirror reproduces the
reference's load-time conversions (against the golden fixtures)."""
import ctypes
import os
import re

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLD = os.path.join(ROOT, "tests", "golden")


def header_functions():
    src = open(os.path.join(ROOT, "include", "paro_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(paro_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    from alpamayo_b200._native import capi
    L = capi()
    names = header_functions()
    assert len(names) >= 12
    for n in names:
        assert hasattr(L, n), f"{n} declared in include/paro_b200.h but not exported"


def test_status_strings_and_version():
    from alpamayo_b200._native import capi
    L = capi()
    assert L.paro_version() >= 100
    assert L.paro_status_string(0) == b"ok"
    assert L.paro_status_string(6) == b"workspace too small"
    assert L.paro_packed_weight_bytes(3584, 3584) == (3584 // 16) * 28 * 1072
    assert L.paro_packed_weight_bytes(3585, 3584) == 0
    # the two-pass activation path: prefill sizes only, about 2 * M * K bytes
    assert L.paro_rotq_int8_workspace_size(8, 3584, 1) == 0
    assert L.paro_rotq_int8_workspace_size(4096, 3584, 0) == 0
    assert L.paro_rotq_int8_workspace_size(4096, 3584, 1) >= 2 * 4096 * 3584


def test_argument_validation_before_launch():
    """Invalid arguments are rejected on the host with a status code (no
    device work is attempted)."""
    from alpamayo_b200._native import capi
    L = capi()
    dummy = ctypes.c_void_p(16)
    # null x
    assert L.paro_rotate(None, 1, 4, 256, None, dummy, 1, dummy, 8, 128, dummy, None) == 1
    # K not a multiple of the group
    assert L.paro_rotate(dummy, 1, 4, 200, None, dummy, 1, dummy, 8, 128, dummy, None) == 2
    # unsupported krot / group
    assert L.paro_rotate(dummy, 1, 4, 256, None, dummy, 1, dummy, 3, 128, dummy, None) == 3
    assert L.paro_rotate(dummy, 1, 4, 256, None, dummy, 1, dummy, 8, 32, dummy, None) == 3
    # bad dtype
    assert L.paro_quant_int8(dummy, 7, 4, 256, dummy, dummy, None) == 3
    # fused kernel only for krot 8, group 128 (rotation_linear.py:18-19)
    assert L.paro_rotq_int8(dummy, 2, 4, 256, None, dummy, 4, 128, 1, dummy, dummy, None) == 3
    # the rotation table is only built for 128-channel groups
    assert L.paro_prepare_rotation(dummy, dummy, 8, 256, 64, dummy, dummy, None) == 3
    # table sizes with and without the per-group matrices (128 x 128 fp32
    # per 128 channels = 128 words per channel)
    assert L.paro_rotation_table_words(3584, 0) == 8 * 3584
    assert L.paro_rotation_table_words(3584, 1) == 136 * 3584
    assert L.paro_rotation_table_words(200, 1) == 0
    assert L.paro_prepare_rotation_matrices(None, 256, None) == 1
    assert L.paro_prepare_rotation_matrices(dummy, 200, None) == 2
    assert L.paro_prepare_rotation_matrices(ctypes.c_void_p(8), 256, None) == 4
    # GEMM shape checks
    assert L.paro_w4a8_gemm(dummy, dummy, 4, 100, 256, dummy, None, 0, dummy, 2, None, 0, None) == 2
    assert L.paro_w4a8_gemm(dummy, dummy, 4, 256, 200, dummy, None, 0, dummy, 2, None, 0, None) == 2
    # misaligned packed weights
    assert L.paro_w4a8_gemm(dummy, dummy, 4, 256, 256, ctypes.c_void_p(8), None, 0, dummy, 2, None, 0,
                            None) == 4
    assert L.paro_prepare_weights(dummy, dummy, dummy, 256, 256, 0, dummy, None) == 2  # G_pad < K/128
    # M == 0 is a no-op success
    assert L.paro_quant_int8(dummy, 2, 0, 256, dummy, dummy, None) == 0
    # explicit-route GEMM: unknown route, shape, misaligned weights, the
    # streaming kernel above 64 tokens and the row-block kernel above 16
    args = (dummy, dummy, 4, 256, 256, dummy, None, 0, dummy, 0, dummy, 1 << 20, None)
    assert L.paro_w4a8_gemm_route(9, *args) == 1
    assert L.paro_w4a8_gemm_route(3, dummy, dummy, 4, 100, 256, dummy, None, 0, dummy, 0, dummy, 1 << 20, None) == 2
    assert L.paro_w4a8_gemm_route(3, dummy, dummy, 4, 256, 256, ctypes.c_void_p(8), None, 0, dummy, 0, dummy,
                                  1 << 20, None) == 4
    assert L.paro_w4a8_gemm_route_workspace_size(1, 65, 256, 256) == 0
    assert L.paro_w4a8_gemm_route_workspace_size(4, 17, 256, 256) == 0
    assert L.paro_w4a8_gemm_route(3, dummy, dummy, 0, 256, 256, dummy, None, 0, dummy, 0, None, 0, None) == 0
    # multicast GEMM: null or misaligned destination, shape
    assert L.paro_w4a8_gemm_multicast(dummy, dummy, 4, 256, 256, dummy, None, 0, None, None) == 1
    assert L.paro_w4a8_gemm_multicast(dummy, dummy, 4, 256, 256, dummy, None, 0, ctypes.c_void_p(20), None) == 4
    assert L.paro_w4a8_gemm_multicast(dummy, dummy, 4, 100, 256, dummy, None, 0, dummy, None) == 2


def test_gemm_kernel_choice_by_shape():
    """The GEMM route is a pure function of the shape (host logic, no device
    work; the SM count falls back to 148 without a GPU): the streaming
    kernel for few tokens, the tensor-core kernel (64-token tiles) from 24
    tokens, from 13 on long rows (K >= 8192) and from 17 on layers with at
    least 0.8 x SMs 256-row tiles (gate_up: N = 37888), and always above 64;
    beyond 64 tokens its tile follows the cost estimate."""
    from alpamayo_b200._native import capi
    import torch
    L = capi()
    sms = torch.cuda.get_device_properties(0).multi_processor_count if torch.cuda.is_available() else 148
    wide = 37888 // 256 * 5 >= sms * 4
    assert L.paro_w4a8_gemm_path(8, 37888, 3584) == 0
    assert L.paro_w4a8_gemm_path(16, 37888, 3584) == 0
    assert L.paro_w4a8_gemm_path(17, 37888, 3584) == (1 if wide else 0)
    assert L.paro_w4a8_gemm_path(23, 4608, 3584) == 0
    assert L.paro_w4a8_gemm_path(24, 4608, 3584) == 1
    assert L.paro_w4a8_gemm_path(12, 3584, 18944) == 0
    assert L.paro_w4a8_gemm_path(13, 3584, 18944) == 1
    assert L.paro_w4a8_gemm_path(64, 3584, 3584) == 1
    assert L.paro_w4a8_gemm_path(65, 4608, 3584) == 1
    assert L.paro_w4a8_gemm_path(65, 100, 3584) == 0   # not a whole number of 16-row records
    if sms == 148:
        # the tile follows the estimate: a split-K 256-token tile for down at
        # 400 tokens (workspace), unsplit 64-token tiles at 300 (none)
        assert L.paro_w4a8_gemm_workspace_size(400, 3584, 18944) > 0
        assert L.paro_w4a8_gemm_workspace_size(300, 3584, 18944) == 0


def test_workspace_sizes_by_route():
    """Workspace sizes are host arithmetic (no device work; the SM count falls
    back to 148 without a GPU): the streaming kernel's [N][M] 64-bit
    fixed-point partial sums plus a counter per 16-row block; the tensor-core
    kernel's split-K sums ([M][N] 64-bit) plus 16 counters per tile (256 rows x
    64 or 256 tokens)
    when its tiles fill fewer than the CTA pairs, else nothing; the linear's
    at least what its route needs."""
    from alpamayo_b200._native import capi
    import torch
    L = capi()
    if torch.cuda.is_available() and torch.cuda.get_device_properties(0).multi_processor_count != 148:
        pytest.skip("sizes below assume 148 SMs")
    al = lambda b: (b + 255) // 256 * 256
    # streaming kernel (8 tokens): one token slice, N / 16 counters
    assert L.paro_w4a8_gemm_workspace_size(8, 3584, 3584) == al(3584 * 8 * 8) + (3584 // 16) * 4
    # tensor-core kernel with split-K: qkv at 65 tokens is 18 x 2 tiles of
    # 256 rows x 64 tokens < 74 pairs
    assert L.paro_w4a8_gemm_workspace_size(65, 4608, 3584) == al(65 * 4608 * 8) + 36 * 16 * 4
    # the explicit routes: 256-token tiles (18 tiles), the streaming kernel
    # only up to 64 tokens
    assert L.paro_w4a8_gemm_route_workspace_size(2, 65, 4608, 3584) == al(65 * 4608 * 8) + 18 * 16 * 4
    assert L.paro_w4a8_gemm_route_workspace_size(3, 65, 4608, 3584) == al(65 * 4608 * 8) + 36 * 16 * 4
    assert L.paro_w4a8_gemm_route_workspace_size(1, 65, 4608, 3584) == 0
    assert L.paro_w4a8_gemm_route_workspace_size(1, 8, 3584, 3584) == al(3584 * 8 * 8) + (3584 // 16) * 4
    assert L.paro_w4a8_gemm_route_workspace_size(0, 65, 4608, 3584) == L.paro_w4a8_gemm_workspace_size(65, 4608, 3584)
    # ... and without: 144 tiles at 2048 tokens fill the pairs
    assert L.paro_w4a8_gemm_workspace_size(2048, 4608, 3584) == 0
    # the linear for down at 64 tokens takes the tensor-core route (14 tiles)
    assert L.paro_w4a8_linear_workspace_size(64, 3584, 18944) >= al(64 * 3584 * 8) + 14 * 16 * 4


def test_header_has_reference_citations():
    src = open(os.path.join(ROOT, "include", "paro_b200.h")).read()
    for cite in ["rotation.cu:456-493", "int8_utils.py", "_custom_ops.py:1277-1318", "paroquant_marlin_w4a8.py"]:
        assert cite in src


def test_python_api_mirror_matches_reference_conversions():
    from alpamayo_b200.quantization import (calculate_zeros_width, pack_awq_int32, pack_intweight,
                                            unpack_wqlinear_qweight, wqlinear_to_awq, dequant_awq,
                                            dequant_wqlinear)
    w = np.load(os.path.join(GOLD, "wq_n128_k1024.npz"))
    codes = torch.from_numpy(w["codes"])
    assert torch.equal(pack_intweight(codes), torch.from_numpy(w["qweight"]))
    qw = torch.from_numpy(w["qweight"])
    assert torch.equal(unpack_wqlinear_qweight(qw, 128, 1024), torch.from_numpy(w["unpacked"]))
    awq = wqlinear_to_awq(qw, torch.from_numpy(w["wq_scales"]), torch.from_numpy(w["wq_scaled_zeros"]),
                          128, 1024, 128)
    assert torch.equal(awq.qweight, torch.from_numpy(w["awq_qweight"]))
    assert torch.equal(awq.qzeros, torch.from_numpy(w["awq_qzeros"]))
    assert torch.equal(awq.zeros, torch.from_numpy(w["awq_zeros"]))
    assert torch.equal(pack_awq_int32(awq.zeros), awq.qzeros)
    a = dequant_wqlinear(awq.int4_values, torch.from_numpy(w["wq_scales"]), torch.from_numpy(w["wq_scaled_zeros"]),
                         128)[:32]
    assert torch.equal(a, torch.from_numpy(w["dequant_wqlinear"]))
    b = dequant_awq(awq.int4_values, awq.zeros, awq.scales, 128)[:32]
    assert torch.equal(b, torch.from_numpy(w["dequant_awq"]))
    assert calculate_zeros_width(3584) * 8 == 32 and calculate_zeros_width(18944) * 8 == 152


def test_module_state_dict_keys_match_reference():
    from alpamayo_b200.quantization import RotateLinearInt4
    m = RotateLinearInt4(1024, 128, True, torch.float16)
    sd = m.state_dict()
    expect = {"rotation.theta": ((8, 512), torch.float16), "rotation.pairs": ((8, 1024), torch.int16),
              "rotation.channel_scales": ((1, 1024), torch.float16), "qlinear.qweight": ((32, 1024), torch.int16),
              "qlinear.scales": ((8, 128), torch.float16), "qlinear.scaled_zeros": ((8, 128), torch.float16),
              "qlinear.bias": ((128,), torch.float16)}
    assert set(sd) == set(expect)
    for k, (shape, dt) in expect.items():
        assert tuple(sd[k].shape) == shape and sd[k].dtype == dt, k
    assert m.buffer_name("rotation.pairs") is m.rotation.pairs
    with pytest.raises(ValueError):
        m.buffer_name("nope")


def test_rotation_rejects_unsupported_config():
    from alpamayo_b200.quantization import Rotation
    with pytest.raises(NotImplementedError):
        Rotation(256, krot=4)


def test_replace_and_wrap_on_fake_model():
    """Module surgery of the loader on a stand-in model with the Alpamayo
    layer path (model.vlm.model.language_model.layers)."""
    import torch.nn as nn
    from alpamayo_b200.quantization import RotateLinearInt4, replace_linears_with_rotate_linear
    from alpamayo_b200.quantization.paroquant_marlin_w4a8 import (_sanitise_channel_scales, _wrap_rotate_linears,
                                                                  BF16RotateLinearWrapper)

    class Attn(nn.Module):
        def __init__(self):
            super().__init__()
            self.q_proj = nn.Linear(256, 256, bias=False)
            self.lm_head = nn.Linear(256, 32, bias=False)

    class Layer(nn.Module):
        def __init__(self):
            super().__init__()
            self.self_attn = Attn()

    model = nn.Module()
    model.vlm = nn.Module()
    model.vlm.model = nn.Module()
    model.vlm.model.language_model = nn.Module()
    model.vlm.model.language_model.layers = nn.ModuleList([Layer(), Layer()])
    replace_linears_with_rotate_linear(model)
    layer0 = model.vlm.model.language_model.layers[0]
    assert isinstance(layer0.self_attn.q_proj, RotateLinearInt4)
    assert isinstance(layer0.self_attn.lm_head, nn.Linear)
    layer0.self_attn.q_proj.rotation.channel_scales[0, :3] = torch.tensor([float("inf"), float("nan"), 1e4])
    assert _sanitise_channel_scales(model) == 1
    cs = layer0.self_attn.q_proj.rotation.channel_scales
    assert torch.isfinite(cs).all() and cs.abs().max() <= 65504 / 128
    _wrap_rotate_linears(model)
    w = layer0.self_attn.q_proj
    assert isinstance(w, BF16RotateLinearWrapper) and w.in_features == 256


def test_selftest_wait_rejects_bad_limits_on_the_host():
    from alpamayo_b200._native import capi
    L = capi()
    assert L.paro_selftest_wait_timeout(0, None) == 1
    assert L.paro_selftest_wait_timeout(3_000_000_000, None) == 1


def test_device_error_recovery_resets_operator_workspaces(monkeypatch):
    """The documented recovery after a non-zero device error word: the
    operator workspaces are zero-filled again before the next call (fakes
    stand in for the two native libraries)."""
    import alpamayo_b200._native as N
    import alpamayo_b200.ops as ops
    calls = {"read": [], "reset": 0}
    word = {"v": 0}

    class FakeCapi:
        def paro_device_error_word(self, clear):
            calls["read"].append(clear)
            v = word["v"]
            if clear:
                word["v"] = 0
            return v

    class FakeShim:
        def paro_torch_reset_workspaces(self):
            calls["reset"] += 1
            return 3

    monkeypatch.setattr(N, "capi", lambda: FakeCapi())
    monkeypatch.setattr(N, "shim", lambda: FakeShim())
    assert ops.device_error_word() == 0 and calls["reset"] == 0   # clean: nothing reset
    word["v"] = 1
    assert ops.device_error_word() == 1 and calls["reset"] == 1   # timed-out wait: workspaces reset
    assert ops.device_error_word() == 0 and calls["reset"] == 1   # cleared by the read
    word["v"] = 2
    assert ops.device_error_word(clear=False) == 2 and calls["reset"] == 2
    assert calls["read"] == [1, 1, 1, 0]

    class BrokenShim:
        def paro_torch_reset_workspaces(self):
            return -1

    monkeypatch.setattr(N, "shim", lambda: BrokenShim())
    with pytest.raises(RuntimeError):
        ops.device_error_word()


# ---------------------------------------------------------------------------
# the product's offline quantisation helpers against the reference's outputs
# ---------------------------------------------------------------------------

def test_product_rotate_tensor_matches_reference_bit_exact():
    from alpamayo_b200.quantization import rotate_tensor
    d = np.load(os.path.join(GOLD, "wq_n128_k1024.npz"))
    w = rotate_tensor(torch.from_numpy(d["W"]), torch.from_numpy(d["theta"]), torch.from_numpy(d["pairs"]),
                      torch.from_numpy(d["channel_scales"]))
    assert np.array_equal(w.numpy(), d["w_rot"])


def test_product_pseudo_quantize_matches_reference_bit_exact():
    from alpamayo_b200.quantization import pseudo_quantize_tensor
    d = np.load(os.path.join(GOLD, "wq_n128_k1024.npz"))
    wq, s, z = pseudo_quantize_tensor(torch.from_numpy(d["w_rot"]), n_bit=4, q_group_size=128, get_scale_zp=True)
    assert np.array_equal(wq.numpy(), d["w_dq"])
    assert np.array_equal(s.numpy(), d["pq_scales"])
    assert np.array_equal(z.numpy(), d["pq_zeros"])


def test_product_from_linear_rotate_weight_matches_reference():
    """RotateLinearInt4.from_linear(rotate_weight=True, init_only=False):
    rotate_tensor -> quantizer -> pseudo_quantize_tensor -> WQLinear, on the
    CPU, equals the reference's checkpoint buffers bit for bit
    (fromlinear_n128_k1024.npz, written by the reference's own from_linear)."""
    from alpamayo_b200.quantization import RotateLinearInt4
    d = np.load(os.path.join(GOLD, "fromlinear_n128_k1024.npz"))
    lin = torch.nn.Linear(1024, 128, bias=False)
    with torch.no_grad():
        lin.weight.copy_(torch.from_numpy(d["W"]))
    m = RotateLinearInt4.from_linear(lin, torch.from_numpy(d["theta"]), torch.from_numpy(d["pairs"]),
                                     torch.from_numpy(d["channel_scales"]), rotate_weight=True, init_only=False)
    assert np.array_equal(m.qlinear.qweight.numpy(), d["qweight"])
    assert np.array_equal(m.qlinear.scales.numpy(), d["scales"])
    assert np.array_equal(m.qlinear.scaled_zeros.numpy(), d["scaled_zeros"])
    assert m.qlinear.qweight.dtype == torch.int16 and m.qlinear.scales.dtype == torch.float16
