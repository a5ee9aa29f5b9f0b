"""The drop-in module API (reference rotation_linear.py, qmodule.py,
paroquant_marlin_w4a8.py) end to end on the GPU, against the oracle."""
import os

import numpy as np
import pytest
import torch

from oracle import paro_oracle as O
from tests.helpers import make_activations, make_quantized_layer, rel_l2

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def load_module(d, N, K, bias=None):
    from alpamayo_b200.quantization import RotateLinearInt4
    m = RotateLinearInt4(K, N, bias is not None, torch.float16)
    sd = {"rotation.theta": torch.from_numpy(d["theta"]), "rotation.pairs": torch.from_numpy(d["pairs"]),
          "rotation.channel_scales": torch.from_numpy(d["channel_scales"]),
          "qlinear.qweight": torch.from_numpy(d["qweight"]), "qlinear.scales": torch.from_numpy(d["wq_scales"]),
          "qlinear.scaled_zeros": torch.from_numpy(d["wq_scaled_zeros"])}
    if bias is not None:
        sd["qlinear.bias"] = torch.from_numpy(bias)
    m.load_state_dict(sd)
    return m.cuda()


def oracle_linear(x, d, N, K, bias=None, variant="fp16"):
    q, s, _ = O.rot_quant_reference(x, d["pairs"], d["theta"].astype(np.float32),
                                    d["channel_scales"].astype(np.float32))
    z = O.recover_zeros(d["wq_scales"], d["wq_scaled_zeros"], N, K)
    codes = O.unpack_wqlinear_qweight(d["qweight"], N, K)
    G = K // 128
    return O.w4a8_linear(q, s, codes, z, d["wq_scales"][:G].astype(np.float32),
                         bias=None if bias is None else bias.astype(np.float32), variant=variant)


def test_golden_checkpoint_through_rotate_linear_and_wrapper():
    from alpamayo_b200.quantization import BF16RotateLinearWrapper, convert_model_to_marlin_w4a8
    d = np.load(os.path.join(GOLD, "wq_n128_k1024.npz"))
    N, K = 128, 1024
    bias = d["bias"].astype(np.float16)
    m = load_module(d, N, K, bias)
    x = torch.from_numpy(d["x"]).to(torch.bfloat16)
    ref = oracle_linear(x.float().numpy(), d, N, K, bias)
    # WQLinear (unconverted) runs the W4A8 path too
    y0 = m(x.cuda()).float().cpu().numpy()
    assert rel_l2(y0, O.round_to_bf16(ref)) <= 1e-3
    holder = torch.nn.Module()
    holder.lin = m
    assert convert_model_to_marlin_w4a8(holder) == 1
    w = BF16RotateLinearWrapper(m)
    y = w(x.cuda())
    assert y.dtype == torch.bfloat16 and y.shape == (16, N)
    assert rel_l2(y.float().cpu().numpy(), O.round_to_bf16(ref)) <= 1e-3
    # the converted module and the checkpoint container run the same kernels
    assert np.array_equal(y.float().cpu().numpy(), y0)
    # against the fake-quant product with the reference's own dequantised weight
    wdq = O.dequant_awq(d["unpacked"], d["awq_zeros"], d["wq_scales"])
    q, s, _ = O.rot_quant_reference(x.float().numpy(), d["pairs"], d["theta"].astype(np.float32),
                                    d["channel_scales"].astype(np.float32))
    fq = (q.astype(np.float32) * s[:, None]) @ wdq.T + bias.astype(np.float32)
    assert rel_l2(y.float().cpu().numpy(), fq) <= 2e-3


def test_fp16_input_returns_fp16_like_marlin_path():
    from alpamayo_b200.quantization import convert_model_to_marlin_w4a8
    N, K = 256, 2048
    d = make_quantized_layer(N, K, seed=7)
    m = load_module(d, N, K)
    holder = torch.nn.Module()
    holder.lin = m
    convert_model_to_marlin_w4a8(holder)
    x = torch.from_numpy(make_activations(8, K, seed=8)).to(torch.float16)
    y = m(x.cuda())
    assert y.dtype == torch.float16
    ref = O.round_to_fp16(oracle_linear(x.float().numpy(), d, N, K, variant="marlin"))
    assert rel_l2(y.float().cpu().numpy(), ref) <= 1e-3


def test_marlin_module_from_awq_buffers():
    from alpamayo_b200.quantization import MarlinW4A8Linear, convert_wqlinear_layer
    d = np.load(os.path.join(GOLD, "wq_n128_k1024.npz"))
    N, K = 128, 1024
    mod = MarlinW4A8Linear(K, N)
    mod.load_from_awq(torch.from_numpy(d["awq_qweight"]).cuda(), torch.from_numpy(d["awq_scales"]).cuda(),
                      torch.from_numpy(d["awq_qzeros"]).cuda())
    xr = torch.from_numpy(O.round_to_fp16(d["x_rotated"])).to(torch.float16).cuda()
    y = mod(xr)
    assert y.dtype == torch.float16
    q, s = O.per_token_quant_int8(xr.float().cpu().numpy())
    ref = O.w4a8_linear(q, s, d["unpacked"], d["awq_zeros"], d["awq_scales"].astype(np.float32))
    assert rel_l2(y.float().cpu().numpy(), O.round_to_fp16(ref)) <= 1e-3
    mod2, awq = convert_wqlinear_layer(torch.from_numpy(d["qweight"]), torch.from_numpy(d["wq_scales"]),
                                       torch.from_numpy(d["wq_scaled_zeros"]), N, K, 128)
    assert torch.equal(mod2.qweight, mod.qweight)
    assert torch.equal(mod2(xr), y)


def test_rotation_module_forward():
    from alpamayo_b200.quantization import Rotation
    d = np.load(os.path.join(GOLD, "rot_m16_k1024.npz"))
    r = Rotation(1024, rotation_angles=torch.from_numpy(d["theta"]).cuda(),
                 rotation_pairs=torch.from_numpy(d["pairs"]).cuda(),
                 channel_scales=torch.from_numpy(d["channel_scales"]).cuda())
    y = r(torch.from_numpy(d["x"]).cuda()).cpu().numpy()
    assert np.abs(y - d["rotated"]).max() <= 2e-5 * np.abs(d["rotated"]).max()


def test_rotate_tensor_weight_side_on_gpu():
    """The weight-side transform on CUDA tensors (the reference runs it on
    CUDA): the same operations as on the CPU, where it is bit-exact against
    the reference's golden; CUDA's sin / cos may differ from the CPU's in
    the last place, hence the float32-level tolerance."""
    from alpamayo_b200.quantization import rotate_tensor
    d = np.load(os.path.join(GOLD, "wq_n128_k1024.npz"))
    w = rotate_tensor(torch.from_numpy(d["W"]).cuda(), torch.from_numpy(d["theta"]).cuda(),
                      torch.from_numpy(d["pairs"]).cuda(), torch.from_numpy(d["channel_scales"]).cuda())
    assert w.is_cuda
    assert np.abs(w.cpu().numpy() - d["w_rot"]).max() <= 2e-6 * np.abs(d["w_rot"]).max()


def test_cuda_graph_capture_and_replay():
    """The fused linear launches on the current stream without syncs or
    host-visible allocation, so it captures into a CUDA graph."""
    from alpamayo_b200.quantization import convert_model_to_marlin_w4a8
    N, K = 512, 1024
    d = make_quantized_layer(N, K, seed=1)
    m = load_module(d, N, K)
    holder = torch.nn.Module()
    holder.lin = m
    convert_model_to_marlin_w4a8(holder)
    x = torch.from_numpy(make_activations(4, K, seed=2)).to(torch.bfloat16).cuda()
    y_eager = m(x)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        m(x)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        y_graph = m(x)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(y_graph, y_eager)
