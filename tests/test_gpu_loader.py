"""The checkpoint -> model load path (load_paroquant_model, mirroring the
reference's src/alpamayo_r1/utils/quantization/paroquant_marlin_w4a8.py:426-510)
on a stand-in model with the Alpamayo layer path
(model.vlm.model.language_model.layers), fed a synthetic ParoQuant state dict
written with the reference's key names (``*.rotation.{theta,pairs,
channel_scales}``, ``*.qlinear.{qweight,scales,scaled_zeros}``) by the
product's offline path (RotateLinearInt4.from_linear, bit-exact against the
reference's).  One layer carries all-zero scales (the loader's zero-scale
diagnostic) and one an infinite and a NaN channel scale (sanitised).
Loaded linears must give the oracle's output for their checkpoint buffers."""
import logging

import numpy as np
import pytest
import torch
import torch.nn as nn

from oracle import paro_oracle as O
from tests.helpers import rel_l2

pytestmark = pytest.mark.gpu
H, I = 256, 512
PROJ = {"self_attn": {"q_proj": (H, H), "k_proj": (128, H), "v_proj": (128, H), "o_proj": (H, H)},
        "mlp": {"gate_proj": (I, H), "up_proj": (I, H), "down_proj": (H, I)}}


class Block(nn.Module):
    def __init__(self):
        super().__init__()
        for part, projs in PROJ.items():
            m = nn.Module()
            for name, (n, k) in projs.items():
                setattr(m, name, nn.Linear(k, n, bias=False))
            setattr(self, part, m)
        self.input_layernorm = nn.LayerNorm(H)


def stand_in(layers=2):
    model = nn.Module()
    model.vlm = nn.Module()
    model.vlm.model = nn.Module()
    model.vlm.model.language_model = nn.Module()
    model.vlm.model.language_model.layers = nn.ModuleList([Block() for _ in range(layers)])
    model.vlm.lm_head = nn.Linear(H, 64, bias=False)
    return model


def synthetic_checkpoint(layers=2, seed=0):
    from alpamayo_b200.quantization import RotateLinearInt4
    g = torch.Generator().manual_seed(seed)
    sd = {}
    for li in range(layers):
        for part, projs in PROJ.items():
            for name, (n, k) in projs.items():
                G = k // 128
                pairs = torch.stack([torch.cat([torch.randperm(128, generator=g) for _ in range(G)])
                                     for _ in range(8)]).to(torch.int16)
                theta = ((torch.rand(8, k // 2, generator=g) * 2 - 1) * np.pi).to(torch.float16)
                cs = (0.5 + 1.5 * torch.rand(1, k, generator=g)).to(torch.float16)
                lin = nn.Linear(k, n, bias=False)
                with torch.no_grad():
                    lin.weight.copy_(torch.randn(n, k, generator=g) * 0.02)
                m = RotateLinearInt4.from_linear(lin, theta, pairs, cs, rotate_weight=True, init_only=False)
                prefix = f"vlm.model.language_model.layers.{li}.{part}.{name}"
                for key, t in m.state_dict().items():
                    sd[f"{prefix}.{key}"] = t.clone()
    return sd


def test_load_paroquant_model_end_to_end(caplog):
    from alpamayo_b200.quantization import RotateLinearInt4, convert_model_to_marlin_w4a8, load_paroquant_model
    from alpamayo_b200.quantization.paroquant_marlin_w4a8 import BF16RotateLinearWrapper, MarlinW4A8Linear
    sd = synthetic_checkpoint()
    zero_key = "vlm.model.language_model.layers.1.mlp.up_proj.qlinear.scales"
    sd[zero_key] = torch.zeros_like(sd[zero_key])
    cs_key = "vlm.model.language_model.layers.0.self_attn.k_proj.rotation.channel_scales"
    sd[cs_key][0, 0] = float("inf")
    sd[cs_key][0, 1] = float("nan")
    made = []

    def factory(path, dtype):
        made.append((path, dtype))
        return stand_in().to(dtype)

    with caplog.at_level(logging.WARNING):
        model = load_paroquant_model("stand-in", sd, model_factory=factory, device="cuda")
    assert made == [("stand-in", torch.bfloat16)]
    assert any("zero scales" in r.getMessage() for r in caplog.records)
    assert any("channel_scales" in r.getMessage() for r in caplog.records)
    layer0 = model.vlm.model.language_model.layers[0]
    assert isinstance(layer0.self_attn.q_proj, BF16RotateLinearWrapper)
    assert isinstance(model.vlm.lm_head, nn.Linear)           # outside the layers: untouched
    assert isinstance(layer0.input_layernorm, nn.LayerNorm)  # not a linear: untouched
    assert next(model.parameters()).is_cuda
    k_cs = layer0.self_attn.k_proj.rotate_linear.rotation.channel_scales
    assert torch.isfinite(k_cs).all() and k_cs.abs().max().item() <= 65504 / 128

    # every loaded linear against the oracle on its checkpoint buffers
    x = torch.from_numpy(np.random.default_rng(1).standard_normal((4, I)).astype(np.float32)).to(torch.bfloat16)
    outs = {}
    for part, projs in PROJ.items():
        for name, (n, k) in projs.items():
            prefix = f"vlm.model.language_model.layers.0.{part}.{name}"
            wrapped = getattr(getattr(layer0, part), name)
            xi = x[:, :k].contiguous().cuda()
            y = wrapped(xi)
            assert y.dtype == torch.bfloat16 and y.shape == (4, n)
            rl = wrapped.rotate_linear
            q, s = rl.rotation.quantize_activations(xi)
            cs = sd[prefix + ".rotation.channel_scales"].float().nan_to_num(nan=65504 / 128, posinf=65504 / 128)
            q_ref, _, _ = O.rot_quant_reference(xi.float().cpu().numpy(), sd[prefix + ".rotation.pairs"].numpy(),
                                                sd[prefix + ".rotation.theta"].float().numpy(), cs.numpy())
            dq = np.abs(q.cpu().numpy().astype(np.int32) - q_ref.astype(np.int32))
            assert dq.max() <= 1 and (dq > 0).mean() <= 1e-3
            codes = O.unpack_wqlinear_qweight(sd[prefix + ".qlinear.qweight"].numpy(), n, k)
            sc = sd[prefix + ".qlinear.scales"].numpy()
            zeros = O.recover_zeros(sc, sd[prefix + ".qlinear.scaled_zeros"].numpy(), n, k)
            ref = O.w4a8_linear(q.cpu().numpy(), s.cpu().numpy().reshape(-1), codes, zeros,
                                sc[:k // 128].astype(np.float32))
            assert rel_l2(y.float().cpu().numpy(), O.round_to_bf16(ref)) <= 1e-3, (part, name)
            outs[(part, name)] = y
    # the zero-scale layer loads (the reference only reports it) and gives zeros
    up1 = model.vlm.model.language_model.layers[1].mlp.up_proj
    assert torch.count_nonzero(up1(x[:, :H].contiguous().cuda())).item() == 0

    # converting to MarlinW4A8Linear keeps every output bit for bit
    assert convert_model_to_marlin_w4a8(model) == 2 * sum(len(p) for p in PROJ.values())
    assert isinstance(layer0.self_attn.q_proj.rotate_linear.qlinear, MarlinW4A8Linear)
    for (part, name), y in outs.items():
        k = PROJ[part][name][1]
        y2 = getattr(getattr(layer0, part), name)(x[:, :k].contiguous().cuda())
        assert torch.equal(y2, y), (part, name)
    assert all(isinstance(m, RotateLinearInt4) for m in [layer0.mlp.down_proj.rotate_linear])
