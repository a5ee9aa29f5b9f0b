"""Asymmetric group quantisation of weights (offline), mirroring
src/alpamayo_r1/utils/quantization/quantization_utils.py (reference)."""
from __future__ import annotations

import torch


def set_op_by_name(layer, name, new_module):
    """Replace the submodule at dotted path ``name`` (quantization_utils.py:4-15)."""
    levels = name.split(".")
    mod = layer
    for lv in levels[:-1]:
        mod = mod[int(lv)] if lv.isdigit() else getattr(mod, lv)
    setattr(mod, levels[-1], new_module)


def pseudo_quantize_tensor(w, n_bit=8, zero_point=True, q_group_size=-1, inplace=False, get_scale_zp=False,
                           qzeros=None, qscales=None):
    """Group quantise-dequantise (quantization_utils.py:18-73):
    s = (max - min).clamp(1e-5) / (2^b - 1), z = clamp(-round(min / s), 0, 2^b - 1),
    w_dq = (clamp(round(w / s) + z, 0, 2^b - 1) - z) * s."""
    shape = w.shape
    if q_group_size > 0:
        assert shape[-1] % q_group_size == 0
        w = w.reshape(-1, q_group_size)
    assert w.dim() == 2
    assert (qscales is None) == (qzeros is None)
    max_int, min_int = 2 ** n_bit - 1, 0
    if qscales is None:
        if not zero_point:
            raise NotImplementedError("only asymmetric (zero-point) quantisation is used")
        max_val = w.amax(dim=1, keepdim=True)
        min_val = w.amin(dim=1, keepdim=True)
        qscales = (max_val - min_val).clamp(min=1e-5) / max_int
        qzeros = (-torch.round(min_val / qscales)).clamp_(min_int, max_int)
    else:
        qscales = qscales.reshape(-1, 1).to(w.dtype)
        qzeros = qzeros.reshape(-1, 1).to(w.dtype)
    assert torch.isnan(qscales).sum() == 0
    assert torch.isnan(w).sum() == 0
    wq = (torch.clamp(torch.round(w / qscales) + qzeros, min_int, max_int) - qzeros) * qscales
    assert torch.isnan(wq).sum() == 0
    if inplace:
        w.copy_(wq)
        wq = w
    wq = wq.reshape(shape)
    if get_scale_zp:
        return wq, qscales.view(wq.shape[0], -1), qzeros.view(wq.shape[0], -1)
    return wq
