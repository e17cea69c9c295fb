"""INT8 attention output projections after the INT8 QKV (mirror of the reference's
opt/int8_attention_out.py).  Container cloning shares the tensors, not the module tables; only the
returned decoder is meant for independent offload / reload."""
from __future__ import annotations

import torch
from torch import nn

from ._containers import clone_containers, selected_indices
from .int8_qkv import clone_qkv_int8_decoder
from .kitchen_int8 import KitchenInt8Linear


def out_linear(block):
    """(attention module, its nn.Linear to_out) of an eval block.  ref: opt/int8_attention_out.py:28-37."""
    attention = getattr(block.attn, "original", block.attn)
    source = getattr(attention, "to_out", None)
    if not isinstance(source, nn.Linear):
        raise ValueError("expected original nn.Linear output projection")
    if (source.in_features, source.out_features) != (2048, 2048):
        raise ValueError("output projection experiment requires K2048/N2048")
    if source.training:
        raise ValueError("output projection inference experiment requires eval()")
    return attention, source


def clone_attention_out_decoder(baseline, *, indices=None):
    """ref: opt/int8_attention_out.py:40-48."""
    chosen = selected_indices(len(baseline.transformer_blocks), indices)
    for i in chosen:
        out_linear(baseline.transformer_blocks[i])
    result = clone_containers(baseline)
    for i in chosen:
        attention, source = out_linear(result.transformer_blocks[i])
        attention.to_out = KitchenInt8Linear(source, require_cuda=True).eval()
    return result


def from_raw_decoder(raw, *, warps=8):
    """INT8 QKV then INT8 attention-out on a raw decoder.  ref: opt/int8_attention_out.py:51-52."""
    return clone_attention_out_decoder(clone_qkv_int8_decoder(raw, warps=warps))


def out_inventory(decoder):
    """ref: opt/int8_attention_out.py:55-67."""
    rows = []
    for i, block in enumerate(decoder.transformer_blocks):
        linear = getattr(block.attn, "original", block.attn).to_out
        if isinstance(linear, KitchenInt8Linear):
            if linear.qweight.dtype != torch.int8 or linear.weight_scale.dtype != torch.float32:
                raise RuntimeError("output projection quantized state has invalid dtype")
            rows.append({"block": i, "shape": list(linear.qweight.shape), "qweight_dtype": str(linear.qweight.dtype),
                         "scale_dtype": str(linear.weight_scale.dtype), "device": str(linear.qweight.device)})
    return rows


__all__ = ["clone_attention_out_decoder", "clone_containers", "from_raw_decoder", "out_inventory", "out_linear"]
