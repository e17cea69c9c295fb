"""INT8 QKV projections on the norm-quant decoder (mirror of the reference's opt/int8_qkv.py).

The selected blocks' to_qkv linears become static-weight INT8 linears (KitchenInt8Linear, the
tcgen05 GEMM); attention, QK norm / RoPE, the output projection and the encoder are unchanged, and
the caller's decoder keeps its original modules."""
from __future__ import annotations

import torch
from torch import nn

from ._containers import selected_indices
from .int8_norm_quant import clone_norm_quant_decoder
from .kitchen_int8 import KitchenInt8Linear


def qkv_linear(block):
    """(attention module, its nn.Linear to_qkv) of an eval block.  ref: opt/int8_qkv.py:12-21."""
    attention = getattr(block.attn, "original", block.attn)
    source = getattr(attention, "to_qkv", None)
    if not isinstance(source, nn.Linear):
        raise ValueError("expected original nn.Linear QKV projection")
    if (source.in_features, source.out_features) != (2048, 6144):
        raise ValueError("QKV experiment requires K2048/N6144")
    if source.training:
        raise ValueError("QKV inference experiment requires eval()")
    return attention, source


def clone_qkv_int8_decoder(raw, *, indices=None, warps=8):
    """Every selected block is validated before the clone; the clone's selected to_qkv linears are
    replaced.  ref: opt/int8_qkv.py:33-41."""
    chosen = selected_indices(len(raw.transformer_blocks), indices)
    for i in chosen:
        qkv_linear(raw.transformer_blocks[i])
    result = clone_norm_quant_decoder(raw, warps)
    for i in chosen:
        attention, source = qkv_linear(result.transformer_blocks[i])
        attention.to_qkv = KitchenInt8Linear(source, require_cuda=True).eval()
    return result


def qkv_inventory(decoder):
    """One row per INT8 QKV projection (block, shape, dtypes, device).  ref: opt/int8_qkv.py:44-56."""
    rows = []
    for i, block in enumerate(decoder.transformer_blocks):
        linear = getattr(block.attn, "original", block.attn).to_qkv
        if isinstance(linear, KitchenInt8Linear):
            if linear.qweight.dtype != torch.int8 or linear.weight_scale.dtype != torch.float32:
                raise RuntimeError("QKV quantized state has invalid dtype")
            rows.append({"block": i, "shape": list(linear.qweight.shape), "qweight_dtype": str(linear.qweight.dtype),
                         "scale_dtype": str(linear.weight_scale.dtype), "device": str(linear.qweight.device)})
    return rows


__all__ = ["clone_qkv_int8_decoder", "qkv_inventory", "qkv_linear", "selected_indices"]
