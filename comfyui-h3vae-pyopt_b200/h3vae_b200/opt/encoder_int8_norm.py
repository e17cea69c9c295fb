"""INT8 norm producer (mirror of the reference's opt/encoder_int8_norm.py): GroupNorm(32) per frame,
SiLU, reflect/causal padding and per-tensor INT8 in one producer with no fp16 scratch tensor."""
from __future__ import annotations

import torch

from .. import kernels as K


def _validate(x, weight, bias, pre_bias):
    """ref: opt/encoder_int8_norm.py:16-31 (the B200 kernels accept any batch and C in 32..2048)."""
    if x.ndim != 5 or x.device.type != "cuda":
        raise ValueError("INT8 norm producer requires a CUDA rank-5 input")
    b, c, d, h, w = x.shape
    if x.dtype != torch.float16 or d < 1 or min(h, w) < 2:
        raise ValueError("INT8 norm producer requires FP16 input with D>=1, H/W>=2")
    for p in (weight, bias) + (() if pre_bias is None else (pre_bias,)):
        if (p is None or p.shape != (c,) or p.dtype != x.dtype or p.device != x.device
                or not p.is_contiguous()):
            raise ValueError("Expected contiguous FP16 channel vectors on input device")


def quantized_temporal_norm_pad(x, weight, bias, eps, *, pre_bias=None):
    """Returns (q int8 NDHWC [B,C,D+2,H+2,W+2], fp32 scale).  ref: opt/encoder_int8_norm.py:77-110."""
    _validate(x, weight, bias, pre_bias)
    return K.norm_pad_quant(x, weight, bias, eps, pre_bias=pre_bias)


__all__ = ["quantized_temporal_norm_pad"]
