"""Exact-order fp32 pixel finalization (mirror of the reference's opt/fp16_finalize.py)."""
from __future__ import annotations

import torch

from .. import kernels as K


def validate(x, std, mean, out=None):
    """ref: opt/fp16_finalize.py:6-15."""
    if x.ndim != 5 or x.shape[1] != 3 or x.numel() == 0:
        raise ValueError("nonempty B,3,T,H,W tensor required")
    if x.dtype not in (torch.float16, torch.float32):
        raise ValueError("FP16 or FP32 decoded pixels required")
    for v in (std, mean):
        if v.numel() != 3 or v.dtype != torch.float32 or not v.is_contiguous() or v.device != x.device:
            raise ValueError("three contiguous FP32 channel constants on same device required")
    if out is not None and (out.shape != x.shape or out.dtype != torch.float32 or out.device != x.device
                            or not out.is_contiguous()):
        raise ValueError("contiguous FP32 output with matching shape/device required")


def finalize_pixels(x, std, mean, out=None):
    """clamp(x * std + mean, 0, 1) in fp32 without FMA, NaN preserved.  ref: opt/fp16_finalize.py:44-54."""
    validate(x, std, mean, out)
    if x.device.type != "cuda":
        raise ValueError("NVIDIA CUDA required")
    if torch.is_grad_enabled():
        raise RuntimeError("inference only")
    return K.finalize_pixels(x, std.reshape(3), mean.reshape(3), out)


__all__ = ["finalize_pixels", "validate"]
