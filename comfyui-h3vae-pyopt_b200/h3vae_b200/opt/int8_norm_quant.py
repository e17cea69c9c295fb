"""Residual + RMSNorm + rowwise INT8 (mirror of the reference's opt/int8_norm_quant.py)."""
from __future__ import annotations

import torch

from .. import kernels as K
from .int8_swiglu_fused import prequantized_linear


def validate(x, a, g, w, eps, warps):
    """ref: opt/int8_norm_quant.py:47-56 (width generic here)."""
    k = x.shape[-1]
    if x.ndim < 2 or x.numel() == 0:
        raise ValueError("nonempty residual rows required")
    if a.shape != x.shape or g.shape != (k,) or w.shape != (k,):
        raise ValueError("residual/scale/RMS weight shape mismatch")
    if any(t.dtype != torch.float16 or not t.is_contiguous() or t.device != x.device for t in (x, a, g, w)):
        raise ValueError("contiguous FP16 tensors on the same device required")
    if not 0 < eps < 1 or warps not in (4, 8, 16):
        raise ValueError("invalid epsilon or warp count")


def residual_quant(x, a, g, w, eps, warps=8, round_stats=False):
    """h = fp16(fma(a, g, x)); act = fp16(h * rsqrt(mean(stat^2) + eps) * w); row INT8 of act.
    Returns (h, q [M,K], s [M,1]).  ref: opt/int8_norm_quant.py:59-70."""
    validate(x, a, g, w, eps, warps)
    if x.device.type != "cuda":
        raise ValueError("NVIDIA CUDA required")
    h, q, s = K.residual_rms_quant(x, a, g, w, eps, round_stats=round_stats)
    return h, q, s


@torch.library.custom_op("h3vae_b200_norm_exp::residual_rms_linear", mutates_args=())
def residual_rms_linear(x: torch.Tensor, a: torch.Tensor, g: torch.Tensor, w: torch.Tensor, qw: torch.Tensor,
                        ws: torch.Tensor, bias: torch.Tensor | None, eps: float,
                        warps: int) -> tuple[torch.Tensor, torch.Tensor]:
    """ref: opt/int8_norm_quant.py:72-80."""
    h, q, s = residual_quant(x, a, g, w, eps, warps)
    return h, prequantized_linear(q, s, qw, ws, bias).reshape(*x.shape[:-1], qw.shape[0])


@residual_rms_linear.register_fake
def _(x, a, g, w, qw, ws, bias, eps, warps):
    return torch.empty_like(x), x.new_empty((*x.shape[:-1], qw.shape[0]))


__all__ = ["residual_quant", "residual_rms_linear", "validate"]
