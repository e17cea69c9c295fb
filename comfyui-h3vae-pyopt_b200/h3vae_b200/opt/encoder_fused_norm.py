"""fp16 GroupNorm + SiLU + reflect/causal pad producers and the residual/downsample pack (mirrors of
the reference's opt/encoder_fused_temporal_norm.py, opt/encoder_fused_norm_bias.py,
opt/encoder_fused_batched_norm.py and opt/encoder_fused_residual_pack.py), with their torch.library
boundaries."""
from __future__ import annotations

import torch

from .. import kernels as K


def _padded_fake(x):
    b, c, d, h, w = x.shape
    return torch.empty((b, c, d + 2, h + 2, w + 2), device=x.device, dtype=x.dtype,
                       memory_format=torch.channels_last_3d)


def fused_temporal_norm_pad(x, weight, bias, eps, config=None):
    """ref: opt/encoder_fused_temporal_norm.py:83-98 (config is accepted and unused)."""
    if x.ndim != 5 or x.dtype != torch.float16 or min(x.shape[-2:]) < 2:
        raise ValueError("FP16 [B,C,D,H,W] input with H/W >= 2 required")
    return K.norm_pad_f16(x, weight, bias, eps)


def fused_bias_temporal_norm_pad(x, pre_bias, weight, bias, eps):
    """ref: opt/encoder_fused_norm_bias.py:75-93."""
    if x.ndim != 5 or x.dtype != torch.float16 or min(x.shape[-2:]) < 2:
        raise ValueError("FP16 [B,C,D,H,W] input with H/W >= 2 required")
    return K.norm_pad_f16(x, weight, bias, eps, pre_bias=pre_bias)


@torch.library.custom_op("h3vae_b200_encoder::temporal_norm_pack", mutates_args=(), device_types="cuda")
def temporal_norm_pack(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, eps: float) -> torch.Tensor:
    return fused_temporal_norm_pad(x, w, b, eps)


@temporal_norm_pack.register_fake
def _(x, w, b, eps):
    return _padded_fake(x)


@torch.library.custom_op("h3vae_b200_encoder::bias_temporal_norm_pack", mutates_args=(), device_types="cuda")
def bias_temporal_norm_pack(x: torch.Tensor, pre_bias: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor,
                            eps: float) -> torch.Tensor:
    return fused_bias_temporal_norm_pad(x, pre_bias, weight, bias, eps)


@bias_temporal_norm_pack.register_fake
def _(x, pre_bias, weight, bias, eps):
    return _padded_fake(x)


@torch.library.custom_op("h3vae_b200_encoder::batched_temporal_norm_pack", mutates_args=(), device_types="cuda")
def batched_temporal_norm_pack(x: torch.Tensor, pre_bias: torch.Tensor | None, weight: torch.Tensor,
                               bias: torch.Tensor, eps: float) -> torch.Tensor:
    """Per-(sample, frame) statistics for a batch of clips.  ref: opt/encoder_fused_batched_norm.py:45-73."""
    return K.norm_pad_f16(x, weight, bias, eps, pre_bias=pre_bias)


@batched_temporal_norm_pack.register_fake
def _(x, pre_bias, weight, bias, eps):
    return _padded_fake(x)


@torch.library.custom_op("h3vae_b200_encoder::residual_downsample_pack", mutates_args=(), device_types="cuda")
def residual_downsample_pack(x: torch.Tensor, residual: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """fp16(r + (x + bias)), right/bottom reflect +1, two causal zero frames.
    ref: opt/encoder_fused_residual_pack.py:35-50."""
    if x.ndim != 5 or min(x.shape[-2:]) < 2 or x.dtype != torch.float16:
        raise ValueError("FP16 [B,C,D,H,W] input with H/W >= 2 required")
    return K.residual_pack(x, residual, bias)


@residual_downsample_pack.register_fake
def _(x, residual, bias):
    b, c, d, h, w = x.shape
    return torch.empty((b, c, d + 2, h + 1, w + 1), device=x.device, dtype=x.dtype,
                       memory_format=torch.channels_last_3d)


__all__ = ["fused_temporal_norm_pad", "fused_bias_temporal_norm_pad", "temporal_norm_pack",
           "bias_temporal_norm_pack", "batched_temporal_norm_pack", "residual_downsample_pack"]
