"""Block-0 RMSNorm and the final residual LayerNorm (mirrors of the reference's
opt/decoder_block0_norm.py and opt/decoder_final_norm.py, shape generic)."""
from __future__ import annotations

import torch

from .. import kernels as K

EPS = 9.999999747378752e-06   # fp32(1e-5), ref: opt/decoder_block0_norm.py:22 and opt/decoder_final_norm.py:13


@torch.library.custom_op("h3vae_b200_norm1_block0::rms_fp16_x2_w16", mutates_args=())
def rms_fp16_x2_w16(x: torch.Tensor, gamma: torch.Tensor) -> torch.Tensor:
    """fp16(x * rsqrt(mean(x^2) + eps) * gamma).  ref: opt/decoder_block0_norm.py:69-89."""
    if x.dtype != torch.float16 or gamma.dtype != torch.float16 or gamma.shape != (x.shape[-1],):
        raise ValueError("expected FP16 rows and a width-K gamma on one device")
    return K.rms_norm_f16(x.contiguous(), gamma, EPS)


@rms_fp16_x2_w16.register_fake
def _(x, gamma):
    return torch.empty_like(x, memory_format=torch.contiguous_format)


@torch.library.custom_op("h3vae_b200_final_ln::residual_ln_w8", mutates_args=())
def final_residual_ln_w8(h: torch.Tensor, o: torch.Tensor, gate: torch.Tensor, gamma: torch.Tensor,
                         beta: torch.Tensor) -> torch.Tensor:
    """LayerNorm(fma(o, gate, h)) * gamma + beta.  ref: opt/decoder_final_norm.py:61-80."""
    if h.shape != o.shape or any(v.shape != (h.shape[-1],) for v in (gate, gamma, beta)):
        raise ValueError("expected contiguous FP16 H/O and width-K vectors on one device")
    return K.final_residual_layernorm(h.contiguous(), o.contiguous(), gate, gamma, beta, EPS)


@final_residual_ln_w8.register_fake
def _(h, o, gate, gamma, beta):
    return torch.empty_like(h, memory_format=torch.contiguous_format)


__all__ = ["rms_fp16_x2_w16", "final_residual_ln_w8"]
