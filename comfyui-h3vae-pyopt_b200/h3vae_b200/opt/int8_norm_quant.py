"""Residual + RMSNorm + rowwise INT8 (mirror of the reference's opt/int8_norm_quant.py)."""
from __future__ import annotations

import os

import torch
from torch import nn

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


class NormQuantBlock(nn.Module):
    """A scaled residual decoder block whose residual add, RMSNorm and FFN run through the INT8
    producers: h = fp16(fma(attn, scale1, x)), out = FFN(RMSNorm(h)), x' = h + out * scale2.  The
    attention module is the block's own, called as attn(norm1(x), rotary_pos_emb, pack_info).
    ref: opt/int8_norm_quant.py:87-124."""

    def __init__(self, block, warps=8):
        super().__init__()
        if not isinstance(block.norm2, nn.RMSNorm) or not block.use_scale:
            raise ValueError("scaled residual block with RMSNorm required")
        if tuple(block.norm2.normalized_shape) != (2048,) or block.norm2.weight is None:
            raise ValueError("affine RMSNorm width 2048 required")
        self.norm1, self.norm2 = block.norm1, block.norm2
        self.attn, self.ff = block.attn, block.ff
        self.scale1, self.scale2 = block.scale1, block.scale2
        self.warps = warps
        self.fuse_ffn_up = self._fused_ffn_available()
        self.train(block.training)

    def _fused_ffn_available(self) -> bool:
        from .int8_ffn_up_fused import supports_fused_ffn_up
        return supports_fused_ffn_up(self.scale1.device)

    def _apply(self, fn, recurse=True):
        result = super()._apply(fn, recurse=recurse)
        self.fuse_ffn_up = self._fused_ffn_available()
        return result

    def forward(self, hidden_states, rotary_pos_emb=None, pack_info=None):
        if self.training or torch.is_grad_enabled():
            raise RuntimeError("eval + inference/no_grad required")
        pack_info = {} if pack_info is None else pack_info
        normed = self.norm1(hidden_states.float()).to(hidden_states.dtype)
        attn = self.attn(normed, rotary_pos_emb, pack_info)
        w1, w2 = self.ff.w1, self.ff.w2
        if self.fuse_ffn_up:
            from .int8_ffn_up_fused import fused_residual_ffn
            h, out = fused_residual_ffn(hidden_states, attn, self.scale1, self.norm2.weight, w1.qweight,
                                        w1.weight_scale, w1.bias, w2.qweight, w2.weight_scale, w2.bias,
                                        self.norm2.eps, self.warps)
        else:
            from .int8_swiglu_fused import swiglu_int8_linear
            h, hidden = residual_rms_linear(hidden_states, attn, self.scale1, self.norm2.weight, w1.qweight,
                                            w1.weight_scale, w1.bias, self.norm2.eps, self.warps)
            out = swiglu_int8_linear(hidden, w2.qweight, w2.weight_scale, w2.bias, 16)
        return h + out * self.scale2


def clone_norm_quant_decoder(raw, warps=8):
    """Container clone of an INT8both decoder with fused FFNs and every block a NormQuantBlock.
    ref: opt/int8_norm_quant.py:127-136."""
    if os.environ.get("MINIMAX_H3_VAE_DECODER_VIT_FP32_NORM", "1").lower() not in ("1", "true", "yes", "on"):
        raise ValueError("experimental fusion requires FP32 norm enabled")
    if warps not in (4, 8, 16):
        raise ValueError("unsupported warp count")
    from .int8_swiglu_fused import clone_fused_decoder
    result = clone_fused_decoder(raw, 16)
    result.transformer_blocks = nn.ModuleList(
        [NormQuantBlock(block, warps).eval() for block in result.transformer_blocks])
    return result


__all__ = ["NormQuantBlock", "clone_norm_quant_decoder", "residual_quant", "residual_rms_linear", "validate"]
