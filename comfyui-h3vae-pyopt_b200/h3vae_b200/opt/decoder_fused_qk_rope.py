"""Per-head QK RMSNorm + rotary (mirror of the reference's opt/decoder_fused_qk_rope.py)."""
from __future__ import annotations

import copy
import os

import torch

from .. import kernels as K


@torch.library.custom_op("h3vae_b200_decoder::qk_rope", mutates_args=(), device_types="cuda")
def qk_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, heads: int, eps: float,
            rows: int) -> tuple[torch.Tensor, torch.Tensor]:
    """x: [b, n, heads*3*64] laid out per head as [q|k|v]; cos/sin [b, n, 1, R] -> q, k [b, n, heads, 64].
    rows is accepted for signature compatibility.  ref: opt/decoder_fused_qk_rope.py:37-49."""
    if rows not in (4, 8, 16, 32):
        raise ValueError("rows must be one of the tested configurations: 4, 8, 16, 32")
    b, n, width = x.shape
    if width % (3 * heads) or width // (3 * heads) != 64:
        raise ValueError("head dim must be 64")
    return K.qk_rope(x.contiguous(), cos.contiguous(), sin.contiguous(), heads, eps)


@qk_rope.register_fake
def _(x, cos, sin, heads, eps, rows):
    shape = (*x.shape[:2], heads, x.shape[-1] // (3 * heads))
    return x.new_empty(shape), x.new_empty(shape)


class FusedQKAttention(torch.nn.Module):
    """An attention module whose QK RMSNorm + RoPE runs as the fused qk_rope op between its own
    to_qkv and its own perform_attention / to_out.  Without rotary tables the original module runs
    unchanged.  ref: opt/decoder_fused_qk_rope.py:55-73."""

    def __init__(self, original, rows=8):
        super().__init__()
        rms = torch.nn.RMSNorm
        if original.spatial_parallel or not isinstance(original.norm_q, rms) or not isinstance(original.norm_k, rms):
            raise ValueError("single-device RMSNorm attention required")
        if (original.norm_q.weight is not None or original.norm_k.weight is not None or original.dim_head != 64
                or original.norm_q.eps != original.norm_k.eps):
            raise ValueError("expected head=64 and unaffined equal-eps QK norms")
        self.original = original
        self.rows = rows

    def forward(self, x, rotary_pos_emb=None, pack_info=None):
        a = self.original
        pack_info = {} if pack_info is None else pack_info
        if rotary_pos_emb is None:
            return a(x, rotary_pos_emb, pack_info)
        b, n, _ = x.shape
        qkv = a.to_qkv(x)
        q, k = qk_rope(qkv, *rotary_pos_emb, a.heads, a.norm_q.eps, self.rows)
        v = qkv.view(b, n, a.heads, 3 * a.dim_head)[..., 2 * a.dim_head:]
        return a.to_out(a.perform_attention(q, k, v, pack_info).reshape(b, n, -1))


def clone_with_qk_fusion(raw, rows=8):
    """A decoder whose blocks are new containers with FusedQKAttention around their attention; the
    weights are shared and `raw` stays intact.  ref: opt/decoder_fused_qk_rope.py:76-89."""
    if raw.training or os.environ.get("MINIMAX_H3_VAE_DECODER_VIT_FP32_NORM", "1").lower() in ("0", "false", "no",
                                                                                              "off"):
        raise ValueError("QK fusion requires eval inference with FP32 norm enabled")
    decoder = copy.copy(raw)
    decoder._modules = dict(raw._modules)
    blocks = []
    for block in raw.transformer_blocks:
        twin = copy.copy(block)
        twin._modules = dict(block._modules)
        twin.attn = FusedQKAttention(block.attn, rows).eval()
        blocks.append(twin)
    decoder.transformer_blocks = torch.nn.ModuleList(blocks)
    return decoder


__all__ = ["FusedQKAttention", "clone_with_qk_fusion", "qk_rope"]
