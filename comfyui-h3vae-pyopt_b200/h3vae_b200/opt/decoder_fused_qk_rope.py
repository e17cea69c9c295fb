"""Per-head QK RMSNorm + rotary (mirror of the reference's opt/decoder_fused_qk_rope.py)."""
from __future__ import annotations

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


__all__ = ["qk_rope"]
