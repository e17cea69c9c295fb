"""norm1 producer feeding the INT8 QKV GEMM, updating the residual in place (mirror of the
reference's opt/int8_norm1_quant.py op residual_qkv)."""
from __future__ import annotations

import torch

from .. import kernels as K
from .int8_swiglu_fused import prequantized_linear


def residual_qkv_impl(h, o, g, w, qw, ws, bias, eps: float = 1.0e-5):
    """h <- fp16(fma(o, g, h)) in place; RMSNorm + row INT8; INT8 QKV GEMM.
    ref: opt/int8_norm1_quant.py:126-149 (any [..., K] width)."""
    if o.shape != h.shape or g.shape != (h.shape[-1],) or w.shape != (h.shape[-1],) or qw.shape[1] != h.shape[-1]:
        raise ValueError("expected matching residual/output rows and width-K vectors")
    if any(t.dtype != torch.float16 or not t.is_contiguous() for t in (h, o, g, w)):
        raise ValueError("contiguous FP16 inputs required")
    if torch.is_grad_enabled():
        raise RuntimeError("norm1 fusion requires inference/no_grad")
    if h.data_ptr() == o.data_ptr():
        raise ValueError("residual H and FFN output must have distinct storage")
    _, q, s = K.residual_rms_quant(h, o, g, w, eps, h_out=h)
    return prequantized_linear(q, s, qw, ws, bias).reshape(*h.shape[:-1], qw.shape[0])


@torch.library.custom_op("h3vae_b200_norm1::residual_qkv", mutates_args=("h",))
def residual_qkv(h: torch.Tensor, o: torch.Tensor, g: torch.Tensor, w: torch.Tensor, qw: torch.Tensor,
                 ws: torch.Tensor, bias: torch.Tensor | None) -> torch.Tensor:
    """ref: opt/int8_norm1_quant.py:152-157."""
    return residual_qkv_impl(h, o, g, w, qw, ws, bias)


@residual_qkv.register_fake
def _(h, o, g, w, qw, ws, bias):
    return h.new_empty((*h.shape[:-1], qw.shape[0]))


__all__ = ["residual_qkv", "residual_qkv_impl"]
