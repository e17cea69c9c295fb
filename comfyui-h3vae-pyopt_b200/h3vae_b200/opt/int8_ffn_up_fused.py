"""INT8 FFN-up GEMM with the SwiGLU epilogue and the fused residual FFN (mirror of the reference's
opt/int8_ffn_up_fused.py; not limited to SM120 or to the H3 widths)."""
from __future__ import annotations

import torch

from .. import kernels as K
from .int8_norm_quant import residual_quant
from .int8_swiglu_fused import prequantized_linear


def supports_fused_ffn_up(device) -> bool:
    """The fused FFN-up kernel exists on the sm_100 build.  ref: opt/int8_ffn_up_fused.py:15-20."""
    device = torch.device(device)
    return (device.type == "cuda" and torch.cuda.is_available()
            and torch.cuda.get_device_capability(device) == (10, 0))


def validate_prequantized(q, scale, weight, weight_scale, bias):
    """ref: opt/int8_ffn_up_fused.py:23-41 (shape generic)."""
    if q.ndim != 2 or q.shape[0] == 0 or weight.ndim != 2 or weight.shape[1] != q.shape[1] or weight.shape[0] % 2:
        raise ValueError("nonempty INT8 activation matrix and a [2F, K] INT8 weight required")
    if q.dtype != torch.int8 or weight.dtype != torch.int8:
        raise ValueError("INT8 activations and weights required")
    if scale.dtype != torch.float32 or weight_scale.dtype != torch.float32:
        raise ValueError("FP32 activation and weight scales required")
    if scale.numel() != q.shape[0] or weight_scale.numel() != weight.shape[0]:
        raise ValueError("one activation/weight scale per row required")
    if bias is not None and (bias.numel() != weight.shape[0] or bias.dtype != torch.float16):
        raise ValueError("FP16 bias with 2F elements required")


def quantize_ffn_up(q, scale, weight, weight_scale, bias=None):
    """act = SwiGLU of the INT8 FFN-up output, then CK-contract row INT8 -> (q, s).
    ref: opt/int8_ffn_up_fused.py:108-130."""
    validate_prequantized(q, scale, weight, weight_scale, bias)
    if torch.is_grad_enabled():
        raise RuntimeError("fused INT8 FFN-up requires inference/no_grad")
    act = K.gemm_i8_swiglu(q, scale.reshape(-1), weight, weight_scale, bias)
    return K.row_quant(act)


@torch.library.custom_op("h3vae_b200_int8_ffn::residual_ffn", mutates_args=())
def fused_residual_ffn(x: torch.Tensor, a: torch.Tensor, g: torch.Tensor, norm_weight: torch.Tensor,
                       up_weight: torch.Tensor, up_scale: torch.Tensor, up_bias: torch.Tensor | None,
                       down_weight: torch.Tensor, down_scale: torch.Tensor, down_bias: torch.Tensor | None,
                       eps: float, warps: int) -> tuple[torch.Tensor, torch.Tensor]:
    """h, ffn(norm2(h)) with h = fp16(fma(a, g, x)).  ref: opt/int8_ffn_up_fused.py:133-160."""
    h, q, s = residual_quant(x, a, g, norm_weight, eps, warps)
    qout, sout = quantize_ffn_up(q, s, up_weight, up_scale, up_bias)
    out = prequantized_linear(qout, sout, down_weight, down_scale, down_bias)
    return h, out.reshape(*x.shape[:-1], down_weight.shape[0])


@fused_residual_ffn.register_fake
def _(x, a, g, norm_weight, up_weight, up_scale, up_bias, down_weight, down_scale, down_bias, eps, warps):
    return torch.empty_like(x), x.new_empty((*x.shape[:-1], down_weight.shape[0]))


__all__ = ["fused_residual_ffn", "quantize_ffn_up", "supports_fused_ffn_up", "validate_prequantized"]
