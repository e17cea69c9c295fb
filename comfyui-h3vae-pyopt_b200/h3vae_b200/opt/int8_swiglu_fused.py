"""SwiGLU + rowwise INT8 and the prequantized INT8 linear (mirror of the reference's
opt/int8_swiglu_fused.py; the CK cutlass_int8_dequant call becomes the tcgen05 GEMM)."""
from __future__ import annotations

import torch
from torch import nn

from .. import kernels as K


def validate_input(x):
    """ref: opt/int8_swiglu_fused.py:44-49."""
    if x.dtype != torch.float16 or x.ndim < 2 or not x.is_contiguous():
        raise ValueError("contiguous FP16 input with at least two dimensions required")
    if x.shape[-1] <= 0 or x.shape[-1] % 2 or x.numel() == 0:
        raise ValueError("nonempty [gate | up] rows of even width required")
    if x.shape[-1] // 2 > 16384:
        raise ValueError("experimental quantizer K exceeds 16384")


def quantize_swiglu(x, *, num_warps=8):
    """act = fp16(silu(gate) * up), CK-contract row quantization -> (q [M,K], s [M,1]).
    ref: opt/int8_swiglu_fused.py:52-66."""
    validate_input(x)
    if x.device.type != "cuda":
        raise ValueError("NVIDIA CUDA required")
    return K.swiglu_quant(x)


def prequantized_linear(q, scale, weight, weight_scale, bias=None):
    """INT8 GEMM consuming already quantized rows.  ref: opt/int8_swiglu_fused.py:78-107."""
    if q.dtype != torch.int8 or weight.dtype != torch.int8 or weight.shape[1] != q.shape[1]:
        raise ValueError("INT8 matrix dimensions/types do not match")
    if scale.dtype != torch.float32 or weight_scale.dtype != torch.float32:
        raise ValueError("FP32 scales required")
    if scale.numel() != q.shape[0] or weight_scale.numel() != weight.shape[0]:
        raise ValueError("one scale per activation/weight row required")
    if q.device.type != "cuda":
        raise ValueError("NVIDIA CUDA required")
    return K.gemm_i8(q, scale.reshape(-1), weight, weight_scale, bias)


@torch.library.custom_op("h3vae_b200_exp::swiglu_int8_linear", mutates_args=())
def swiglu_int8_linear(x: torch.Tensor, weight: torch.Tensor, weight_scale: torch.Tensor,
                       bias: torch.Tensor | None, warps: int) -> torch.Tensor:
    """ref: opt/int8_swiglu_fused.py:110-117."""
    q, s = quantize_swiglu(x, num_warps=warps)
    return prequantized_linear(q, s, weight, weight_scale, bias).reshape(*x.shape[:-1], weight.shape[0])


@swiglu_int8_linear.register_fake
def _(x, weight, weight_scale, bias, warps):
    return x.new_empty((*x.shape[:-1], weight.shape[0]))


class FusedFFN(nn.Module):
    """An INT8both FFN whose SwiGLU, activation quantization and w2 GEMM run as one op after w1.
    ref: opt/int8_swiglu_fused.py:124-138."""

    def __init__(self, original, warps=8):
        super().__init__()
        if getattr(original, "mode", None) != "INT8both":
            raise ValueError("requires an existing INT8both FFN")
        self.w1, self.w2 = original.w1, original.w2
        self.warps = warps
        self.train(original.training)

    def forward(self, x):
        if self.training or torch.is_grad_enabled():
            raise RuntimeError("eval + no_grad/inference_mode required")
        return swiglu_int8_linear(self.w1(x), self.w2.qweight, self.w2.weight_scale, self.w2.bias, self.warps)


def clone_fused_decoder(raw, warps=8):
    """A container clone of `raw` (weights shared) with every block's FFN wrapped in FusedFFN.
    ref: opt/int8_swiglu_fused.py:141-155."""
    from ._containers import clone_containers, require_backend
    require_backend()
    if raw.training:
        raise ValueError("decoder.eval() required")
    result = clone_containers(raw)
    for block in result.transformer_blocks:
        block.ff = FusedFFN(block.ff, warps).eval()
    return result


__all__ = ["FusedFFN", "clone_fused_decoder", "quantize_swiglu", "prequantized_linear", "swiglu_int8_linear",
           "validate_input"]
