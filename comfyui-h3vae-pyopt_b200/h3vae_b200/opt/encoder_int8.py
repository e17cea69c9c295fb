"""INT8 implicit-GEMM causal conv3d (mirror of the reference's opt/encoder_int8.py).

The reference's Triton kernels are replaced by the tcgen05 kind::i8 kernel of libh3vae_b200.so;
activations are quantized once per call with one fp32 tensor scale, weights once per output
channel, accumulation is int32 and the fp16 epilogue is fused.  There is no fp16 fallback.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
from torch import nn

from .. import kernels as K
from ..model import prepare_int8_weight as _pack_weight

_TILE_VARIANTS = ("64x64x64", "128x64x64", "128x64x128", "128x128x64", "128x128x64_pipeline4", "tcgen05")


@dataclass(frozen=True)
class Int8Conv3DConfig:
    """Static configuration of the valid convolution contract.  ref: opt/encoder_int8.py:42-51."""
    in_channels: int
    out_channels: int
    kernel_size: tuple[int, int, int]
    stride: tuple[int, int, int]
    dilation: tuple[int, int, int] = (1, 1, 1)
    groups: int = 1


def int32_accumulator_bound(config: Int8Conv3DConfig) -> int:
    """Worst-case |int32 dot| for symmetric int8 operands.  ref: opt/encoder_int8.py:54-58."""
    return config.in_channels * math.prod(config.kernel_size) * 127 * 127


def validate_int8_weight_buffers(qweight, weight_scale, config: Int8Conv3DConfig) -> None:
    """One-time (synchronizing) validation of the static buffers.  ref: opt/encoder_int8.py:61-91."""
    expected = (config.out_channels, math.prod(config.kernel_size) * config.in_channels)
    if tuple(qweight.shape) != expected:
        raise ValueError(f"qweight shape {tuple(qweight.shape)} != packed {expected}")
    if qweight.dtype != torch.int8 or not qweight.is_contiguous():
        raise ValueError("qweight must be contiguous torch.int8")
    if tuple(weight_scale.shape) != (config.out_channels,):
        raise ValueError("weight_scale must be [out_channels]")
    if weight_scale.dtype != torch.float32 or not weight_scale.is_contiguous():
        raise ValueError("weight_scale must be contiguous FP32")
    if not bool(torch.isfinite(weight_scale).all().item()) or not bool((weight_scale > 0).all().item()):
        raise ValueError("weight_scale must be finite and positive")


def _validate_conv_config(weight, stride, dilation, groups) -> Int8Conv3DConfig:
    """ref: opt/encoder_int8.py:275-300."""
    if weight.ndim != 5:
        raise ValueError("weight must be [out_channels, in_channels, kd, kh, kw]")
    if groups != 1:
        raise ValueError("INT8 implicit conv currently supports groups=1 only")
    if tuple(dilation) != (1, 1, 1):
        raise ValueError("INT8 implicit conv currently supports dilation=1 only")
    stride = tuple(int(v) for v in stride)
    if any(v not in (1, 2) for v in stride):
        raise ValueError("INT8 implicit conv supports stride values 1 or 2")
    kernel_size = tuple(int(v) for v in weight.shape[-3:])
    if any(v not in (1, 3) for v in kernel_size):
        raise ValueError("INT8 implicit conv supports kernel dimensions 1 or 3")
    return Int8Conv3DConfig(int(weight.shape[1]), int(weight.shape[0]), kernel_size, stride)


def prepare_int8_weight(weight: torch.Tensor, *, stride=(1, 1, 1), dilation=(1, 1, 1), groups=1):
    """Packed [O, kd*kh*kw*C] int8 weights + fp32 per-channel scales.  ref: opt/encoder_int8.py:303-327."""
    if weight.numel() == 0 or not weight.is_floating_point():
        raise ValueError("source weight must be a non-empty floating tensor")
    if not bool(torch.isfinite(weight.detach()).all().item()):
        raise ValueError("source weight contains non-finite values")
    config = _validate_conv_config(weight, stride, dilation, groups)
    bound = int32_accumulator_bound(config)
    if bound >= 2**31:
        raise ValueError(f"INT32 accumulator bound {bound} exceeds signed INT32 range")
    q, s = _pack_weight(weight)
    return q, s, config


@torch.no_grad()
def quantize_activation_tensor(x: torch.Tensor, *, check_finite: bool = False):
    """One fp32 scale per tensor, half-away rounding, NDHWC int8.  ref: opt/encoder_int8.py:384-426."""
    if x.ndim != 5:
        raise ValueError("activation must be [B,C,D,H,W]")
    if x.dtype != torch.float16:
        raise ValueError("INT8 implicit conv currently requires FP16 activations")
    if not x.is_cuda:
        raise RuntimeError("INT8 activation quantization requires CUDA")
    if check_finite and not bool(torch.isfinite(x).all().item()):
        raise ValueError("INT8 activation quantization rejects non-finite input")
    if x.numel() == 0:
        raise ValueError("INT8 activation quantization requires a nonempty tensor")
    return K.quantize_tensor_i8(x)


def _valid_output_shape(x_shape, config: Int8Conv3DConfig):
    """ref: opt/encoder_int8.py:433-450."""
    b, _, d, h, w = x_shape
    out = tuple((n - k) // s + 1 for n, k, s in zip((d, h, w), config.kernel_size, config.stride))
    if any(v <= 0 for v in out):
        raise ValueError(f"input shape {tuple(x_shape)} is too small for valid conv")
    return (b, config.out_channels, *out)


def _conv3d_from_quantized(qx, activation_scale, qweight, weight_scale, *, config: Int8Conv3DConfig, bias,
                           tile_variant: str = "tcgen05", causal_prefix_zero: bool = False):
    """Valid INT8 conv of a validated NDHWC int8 input.  causal_prefix_zero: the producer guarantees
    two leading zero frames, whose temporal taps are skipped.  ref: opt/encoder_int8.py:509-588."""
    if tile_variant not in _TILE_VARIANTS:
        raise ValueError(f"unknown tile variant {tile_variant!r}")
    _valid_output_shape(tuple(qx.shape), config)
    return K.conv3d_i8(qx, activation_scale, qweight, weight_scale, bias, config.kernel_size, config.stride,
                       causal_zero_frames=2 if causal_prefix_zero else 0)


@torch.no_grad()
def int8_valid_conv3d(x, qweight, weight_scale, *, config: Int8Conv3DConfig, bias=None,
                      tile_variant: str = "tcgen05"):
    """Quantize + valid INT8 conv with no fp16 fallback.  ref: opt/encoder_int8.py:454-506."""
    if tile_variant not in _TILE_VARIANTS:
        raise ValueError(f"unknown tile variant {tile_variant!r}")
    if x.ndim != 5 or x.device.type != "cuda":
        raise RuntimeError("INT8 implicit conv requires a CUDA 5-D activation")
    if x.dtype != torch.float16:
        raise ValueError("INT8 implicit conv currently requires FP16 activations")
    if qweight.dtype != torch.int8 or qweight.device != x.device:
        raise ValueError("qweight must be CUDA torch.int8")
    if not qweight.is_contiguous():
        raise ValueError("qweight must use packed contiguous layout")
    if weight_scale.dtype != torch.float32 or weight_scale.device != x.device:
        raise ValueError("weight_scale must be CUDA FP32")
    if tuple(weight_scale.shape) != (config.out_channels,) or not weight_scale.is_contiguous():
        raise ValueError("weight_scale must be [out_channels]")
    expected = (config.out_channels, math.prod(config.kernel_size) * config.in_channels)
    if tuple(qweight.shape) != expected:
        raise ValueError(f"qweight shape {tuple(qweight.shape)} != packed {expected}")
    if x.shape[1] != config.in_channels:
        raise ValueError("activation channel count does not match qweight")
    if bias is not None and (bias.device != x.device or bias.dtype != torch.float16 or bias.ndim != 1
                             or bias.numel() != config.out_channels or not bias.is_contiguous()):
        raise ValueError("bias must be contiguous CUDA FP16 [out_channels]")
    qx, scale = quantize_activation_tensor(x)
    return _conv3d_from_quantized(qx, scale, qweight, weight_scale, config=config, bias=bias, tile_variant=tile_variant)


class Int8Conv3d(nn.Module):
    """Inference-only INT8 replacement of one (already padded) Conv3d.  ref: opt/encoder_int8.py:653-717."""

    def __init__(self, original: nn.Module, *, assume_padded: bool = True):
        super().__init__()
        if not isinstance(original, nn.Conv3d):
            raise ValueError("expected an nn.Conv3d-compatible source module")
        if not assume_padded:
            raise ValueError("only pre-padded inputs are supported (assume_padded=True)")
        config = _validate_conv_config(original.weight, tuple(original.stride), tuple(original.dilation),
                                       int(original.groups))
        qweight, scale, _ = prepare_int8_weight(original.weight, stride=config.stride)
        validate_int8_weight_buffers(qweight, scale, config)
        self.qweight = nn.Parameter(qweight, requires_grad=False)
        self.register_buffer("weight_scale", scale, persistent=True)
        if original.bias is None:
            self.register_buffer("bias", None, persistent=True)
        else:
            if not bool(torch.isfinite(original.bias.detach()).all().item()):
                raise ValueError("source bias contains non-finite values")
            self.bias = nn.Parameter(original.bias.detach().clone().half().contiguous(), requires_grad=False)
        self.config = config

    def _apply(self, fn, recurse=True):
        scale = self.weight_scale.detach().clone()
        out = super()._apply(fn, recurse=recurse)
        self.qweight.data = self.qweight.data.to(dtype=torch.int8)
        self.weight_scale.data = scale.to(device=self.qweight.device, dtype=torch.float32)
        return out

    @torch.no_grad()
    def forward(self, x):
        return int8_valid_conv3d(x, self.qweight, self.weight_scale, config=self.config, bias=self.bias)


TritonInt8Conv3d = Int8Conv3d  # the reference's class name (ref: opt/encoder_int8.py:653)

__all__ = ["Int8Conv3DConfig", "Int8Conv3d", "TritonInt8Conv3d", "int8_valid_conv3d", "prepare_int8_weight",
           "quantize_activation_tensor", "int32_accumulator_bound", "validate_int8_weight_buffers"]
