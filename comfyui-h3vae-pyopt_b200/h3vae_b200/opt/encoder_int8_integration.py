"""torch.library boundaries of the INT8 encoder convolutions and the static-weight wrapper (mirror of
the reference's opt/encoder_int8_integration.py).  The module-graph installer of the reference
(install_int8_encoder_prefix) targets the external klvae model and is not reproduced; the
synthetic H3 encoder of h3vae_b200.model wires the same ops directly."""
from __future__ import annotations

import torch
from torch import nn

from .encoder_int8 import (Int8Conv3DConfig, _conv3d_from_quantized, _valid_output_shape, int8_valid_conv3d,
                           prepare_int8_weight)
from .encoder_int8_norm import quantized_temporal_norm_pad

INT8_ENCODER_POLICY = {
    "stages": (0, 1),
    "blocks_per_stage": 2,
    "convolutions_per_block": ("first", "second"),
    "quantized_conv_count": 8,
    "kernel": (3, 3, 3),
    "excluded": ("conv_in", "conv_out", "downsample", "nin_shortcut", "encoder suffix", "quant_conv"),
}


@torch.library.custom_op("h3vae_b200_encoder::int8_valid_conv3d_integration", mutates_args=(),
                         device_types="cuda")
def int8_valid_conv3d_integration(x: torch.Tensor, qweight: torch.Tensor, weight_scale: torch.Tensor,
                                  bias: torch.Tensor, kernel_d: int, kernel_h: int, kernel_w: int, stride_d: int,
                                  stride_h: int, stride_w: int, apply_bias: bool, tile_variant: str) -> torch.Tensor:
    """ref: opt/encoder_int8_integration.py:105-139."""
    taps = int(kernel_d) * int(kernel_h) * int(kernel_w)
    config = Int8Conv3DConfig(int(qweight.shape[1]) // taps, int(qweight.shape[0]),
                              (int(kernel_d), int(kernel_h), int(kernel_w)), (int(stride_d), int(stride_h), int(stride_w)))
    return int8_valid_conv3d(x, qweight, weight_scale, config=config, bias=bias if apply_bias else None)


@int8_valid_conv3d_integration.register_fake
def _(x, qweight, weight_scale, bias, kernel_d, kernel_h, kernel_w, stride_d, stride_h, stride_w, apply_bias,
      tile_variant):
    taps = int(kernel_d) * int(kernel_h) * int(kernel_w)
    config = Int8Conv3DConfig(int(qweight.shape[1]) // taps, int(qweight.shape[0]),
                              (int(kernel_d), int(kernel_h), int(kernel_w)), (int(stride_d), int(stride_h), int(stride_w)))
    return torch.empty(_valid_output_shape(tuple(x.shape), config), device=x.device, dtype=x.dtype,
                       memory_format=torch.channels_last_3d)


@torch.library.custom_op("h3vae_b200_encoder::int8_norm_conv3d", mutates_args=(), device_types="cuda")
def int8_norm_conv3d(x: torch.Tensor, norm_weight: torch.Tensor, norm_bias: torch.Tensor,
                     pre_bias: torch.Tensor | None, eps: float, qweight: torch.Tensor, weight_scale: torch.Tensor,
                     bias: torch.Tensor | None) -> torch.Tensor:
    """GroupNorm/SiLU/padding/quantization then the causal INT8 3x3x3 conv (the producer guarantees the
    two zero causal frames, so their taps are skipped).  ref: opt/encoder_int8_integration.py:172-201."""
    qx, scale = quantized_temporal_norm_pad(x, norm_weight, norm_bias, eps, pre_bias=pre_bias)
    return _conv3d_from_quantized(qx, scale, qweight, weight_scale,
                                  config=Int8Conv3DConfig(x.shape[1], qweight.shape[0], (3, 3, 3), (1, 1, 1)),
                                  bias=bias, causal_prefix_zero=True)


@int8_norm_conv3d.register_fake
def _(x, norm_weight, norm_bias, pre_bias, eps, qweight, weight_scale, bias):
    return torch.empty((x.shape[0], qweight.shape[0], *x.shape[2:]), device=x.device, dtype=x.dtype,
                       memory_format=torch.channels_last_3d)


class Int8FusedValidConv3d(nn.Module):
    """Static-weight INT8 wrapper of a 3x3x3 source conv.  ref: opt/encoder_int8_integration.py:212-318."""

    def __init__(self, source: nn.Module, *, apply_bias: bool, tile_variant: str = "tcgen05") -> None:
        super().__init__()
        w = getattr(source, "weight", None)
        b = getattr(source, "bias", None)
        if not isinstance(w, torch.Tensor) or w.ndim != 5:
            raise ValueError("INT8 encoder source must expose a rank-5 weight")
        if b is None or b.ndim != 1 or b.shape[0] != w.shape[0]:
            raise ValueError("INT8 encoder integration requires a source bias matching the output channels")
        if tuple(w.shape[-3:]) != (3, 3, 3):
            raise ValueError("the initial INT8 encoder policy only supports 3x3x3")
        qweight, scale, config = prepare_int8_weight(w, stride=tuple(getattr(source, "stride", (1, 1, 1))))
        self.qweight = nn.Parameter(qweight.contiguous(), requires_grad=False)
        self.register_buffer("weight_scale", scale.float().contiguous(), persistent=True)
        self.bias = nn.Parameter(b.detach().clone().half().contiguous(), requires_grad=False)
        self.config = config
        self.apply_bias = bool(apply_bias)
        self.tile_variant = str(tile_variant)
        self.fuse_norm = config.stride == (1, 1, 1)

    def _apply(self, fn, recurse=True):
        scale = self.weight_scale.detach().clone()
        out = super()._apply(fn, recurse=recurse)
        self.qweight.data = self.qweight.data.to(dtype=torch.int8)
        self.weight_scale.data = scale.to(device=self.weight_scale.device, dtype=torch.float32)
        self.bias.data = self.bias.data.to(dtype=torch.float16)
        return out

    def forward_norm(self, x, norm_weight, norm_bias, eps, pre_bias=None):
        if not self.fuse_norm:
            raise RuntimeError("INT8 norm fusion is not enabled for this convolution")
        if x.dtype != torch.float16:
            raise RuntimeError("INT8 encoder convolution requires FP16 activations")
        if x.device != self.qweight.device:
            raise RuntimeError("INT8 encoder activation and qweight must be on the same device")
        return int8_norm_conv3d(x, norm_weight, norm_bias, pre_bias, eps, self.qweight, self.weight_scale,
                                self.bias if self.apply_bias else None)

    def forward(self, x):
        if x.dtype != torch.float16:
            raise RuntimeError("INT8 encoder convolution requires FP16 activations")
        if x.device != self.qweight.device:
            raise RuntimeError("INT8 encoder activation and qweight must be on the same device")
        k, s = self.config.kernel_size, self.config.stride
        return int8_valid_conv3d_integration(x, self.qweight, self.weight_scale, self.bias, k[0], k[1], k[2], s[0],
                                             s[1], s[2], self.apply_bias, self.tile_variant)


__all__ = ["INT8_ENCODER_POLICY", "Int8FusedValidConv3d", "int8_valid_conv3d_integration", "int8_norm_conv3d"]
