"""FP16-input, FP32-accumulate FFN-up GEMM with the SwiGLU epilogue (mirror of the reference's
opt/fp16_swiglu_gemm.py; its Triton kernel becomes the tcgen05 kind::f16 GEMM h3b_gemm_f16_swiglu).

Numerics follow the reference: fp32 accumulation, the bias added in fp32, gate and up rounded to
fp16, silu(gate) * up in fp32, one rounding to the fp16 output.  The reference's five-integer
Triton tile config (bm, bn, bk, warps, stages) is validated against the reference's accepted
values so existing callers and saved prompts keep working; the sm_100a kernel picks its own tiles
(128 rows x 128 gate + 128 up columns, 4 stages), so the config does not change the result.
"""
from __future__ import annotations

import torch
from torch import nn

from .. import kernels as K
from ._containers import clone_containers

_BM = (32, 64, 128, 256)
_BN = (32, 64, 128)
_BK = (32, 64, 128)
_WARPS = (4, 8)
_STAGES = (2, 3, 4, 5)


def validate(x, w, bias, config):
    """Contract checks before any launch.  ref: opt/fp16_swiglu_gemm.py:50-63."""
    if x.dtype != torch.float16 or w.dtype != torch.float16:
        raise ValueError("FP16 activations and weights required")
    if x.ndim < 2 or w.ndim != 2 or x.shape[-1] != w.shape[1] or w.shape[0] % 2:
        raise ValueError("expected matching K and paired gate/up output rows")
    if x.numel() == 0 or w.numel() == 0 or not x.is_contiguous() or not w.is_contiguous():
        raise ValueError("nonempty contiguous tensors required")
    if bias is not None and (tuple(bias.shape) != (w.shape[0],) or bias.dtype != x.dtype
                             or not bias.is_contiguous()):
        raise ValueError("contiguous FP16 bias with output width required")
    if len(config) != 5 or any(type(v) is not int for v in config):
        raise ValueError("five integer config values required")
    bm, bn, bk, warps, stages = config
    if bm not in _BM or bn not in _BN or bk not in _BK or warps not in _WARPS or stages not in _STAGES:
        raise ValueError("unsupported kernel configuration")


def fused_w1_swiglu(x, w, bias=None, config=(64, 64, 64, 4, 3)):
    """act[..., j] = fp16(silu(g) * u) with g, u = fp16(x @ w[j]^T + b[j]), fp16(x @ w[F+j]^T + b[F+j]).
    ref: opt/fp16_swiglu_gemm.py:66-80."""
    validate(x, w, bias, config)
    if x.device.type != "cuda" or torch.version.hip is not None:
        raise ValueError("NVIDIA CUDA required")
    if w.device != x.device or (bias is not None and bias.device != x.device):
        raise ValueError("same device required")
    k = x.shape[-1]
    act = K.gemm_f16_swiglu(x.reshape(-1, k), w, bias)
    return act.reshape(*x.shape[:-1], w.shape[0] // 2)


@torch.library.custom_op("h3vae_b200_fp16_exp::w1_swiglu", mutates_args=())
def w1_swiglu(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None,
              bm: int, bn: int, bk: int, warps: int, stages: int) -> torch.Tensor:
    """ref: opt/fp16_swiglu_gemm.py:83-86."""
    return fused_w1_swiglu(x, w, bias, (bm, bn, bk, warps, stages))


@w1_swiglu.register_fake
def _(x, w, bias, bm, bn, bk, warps, stages):
    return x.new_empty((*x.shape[:-1], w.shape[0] // 2))


class FusedFP16FFN(nn.Module):
    """A gated-SiLU FFN whose w1 + SwiGLU runs as one fused GEMM; w2 stays the model's own linear.
    ref: opt/fp16_swiglu_gemm.py:94-110."""

    def __init__(self, original, config):
        super().__init__()
        if original.training or not original.use_gated or not isinstance(original.act_fn, nn.SiLU):
            raise ValueError("eval gated SiLU FFN required")
        if not isinstance(original.w1, nn.Linear) or not isinstance(original.w2, nn.Linear):
            raise ValueError("original FP16 nn.Linear FFN required")
        if original.w1.out_features != 2 * original.w2.in_features:
            raise ValueError("gate/up dimensions do not match w2")
        self.w1, self.w2 = original.w1, original.w2
        self.config = tuple(config)
        self.eval()

    def forward(self, x):
        if self.training or torch.is_grad_enabled():
            raise RuntimeError("inference only")
        return self.w2(w1_swiglu(x, self.w1.weight, self.w1.bias, *self.config))


def clone_fp16_decoder(raw, config):
    """The decoder with every transformer block's FFN replaced by FusedFP16FFN; the original module
    tree is left untouched and the weights are shared, not copied.  ref: opt/fp16_swiglu_gemm.py:113-124."""
    if raw.training:
        raise ValueError("eval decoder required")
    result = clone_containers(raw)
    for block in result.transformer_blocks:
        block.ff = FusedFP16FFN(block.ff, config)
    return result


__all__ = ["validate", "fused_w1_swiglu", "w1_swiglu", "FusedFP16FFN", "clone_fp16_decoder"]
