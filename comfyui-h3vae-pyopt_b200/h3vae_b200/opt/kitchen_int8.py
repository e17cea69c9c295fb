"""Decoder INT8 linears with static rowwise weights (mirror of the reference's opt/kitchen_int8.py).

The reference delegates the GEMM and the dynamic per-row activation quantization to comfy-kitchen
0.2.34 (a closed CUTLASS binary).  Here the activation is row-quantized with the CK contract the
reference restates (scale = max(amax/127, 1e-30), q = rint(fp16(x / fp16(scale)))) and the product
runs on the tcgen05 kind::i8 GEMM with the dequantizing fp16 epilogue."""
from __future__ import annotations

import torch
from torch import nn

from .. import kernels as K
from ..model import quantize_rowwise_weight


@torch.library.custom_op("h3vae_b200::int8_linear", mutates_args=())
def int8_linear(x: torch.Tensor, qweight: torch.Tensor, weight_scale: torch.Tensor,
                bias: torch.Tensor | None) -> torch.Tensor:
    """out = x @ dequant(qweight)^T (+ bias) with per-row dynamic INT8 activations.
    ref: opt/kitchen_int8.py:20-37."""
    q, s = K.row_quant(x.reshape(-1, x.shape[-1]).contiguous())
    return K.gemm_i8(q, s, qweight, weight_scale, bias).reshape(*x.shape[:-1], qweight.shape[0])


@int8_linear.register_fake
def _(x, qweight, weight_scale, bias):
    return x.new_empty((*x.shape[:-1], qweight.shape[0]))


def quantize_static_weight(original: nn.Linear, *, quantize_fn=None, require_cuda: bool = False):
    """Static per-output-row INT8 weights; an all-zero row becomes q = 0, scale = 1.
    ref: opt/kitchen_int8.py:88-145."""
    if not isinstance(original, nn.Linear):
        raise ValueError("kitchen INT8 replacement requires nn.Linear")
    if not bool(torch.isfinite(original.weight.detach()).all()):
        raise ValueError("kitchen INT8 rejects non-finite source weights")
    if require_cuda and (original.weight.device.type != "cuda" or original.weight.dtype != torch.float16):
        raise ValueError("kitchen INT8 decoder requires CUDA FP16 weights")
    if quantize_fn is None:
        return quantize_rowwise_weight(original.weight)
    q, s = quantize_fn(original.weight.detach(), stochastic_rounding=0)
    s = s.reshape(-1).contiguous()
    zero = torch.all(original.weight.detach() == 0, dim=1)
    if bool(zero.any()):
        q, s = q.clone(), s.clone()
        q[zero] = 0
        s[zero] = 1.0
    return q.contiguous(), s


class KitchenInt8Linear(nn.Module):
    """Inference-only linear with static rowwise INT8 weights.  ref: opt/kitchen_int8.py:148-219."""

    def __init__(self, original: nn.Linear, *, quantize_fn=None, require_cuda: bool = False):
        super().__init__()
        q, s = quantize_static_weight(original, quantize_fn=quantize_fn, require_cuda=require_cuda)
        self.register_buffer("qweight", q)
        self.register_buffer("weight_scale", s)
        self.bias = original.bias
        self.in_features, self.out_features = original.in_features, original.out_features
        self.source_dtype = original.weight.dtype
        self.extra_weight_bytes = q.numel() * q.element_size() + s.numel() * s.element_size()
        self.train(original.training)

    def _apply(self, fn, recurse=True):
        scale = self.weight_scale
        out = super()._apply(fn, recurse=recurse)
        self.weight_scale = scale.to(device=self.qweight.device, dtype=torch.float32)
        return out

    def forward(self, x):
        if self.training:
            raise RuntimeError("kitchen INT8 candidate is inference-only; call eval()")
        if torch.is_grad_enabled():
            raise RuntimeError("kitchen INT8 candidate requires torch.no_grad()")
        if x.shape[-1] != self.in_features:
            raise ValueError(f"INT8 input K={x.shape[-1]} does not match K={self.in_features}")
        if x.dtype != self.source_dtype:
            raise ValueError(f"INT8 input dtype must match source dtype {self.source_dtype}, got {x.dtype}")
        return int8_linear(x, self.qweight, self.weight_scale, self.bias)


class KitchenInt8FFN(nn.Module):
    """Gated SiLU FFN with w1 and/or w2 as static-weight INT8 linears (modes INT8both, INT8w1,
    INT8w2); the branch not selected keeps the source linear.  ref: opt/kitchen_int8.py:222-280."""

    MODES = frozenset(("INT8both", "INT8w1", "INT8w2"))

    def __init__(self, original: nn.Module, mode: str = "INT8both", *, quantize_fn=None,
                 require_cuda: bool = False):
        super().__init__()
        if mode not in self.MODES:
            raise ValueError(f"unsupported INT8 FFN mode: {mode}")
        if not bool(getattr(original, "use_gated", False)):
            raise ValueError("kitchen INT8 experiment requires a gated FFN")
        if not isinstance(getattr(original, "act_fn", None), nn.SiLU):
            raise ValueError("kitchen INT8 experiment requires a SiLU FFN")
        for name in ("w1", "w2"):
            if not isinstance(getattr(original, name, None), nn.Linear):
                raise ValueError(f"kitchen INT8 FFN requires an nn.Linear {name}")

        def convert(linear, selected):
            if not selected:
                return linear
            return KitchenInt8Linear(linear, quantize_fn=quantize_fn, require_cuda=require_cuda)

        self.mode = mode
        self.use_gated = True
        self.act_fn = original.act_fn
        self.w1 = convert(original.w1, mode in ("INT8both", "INT8w1"))
        self.w2 = convert(original.w2, mode in ("INT8both", "INT8w2"))
        self.train(original.training)

    @property
    def extra_weight_bytes(self) -> int:
        return sum(getattr(m, "extra_weight_bytes", 0) for m in (self.w1, self.w2))

    def forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
        gate, up = self.w1(hidden_states).chunk(2, dim=-1)
        return self.w2(self.act_fn(gate) * up)


def install_kitchen_int8_ffn(decoder: nn.Module, mode: str = "INT8both", *, require_cuda: bool = True) -> int:
    """Replace every transformer block's FFN of `decoder` in place (the caller owns any clone);
    all blocks are converted before the first assignment, so a block that fails validation leaves
    the decoder unchanged.  Returns the number of FFNs replaced.  ref: opt/kitchen_int8.py:283-310."""
    if decoder.training:
        raise ValueError("kitchen INT8 candidate requires decoder.eval()")
    blocks = getattr(decoder, "transformer_blocks", None)
    if blocks is None:
        raise ValueError("decoder has no transformer_blocks")
    from ._containers import require_backend
    require_backend()
    replacements = [KitchenInt8FFN(block.ff, mode, require_cuda=require_cuda) for block in blocks]
    for block, replacement in zip(blocks, replacements):
        block.ff = replacement
    decoder._h3vae_kitchen_int8_ffn_mode = mode
    return len(replacements)


__all__ = ["KitchenInt8FFN", "KitchenInt8Linear", "install_kitchen_int8_ffn", "int8_linear",
           "quantize_static_weight"]
