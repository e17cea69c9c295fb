"""norm1 producer feeding the INT8 QKV GEMM, updating the residual in place, and the block chain
that carries (h, out, scale2) from one decoder block into the next block's norm1 producer and the
final LayerNorm (mirror of the reference's opt/int8_norm1_quant.py).

The reference enables the chain only on its validated SM120 recipe and only for the H3 B4 shape;
here the gate is this library on an sm_100 device and the kernels take any row count of the
width-2048 block contract."""
from __future__ import annotations

from functools import lru_cache

import torch
import torch.nn.functional as F
from torch import nn

from .. import kernels as K
from .int8_swiglu_fused import prequantized_linear

_EPS = 1.0e-5
_WIDTH = 2048
_FFN_WARPS = 8


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


@lru_cache(maxsize=8)
def _device_supports_norm1_quant(index: int) -> bool:
    try:
        return torch.cuda.get_device_capability(index) == (10, 0)
    except Exception:  # noqa: BLE001 - an unusable device simply does not qualify
        return False


def supports_norm1_quant(device) -> bool:
    """The fused chain runs on an sm_100 CUDA device.  ref: opt/int8_norm1_quant.py:63-82."""
    device = torch.device(device)
    if device.type != "cuda" or torch.version.hip is not None or not torch.cuda.is_available():
        return False
    return _device_supports_norm1_quant(torch.cuda.current_device() if device.index is None else device.index)


class _FinalNormAdapter(nn.Module):
    """The decoder's final LayerNorm, also accepting the last block's (h, out, gate) carry, whose
    residual add is then fused into the LayerNorm.  ref: opt/int8_norm1_quant.py:31-46."""

    def __init__(self, original):
        super().__init__()
        self.weight, self.bias = original.weight, original.bias
        self.normalized_shape, self.eps = original.normalized_shape, original.eps
        self.train(original.training)

    def forward(self, states):
        if not isinstance(states, tuple):
            return F.layer_norm(states, self.normalized_shape, self.weight, self.bias, self.eps)
        if self.training or torch.is_grad_enabled():
            raise RuntimeError("eval + inference/no_grad required")
        from .decoder_norms import final_residual_ln_w8
        h, out, gate = states
        return final_residual_ln_w8(h, out, gate, self.weight, self.bias)


def _carry_safe_unpad(original_unpad):
    """Wrap the decoder's sequence unpadding so a carry tuple passes only unchanged (zero padding).
    ref: opt/int8_norm1_quant.py:49-60."""
    def unpad(states, pad_len):
        if not isinstance(states, tuple):
            return original_unpad(states, pad_len)
        if pad_len != 0:
            raise RuntimeError("final residual carry requires zero sequence padding")
        result = original_unpad(states, pad_len)
        if result is not states:
            raise RuntimeError("zero unpadding must preserve final residual carry")
        return result
    return unpad


def _qk_rope_for(attn):
    """The fused QK-norm + RoPE op behind a FusedQKAttention.  ref: opt/int8_norm1_quant.py:165-173."""
    from .decoder_fused_qk_rope import FusedQKAttention, qk_rope
    if not isinstance(attn, FusedQKAttention):
        raise ValueError("expected the runtime FusedQKAttention class")
    return qk_rope


def _attention_from_qkv(attn, qkv, rotary, pack_info, qk_rope):
    """The attention of a FusedQKAttention from an already computed qkv.  ref: opt/int8_norm1_quant.py:176-182."""
    a = attn.original
    b, n, _ = qkv.shape
    q, k = qk_rope(qkv, *rotary, a.heads, a.norm_q.eps, attn.rows)
    v = qkv.view(b, n, a.heads, 3 * a.dim_head)[..., 2 * a.dim_head:]
    return a.to_out(a.perform_attention(q, k, v, pack_info).reshape(b, n, -1))


class _Norm1QuantBlock(nn.Module):
    """A NormQuantBlock in the carry chain: it returns (h, out, scale2) instead of h + out * scale2
    when the next block can fold that residual add into its norm1 producer (residual_qkv), block 0
    normalizes with the fused RMSNorm, and the last block hands its carry to the final LayerNorm.
    ref: opt/int8_norm1_quant.py:185-252."""

    def __init__(self, src, first, last, norm1_enabled):
        super().__init__()
        self.norm1, self.norm2, self.attn, self.ff = src.norm1, src.norm2, src.attn, src.ff
        self.scale1, self.scale2 = src.scale1, src.scale2
        self.warps, self.fuse_ffn_up = src.warps, src.fuse_ffn_up
        self.norm1_enabled = bool(norm1_enabled)
        self.fuse_norm1 = self.norm1_enabled and supports_norm1_quant(self.scale1.device)
        self.qk_rope = _qk_rope_for(self.attn)
        self.first, self.last = first, last
        self.train(src.training)

    def _apply(self, fn, recurse=True):
        from .int8_ffn_up_fused import supports_fused_ffn_up
        out = super()._apply(fn, recurse=recurse)
        self.fuse_ffn_up = supports_fused_ffn_up(self.scale1.device)
        self.fuse_norm1 = self.norm1_enabled and supports_norm1_quant(self.scale1.device)
        return out

    def _ffn_pair(self, h, attn):
        w1, w2 = self.ff.w1, self.ff.w2
        if self.fuse_ffn_up:
            from .int8_ffn_up_fused import fused_residual_ffn
            return fused_residual_ffn(h, attn, self.scale1, self.norm2.weight, w1.qweight, w1.weight_scale, w1.bias,
                                      w2.qweight, w2.weight_scale, w2.bias, self.norm2.eps, self.warps)
        from .int8_norm_quant import residual_rms_linear
        from .int8_swiglu_fused import swiglu_int8_linear
        h, hidden = residual_rms_linear(h, attn, self.scale1, self.norm2.weight, w1.qweight, w1.weight_scale,
                                        w1.bias, self.norm2.eps, self.warps)
        return h, swiglu_int8_linear(hidden, w2.qweight, w2.weight_scale, w2.bias, 16)

    def _target_shape(self, h):
        return (self.fuse_norm1 and h.ndim == 3 and h.shape[-1] == _WIDTH and h.dtype == torch.float16
                and h.is_cuda and h.is_contiguous())

    def forward(self, states, rotary_pos_emb=None, pack_info=None):
        if self.training or torch.is_grad_enabled():
            raise RuntimeError("eval + inference/no_grad required")
        pack_info = {} if pack_info is None else pack_info
        chain = False
        if isinstance(states, tuple):
            h, prev_out, prev_scale2 = states
            if (not self.first and rotary_pos_emb is not None and self._target_shape(h)
                    and prev_out.shape == h.shape and prev_out.dtype == torch.float16 and prev_out.is_contiguous()):
                linear = self.attn.original.to_qkv
                qkv = residual_qkv(h, prev_out, prev_scale2, self.norm1.weight, linear.qweight,
                                   linear.weight_scale, linear.bias)   # h += prev_out * prev_scale2
                attn = _attention_from_qkv(self.attn, qkv, rotary_pos_emb, pack_info, self.qk_rope)
                states, chain = h, True
            else:
                states = h + prev_out * prev_scale2
                attn = self.attn(self.norm1(states.float()).to(states.dtype), rotary_pos_emb, pack_info)
        else:
            if self.first and self._target_shape(states):
                from .decoder_norms import rms_fp16_x2_w16
                normed = rms_fp16_x2_w16(states, self.norm1.weight)
            else:
                normed = self.norm1(states.float()).to(states.dtype)
            attn = self.attn(normed, rotary_pos_emb, pack_info)
            chain = self._target_shape(states) and rotary_pos_emb is not None
        h, out = self._ffn_pair(states, attn)
        if self.last:
            return (h, out, self.scale2) if self._target_shape(h) else h + out * self.scale2
        return (h, out, self.scale2) if chain else h + out * self.scale2


def _validate_blocks(blocks):
    """The fused chain's block contract: 36 eval NormQuantBlocks of width 2048 (fp16 RMSNorms with
    eps 1e-5, fp16 scales), FusedQKAttention, and already-INT8 QKV / out / FFN linears.
    ref: opt/int8_norm1_quant.py:255-279."""
    from .kitchen_int8 import KitchenInt8Linear
    if len(blocks) != 36:
        raise ValueError("norm1 fusion expects 36 decoder blocks")
    for block in blocks:
        norms_ok = all(isinstance(n, nn.RMSNorm) and tuple(n.normalized_shape) == (_WIDTH,) and n.weight is not None
                       and n.eps == _EPS and n.weight.dtype == torch.float16 for n in (block.norm1, block.norm2))
        scales_ok = all(t.shape == (_WIDTH,) and t.dtype == torch.float16 for t in (block.scale1, block.scale2))
        if block.training or block.warps != _FFN_WARPS or not norms_ok or not scales_ok:
            raise ValueError("norm1 fusion requires the validated FP16 width-2048 block contract")
        _qk_rope_for(block.attn)
        a = block.attn.original
        linears = (a.to_qkv, a.to_out, block.ff.w1, block.ff.w2)
        if (not all(isinstance(m, KitchenInt8Linear) for m in linears)
                or tuple(a.to_qkv.qweight.shape) != (6144, _WIDTH) or tuple(a.to_qkv.weight_scale.shape) != (6144,)):
            raise ValueError("expected an already-quantized INT8 decoder; refusing requantization")


def clone_norm1_quant_decoder(raw, *, enabled=False):
    """Container clone of an already-INT8 36-block decoder; with enabled=True its blocks become the
    carry chain and its final LayerNorm / unpadding accept the carry.  ref: opt/int8_norm1_quant.py:282-319."""
    from ._containers import clone_containers, require_backend
    if raw.training:
        raise ValueError("eval decoder required")
    blocks = getattr(raw, "transformer_blocks", None)
    if blocks is None or len(blocks) != 36:
        raise ValueError("expected a 36-block decoder")
    result = clone_containers(raw)
    try:
        device = next(raw.parameters()).device
    except StopIteration:
        raise ValueError("decoder has no parameters") from None
    if not enabled:
        result._h3vae_norm1_quant_enabled = False
        return result.eval()
    if not supports_norm1_quant(device):
        raise RuntimeError("norm1 fusion requires an sm_100 CUDA device")
    require_backend()
    # a carry tuple cannot pass a sequence-parallel gather or nonzero unpadding
    if getattr(raw, "spatial_parallel", True):
        raise RuntimeError("authored final LayerNorm requires spatial_parallel=false")
    norm = getattr(raw, "norm_out", None)
    if (type(norm) is not nn.LayerNorm or "forward" in vars(norm) or tuple(norm.normalized_shape) != (_WIDTH,)
            or norm.eps != _EPS or norm.weight is None or norm.bias is None
            or norm.weight.dtype != torch.float16 or norm.bias.dtype != torch.float16):
        raise ValueError("final LayerNorm requires affine FP16 width-2048/eps-1e-5")
    chain = list(result.transformer_blocks)
    _validate_blocks(chain)
    result.transformer_blocks = nn.ModuleList(
        [_Norm1QuantBlock(block, i == 0, i == len(chain) - 1, norm1_enabled=True).eval()
         for i, block in enumerate(chain)])
    result.norm_out = _FinalNormAdapter(result.norm_out).eval()
    result._unpad_for_sp = _carry_safe_unpad(result._unpad_for_sp)
    result._h3vae_norm1_quant_enabled = True
    return result.eval()


__all__ = ["clone_norm1_quant_decoder", "residual_qkv", "residual_qkv_impl", "supports_norm1_quant"]
