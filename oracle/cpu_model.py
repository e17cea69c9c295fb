"""CPU forward passes of the H3-structured encoder and decoder, for the CPU baseline and model-level checks.

TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs may
import this module; the product path never does.

It runs one encoder work item (a clip batch of one spatial tile) or one decoder tile task on the host
cores with the arithmetic of the reference's CPU path, taking the weights from the model objects
(h3vae_b200.model.H3Encoder / H3Decoder, duck-typed: only their weight attributes are read):

* INT8 convolutions as the reference's CPU oracle computes them (opt/encoder_int8.py:591-619): the
  per-tensor quantized activation and the per-channel quantized weight dequantized to fp32 and
  convolved in fp32 (dtype=torch.float64 instead gives the exact integer sums of the GPU path);
* the GroupNorm(32) + SiLU + reflect / causal pad producers with their fp16 rounding points
  (opt/encoder_int8_norm_recompute.py:27-49), the residual pack (opt/encoder_fused_residual_pack.py:13-32);
* fp16 convolutions as fp32 convolutions rounded to fp16;
* the decoder block chain of the INT8 profile (opt/int8_norm1_quant.py:185-252): CK row quantization,
  INT8 linears as dequantized fp32 matmuls (float64: exact), QK RMSNorm + rotary, attention
  (torch SDPA on the CPU), residual + RMSNorm + row quantization, FFN-up + SwiGLU, final LayerNorm;
* nearest x2 spatial / causal x2 temporal upsampling before each decoder producer.

`timer` (an OpTimer) splits the wall time into work that grows linearly with the number of positions
(every convolution, producer and linear) and attention (quadratic in the tokens of a tile), so a timed
sample on a spatial crop can be scaled to the full tile exactly by op count.
"""
from __future__ import annotations

import math
import time
from contextlib import contextmanager

import torch
import torch.nn.functional as F

F16 = torch.float16
RECIP_127 = torch.tensor(1.0, dtype=torch.float32) / torch.tensor(127.0, dtype=torch.float32)


class OpTimer:
    """Wall seconds per cost class: 'linear' (scales with positions) and 'attention' (quadratic)."""

    def __init__(self):
        self.seconds = {"linear": 0.0, "attention": 0.0}

    @contextmanager
    def __call__(self, kind: str):
        t0 = time.perf_counter()
        try:
            yield
        finally:
            self.seconds[kind] += time.perf_counter() - t0


class _NoTimer:
    @contextmanager
    def __call__(self, kind: str):
        yield


def _t(x, dtype=torch.float32):
    return x.detach().to("cpu", dtype)


def _f16(x):
    return x.to(F16).to(torch.float32)


# ---------------------------------------------------------------------------
# producers
# ---------------------------------------------------------------------------
def _reflect_causal_pad(z):
    """Reflect pad 1 in H and W (zero pad for a 1-pixel axis), two zero frames in front."""
    if min(z.shape[-2:]) > 1:
        z = F.pad(z, (1, 1, 1, 1, 0, 0), mode="reflect")
    else:
        z = F.pad(z, (1, 1, 1, 1, 0, 0))
    return F.pad(z, (0, 0, 0, 0, 2, 0))


def _upsample(x, spatial: bool, temporal: bool):
    """Nearest x2 spatial; causal x2 temporal (frame 0 once, later frames twice: D -> 2D-1)."""
    if spatial:
        x = x.repeat_interleave(2, dim=-1).repeat_interleave(2, dim=-2)
    if temporal and x.shape[2] > 1:
        idx = torch.tensor([(f + 1) // 2 for f in range(2 * x.shape[2] - 1)])
        x = x.index_select(2, idx)
    return x


def norm_silu(x, gamma, beta, eps, pre_bias=None, groups: int = 32):
    """fp16 GroupNorm per (batch, frame, group) -> fp16 -> SiLU -> fp16 (fp32 values of fp16 numbers)."""
    v = x.to(torch.float32)
    if pre_bias is not None:
        v = _f16(v + _t(pre_bias).view(1, -1, 1, 1, 1))
    b, c, d, h, w = v.shape
    g = v.view(b, groups, c // groups, d, h, w)
    mean = g.mean(dim=(2, 4, 5), keepdim=True)
    var = ((g - mean) ** 2).mean(dim=(2, 4, 5), keepdim=True)
    z = (g - mean) * torch.rsqrt(var.clamp_min(0) + eps)
    z = _f16(z.view(b, c, d, h, w) * _t(gamma).view(1, -1, 1, 1, 1) + _t(beta).view(1, -1, 1, 1, 1))
    return _f16(z / (1.0 + torch.exp(-z)))


def quantize_tensor(y):
    """Per-tensor scale absmax * fp32(1/127) (0 -> 1), half-away rounding, clamp +-127."""
    scale = y.abs().amax() * RECIP_127
    scale = torch.where(scale > 0, scale, torch.ones_like(scale))
    s = y / scale
    q = torch.where(s >= 0, torch.floor(s + 0.5), -torch.floor(-s + 0.5)).clamp_(-127, 127)
    return q, scale


def residual_pack(x, r, bias):
    """fp16(r + (x + bias)); right/bottom reflect +1; two zero frames in front."""
    y = _f16(r.to(torch.float32) + (x.to(torch.float32) + _t(bias).view(1, -1, 1, 1, 1)))
    y = torch.cat([y, y[..., -2:-1, :]], dim=-2)
    y = torch.cat([y, y[..., -2:-1]], dim=-1)
    return F.pad(y, (0, 0, 0, 0, 2, 0))


# ---------------------------------------------------------------------------
# convolutions
# ---------------------------------------------------------------------------
def conv_f16(x, w, b, stride=(1, 1, 1)):
    y = F.conv3d(x.to(torch.float32), _t(w), None if b is None else _t(b), stride=stride)
    return _f16(y)


def conv_i8(q, scale, qw, ws, bias, kernel, acc_dtype):
    """Valid conv of the quantized activation with the packed int8 weights [O, kd*kh*kw*C]."""
    o, c = qw.shape[0], q.shape[1]
    wt = _t(qw, acc_dtype).view(o, *kernel, c).permute(0, 4, 1, 2, 3)
    if acc_dtype == torch.float64:          # exact integer sums, then the GPU epilogue's order
        acc = F.conv3d(q.to(torch.float64), wt)
        y = (acc.to(torch.float32) * scale) * _t(ws).view(1, -1, 1, 1, 1)
    else:                                   # the reference CPU oracle: dequantized fp32 operands
        y = F.conv3d(q * scale, wt * _t(ws).view(-1, 1, 1, 1, 1))
    if bias is not None:
        y = y + _t(bias).view(1, -1, 1, 1, 1)
    return _f16(y)


# ---------------------------------------------------------------------------
# encoder
# ---------------------------------------------------------------------------
def _res_block(blk, x, pack: bool, acc_dtype, timer):
    with timer("linear"):
        skip = x if blk.nin is None else conv_f16(x, blk.nin_w, blk.nin_b)
        if blk.int8:
            q1, s1 = quantize_tensor(_reflect_causal_pad(norm_silu(x, blk.gn1_w, blk.gn1_b, blk.eps)))
            h = conv_i8(q1, s1, blk.q1, blk.s1, None, (3, 3, 3), acc_dtype)
            q2, s2 = quantize_tensor(_reflect_causal_pad(norm_silu(h, blk.gn2_w, blk.gn2_b, blk.eps, blk.b1)))
            if pack:
                return residual_pack(conv_i8(q2, s2, blk.q2, blk.s2, None, (3, 3, 3), acc_dtype), skip, blk.b2)
            return _f16(conv_i8(q2, s2, blk.q2, blk.s2, blk.b2, (3, 3, 3), acc_dtype) + skip)
        y1 = _f16(_reflect_causal_pad(norm_silu(x, blk.gn1_w, blk.gn1_b, blk.eps)))
        h = conv_f16(y1, blk.w1, None)
        y2 = _reflect_causal_pad(norm_silu(h, blk.gn2_w, blk.gn2_b, blk.eps, blk.b1))
        if pack:
            return residual_pack(conv_f16(y2, blk.w2, None), skip, blk.b2)
        return _f16(conv_f16(y2, blk.w2, blk.b2) + skip)


@torch.no_grad()
def encoder_forward(enc, x, mean, std, *, acc_dtype=torch.float32, timer=None):
    """x: fp16 [B,3,T,H,W] pixels in [-1,1] of one causal clip batch -> fp16-valued moments
    [B, 2*latent, T', H/r, W/r] (fp32 tensor).  mean/std: the 3 ImageNet channel constants."""
    timer = timer or _NoTimer()
    with timer("linear"):
        xn = _f16(((x.to(torch.float32) + 1.0) * 0.5 - _t(mean).view(1, 3, 1, 1, 1)) / _t(std).view(1, 3, 1, 1, 1))
        h = conv_f16(_reflect_causal_pad(xn), enc.conv_in_w, enc.conv_in_b)
    for blocks, down in zip(enc.stages, enc.down):
        for j, blk in enumerate(blocks):
            h = _res_block(blk, h, j == len(blocks) - 1 and down is not None, acc_dtype, timer)
        if down is not None:
            with timer("linear"):
                h = conv_f16(h, down.w, down.b, down.stride)
    with timer("linear"):
        y = _reflect_causal_pad(norm_silu(h, enc.norm_out_w, enc.norm_out_b, enc.cfg.eps))
        moments = conv_f16(y, enc.conv_out_w, enc.conv_out_b)
        return conv_f16(moments, enc.quant_w, enc.quant_b)


# ---------------------------------------------------------------------------
# decoder
# ---------------------------------------------------------------------------
def row_quant_ck(act):
    """CK row quantization: s = max(amax * fp32(1/127), 1e-30); q = clamp(rint(fp16(act / fp16(s))))."""
    amax = act.abs().amax(dim=-1, keepdim=True)
    s = torch.clamp_min(amax * RECIP_127, 1e-30)
    v = torch.round(_f16(act / _f16(s)))
    v = torch.nan_to_num(v, nan=-128.0).clamp_(-128, 127)
    return v, s


def linear_i8(q, s, qw, ws, bias, acc_dtype):
    if acc_dtype == torch.float64:
        acc = (q.to(torch.float64) @ _t(qw, torch.float64).T).to(torch.float32)
        v = acc * s
    else:
        v = (q @ _t(qw).T) * s
    v = v * _t(ws).view(1, -1)
    if bias is not None:
        v = v + _t(bias).view(1, -1)
    return _f16(v)


def _rms(x, w, eps):
    return _f16(x * torch.rsqrt((x * x).mean(dim=-1, keepdim=True) + eps) * _t(w))


def _qk_rope(qkv, cos, sin, heads, eps):
    b, n, _ = qkv.shape
    x = qkv.view(b, n, heads, 3, 64)
    r = cos.shape[-1]
    outs = []
    for part in (0, 1):
        v = x[:, :, :, part]
        v = _f16(v * torch.rsqrt((v * v).mean(dim=-1, keepdim=True) + eps))
        rot = torch.cat([-v[..., r // 2:r], v[..., : r // 2]], dim=-1)
        rope = _f16(v[..., :r] * cos) + _f16(rot * sin)
        outs.append(_f16(torch.cat([rope, v[..., r:]], dim=-1)))
    return outs[0], outs[1], x[:, :, :, 2]


@torch.no_grad()
def decoder_forward(dec, z, *, acc_dtype=torch.float32, timer=None):
    """z: fp16 [B, latent, t, h, w] (de-normalized latents) -> raw fp16-valued pixels [B, 3, T, H, W]."""
    timer = timer or _NoTimer()
    b, _, t, hh, ww = z.shape
    with timer("linear"):
        tokens = decoder_tokens(dec, z)
    y = decoder_blocks(dec, tokens, (t, hh, ww), acc_dtype=acc_dtype, timer=timer)
    return decoder_upsample(dec, y, (t, hh, ww), timer=timer)


def decoder_tokens(dec, z):
    """Latent conv-in: fp16-valued tokens [B, t*h*w, hidden]."""
    b, _, t, hh, ww = z.shape
    feat = conv_f16(_reflect_causal_pad(z.to(torch.float32)), dec.conv_in_w, dec.conv_in_b)
    return feat.permute(0, 2, 3, 4, 1).reshape(b, t * hh * ww, dec.cfg.hidden)


@torch.no_grad()
def decoder_blocks(dec, tokens, grid, *, acc_dtype=torch.float32, timer=None):
    """The INT8 block chain and the final residual + LayerNorm: tokens [B, n, hidden] -> [B, n, hidden]."""
    timer = timer or _NoTimer()
    cfg = dec.cfg
    b, n, d = tokens.shape
    t, hh, ww = grid
    with timer("linear"):
        x = tokens.to(torch.float32).reshape(b * n, d)
        cos, sin = (_t(v).view(1, n, 1, -1) for v in dec._rope(1, t, hh, ww))
        cos, sin = cos.expand(b, n, 1, -1), sin.expand(b, n, 1, -1)
    h_state, out, prev = x, None, None
    for i, blk in enumerate(dec.blocks):
        with timer("linear"):
            if i == 0:
                q1, s1 = row_quant_ck(_rms(x, blk.norm1_w, cfg.eps))
            else:
                raw = torch.addcmul(h_state, out, _t(prev))
                h_state = _f16(raw)
                x = h_state
                q1, s1 = row_quant_ck(_f16(h_state * torch.rsqrt((raw * raw).mean(-1, keepdim=True) + cfg.eps)
                                           * _t(blk.norm1_w)))
            qkv = linear_i8(q1, s1, blk.qkv_q, blk.qkv_s, blk.qkv_b, acc_dtype).view(b, n, 3 * d)
            q, k, v = _qk_rope(qkv, cos, sin, cfg.heads, cfg.qk_eps)
        with timer("attention"):
            y = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), scale=0.125)
        with timer("linear"):
            qy, sy = row_quant_ck(_f16(y.transpose(1, 2).reshape(b * n, d)))
            a = linear_i8(qy, sy, blk.out_q, blk.out_s, blk.out_b, acc_dtype)
            raw = torch.addcmul(x, a, _t(blk.scale1))
            h_state = _f16(raw)
            q2, s2 = row_quant_ck(_f16(h_state * torch.rsqrt((raw * raw).mean(-1, keepdim=True) + cfg.eps)
                                       * _t(blk.norm2_w)))
            lin = linear_i8(q2, s2, blk.up_q, blk.up_s, blk.up_b, acc_dtype)
            f = lin.shape[1] // 2
            act = _f16(lin[:, :f] / (1.0 + torch.exp(-lin[:, :f])) * lin[:, f:])
            qf, sf = row_quant_ck(act)
            out = linear_i8(qf, sf, blk.down_q, blk.down_s, blk.down_b, acc_dtype)
            prev = blk.scale2
    with timer("linear"):
        raw = torch.addcmul(h_state, out, _t(prev))
        return _f16(F.layer_norm(raw, (d,), _t(dec.ln_w), _t(dec.ln_b), cfg.eps)).view(b, n, d)


@torch.no_grad()
def decoder_upsample(dec, y, grid, *, timer=None):
    """After the blocks: [B, n, hidden] tokens of a (t, h, w) grid -> raw pixels [B, 3, T, H, W] through the
    upsampling stages (GroupNorm + SiLU + pad of the upsampled tensor, fp16 conv) and the RGB conv."""
    timer = timer or _NoTimer()
    cfg = dec.cfg
    b, n, d = y.shape
    t, hh, ww = grid
    with timer("linear"):
        x = y.to(torch.float32).reshape(b, t, hh, ww, d).permute(0, 4, 1, 2, 3)
        gns = [(gw, gb) for gw, gb, _, _ in dec.up] + [(dec.out_gn_w, dec.out_gn_b)]
        pending, up_s, up_t = None, False, False
        for k_, (gw, gb, wt, bs) in enumerate(dec.up):
            xu = _upsample(x, up_s, up_t)
            y = _reflect_causal_pad(norm_silu(xu, gns[k_][0], gns[k_][1], cfg.gn_eps, pending))
            x = conv_f16(y, wt, None)
            pending, up_s, up_t = bs, cfg.up_spatial[k_], cfg.up_temporal[k_]
        xu = _upsample(x, up_s, up_t)
        y = _reflect_causal_pad(norm_silu(xu, dec.out_gn_w, dec.out_gn_b, cfg.gn_eps, pending))
        return conv_f16(y, dec.conv_out_w, dec.conv_out_b)


def scale_sample(timer: OpTimer, area_ratio: float) -> float:
    """Seconds of the full-size work item from a sample on a spatial crop `area_ratio` times smaller:
    position-linear work scales with the area, attention with its square."""
    return timer.seconds["linear"] * area_ratio + timer.seconds["attention"] * area_ratio ** 2


def encoder_item_seconds(enc, frames: int, crop: int, tile: int, mean, std, seed: int = 0) -> tuple[float, dict]:
    """Time one encoder work item (one clip of `frames` frames of one tile) on a crop x crop window
    and scale it to the tile x tile item."""
    g = torch.Generator().manual_seed(seed)
    x = (torch.rand((1, 3, frames, crop, crop), generator=g) * 2 - 1).to(F16)
    timer = OpTimer()
    encoder_forward(enc, x, mean, std, timer=timer)
    ratio = (tile / crop) ** 2
    return scale_sample(timer, ratio), dict(timer.seconds, area_ratio=ratio)


def decoder_task_seconds(dec, tokens_t: int, crop: int, tile: int, seed: int = 0) -> tuple[float, dict]:
    """Time one decoder tile task (tokens_t latent frames of one tile) on a crop x crop latent window
    and scale it to the tile x tile task."""
    g = torch.Generator().manual_seed(seed)
    z = torch.randn((1, dec.cfg.latent_channels, tokens_t, crop, crop), generator=g).to(F16)
    timer = OpTimer()
    decoder_forward(dec, z, timer=timer)
    ratio = (tile / crop) ** 2
    return scale_sample(timer, ratio), dict(timer.seconds, area_ratio=ratio)


def cpu_threads() -> int:
    return torch.get_num_threads()


__all__ = ["OpTimer", "encoder_forward", "decoder_forward", "decoder_tokens", "decoder_blocks", "decoder_upsample",
           "encoder_item_seconds", "decoder_task_seconds", "scale_sample", "cpu_threads", "math"]
