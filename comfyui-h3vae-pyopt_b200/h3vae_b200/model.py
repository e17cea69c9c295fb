"""H3-structured video VAE assembled from the sm_100a kernels.

The reference wraps the external klvae model (video_vae.klvae, not distributed).  This module
re-creates the parts of its structure that the INT8 hot path exercises, with random-init weights
(no checkpoint is available), following the reference's block contracts:

Encoder (ref: opt/encoder_fused_norm_bias.py:108-140, opt/encoder_fused_residual_pack.py:57-85,
opt/encoder_int8_integration.py:32-52,350-459):
  conv_in (fp16) -> stages of residual blocks
     block: q1 = norm_pad_quant(x; GN1)           [temporal-isolated GroupNorm(32), SiLU, reflect/causal pad, INT8]
            h  = conv1_i8(q1)                     [bias deferred: becomes GN2's pre_bias]
            q2 = norm_pad_quant(h; GN2, pre_bias=b1)
            y  = conv2_i8(q2) + b2 + shortcut(x)  [skip add fused in the conv epilogue]
     a stage that downsamples ends with residual_pack(h, x, b2) feeding a strided fp16 conv
  norm_out + SiLU + conv_out (fp16) -> quant_conv (1x1x1) -> moments (mean = first half).

Decoder (ref: opt/int8_norm1_quant.py:185-252, opt/int8_ffn_up_fused.py:133-160,
opt/decoder_fused_qk_rope.py:56-74, opt/decoder_final_norm.py:35-72):
  conv_in (fp16) -> tokens; per block with the (h, out, scale2) carry:
     norm1 producer (residual + RMSNorm + row INT8) -> INT8 QKV GEMM with fused QK RMSNorm + RoPE
     -> fp16 attention -> row INT8 -> INT8 out-proj -> residual + RMSNorm + row INT8
     -> INT8 FFN-up GEMM with fused SwiGLU -> row INT8 -> INT8 down-proj
  final residual + LayerNorm -> causal conv3d upsampling stages (fp16) -> RGB.

INT8 convolutions and linears run on the tcgen05 kernels, and so do the fp16 convolutions outside
the INT8 scope (the encoder's input conv, strided downsamples, 1x1x1 shortcuts, conv_out and the
decoder's upsampling and RGB convs, which the reference leaves in fp16 on cuDNN).  The two convs
whose inputs are narrower than one 128-byte K row of the implicit-GEMM conv run as tcgen05 fp16
GEMMs: the decoder's 16-channel latent conv-in on rows unrolled by h3b_im2col_causal_f16, the
encoder's 32-channel 1x1x1 quant conv on the channels-last moments as they are.  cuDNN (through
torch) remains only for conv geometries outside these kernels' contracts (none in the H3 configs).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from . import kernels as K

CL3 = torch.channels_last_3d


# ---------------------------------------------------------------------------
# Load-time weight quantizers (not on the timed path)
# ---------------------------------------------------------------------------
def prepare_int8_weight(weight: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """[O,C,kd,kh,kw] -> int8 [O, kd*kh*kw*C] (tap-major, channel-minor) + fp32 per-channel scale
    amax/127 (0 -> 1), round-half-even, clamp +-127.  ref: opt/encoder_int8.py:303-327."""
    source = weight.detach().float().contiguous()
    packed = source.permute(0, 2, 3, 4, 1).reshape(source.shape[0], -1)
    scale = packed.abs().amax(dim=1).div(127.0)
    scale = torch.where(scale > 0, scale, torch.ones_like(scale))
    q = torch.round(packed / scale[:, None]).clamp(-127, 127).to(torch.int8)
    return q.contiguous(), scale.float().contiguous()


def quantize_rowwise_weight(weight: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Static per-output-row weight quantization (the comfy-kitchen rowwise contract the reference
    uses): scale = max(amax/127, 1e-30), round, clamp [-128,127]; a zero row -> q 0, scale 1.
    ref: opt/kitchen_int8.py:88-145, tests/test_kitchen_int8.py:19-26."""
    w = weight.detach().float()
    scale = (w.abs().amax(dim=-1, keepdim=True) / 127.0).clamp(min=1e-30)
    q = (w / scale).round().clamp(-128, 127).to(torch.int8)
    scale = scale.reshape(-1).contiguous()
    zero = torch.all(w == 0, dim=1)
    q = torch.where(zero[:, None], torch.zeros_like(q), q)
    scale = torch.where(zero, torch.ones_like(scale), scale)
    return q.contiguous(), scale.contiguous()


# ---------------------------------------------------------------------------
# fp16 helpers: padding and the cuDNN reference conv for geometries outside the kernels' contracts;
# the narrow-input convs as tcgen05 GEMMs
# ---------------------------------------------------------------------------
def causal_reflect_pad(x: torch.Tensor) -> torch.Tensor:
    """Reflect pad 1 in H/W, two zero frames in front (the causal 3x3x3 conv input)."""
    x = F.pad(x, (1, 1, 1, 1, 0, 0), mode="reflect") if min(x.shape[-2:]) > 1 else F.pad(x, (1, 1, 1, 1, 0, 0))
    return F.pad(x, (0, 0, 0, 0, 2, 0)).contiguous(memory_format=CL3)


def conv_f16(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None, stride=(1, 1, 1)) -> torch.Tensor:
    return F.conv3d(x, w, b, stride=stride).contiguous(memory_format=CL3)


def conv1x1_f16(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None) -> torch.Tensor:
    """1x1x1 conv of a channels-last fp16 [B, C, T, H, W] tensor as one tcgen05 fp16 GEMM
    (positions x C times the [O, C] weight); returns channels-last [B, O, T, H, W]."""
    bsz, c, t, h, w_ = x.shape
    o = w.shape[0]
    rows = x.permute(0, 2, 3, 4, 1).reshape(-1, c)        # a view of channels-last storage
    y = K.gemm_f16(rows.contiguous(), w.reshape(o, c), b)
    return y.view(bsz, t, h, w_, o).permute(0, 4, 1, 2, 3)


def causal_conv3_rows_f16(z: torch.Tensor, w_rows: torch.Tensor, b: torch.Tensor | None) -> torch.Tensor:
    """Causal 3x3x3 conv (two zero frames in front, reflect 1 in H/W) of fp16 [B, C, T, H, W] with
    C % 8 == 0 as unrolled rows times the [O, 27*C] weight rows: fp16 [B*T*H*W, O], rows in
    (b, t, h, w) order -- the input conv of the 16-channel latents, narrower than one 128-byte K
    row of the implicit-GEMM conv."""
    return K.gemm_f16(K.im2col_causal_f16(z), w_rows, b)


class Conv3dF16:
    """One fp16 valid conv of the model.  Input channel counts that are a multiple of 64 with at
    least 16 outputs run on the tcgen05 fp16 implicit-GEMM kernel (bias and an optional residual
    add fused, stride-2 through TMA element strides); the 3-channel RGB output conv runs on the
    tap-packing kernel (h3b_conv3d_rgb_f16).  Other geometries (none in the H3 configurations)
    fall back to cuDNN through torch."""

    def __init__(self, w: torch.Tensor, b: torch.Tensor | None, stride=(1, 1, 1)):
        self.w, self.b, self.stride = w, b, tuple(stride)
        self.kernel = tuple(int(k) for k in w.shape[2:])
        self.packed = K.pack_conv_weight_f16(w) if (w.shape[1] % 64 == 0 and w.shape[0] >= 16) else None
        self.rgb = (K.pack_rgb_weight(w) if (w.shape[0] == 3 and w.shape[1] % 64 == 0 and w.shape[1] <= 256
                                             and self.kernel == (3, 3, 3) and self.stride == (1, 1, 1)) else None)

    def __call__(self, x: torch.Tensor, *, residual: torch.Tensor | None = None, causal: bool = False,
                 bias: bool = True) -> torch.Tensor:
        b = self.b if bias else None
        if self.rgb is not None and residual is None:
            return K.conv3d_rgb_f16(K.ndhwc(x), self.rgb, b)
        if self.packed is not None:
            return K.conv3d_f16(K.ndhwc(x), self.packed, b, self.kernel, self.stride,
                                causal_zero_frames=2 if causal else 0, residual=residual)
        y = conv_f16(x, self.w, b, self.stride)
        return y if residual is None else (y + residual).contiguous(memory_format=CL3)


def _randn(gen, shape, std, device, dtype=torch.float16):
    return (torch.randn(*shape, generator=gen) * std).to(device=device, dtype=dtype)


# ---------------------------------------------------------------------------
# Encoder
# ---------------------------------------------------------------------------
@dataclass
class EncoderConfig:
    """Config 3 by default: stages 128/256/512/512, 2 residual blocks per stage, spatial /2 after
    stages 1-3 and temporal /2 (causal) after stages 2-3, 16-channel latent."""
    in_channels: int = 3
    channels: tuple[int, ...] = (128, 256, 512, 512)
    blocks_per_stage: int = 2
    spatial_down: tuple[bool, ...] = (True, True, True, False)
    temporal_down: tuple[bool, ...] = (False, True, True, False)
    latent_channels: int = 16
    groups: int = 32
    eps: float = 1e-6
    int8_stages: tuple[int, ...] = (0, 1, 2, 3)   # "reference" scope is (0, 1): the 8 prefix convs
    act_scale_mode: str = "tensor"                 # "tensor" (the reference's scheme) or "token"

    @property
    def spatial_ratio(self) -> int:
        return 2 ** sum(self.spatial_down)

    @property
    def temporal_ratio(self) -> int:
        return 2 ** sum(self.temporal_down)


class _ResBlock:
    def __init__(self, cin, cout, int8, gen, device, cfg: EncoderConfig):
        self.cin, self.cout, self.int8, self.eps = cin, cout, int8, cfg.eps
        if cfg.act_scale_mode not in ("tensor", "token"):
            raise ValueError("act_scale_mode must be 'tensor' or 'token'")
        self.quant = K.norm_pad_quant_token if cfg.act_scale_mode == "token" else K.norm_pad_quant
        std1 = 1.0 / math.sqrt(cin * 27)
        std2 = 1.0 / math.sqrt(cout * 27)
        self.gn1_w = (1.0 + 0.1 * torch.randn(cin, generator=gen)).half().to(device)
        self.gn1_b = (0.1 * torch.randn(cin, generator=gen)).half().to(device)
        self.gn2_w = (1.0 + 0.1 * torch.randn(cout, generator=gen)).half().to(device)
        self.gn2_b = (0.1 * torch.randn(cout, generator=gen)).half().to(device)
        self.w1 = _randn(gen, (cout, cin, 3, 3, 3), std1, device).contiguous(memory_format=CL3)
        self.b1 = _randn(gen, (cout,), 0.02, device)
        self.w2 = _randn(gen, (cout, cout, 3, 3, 3), std2, device).contiguous(memory_format=CL3)
        self.b2 = _randn(gen, (cout,), 0.02, device)
        self.nin_w = None
        self.nin_b = None
        if cin != cout:
            self.nin_w = _randn(gen, (cout, cin, 1, 1, 1), 1.0 / math.sqrt(cin), device).contiguous(memory_format=CL3)
            self.nin_b = _randn(gen, (cout,), 0.02, device)
        if int8:
            self.q1, self.s1 = prepare_int8_weight(self.w1)
            self.q2, self.s2 = prepare_int8_weight(self.w2)
        self.conv1 = Conv3dF16(self.w1, self.b1)
        self.conv2 = Conv3dF16(self.w2, self.b2)
        self.nin = Conv3dF16(self.nin_w, self.nin_b) if self.nin_w is not None else None

    def shortcut(self, x):
        if self.nin is None:
            return x
        return self.nin(x)

    def __call__(self, x: torch.Tensor, *, pack_for_downsample: bool) -> torch.Tensor:
        """Returns the block output, or when pack_for_downsample the residual-packed (padded) tensor
        [B,C,D+2,H+1,W+1] that the strided downsample conv consumes."""
        skip = self.shortcut(x)
        if self.int8:
            q1, s1 = self.quant(x, self.gn1_w, self.gn1_b, self.eps)
            h = K.conv3d_i8(q1, s1, self.q1, self.s1, None, (3, 3, 3), causal_zero_frames=2)
            q2, s2 = self.quant(h, self.gn2_w, self.gn2_b, self.eps, pre_bias=self.b1)
            if pack_for_downsample:
                h2 = K.conv3d_i8(q2, s2, self.q2, self.s2, None, (3, 3, 3), causal_zero_frames=2)
                return K.residual_pack(h2, skip, self.b2)
            return K.conv3d_i8(q2, s2, self.q2, self.s2, self.b2, (3, 3, 3), causal_zero_frames=2, residual=skip)
        y1 = K.norm_pad_f16(x, self.gn1_w, self.gn1_b, self.eps)
        h = self.conv1(y1, bias=False, causal=True)
        y2 = K.norm_pad_f16(h, self.gn2_w, self.gn2_b, self.eps, pre_bias=self.b1)
        if pack_for_downsample:
            return K.residual_pack(self.conv2(y2, bias=False, causal=True), skip, self.b2)
        return self.conv2(y2, causal=True, residual=skip)


class H3Encoder:
    """Synthetic H3-structured causal video encoder (random init, seeded)."""

    def __init__(self, cfg: EncoderConfig | None = None, device="cuda", seed: int = 0):
        self.cfg = cfg = cfg or EncoderConfig()
        gen = torch.Generator().manual_seed(seed)
        c0 = cfg.channels[0]
        self.conv_in_w = _randn(gen, (c0, cfg.in_channels, 3, 3, 3), 1.0 / math.sqrt(cfg.in_channels * 27),
                                device).contiguous(memory_format=CL3)
        self.conv_in_b = _randn(gen, (c0,), 0.02, device)
        self.stages: list[list[_ResBlock]] = []
        self.down: list[tuple | None] = []
        cin = c0
        for s, cout in enumerate(cfg.channels):
            blocks = []
            for j in range(cfg.blocks_per_stage):
                blocks.append(_ResBlock(cin if j == 0 else cout, cout, s in cfg.int8_stages, gen, device, cfg))
            cin = cout
            self.stages.append(blocks)
            if cfg.spatial_down[s] or cfg.temporal_down[s]:
                stride = (2 if cfg.temporal_down[s] else 1, 2 if cfg.spatial_down[s] else 1,
                          2 if cfg.spatial_down[s] else 1)
                w = _randn(gen, (cout, cout, 3, 3, 3), 1.0 / math.sqrt(cout * 27), device).contiguous(memory_format=CL3)
                self.down.append(Conv3dF16(w, _randn(gen, (cout,), 0.02, device), stride))
            else:
                self.down.append(None)
        cl = cfg.channels[-1]
        self.norm_out_w = (1.0 + 0.1 * torch.randn(cl, generator=gen)).half().to(device)
        self.norm_out_b = (0.1 * torch.randn(cl, generator=gen)).half().to(device)
        self.conv_out_w = _randn(gen, (2 * cfg.latent_channels, cl, 3, 3, 3), 1.0 / math.sqrt(cl * 27),
                                 device).contiguous(memory_format=CL3)
        self.conv_out_b = _randn(gen, (2 * cfg.latent_channels,), 0.02, device)
        lc = 2 * cfg.latent_channels
        self.quant_w = _randn(gen, (lc, lc, 1, 1, 1), 1.0 / math.sqrt(lc), device).contiguous(memory_format=CL3)
        self.quant_b = _randn(gen, (lc,), 0.02, device)
        self.conv_out = Conv3dF16(self.conv_out_w, self.conv_out_b)

    @property
    def int8_conv_count(self) -> int:
        return sum(2 for blocks in self.stages for b in blocks if b.int8)

    @torch.no_grad()
    def __call__(self, x: torch.Tensor, norm: tuple[torch.Tensor, torch.Tensor] | None = None) -> torch.Tensor:
        """x: fp16 [B,3,T,H,W] pixels of one causal clip -> moments [B, 2*latent, T', H/ratio, W/ratio]
        (fp16).  With norm=(mean, std), x is in [-1, 1] and the input conv applies the ImageNet
        normalization fp16(((x + 1) / 2 - mean) / std) itself; otherwise x is already normalized."""
        if x.device.type != "cuda":
            raise RuntimeError("H3Encoder requires CUDA input (no CPU fallback)")
        if self.conv_in_w.shape[0] == 128 and x.shape[1] <= 4:
            h = K.conv_in_f16(x.half(), self.conv_in_w, self.conv_in_b, norm)
        else:
            if norm is not None:
                mean, std = (v.float().view(1, -1, 1, 1, 1) for v in norm)
                x = (((x.float() + 1.0) * 0.5 - mean) / std).half()
            h = conv_f16(causal_reflect_pad(x.half()), self.conv_in_w, self.conv_in_b)
        for blocks, down in zip(self.stages, self.down):
            for j, blk in enumerate(blocks):
                last = j == len(blocks) - 1
                h = blk(h, pack_for_downsample=last and down is not None)
            if down is not None:
                # h is the residual-packed [B,C,D+2,H+1,W+1] tensor (two zero frames in front):
                # valid strided conv
                h = down(h, causal=True)
        y = K.norm_pad_f16(h, self.norm_out_w, self.norm_out_b, self.cfg.eps)
        moments = self.conv_out(y, causal=True)
        return conv1x1_f16(moments, self.quant_w, self.quant_b)


# ---------------------------------------------------------------------------
# Decoder
# ---------------------------------------------------------------------------
@dataclass
class DecoderConfig:
    """Config 4 by default: 16-ch latent, conv-in to hidden 1024, 6 blocks (16 heads x 64, FFN
    2 x 4096 SwiGLU), then causal upsampling stages 512/256/128 to RGB."""
    latent_channels: int = 16
    hidden: int = 1024
    heads: int = 16
    blocks: int = 6
    ffn: int = 4096
    rot_dims: int = 48
    up_channels: tuple[int, ...] = (512, 256, 128)
    up_spatial: tuple[bool, ...] = (True, True, True)
    up_temporal: tuple[bool, ...] = (True, True, False)
    out_channels: int = 3
    eps: float = 1e-5
    qk_eps: float = 1e-6
    gn_eps: float = 1e-6


def rope_tables(t: int, h: int, w: int, rot_dims: int, device, base: float = 10000.0):
    """3-axis rotary tables over a (t, h, w) token grid: the first rot_dims dims of each head are
    split evenly over the three axes (rot_dims/3 dims, rot_dims/6 frequencies each) in the
    rotate-half convention (pairs d, d + rot_dims/2).  Returns cos, sin fp16 [t*h*w, rot_dims]."""
    if rot_dims == 0:
        z = torch.empty(t * h * w, 0, dtype=torch.float16, device=device)
        return z, z
    assert rot_dims % 6 == 0
    nf = rot_dims // 6
    inv = 1.0 / (base ** (torch.arange(nf, dtype=torch.float64) / nf))
    tt, hh, ww = torch.meshgrid(torch.arange(t), torch.arange(h), torch.arange(w), indexing="ij")
    angles = torch.cat([p.reshape(-1, 1).double() * inv for p in (tt, hh, ww)], dim=1)  # [n, rot/2]
    angles = torch.cat([angles, angles], dim=1)
    return angles.cos().half().to(device), angles.sin().half().to(device)


class _DecoderBlock:
    def __init__(self, cfg: DecoderConfig, gen, device):
        d, f, H = cfg.hidden, cfg.ffn, cfg.heads
        assert d == H * 64
        std = 0.02
        self.norm1_w = (1.0 + 0.1 * torch.randn(d, generator=gen)).half().to(device)
        self.norm2_w = (1.0 + 0.1 * torch.randn(d, generator=gen)).half().to(device)
        self.scale1 = (0.5 + 0.1 * torch.randn(d, generator=gen)).half().to(device)
        self.scale2 = (0.5 + 0.1 * torch.randn(d, generator=gen)).half().to(device)
        # to_qkv rows are laid out per head as [q(64) | k(64) | v(64)]
        self.qkv_w = _randn(gen, (3 * d, d), std, device)
        self.qkv_b = _randn(gen, (3 * d,), std, device)
        self.out_w = _randn(gen, (d, d), std, device)
        self.out_b = _randn(gen, (d,), std, device)
        self.up_w = _randn(gen, (2 * f, d), std, device)      # rows 0..f-1 gate, f..2f-1 up
        self.up_b = _randn(gen, (2 * f,), std, device)
        self.down_w = _randn(gen, (d, f), std, device)
        self.down_b = _randn(gen, (d,), std, device)
        self.qkv_q, self.qkv_s = quantize_rowwise_weight(self.qkv_w)
        self.out_q, self.out_s = quantize_rowwise_weight(self.out_w)
        self.up_q, self.up_s = quantize_rowwise_weight(self.up_w)
        self.down_q, self.down_s = quantize_rowwise_weight(self.down_w)


class H3Decoder:
    """Synthetic H3-structured decoder (random init, seeded).  int8=True runs the fused INT8 block
    chain (the int8_decode + decode_fusions profile); int8=False runs the fp16 profile: fp16
    tcgen05 linears (the FFN-up with the fused SwiGLU epilogue of opt/fp16_swiglu_gemm.py), the
    tcgen05 attention, and the fused QK RMSNorm + RoPE and RMSNorm kernels."""

    def __init__(self, cfg: DecoderConfig | None = None, device="cuda", seed: int = 1, int8: bool = True):
        self.cfg = cfg = cfg or DecoderConfig()
        self.int8 = bool(int8)
        gen = torch.Generator().manual_seed(seed)
        self.device = torch.device(device)
        lc, d = cfg.latent_channels, cfg.hidden
        self.conv_in_w = _randn(gen, (d, lc, 3, 3, 3), 1.0 / math.sqrt(lc * 27), device).contiguous(memory_format=CL3)
        self.conv_in_b = _randn(gen, (d,), 0.02, device)
        self._conv_in_rows: tuple[torch.Tensor, torch.Tensor] | None = None
        self.blocks = [_DecoderBlock(cfg, gen, device) for _ in range(cfg.blocks)]
        self.ln_w = (1.0 + 0.1 * torch.randn(d, generator=gen)).half().to(device)
        self.ln_b = (0.1 * torch.randn(d, generator=gen)).half().to(device)
        self.up = []
        self.up_convs: list[Conv3dF16] = []
        cin = d
        for cout in cfg.up_channels:
            gw = (1.0 + 0.1 * torch.randn(cin, generator=gen)).half().to(device)
            gb = (0.1 * torch.randn(cin, generator=gen)).half().to(device)
            w = _randn(gen, (cout, cin, 3, 3, 3), 1.0 / math.sqrt(cin * 27), device).contiguous(memory_format=CL3)
            b = _randn(gen, (cout,), 0.02, device)
            self.up.append((gw, gb, w, b))
            self.up_convs.append(Conv3dF16(w, b))
            cin = cout
        self.out_gn_w = (1.0 + 0.1 * torch.randn(cin, generator=gen)).half().to(device)
        self.out_gn_b = (0.1 * torch.randn(cin, generator=gen)).half().to(device)
        self.conv_out_w = _randn(gen, (cfg.out_channels, cin, 3, 3, 3), 1.0 / math.sqrt(cin * 27),
                                 device).contiguous(memory_format=CL3)
        self.conv_out_b = _randn(gen, (cfg.out_channels,), 0.02, device)
        self.conv_out = Conv3dF16(self.conv_out_w, self.conv_out_b)
        self._rope_cache: dict = {}

    @property
    def spatial_ratio(self) -> int:
        return 2 ** sum(self.cfg.up_spatial)

    @property
    def temporal_ratio(self) -> int:
        return 2 ** sum(self.cfg.up_temporal)

    def frames_for(self, tokens_t: int) -> int:
        f = tokens_t
        for up in self.cfg.up_temporal:
            if up:
                f = 1 + 2 * (f - 1)
        return f

    def _rope(self, b, t, h, w):
        """cos, sin fp16 [b, n, 1, rot_dims] for a (t, h, w) token grid, built once per shape."""
        key = (b, t, h, w)
        if key not in self._rope_cache:
            cos, sin = rope_tables(t, h, w, self.cfg.rot_dims, self.device)
            n = t * h * w
            self._rope_cache[key] = (cos.view(1, n, 1, -1).expand(b, n, 1, cos.shape[-1]).contiguous(),
                                     sin.view(1, n, 1, -1).expand(b, n, 1, sin.shape[-1]).contiguous())
        return self._rope_cache[key]

    def transformer_fp16(self, x: torch.Tensor, grid: tuple[int, int, int]) -> torch.Tensor:
        """fp16 profile of the block chain (ref: opt/int8_norm_quant.py:106-124 block structure;
        FFN-up + SwiGLU fused as opt/fp16_swiglu_gemm.py:94-110 FusedFP16FFN)."""
        cfg = self.cfg
        b, n, d = x.shape
        cos, sin = self._rope(b, *grid)
        x = x.reshape(b * n, d).contiguous()
        h, out, prev_scale2 = x, None, None
        for i, blk in enumerate(self.blocks):
            if i == 0:
                n1 = K.rms_norm_f16(x, blk.norm1_w, cfg.eps)
            else:
                # x = h + out * scale2 (in place) and its RMSNorm in one pass
                h, _, _, n1 = K.residual_rms_quant(h, out, prev_scale2, blk.norm1_w, cfg.eps, h_out=h,
                                                   return_norm=True)
                x = h
            qkv = K.gemm_f16(n1, blk.qkv_w, blk.qkv_b).view(b, n, 3 * d)
            q, k = K.qk_rope(qkv, cos, sin, cfg.heads, cfg.qk_eps)
            v = qkv.view(b, n, cfg.heads, 192)[..., 128:]
            y = K.attention_f16(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), 1.0 / 8.0)
            a = K.gemm_f16(y.transpose(1, 2).reshape(b * n, d), blk.out_w, blk.out_b)
            h, _, _, n2 = K.residual_rms_quant(x, a, blk.scale1, blk.norm2_w, cfg.eps, return_norm=True)
            act = K.gemm_f16_swiglu(n2, blk.up_w, blk.up_b)
            out = K.gemm_f16(act, blk.down_w, blk.down_b)
            prev_scale2 = blk.scale2
        y = K.final_residual_layernorm(h, out, prev_scale2, self.ln_w, self.ln_b, cfg.eps)
        return y.view(b, n, d)

    def transformer(self, x: torch.Tensor, grid: tuple[int, int, int]) -> torch.Tensor:
        """x: fp16 [B, n, hidden] tokens -> fp16 [B, n, hidden] after the blocks and final LayerNorm."""
        if not self.int8:
            return self.transformer_fp16(x, grid)
        cfg = self.cfg
        b, n, d = x.shape
        cos, sin = self._rope(b, *grid)
        x = x.reshape(b * n, d).contiguous()
        h_state = x
        out = None
        prev_scale2 = None
        for i, blk in enumerate(self.blocks):
            if i == 0:
                q1, s1 = K.rms_quant(x, blk.norm1_w, cfg.eps)
            else:
                # norm1 producer: x = h + out * scale2 (in place), RMSNorm, row INT8
                h_state, q1, s1 = K.residual_rms_quant(h_state, out, prev_scale2, blk.norm1_w, cfg.eps, h_out=h_state)
                x = h_state
            q, k, v = K.gemm_i8_qkv_rope(q1, s1, blk.qkv_q, blk.qkv_s, blk.qkv_b, b, n, cfg.heads, cos, sin,
                                         cfg.qk_eps)
            y = K.attention_f16(q, k, v, 1.0 / 8.0)            # [B, n, H, 64] storage
            qy, sy = K.row_quant(y.transpose(1, 2).reshape(b * n, d))
            # attention-out GEMM with the residual (h = x + a * scale1) and norm2's sums of squares in
            # its epilogue, then norm2 + the FFN-up's row quantization
            h_state, sumsq = K.gemm_i8_residual(qy, sy, blk.out_q, blk.out_s, blk.out_b, x, blk.scale1)
            q2, s2 = K.rms_quant_parts(h_state, sumsq, blk.norm2_w, cfg.eps)
            act = K.gemm_i8_swiglu(q2, s2, blk.up_q, blk.up_s, blk.up_b)
            qf, sf = K.row_quant(act)
            out = K.gemm_i8(qf, sf, blk.down_q, blk.down_s, blk.down_b)
            prev_scale2 = blk.scale2
        y = K.final_residual_layernorm(h_state, out, prev_scale2, self.ln_w, self.ln_b, cfg.eps)
        return y.view(b, n, d)

    def conv_in_rows(self) -> torch.Tensor:
        """The conv-in weight as [hidden, 27*latent] GEMM rows, rebuilt only when conv_in_w is replaced."""
        if self._conv_in_rows is None or self._conv_in_rows[0] is not self.conv_in_w:
            self._conv_in_rows = (self.conv_in_w, K.conv_weight_rows(self.conv_in_w))
        return self._conv_in_rows[1]

    @torch.no_grad()
    def __call__(self, z: torch.Tensor) -> torch.Tensor:
        """z: fp16 [B, latent, t, h, w] -> raw decoder output fp16 [B, 3, T, H, W] (before finalize)."""
        if z.device.type != "cuda":
            raise RuntimeError("H3Decoder requires CUDA input (no CPU fallback)")
        cfg = self.cfg
        b, _, t, h, w = z.shape
        tokens = causal_conv3_rows_f16(z.half(), self.conv_in_rows(), self.conv_in_b).view(b, t * h * w, cfg.hidden)
        y = self.transformer(tokens, (t, h, w))
        x = y.view(b, t, h, w, cfg.hidden).permute(0, 4, 1, 2, 3)                      # NDHWC logical [B,d,t,h,w]
        # Each stage: GN + SiLU + pad -> conv (its bias is carried as the next producer's pre_bias,
        # the same fp16(conv + bias) rounding), then the x2 upsampling, which the next producer
        # reads through its index map instead of materializing it.
        gns = [(gw, gb) for gw, gb, _, _ in self.up] + [(self.out_gn_w, self.out_gn_b)]
        pending_bias, up_s, up_t = None, False, False
        for k, (wt, bs, sp, tp) in enumerate(zip([u[2] for u in self.up], [u[3] for u in self.up], cfg.up_spatial,
                                                 cfg.up_temporal)):
            gw, gb = gns[k]
            y = K.upsample_norm_pad_f16(x, gw, gb, cfg.gn_eps, spatial=up_s, temporal=up_t, pre_bias=pending_bias)
            x = self.up_convs[k](y, bias=False, causal=True)
            pending_bias, up_s, up_t = bs, sp, tp
        y = K.upsample_norm_pad_f16(x, self.out_gn_w, self.out_gn_b, cfg.gn_eps, spatial=up_s, temporal=up_t,
                                    pre_bias=pending_bias)
        return self.conv_out(y, causal=True)
