"""Tensor-level wrappers over the C ABI.

Each function validates dtypes / devices / layouts on the host (raising
ValueError before any launch), allocates outputs and workspaces with the
PyTorch caching allocator, and launches on the caller's current CUDA stream.
These are the only functions in the package that touch the native library.
"""
from __future__ import annotations

import torch

from . import _lib

F16 = torch.float16
I8 = torch.int8
F32 = torch.float32

# Kernel-launch accounting (bench.py reads it): number of library kernels each wrapper launches.
LAUNCHES = {"count": 0}
# Optional per-call CUDA-event timing of the INT8 conv (bench.py's live roofline measurement):
# when CONV_TIMING is a list, conv3d_i8 appends (start_event, end_event, int8_ops) per launch.
CONV_TIMING: list | None = None


def _count(n: int) -> None:
    LAUNCHES["count"] += n


def conv3d_int8_ops(b, c, d_out, h_out, w_out, o, kernel, causal_zero_frames) -> int:
    """Algorithmic INT8 ops (2 per MAC) of one conv launch, excluding the skipped causal taps."""
    kd, kh, kw = kernel
    if causal_zero_frames == 2 and kd == 3:
        taps = sum(min(t + 1, 3) for t in range(d_out)) * kh * kw
    else:
        taps = d_out * kd * kh * kw
    return 2 * b * h_out * w_out * o * c * taps


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*tensors: torch.Tensor | None) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if t.device.type != "cuda":
            raise RuntimeError("h3vae_b200 kernels require CUDA tensors (no CPU fallback)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError("all tensors must be on the same CUDA device")
    if dev is None:
        raise ValueError("no tensor given")
    return dev


def _require(t: torch.Tensor | None, dtype: torch.dtype, name: str, contiguous: bool = True) -> None:
    if t is None:
        return
    if t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")
    if contiguous and not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def ndhwc(x: torch.Tensor) -> torch.Tensor:
    """Return x in channels_last_3d layout (a copy only when needed)."""
    return x.contiguous(memory_format=torch.channels_last_3d)


def is_ndhwc(x: torch.Tensor) -> bool:
    return x.ndim == 5 and x.is_contiguous(memory_format=torch.channels_last_3d)


# ---------------------------------------------------------------------------
# Encoder
# ---------------------------------------------------------------------------
def conv3d_i8(qx: torch.Tensor, x_scale: torch.Tensor, qweight: torch.Tensor, weight_scale: torch.Tensor,
              bias: torch.Tensor | None, kernel: tuple[int, int, int], stride: tuple[int, int, int] = (1, 1, 1),
              *, causal_zero_frames: int = 0, out: torch.Tensor | None = None,
              residual: torch.Tensor | None = None, acc_out: torch.Tensor | None = None) -> torch.Tensor:
    """Valid INT8 conv3d of a padded NDHWC int8 activation (logical [B,C,D,H,W]).

    x_scale is one fp32 value (per-tensor quantization, the reference's scheme) or fp32 [B,D,H,W]
    scales per padded input position (per-token quantization).  With `residual` (fp16, same
    shape and strides as the output) the epilogue returns fp16(fp16(conv) + residual), the
    residual block's skip add."""
    dev = _require_cuda(qx, x_scale, qweight, weight_scale, bias, out, acc_out, residual)
    if qx.ndim != 5 or qx.dtype != I8 or not is_ndhwc(qx):
        raise ValueError("qx must be a channels_last_3d int8 [B,C,D,H,W] tensor")
    _require(qweight, I8, "qweight")
    _require(weight_scale, F32, "weight_scale")
    _require(bias, F16, "bias")
    b, c, d, h, w = qx.shape
    per_token = x_scale.ndim == 4
    if x_scale.dtype != F32 or (x_scale.numel() != 1 and not per_token):
        raise ValueError("x_scale must be one fp32 value or per-position fp32 scales [B,D,H,W]")
    if per_token and (tuple(x_scale.shape) != (b, d, h, w) or not x_scale.is_contiguous()):
        raise ValueError("per-token x_scale must be contiguous fp32 [B,D,H,W] of the padded input")
    if per_token and acc_out is not None:
        raise ValueError("acc_out is not available with per-token scales (the int32 partials are per k-block)")
    kd, kh, kw = (int(k) for k in kernel)
    sd, sh, sw = (int(s) for s in stride)
    o = qweight.shape[0]
    if qweight.ndim != 2 or qweight.shape[1] != kd * kh * kw * c:
        raise ValueError(f"qweight shape {tuple(qweight.shape)} != packed {(o, kd * kh * kw * c)}")
    if weight_scale.shape != (o,) or (bias is not None and bias.shape != (o,)):
        raise ValueError("weight_scale / bias must be [out_channels]")
    do, ho, wo = (d - kd) // sd + 1, (h - kh) // sh + 1, (w - kw) // sw + 1
    if min(do, ho, wo) <= 0:
        raise ValueError(f"input shape {tuple(qx.shape)} is too small for valid conv")
    if out is None:
        out = torch.empty((b, o, do, ho, wo), device=dev, dtype=F16, memory_format=torch.channels_last_3d)
    elif out.shape != (b, o, do, ho, wo) or out.dtype != F16 or out.stride(1) != 1:
        raise ValueError("out must be fp16 [B,O,Do,Ho,Wo] with unit channel stride")
    if acc_out is not None and (acc_out.dtype != torch.int32 or acc_out.shape != (b, o, do, ho, wo)
                                or not is_ndhwc(acc_out)):
        raise ValueError("acc_out must be a channels_last_3d int32 [B,O,Do,Ho,Wo] tensor")
    if residual is not None and (residual.dtype != F16 or residual.shape != out.shape
                                 or residual.stride() != out.stride()):
        raise ValueError("residual must be fp16 with the output's shape and strides")
    lib = _lib.load()
    timing = CONV_TIMING
    if timing is not None:
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record()
    if per_token:
        _lib.check(lib.h3b_conv3d_i8_token(
            qx.data_ptr(), _lib.i64_array((b, d, h, w, c)), qweight.data_ptr(), o, kd, kh, kw, sd, sh, sw,
            x_scale.data_ptr(), weight_scale.data_ptr(), _ptr(bias), out.data_ptr(),
            _lib.i64_array((out.stride(0), out.stride(2), out.stride(3), out.stride(4))), _ptr(residual),
            int(causal_zero_frames), _stream(dev)))
    else:
        _lib.check(lib.h3b_conv3d_i8(
            qx.data_ptr(), _lib.i64_array((b, d, h, w, c)), qweight.data_ptr(), o, kd, kh, kw, sd, sh, sw,
            x_scale.data_ptr(), weight_scale.data_ptr(), _ptr(bias), out.data_ptr(),
            _lib.i64_array((out.stride(0), out.stride(2), out.stride(3), out.stride(4))), _ptr(residual),
            _ptr(acc_out), int(causal_zero_frames), _stream(dev)))
    _count(1)
    if timing is not None:
        ev1.record()
        timing.append((ev0, ev1, conv3d_int8_ops(b, c, do, ho, wo, o, (kd, kh, kw), causal_zero_frames)))
    return out


def pack_conv_weight_f16(weight: torch.Tensor) -> torch.Tensor:
    """[O, C, kd, kh, kw] -> fp16 [O, kd*kh*kw*C] (tap-major, channel-minor), the B operand layout."""
    o = weight.shape[0]
    return weight.detach().permute(0, 2, 3, 4, 1).reshape(o, -1).to(F16).contiguous()


def conv3d_f16(x: torch.Tensor, wpacked: torch.Tensor, bias: torch.Tensor | None, kernel: tuple[int, int, int],
               stride: tuple[int, int, int] = (1, 1, 1), *, causal_zero_frames: int = 0,
               residual: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """Valid fp16 conv3d (fp32 accumulate) of a padded NDHWC fp16 activation (logical [B,C,D,H,W])
    on the tcgen05 tensor cores; bias and the optional residual add are fused in the epilogue."""
    dev = _require_cuda(x, wpacked, bias, residual, out)
    if x.ndim != 5 or x.dtype != F16 or not is_ndhwc(x):
        raise ValueError("x must be a channels_last_3d fp16 [B,C,D,H,W] tensor")
    _require(wpacked, F16, "weight")
    _require(bias, F16, "bias")
    b, c, d, h, w = x.shape
    kd, kh, kw = (int(k) for k in kernel)
    sd, sh, sw = (int(s) for s in stride)
    o = wpacked.shape[0]
    if wpacked.ndim != 2 or wpacked.shape[1] != kd * kh * kw * c:
        raise ValueError(f"weight shape {tuple(wpacked.shape)} != packed {(o, kd * kh * kw * c)}")
    if bias is not None and bias.shape != (o,):
        raise ValueError("bias must be [out_channels]")
    do, ho, wo = (d - kd) // sd + 1, (h - kh) // sh + 1, (w - kw) // sw + 1
    if min(do, ho, wo) <= 0:
        raise ValueError(f"input shape {tuple(x.shape)} is too small for valid conv")
    if out is None:
        out = torch.empty((b, o, do, ho, wo), device=dev, dtype=F16, memory_format=torch.channels_last_3d)
    elif out.shape != (b, o, do, ho, wo) or out.dtype != F16 or out.stride(1) != 1:
        raise ValueError("out must be fp16 [B,O,Do,Ho,Wo] with unit channel stride")
    if residual is not None and (residual.dtype != F16 or residual.shape != out.shape
                                 or residual.stride() != out.stride()):
        raise ValueError("residual must be fp16 with the output's shape and strides")
    _lib.check(_lib.load().h3b_conv3d_f16(
        x.data_ptr(), _lib.i64_array((b, d, h, w, c)), wpacked.data_ptr(), o, kd, kh, kw, sd, sh, sw, _ptr(bias),
        out.data_ptr(), _lib.i64_array((out.stride(0), out.stride(2), out.stride(3), out.stride(4))),
        _ptr(residual), int(causal_zero_frames), _stream(dev)))
    _count(1)
    return out


def pack_rgb_weight(weight: torch.Tensor) -> torch.Tensor:
    """[3, C, 3, 3, 3] -> fp16 [3*32, C]: row kd*32 + kh*9 + kw*3 + o = W[o, :, kd, kh, kw], rest zero."""
    o, c = weight.shape[:2]
    if o != 3 or tuple(weight.shape[2:]) != (3, 3, 3):
        raise ValueError("RGB conv weight must be [3, C, 3, 3, 3]")
    w = weight.detach().to(F16)
    packed = torch.zeros((3, 32, c), dtype=F16, device=weight.device)
    packed[:, :27] = w.permute(2, 3, 4, 0, 1).reshape(3, 27, c)   # [kd, kh*9 + kw*3 + o, C]
    return packed.reshape(3 * 32, c).contiguous()


def conv3d_rgb_f16(x: torch.Tensor, wpacked: torch.Tensor, bias: torch.Tensor | None) -> torch.Tensor:
    """Valid 3x3x3 conv of a padded NDHWC fp16 activation to 3 channels (+bias) -> planar fp16
    [B, 3, T, H, W]."""
    dev = _require_cuda(x, wpacked, bias)
    if x.ndim != 5 or x.dtype != F16 or not is_ndhwc(x):
        raise ValueError("x must be a channels_last_3d fp16 [B,C,D,H,W] tensor")
    _require(wpacked, F16, "weight")
    _require(bias, F16, "bias")
    b, c, d, h, w = x.shape
    if wpacked.shape != (3 * 32, c) or (bias is not None and bias.shape != (3,)):
        raise ValueError("packed RGB weight must be [96, C] and bias [3]")
    if min(d, h, w) < 3:
        raise ValueError("input too small for a valid 3x3x3 conv")
    out = torch.empty((b, 3, d - 2, h - 2, w - 2), device=dev, dtype=F16)
    _lib.check(_lib.load().h3b_conv3d_rgb_f16(x.data_ptr(), _lib.i64_array((b, d, h, w, c)), wpacked.data_ptr(),
                                              _ptr(bias), out.data_ptr(), _stream(dev)))
    _count(1)
    return out


def conv_in_f16(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None,
                norm: tuple[torch.Tensor, torch.Tensor] | None = None) -> torch.Tensor:
    """Encoder input conv: optional pixel normalization fp16(((x+1)*0.5 - mean)/std), causal +
    reflect pad and the 3x3x3 conv (+bias) to 128 channels, fp32 accumulate on the tensor cores.
    x fp16 [B, Cin<=4, T, H, W] (any strides); weight fp16 [128, Cin, 3, 3, 3] -> NDHWC fp16."""
    dev = _require_cuda(x, weight, bias, *(norm or ()))
    if x.ndim != 5 or x.dtype != F16:
        raise ValueError("x must be fp16 [B,C,T,H,W]")
    b, cin, t, h, w = x.shape
    if weight.shape != (weight.shape[0], cin, 3, 3, 3) or weight.dtype != F16:
        raise ValueError("weight must be fp16 [O, Cin, 3, 3, 3]")
    o = weight.shape[0]
    _require(bias, F16, "bias")
    wp = weight.detach().permute(0, 2, 3, 4, 1).reshape(o, -1).contiguous()
    mean = std = None
    if norm is not None:
        mean, std = (v.reshape(-1).to(F32).contiguous() for v in norm)
        if mean.numel() != cin or std.numel() != cin:
            raise ValueError("normalization vectors must have one value per input channel")
    lib = _lib.load()
    ws_bytes = lib.h3b_conv_in_workspace_size(b, t, h, w)
    ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
    out = torch.empty((b, o, t, h, w), device=dev, dtype=F16, memory_format=torch.channels_last_3d)
    _lib.check(lib.h3b_conv_in_f16(x.data_ptr(), _lib.i64_array(x.shape), _lib.i64_array(x.stride()), _ptr(mean),
                                   _ptr(std), wp.data_ptr(), o, _ptr(bias), out.data_ptr(), ws.data_ptr(), ws_bytes,
                                   _stream(dev)))
    _count(2)
    return out


def im2col_causal_f16(x: torch.Tensor) -> torch.Tensor:
    """GEMM rows of a causal 3x3x3 conv: x fp16 [B, C, T, H, W] (any strides, C % 8 == 0) ->
    fp16 [B*T*H*W, 27*C], column (kd, kh, kw, c), the two causal zero frames in front and reflect
    padding 1 in H/W (zero when H or W is 1).  Times a [N, 27*C] weight it is the conv."""
    dev = _require_cuda(x)
    if x.ndim != 5 or x.dtype != F16:
        raise ValueError("x must be fp16 [B,C,T,H,W]")
    b, c, t, h, w = x.shape
    out = torch.empty((b * t * h * w, 27 * c), device=dev, dtype=F16)
    _lib.check(_lib.load().h3b_im2col_causal_f16(x.data_ptr(), _lib.i64_array(x.shape), _lib.i64_array(x.stride()),
                                                 out.data_ptr(), _stream(dev)))
    _count(1)
    return out


def conv_weight_rows(weight: torch.Tensor) -> torch.Tensor:
    """fp16 [N, C, kd, kh, kw] conv weight -> [N, kd*kh*kw*C] rows in (kd, kh, kw, c) order."""
    n = weight.shape[0]
    return weight.detach().permute(0, 2, 3, 4, 1).reshape(n, -1).contiguous()


def quantize_tensor_i8(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-tensor half-away INT8 quantization of fp16 [B,C,D,H,W] (any strides) to NDHWC int8."""
    dev = _require_cuda(x)
    if x.ndim != 5:
        raise ValueError("activation must be [B,C,D,H,W]")
    if x.dtype != F16:
        raise ValueError("INT8 quantization requires FP16 activations")
    if x.numel() == 0:
        raise ValueError("INT8 activation quantization requires a nonempty tensor")
    lib = _lib.load()
    q = torch.empty(x.shape, device=dev, dtype=I8, memory_format=torch.channels_last_3d)
    scale = torch.empty((), device=dev, dtype=F32)
    ws_bytes = int(lib.h3b_quantize_tensor_workspace_size())
    ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
    _lib.check(lib.h3b_quantize_tensor_i8(x.data_ptr(), _lib.i64_array(x.shape), _lib.i64_array(x.stride()),
                                          q.data_ptr(), scale.data_ptr(), ws.data_ptr(), ws_bytes, _stream(dev)))
    _count(2)
    return q, scale


def _norm_common(x, pre_bias, gamma, beta):
    dev = _require_cuda(x, pre_bias, gamma, beta)
    if x.ndim != 5 or x.dtype != F16:
        raise ValueError("norm producer requires an FP16 rank-5 input")
    b, c, d, h, w = x.shape
    for name, t in (("gamma", gamma), ("beta", beta), ("pre_bias", pre_bias)):
        if t is not None and (t.shape != (c,) or t.dtype != F16 or not t.is_contiguous()):
            raise ValueError(f"Expected contiguous FP16 channel vectors on input device ({name})")
    x = ndhwc(x)
    lib = _lib.load()
    ws_bytes = int(lib.h3b_norm_workspace_size(b, c, d, h, w))
    if ws_bytes == 0:
        raise ValueError(f"unsupported norm producer shape {tuple(x.shape)} (H,W >= 2; C a power of two 32..2048)")
    ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
    return dev, x, lib, ws, ws_bytes


def norm_pad_quant(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, eps: float,
                   pre_bias: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """GroupNorm(32)->SiLU->reflect/causal pad->per-tensor INT8 (NDHWC [B,C,D+2,H+2,W+2])."""
    dev, x, lib, ws, ws_bytes = _norm_common(x, pre_bias, gamma, beta)
    b, c, d, h, w = x.shape
    q = torch.empty((b, c, d + 2, h + 2, w + 2), device=dev, dtype=I8, memory_format=torch.channels_last_3d)
    scale = torch.empty((), device=dev, dtype=F32)
    _lib.check(lib.h3b_norm_pad_quant(x.data_ptr(), b, c, d, h, w, _ptr(pre_bias), gamma.data_ptr(),
                                      beta.data_ptr(), float(eps), q.data_ptr(), scale.data_ptr(), ws.data_ptr(),
                                      ws_bytes, _stream(dev)))
    _count(4)
    return q, scale


def norm_pad_quant_token(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, eps: float,
                         pre_bias: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """GroupNorm(32)->SiLU->reflect/causal pad->INT8 with one scale per padded position:
    (q NDHWC [B,C,D+2,H+2,W+2], scales fp32 [B,D+2,H+2,W+2])."""
    dev, x, lib, ws, ws_bytes = _norm_common(x, pre_bias, gamma, beta)
    b, c, d, h, w = x.shape
    q = torch.empty((b, c, d + 2, h + 2, w + 2), device=dev, dtype=I8, memory_format=torch.channels_last_3d)
    scales = torch.empty((b, d + 2, h + 2, w + 2), device=dev, dtype=F32)
    _lib.check(lib.h3b_norm_pad_quant_token(x.data_ptr(), b, c, d, h, w, _ptr(pre_bias), gamma.data_ptr(),
                                            beta.data_ptr(), float(eps), q.data_ptr(), scales.data_ptr(),
                                            ws.data_ptr(), ws_bytes, _stream(dev)))
    _count(3)
    return q, scales


def norm_pad_f16(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, eps: float,
                 pre_bias: torch.Tensor | None = None) -> torch.Tensor:
    """GroupNorm(32)->SiLU->reflect/causal pad, fp16 NDHWC [B,C,D+2,H+2,W+2]."""
    dev, x, lib, ws, ws_bytes = _norm_common(x, pre_bias, gamma, beta)
    b, c, d, h, w = x.shape
    y = torch.empty((b, c, d + 2, h + 2, w + 2), device=dev, dtype=F16, memory_format=torch.channels_last_3d)
    _lib.check(lib.h3b_norm_pad_f16(x.data_ptr(), b, c, d, h, w, _ptr(pre_bias), gamma.data_ptr(),
                                    beta.data_ptr(), float(eps), y.data_ptr(), ws.data_ptr(), ws_bytes,
                                    _stream(dev)))
    _count(3)
    return y


def upsample_norm_pad_f16(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, eps: float, *,
                          spatial: bool, temporal: bool, pre_bias: torch.Tensor | None = None) -> torch.Tensor:
    """pad(silu(GN(up(x) [+ pre_bias]))) with nearest x2 spatial / causal x2 temporal upsampling folded
    into the producer; fp16 NDHWC [B, C, D'+2, H'+2, W'+2] with D' = 2D-1 (temporal) and H' = 2H."""
    dev, x, lib, ws, ws_bytes = _norm_common(x, pre_bias, gamma, beta)
    b, c, d, h, w = x.shape
    us, ut = (2 if spatial else 1), (1 if temporal and d > 1 else 0)
    du = 2 * d - 1 if ut else d
    y = torch.empty((b, c, du + 2, h * us + 2, w * us + 2), device=dev, dtype=F16,
                    memory_format=torch.channels_last_3d)
    _lib.check(lib.h3b_upsample_norm_pad_f16(x.data_ptr(), b, c, d, h, w, us, ut, _ptr(pre_bias), gamma.data_ptr(),
                                             beta.data_ptr(), float(eps), y.data_ptr(), ws.data_ptr(), ws_bytes,
                                             _stream(dev)))
    _count(3)
    return y


def residual_pack(x: torch.Tensor, residual: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """fp16(r + (x + bias)), right/bottom reflect +1, two causal zero frames; NDHWC [B,C,D+2,H+1,W+1]."""
    dev = _require_cuda(x, residual, bias)
    if x.ndim != 5 or x.dtype != F16 or residual.shape != x.shape or residual.dtype != F16:
        raise ValueError("Residual must match input")
    b, c, d, h, w = x.shape
    if bias.shape != (c,) or bias.dtype != F16 or not bias.is_contiguous():
        raise ValueError("Expected contiguous FP16 channel bias")
    x, residual = ndhwc(x), ndhwc(residual)
    y = torch.empty((b, c, d + 2, h + 1, w + 1), device=dev, dtype=F16, memory_format=torch.channels_last_3d)
    _lib.check(_lib.load().h3b_residual_pack(x.data_ptr(), residual.data_ptr(), bias.data_ptr(), b, c, d, h, w,
                                             y.data_ptr(), _stream(dev)))
    _count(1)
    return y


def finalize_pixels(x: torch.Tensor, std: torch.Tensor, mean: torch.Tensor,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    dev = _require_cuda(x, std, mean, out)
    if x.ndim != 5 or x.shape[1] != 3 or x.numel() == 0:
        raise ValueError("nonempty B,3,T,H,W tensor required")
    if x.dtype not in (F16, F32):
        raise ValueError("FP16 or FP32 decoded pixels required")
    for v in (std, mean):
        if v.numel() != 3 or v.dtype != F32 or not v.is_contiguous():
            raise ValueError("three contiguous FP32 channel constants on same device required")
    if out is None:
        out = torch.empty(x.shape, device=dev, dtype=F32)
    elif out.shape != x.shape or out.dtype != F32 or not out.is_contiguous():
        raise ValueError("contiguous FP32 output with matching shape/device required")
    _lib.check(_lib.load().h3b_finalize_pixels(x.data_ptr(), 1 if x.dtype == F16 else 0, _lib.i64_array(x.shape),
                                               _lib.i64_array(x.stride()), std.data_ptr(), mean.data_ptr(),
                                               out.data_ptr(), _stream(dev)))
    _count(1)
    return out


def blend_accumulate(canvas: torch.Tensor, tile: torch.Tensor, weight: torch.Tensor) -> None:
    """canvas += tile.float() * weight in place; canvas is a [C,T,H,W] FP32 window (any strides) of
    the blend canvas, tile FP16/FP32 [C,T,H,W], weight FP32 [H,W] contiguous (the tile's weight map).
    ref: h3vae_runtime.py:623-639 (the blend and trim these weights restate)."""
    dev = _require_cuda(canvas, tile, weight)
    if canvas.ndim != 4 or tile.shape != canvas.shape or canvas.numel() == 0:
        raise ValueError("nonempty C,T,H,W tile matching the canvas window required")
    if canvas.dtype != F32 or tile.dtype not in (F16, F32):
        raise ValueError("FP32 canvas and FP16/FP32 tile required")
    if weight.dtype != F32 or weight.shape != canvas.shape[2:] or not weight.is_contiguous():
        raise ValueError("contiguous FP32 [H,W] weight map required")
    _lib.check(_lib.load().h3b_blend_accumulate(tile.data_ptr(), 1 if tile.dtype == F16 else 0,
                                                _lib.i64_array(tile.shape), _lib.i64_array(tile.stride()),
                                                weight.data_ptr(), canvas.data_ptr(),
                                                _lib.i64_array(canvas.stride()), _stream(dev)))
    _count(1)


# ---------------------------------------------------------------------------
# Decoder
# ---------------------------------------------------------------------------
def _rows(x: torch.Tensor) -> tuple[int, int]:
    k = x.shape[-1]
    return x.numel() // k, k


def gemm_i8(q: torch.Tensor, scale: torch.Tensor, qweight: torch.Tensor, weight_scale: torch.Tensor,
            bias: torch.Tensor | None = None, *, out: torch.Tensor | None = None,
            acc_out: torch.Tensor | None = None) -> torch.Tensor:
    """out[M,N] = fp16(fma(acc*scale[m], weight_scale[n], bias[n])), int8 q [M,K] x qweight [N,K]^T."""
    dev = _require_cuda(q, scale, qweight, weight_scale, bias, out, acc_out)
    if q.ndim != 2 or qweight.ndim != 2 or q.shape[1] != qweight.shape[1]:
        raise ValueError("INT8 matrix dimensions/types do not match")
    _require(q, I8, "q")
    _require(qweight, I8, "qweight")
    _require(scale, F32, "scale")
    _require(weight_scale, F32, "weight_scale")
    _require(bias, F16, "bias")
    m, k = q.shape
    n = qweight.shape[0]
    if scale.numel() != m or weight_scale.numel() != n or (bias is not None and bias.numel() != n):
        raise ValueError("one scale per activation/weight row required")
    if out is None:
        out = torch.empty((m, n), device=dev, dtype=F16)
    elif out.dtype != F16 or out.shape != (m, n) or out.stride(1) != 1:
        raise ValueError("out must be fp16 [M,N] with unit column stride")
    if acc_out is not None and (acc_out.dtype != torch.int32 or acc_out.shape != (m, n) or not acc_out.is_contiguous()):
        raise ValueError("acc_out must be contiguous int32 [M,N]")
    _lib.check(_lib.load().h3b_gemm_i8(q.data_ptr(), scale.data_ptr(), qweight.data_ptr(), weight_scale.data_ptr(),
                                       _ptr(bias), m, n, k, out.data_ptr(), out.stride(0), _ptr(acc_out),
                                       _stream(dev)))
    _count(1)
    return out


def gemm_i8_residual(q: torch.Tensor, scale: torch.Tensor, qweight: torch.Tensor, weight_scale: torch.Tensor,
                     bias: torch.Tensor | None, x: torch.Tensor, gate: torch.Tensor, *, round_stats: bool = False,
                     h_out: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Attention-out INT8 GEMM with the residual fused into its epilogue: h = fp16(fma(a, gate, x)) for
    a = fp16(linear), written instead of a, plus per-row partial sums of squares for rms_quant_parts.
    Returns (h [M, N] fp16, row_sumsq [M, parts] fp32)."""
    dev = _require_cuda(q, scale, qweight, weight_scale, bias, x, gate, h_out)
    _require(q, I8, "q")
    _require(qweight, I8, "qweight")
    _require(scale, F32, "scale")
    _require(weight_scale, F32, "weight_scale")
    _require(bias, F16, "bias")
    _require(x, F16, "x")
    _require(gate, F16, "gate")
    m, k = _rows(q)
    n = qweight.shape[0]
    if x.shape[-1] != n or x.numel() != m * n or gate.shape != (n,):
        raise ValueError("x must be [M, N] and gate [N] for an [N, K] weight")
    lib = _lib.load()
    h = torch.empty((m, n), device=dev, dtype=F16) if h_out is None else h_out
    parts = int(lib.h3b_gemm_i8_residual_parts(n))
    sums = torch.empty((m, parts), device=dev, dtype=F32)
    _lib.check(lib.h3b_gemm_i8_residual(q.data_ptr(), scale.data_ptr(), qweight.data_ptr(), weight_scale.data_ptr(),
                                        _ptr(bias), m, n, k, x.data_ptr(), gate.data_ptr(), 1 if round_stats else 0,
                                        h.data_ptr(), n, sums.data_ptr(), _stream(dev)))
    _count(1)
    return h, sums


def rms_quant_parts(h: torch.Tensor, row_sumsq: torch.Tensor, w: torch.Tensor, eps: float, *,
                    return_norm: bool = False):
    """act = fp16(h * rsqrt(sum(row_sumsq[m]) / K + eps) * w) and CK row quantization -> (q, s[, act])."""
    dev = _require_cuda(h, row_sumsq, w)
    _require(h, F16, "h")
    _require(w, F16, "w")
    _require(row_sumsq, F32, "row_sumsq")
    m, k = _rows(h)
    if w.shape != (k,) or row_sumsq.shape[0] != m:
        raise ValueError("w must be [K] and row_sumsq [M, parts]")
    q = torch.empty((m, k), device=dev, dtype=I8)
    s = torch.empty((m, 1), device=dev, dtype=F32)
    norm = torch.empty_like(h) if return_norm else None
    _lib.check(_lib.load().h3b_rms_quant_parts(h.data_ptr(), row_sumsq.data_ptr(), row_sumsq.shape[1], w.data_ptr(),
                                               m, k, float(eps), q.data_ptr(), s.data_ptr(), _ptr(norm), _stream(dev)))
    _count(1)
    return (q, s, norm) if return_norm else (q, s)


def gemm_i8_swiglu(q: torch.Tensor, scale: torch.Tensor, qweight: torch.Tensor, weight_scale: torch.Tensor,
                   bias: torch.Tensor | None = None) -> torch.Tensor:
    """FFN-up INT8 GEMM with the SwiGLU epilogue: returns fp16 act [M, F] for a [2F, K] weight."""
    dev = _require_cuda(q, scale, qweight, weight_scale, bias)
    _require(q, I8, "q")
    _require(qweight, I8, "qweight")
    _require(scale, F32, "scale")
    _require(weight_scale, F32, "weight_scale")
    _require(bias, F16, "bias")
    m, k = q.shape
    n2 = qweight.shape[0]
    if qweight.shape[1] != k or n2 % 2 or scale.numel() != m or weight_scale.numel() != n2:
        raise ValueError("INT8 FFN-up shapes do not match")
    if bias is not None and bias.numel() != n2:
        raise ValueError("FP16 bias matching output channels required")
    f = n2 // 2
    act = torch.empty((m, f), device=dev, dtype=F16)
    _lib.check(_lib.load().h3b_gemm_i8_swiglu(q.data_ptr(), scale.data_ptr(), qweight.data_ptr(),
                                              weight_scale.data_ptr(), _ptr(bias), m, f, k, act.data_ptr(),
                                              _stream(dev)))
    _count(1)
    return act


def _f16_operands(a: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None, rows: int) -> None:
    _require(a, F16, "a")
    _require(w, F16, "w")
    _require(bias, F16, "bias")
    if a.ndim != 2 or w.ndim != 2 or a.shape[1] != w.shape[1]:
        raise ValueError("FP16 matrix dimensions do not match")
    if a.shape[1] % 8 or a.data_ptr() % 16 or w.data_ptr() % 16:
        raise ValueError("K must be a multiple of 8 and the operands 16-byte aligned")
    if bias is not None and bias.numel() != rows:
        raise ValueError("FP16 bias matching output channels required")


def gemm_f16(a: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None, *,
             out: torch.Tensor | None = None) -> torch.Tensor:
    """out[M,N] = fp16(a[M,K] @ w[N,K]^T + bias) with an fp32 accumulator (fp16 decoder profile linear)."""
    dev = _require_cuda(a, w, bias, out)
    _f16_operands(a, w, bias, w.shape[0])
    m, k = a.shape
    n = w.shape[0]
    if out is None:
        out = torch.empty((m, n), device=dev, dtype=F16)
    elif out.dtype != F16 or out.shape != (m, n) or out.stride(1) != 1:
        raise ValueError("out must be fp16 [M,N] with unit column stride")
    _lib.check(_lib.load().h3b_gemm_f16(a.data_ptr(), w.data_ptr(), _ptr(bias), m, n, k, out.data_ptr(),
                                        out.stride(0), _stream(dev)))
    _count(1)
    return out


def gemm_f16_swiglu(a: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """FFN-up fp16 GEMM with the SwiGLU epilogue: fp16 act [M, F] for a [2F, K] weight.
    ref: opt/fp16_swiglu_gemm.py:66-80 (fused_w1_swiglu)."""
    dev = _require_cuda(a, w, bias)
    _f16_operands(a, w, bias, w.shape[0])
    if w.shape[0] % 2:
        raise ValueError("expected matching K and paired gate/up output rows")
    m, k = a.shape
    f = w.shape[0] // 2
    act = torch.empty((m, f), device=dev, dtype=F16)
    _lib.check(_lib.load().h3b_gemm_f16_swiglu(a.data_ptr(), w.data_ptr(), _ptr(bias), m, f, k, act.data_ptr(),
                                               _stream(dev)))
    _count(1)
    return act


def gemm_i8_qkv_rope(q: torch.Tensor, scale: torch.Tensor, qweight: torch.Tensor, weight_scale: torch.Tensor,
                     bias: torch.Tensor | None, batch: int, tokens: int, heads: int, cos: torch.Tensor,
                     sin: torch.Tensor, eps: float) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """INT8 QKV GEMM with fused QK RMSNorm + RoPE; returns q, k, v as fp16 [batch, heads, tokens, 64]."""
    dev = _require_cuda(q, scale, qweight, weight_scale, bias, cos, sin)
    _require(q, I8, "q")
    _require(qweight, I8, "qweight")
    _require(cos, F16, "cos")
    _require(sin, F16, "sin")
    m, k = q.shape
    if m != batch * tokens or qweight.shape != (heads * 192, k):
        raise ValueError("QKV shapes do not match [heads*192, K] per-head layout")
    r = cos.shape[-1]
    if cos.numel() != m * r or sin.shape != cos.shape:
        raise ValueError("cos/sin must be [batch, tokens, 1, R]")
    qo = torch.empty((batch, heads, tokens, 64), device=dev, dtype=F16)
    ko = torch.empty_like(qo)
    vo = torch.empty_like(qo)
    _lib.check(_lib.load().h3b_gemm_i8_qkv_rope(q.data_ptr(), scale.data_ptr(), qweight.data_ptr(),
                                                weight_scale.data_ptr(), _ptr(bias), batch, tokens, heads, k,
                                                cos.data_ptr(), sin.data_ptr(), r, float(eps), qo.data_ptr(),
                                                ko.data_ptr(), vo.data_ptr(), _stream(dev)))
    _count(1)
    return qo, ko, vo


def row_quant(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """CK-contract per-row INT8 quantization of fp16 [..., K] -> (q [M,K], s [M,1])."""
    dev = _require_cuda(x)
    _require(x, F16, "x")
    m, k = _rows(x)
    q = torch.empty((m, k), device=dev, dtype=I8)
    s = torch.empty((m, 1), device=dev, dtype=F32)
    _lib.check(_lib.load().h3b_row_quant(x.data_ptr(), m, k, k, q.data_ptr(), s.data_ptr(), _stream(dev)))
    _count(1)
    return q, s


def swiglu_quant(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    dev = _require_cuda(x)
    if x.dtype != F16 or x.ndim < 2 or not x.is_contiguous():
        raise ValueError("contiguous FP16 input with at least two dimensions required")
    if x.shape[-1] <= 0 or x.shape[-1] % 2 or x.numel() == 0:
        raise ValueError("nonempty [gate | up] rows of even width required")
    k = x.shape[-1] // 2
    m = x.numel() // (2 * k)
    q = torch.empty((m, k), device=dev, dtype=I8)
    s = torch.empty((m, 1), device=dev, dtype=F32)
    _lib.check(_lib.load().h3b_swiglu_quant(x.data_ptr(), m, k, q.data_ptr(), s.data_ptr(), _stream(dev)))
    _count(1)
    return q, s


def residual_rms_quant(x: torch.Tensor, a: torch.Tensor, g: torch.Tensor, w: torch.Tensor, eps: float, *,
                       round_stats: bool = False, h_out: torch.Tensor | None = None,
                       return_norm: bool = False):
    """raw=fma(a,g,x); h=fp16(raw); act=fp16(h*rsqrt(mean(stat^2)+eps)*w); row quant.

    Returns (h, q, s[, norm]).  Pass h_out=x for the in-place residual update.
    """
    dev = _require_cuda(x, a, g, w, h_out)
    for name, t in (("x", x), ("a", a), ("g", g), ("w", w)):
        _require(t, F16, name)
    m, k = _rows(x)
    if a.shape != x.shape or g.shape != (k,) or w.shape != (k,):
        raise ValueError("residual/scale/RMS weight shape mismatch")
    h = torch.empty_like(x) if h_out is None else h_out
    q = torch.empty((m, k), device=dev, dtype=I8)
    s = torch.empty((m, 1), device=dev, dtype=F32)
    norm = torch.empty_like(x) if return_norm else None
    _lib.check(_lib.load().h3b_residual_rms_quant(x.data_ptr(), a.data_ptr(), g.data_ptr(), w.data_ptr(), m, k,
                                                  float(eps), 1 if round_stats else 0, h.data_ptr(), q.data_ptr(),
                                                  s.data_ptr(), _ptr(norm), _stream(dev)))
    _count(1)
    return (h, q, s, norm) if return_norm else (h, q, s)


def rms_norm_f16(x: torch.Tensor, gamma: torch.Tensor, eps: float) -> torch.Tensor:
    dev = _require_cuda(x, gamma)
    _require(x, F16, "x")
    _require(gamma, F16, "gamma")
    m, k = _rows(x)
    y = torch.empty_like(x, memory_format=torch.contiguous_format)
    _lib.check(_lib.load().h3b_rms_norm_f16(x.data_ptr(), gamma.data_ptr(), m, k, float(eps), y.data_ptr(),
                                            _stream(dev)))
    _count(1)
    return y


def rms_quant(x: torch.Tensor, gamma: torch.Tensor, eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    dev = _require_cuda(x, gamma)
    _require(x, F16, "x")
    _require(gamma, F16, "gamma")
    m, k = _rows(x)
    q = torch.empty((m, k), device=dev, dtype=I8)
    s = torch.empty((m, 1), device=dev, dtype=F32)
    _lib.check(_lib.load().h3b_rms_quant(x.data_ptr(), gamma.data_ptr(), m, k, float(eps), q.data_ptr(),
                                         s.data_ptr(), _stream(dev)))
    _count(1)
    return q, s


def final_residual_layernorm(h: torch.Tensor, o: torch.Tensor, gate: torch.Tensor, gamma: torch.Tensor,
                             beta: torch.Tensor, eps: float) -> torch.Tensor:
    dev = _require_cuda(h, o, gate, gamma, beta)
    for name, t in (("h", h), ("o", o), ("gate", gate), ("gamma", gamma), ("beta", beta)):
        _require(t, F16, name)
    m, k = _rows(h)
    if o.shape != h.shape or any(v.shape != (k,) for v in (gate, gamma, beta)):
        raise ValueError("expected matching H/O and width-K vectors")
    y = torch.empty_like(h, memory_format=torch.contiguous_format)
    _lib.check(_lib.load().h3b_final_residual_layernorm(h.data_ptr(), o.data_ptr(), gate.data_ptr(),
                                                        gamma.data_ptr(), beta.data_ptr(), m, k, float(eps),
                                                        y.data_ptr(), _stream(dev)))
    _count(1)
    return y


def qk_rope(qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, heads: int,
            eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    dev = _require_cuda(qkv, cos, sin)
    _require(qkv, F16, "qkv")
    _require(cos, F16, "cos")
    _require(sin, F16, "sin")
    b, n, width = qkv.shape
    if width != heads * 192:
        raise ValueError("qkv width must be heads * 3 * 64")
    r = cos.shape[-1]
    if cos.shape != (b, n, 1, r) or sin.shape != cos.shape:
        raise ValueError("cos/sin must be [b, n, 1, R]")
    q = torch.empty((b, n, heads, 64), device=dev, dtype=F16)
    k = torch.empty_like(q)
    _lib.check(_lib.load().h3b_qk_rope(qkv.data_ptr(), cos.data_ptr(), sin.data_ptr(), b, n, heads, r, float(eps),
                                       q.data_ptr(), k.data_ptr(), _stream(dev)))
    _count(1)
    return q, k


def attention_f16(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """softmax(q k^T * scale) v for [B, H, S, 64] views (any batch/head/token strides, unit dim stride).

    The result is written to `out` (default: a new [B, S, H, 64] fp16 tensor, returned as the
    [B, H, S, 64] view of it).
    """
    dev = _require_cuda(q, k, v, out)
    for name, t in (("q", q), ("k", k), ("v", v)):
        if t.dtype != F16 or t.ndim != 4 or t.shape[-1] != 64 or t.stride(-1) != 1:
            raise ValueError(f"{name} must be fp16 [B,H,S,64] with unit dim stride")
    bsz, heads, sq, _ = q.shape
    skv = k.shape[2]
    if k.shape != (bsz, heads, skv, 64) or v.shape != k.shape:
        raise ValueError("k/v shape mismatch")
    if out is None:
        out = torch.empty((bsz, sq, heads, 64), device=dev, dtype=F16).transpose(1, 2)
    strides = lambda t: _lib.i64_array((t.stride(0), t.stride(1), t.stride(2)))  # noqa: E731
    _lib.check(_lib.load().h3b_attention_f16(q.data_ptr(), strides(q), k.data_ptr(), strides(k), v.data_ptr(),
                                             strides(v), out.data_ptr(), strides(out), bsz, heads, sq, skv,
                                             float(scale), _stream(dev)))
    _count(1)
    return out
