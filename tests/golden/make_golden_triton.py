"""Generate tests/golden/golden_v2.npz by running the reference's own Triton kernels on the CPU.

TEST INFRASTRUCTURE ONLY (fixture generator).  Run once in a container that has the reference
checkout (fishelegs/ComfyUI-H3VAE-PyOpt 0.2.0) and Triton; the checkout path is a required argument:

    python tests/golden/make_golden_triton.py <path-to-reference-checkout>

Triton's interpreter (TRITON_INTERPRET=1) executes each @triton.jit kernel of the reference with
numpy, program instance by program instance, so no GPU is needed and the GPU box never runs this
script: the tests read only the committed .npz.  Each fixture launches the reference kernel with the
grid, block sizes and argument order of the reference wrapper named beside it (the wrappers
themselves refuse CPU tensors).  What the interpreter cannot execute is emulated, and that is the
only departure from the compiled kernels:
  * libdevice calls (exp, rsqrt, nearbyint, fma) become interpreter-executable equivalents
    (numpy exp / 1/sqrt, round-half-to-even, an fp32 fma through an exact float64 product);
  * tl.exp, `/` and tl.sum run in numpy (IEEE exp and division, numpy's pairwise summation order),
    where the compiled kernels use the SFU's approximate exp2 / division and a tree reduction.
So index arithmetic, padding, reduction structure (chunk sizes, Chan merges), fp16 rounding points
and the integer paths are the reference's own; transcendental results may differ from the compiled
kernels in the last bits, which the tests' tolerances cover.

Fixtures (all seeded):
  np_*   quantized_temporal_norm_pad (opt/encoder_int8_norm.py:16-50, 77-110): GroupNorm statistics
         (_partial / _partial_bias + _merge, opt/encoder_fused_temporal_norm.py:13-51,
         opt/encoder_fused_norm_bias.py:15-40), the recompute producer's two passes
         (opt/encoder_int8_norm_recompute.py:11-49) and the absmax/scale kernels
         (opt/encoder_int8.py:343-364); with and without pre_bias; plus the fp16 padded pack
         _norm_pack_with_maxima (opt/encoder_int8_norm.py:53-74)
  rp_*   residual_downsample_pack (opt/encoder_fused_residual_pack.py:12-50)
  aq_*   quantize_activation_tensor (opt/encoder_int8.py:384-426)
  cv_*   _conv3d_from_quantized (opt/encoder_int8.py:509-588) with the pipelined kernel and
         causal_prefix_zero=True (opt/encoder_int8_pipeline.py:16-121), with and without bias,
         and the default 64x64x64 kernel on a stride-(2,1,2) (1,3,3) conv (opt/encoder_int8.py:157-269)
  qk_*   qk_rope (opt/decoder_fused_qk_rope.py:12-49)
  sw_*   quantize_swiglu (opt/int8_swiglu_fused.py:16-66)
  rq_*   residual_quant (opt/int8_norm_quant.py:17-70), round_stats False and True
  ln_*   final_residual_ln_w8 (opt/decoder_final_norm.py:28-82)
  fu_*   quantize_ffn_up (opt/int8_ffn_up_fused.py:45-130): INT8 GEMM + fma epilogue + SwiGLU, row quant
  b0_*   block-0 RMS (opt/decoder_block0_norm.py:33-82)
  fp_*   finalize_pixels (opt/fp16_finalize.py:19-54), contiguous fp16 and strided fp32 inputs
"""
from __future__ import annotations

import importlib
import os
import sys
import types
from pathlib import Path

import numpy as np


def _libdevice_shim(triton, tl):
    # the interpreter resolves triton.language through the jit functions' module globals
    globals()["tl"], globals()["triton"] = tl, triton

    @triton.jit
    def exp(x):
        return tl.exp(x)

    @triton.jit
    def rsqrt(x):
        return tl.rsqrt(x)

    @triton.jit
    def nearbyint(x):
        # round half to even (exact for the |x| < 2^22 this is used on)
        r = tl.floor(x + 0.5)
        odd = (r - 2.0 * tl.floor(r * 0.5)) != 0.0
        return tl.where(((r - x) == 0.5) & odd, r - 1.0, r)

    @triton.jit
    def fma(a, b, c):
        return (a.to(tl.float64) * b.to(tl.float64) + c.to(tl.float64)).to(tl.float32)

    return types.SimpleNamespace(exp=exp, rsqrt=rsqrt, nearbyint=nearbyint, fma=fma)


def main(ref_root: str) -> None:
    os.environ["TRITON_INTERPRET"] = "1"
    ref = Path(ref_root)
    if not (ref / "opt" / "encoder_int8.py").is_file():
        raise SystemExit(f"{ref} is not a ComfyUI-H3VAE-PyOpt checkout")
    sys.path.insert(0, str(ref))
    sys.path.insert(0, str(ref / "opt"))
    import torch
    import triton
    import triton.language as tl
    from torch._inductor.runtime import triton_helpers

    shim = _libdevice_shim(triton, tl)
    mods = {}
    for name in ("opt.encoder_int8", "opt.encoder_int8_pipeline", "opt.encoder_int8_norm_recompute",
                 "encoder_fused_temporal_norm", "encoder_fused_norm_bias", "encoder_fused_residual_pack",
                 "decoder_fused_qk_rope", "opt.int8_swiglu_fused", "opt.int8_norm_quant", "opt.decoder_final_norm",
                 "opt.int8_ffn_up_fused", "opt.decoder_block0_norm", "opt.fp16_finalize"):
        m = importlib.import_module(name)
        # the kernels are closures of lazy factory functions; the interpreter resolves their names in
        # the module globals, so the factory-local imports are provided there
        m.triton, m.tl, m.libdevice, m.triton_helpers = triton, tl, shim, triton_helpers
        mods[name] = m

    CL3 = torch.channels_last_3d
    out: dict[str, np.ndarray] = {}
    g = torch.Generator().manual_seed(20261202)

    def randn(*shape, std=1.0, mean=0.0):
        return torch.randn(*shape, generator=g) * std + mean

    # ------------------------------------------------------------------ norm producer
    norm_stat = mods["encoder_fused_temporal_norm"]
    norm_bias = mods["encoder_fused_norm_bias"]
    recompute = mods["opt.encoder_int8_norm_recompute"].recompute_pack_kernel()
    reduce_k, scale_k, quant_k = mods["opt.encoder_int8"]._quantization_kernels()

    def norm_statistics(x, eps, pre_bias):
        # opt/encoder_int8_norm.py:16-50
        b, c, d, h, w = x.shape
        bs, bc, warps = 128, 64, 8
        nparts = triton.cdiv(h * w, bs)
        p = torch.empty((d, nparts, 32), dtype=torch.float32)
        q = torch.empty_like(p)
        stats = torch.empty((d, 32, 2), dtype=torch.float32)
        grid = (nparts, triton.cdiv(c, bc), d)
        strides = (x.stride(2), x.stride(1), x.stride(3), x.stride(4))
        args = (p, q, c, h, w, *strides, 32, nparts, bs, bc)
        if pre_bias is None:
            norm_stat._partial[grid](x, *args, num_warps=warps)
        else:
            norm_bias._partial_bias[grid](x, pre_bias, *args, num_warps=warps)
        norm_stat._merge[(32, d)](p, q, stats, h, w, c, 32, nparts, bs, eps, triton.next_power_of_2(nparts),
                                  num_warps=4)
        return stats

    def norm_pad_quant(x, weight, bias, eps, pre_bias):
        # opt/encoder_int8_norm.py:77-110
        stats = norm_statistics(x, eps, pre_bias)
        b, c, d, h, w = x.shape
        qy = torch.empty((b, c, d + 2, h + 2, w + 2), dtype=torch.int8, memory_format=CL3)
        block = 4096
        count = triton.cdiv(qy.numel(), block)
        maxima = torch.empty((count,), dtype=torch.float32)
        act_scale = torch.empty((), dtype=torch.float32)
        args = (x, pre_bias if pre_bias is not None else bias, weight, bias, stats, qy, maxima, act_scale,
                c, d, h, w, x.stride(2), x.stride(1), x.stride(3), x.stride(4), pre_bias is not None)
        recompute[(count,)](*args, False, block, num_warps=4, enable_fp_fusion=False)
        nparts = triton.cdiv(count, 8192)
        partials = torch.empty((nparts,), dtype=torch.float32)
        reduce_k[(nparts,)](maxima, partials, count, GRID=nparts, BLOCK=8192, num_warps=4)
        scale_k[(1,)](partials, act_scale, N=nparts, BLOCK=triton.next_power_of_2(nparts), num_warps=4)
        recompute[(count,)](*args, True, block, num_warps=4, enable_fp_fusion=False)
        return stats, qy, act_scale

    def norm_pack_f16(x, weight, bias, eps, pre_bias):
        # opt/encoder_int8_norm.py:53-74
        stats = norm_statistics(x, eps, pre_bias)
        b, c, d, h, w = x.shape
        strides = (x.stride(2), x.stride(1), x.stride(3), x.stride(4))
        y = torch.empty((b, c, d + 2, h + 2, w + 2), dtype=x.dtype, memory_format=CL3)
        count = triton.cdiv(y.numel(), 1024)
        maxima = torch.empty((count,), dtype=torch.float32)
        args = (weight, bias, stats, y, c, d, h, w, *strides, 32, 1024)
        opts = dict(Maxima=maxima, WRITE_MAX=True, num_warps=4, enable_fp_fusion=False)
        if pre_bias is None:
            norm_stat._normalize_pack[(count,)](x, *args, **opts)
        else:
            norm_bias._normalize_pack_bias[(count,)](x, pre_bias, *args, **opts)
        return y

    for k, (shape, with_bias) in enumerate((((1, 128, 2, 12, 20), False), ((1, 256, 3, 9, 15), True))):
        c = shape[1]
        x = randn(*shape, std=1.5, mean=0.3).half().contiguous(memory_format=CL3)
        wgt = (1.0 + 0.3 * randn(c)).half()
        bia = (0.2 * randn(c)).half()
        pre = (0.5 * randn(c)).half() if with_bias else None
        eps = 1e-6
        stats, qy, sc = norm_pad_quant(x, wgt, bia, eps, pre)
        y16 = norm_pack_f16(x, wgt, bia, eps, pre)
        out[f"np{k}_x"], out[f"np{k}_w"], out[f"np{k}_b"] = x.numpy(), wgt.numpy(), bia.numpy()
        if pre is not None:
            out[f"np{k}_pre"] = pre.numpy()
        out[f"np{k}_stats"] = stats.numpy()
        out[f"np{k}_q"] = qy.numpy()                  # logical [B,C,D+2,H+2,W+2]
        out[f"np{k}_scale"] = sc.numpy().reshape(1)
        out[f"np{k}_y16"] = y16.numpy()
        print(f"norm producer {k}: scale {float(sc):.6g}")

    # ------------------------------------------------------------------ residual pack
    rp = mods["encoder_fused_residual_pack"]
    b, c, d, h, w = 1, 256, 3, 6, 7
    x = randn(b, c, d, h, w).half().contiguous(memory_format=CL3)
    r = randn(b, c, d, h, w).half().contiguous(memory_format=CL3)
    bias = (0.1 * randn(c)).half()
    y = torch.empty((b, c, d + 2, h + 1, w + 1), dtype=torch.float16, memory_format=CL3)
    rp._residual_pack[(triton.cdiv(y.numel(), 1024),)](
        x, r, bias, y, c, d, h, w, x.stride(2), x.stride(1), x.stride(3), x.stride(4),
        r.stride(2), r.stride(1), r.stride(3), r.stride(4), 1024, num_warps=4, enable_fp_fusion=False)
    out["rp_x"], out["rp_r"], out["rp_b"], out["rp_y"] = x.numpy(), r.numpy(), bias.numpy(), y.numpy()

    # ------------------------------------------------------------------ per-tensor activation quant
    xq = randn(1, 16, 4, 6, 7, std=2.0).half().contiguous(memory_format=CL3)
    xq[0, :7, 0, 0, 0] = torch.tensor([-127.0, -0.5, -1.5, 0.0, 0.5, 1.5, 127.0]).half()
    n_el = xq.numel()
    pcount = min(triton.cdiv(n_el, 8192), 2048)
    partials = torch.empty((pcount,), dtype=torch.float32)
    ascale = torch.empty((), dtype=torch.float32)
    qx = torch.empty(xq.shape, dtype=torch.int8, memory_format=CL3)
    reduce_k[(pcount,)](xq, partials, n_el, GRID=pcount, BLOCK=8192, num_warps=4)
    scale_k[(1,)](partials, ascale, N=pcount, BLOCK=1 << (pcount - 1).bit_length(), num_warps=4)
    quant_k[(triton.cdiv(n_el, 1024),)](xq, qx, ascale, n_el, BLOCK=1024, num_warps=4)
    out["aq_x"], out["aq_q"], out["aq_scale"] = xq.numpy(), qx.numpy(), ascale.numpy().reshape(1)

    # ------------------------------------------------------------------ INT8 implicit-GEMM conv
    enc = mods["opt.encoder_int8"]
    pipelined = mods["opt.encoder_int8_pipeline"].pipelined_conv3d_kernel()
    _, generic = enc._triton_kernels()

    def conv(qx, qw, xs, ws, bias, kernel, stride, variant, causal):
        # opt/encoder_int8.py:509-588
        b, c, d, h, w = qx.shape
        od, oh, ow = ((n - k) // s + 1 for n, k, s in zip((d, h, w), kernel, stride))
        o = qw.shape[0]
        y = torch.empty((b, o, od, oh, ow), dtype=torch.float16, memory_format=CL3)
        bm, bn, bk = {"64x64x64": (64, 64, 64), "128x128x64_pipeline4": (128, 128, 64)}[variant]
        pipe = variant == "128x128x64_pipeline4"
        opts = {}
        if pipe:
            opts["SKIP_CAUSAL_ZEROS"] = bool(causal and kernel == (3, 3, 3) and stride == (1, 1, 1)
                                             and (oh * ow) % bm == 0 and (9 * c) % bk == 0)
        grid = (triton.cdiv(b * od * oh * ow, bm), triton.cdiv(o, bn))
        has_bias = bias is not None
        bptr = bias if has_bias else torch.empty((1,), dtype=torch.float16)
        (pipelined if pipe else generic)[grid](
            qx, qw, xs, ws, bptr, y, b, c, d, h, w, o, od, oh, ow, *qx.stride(), *y.stride(), *stride,
            KERNEL_D=kernel[0], KERNEL_H=kernel[1], KERNEL_W=kernel[2], BLOCK_M=bm, BLOCK_N=bn, BLOCK_K=bk,
            HAS_BIAS=has_bias, num_warps=4, num_stages=4 if pipe else 2, **opts)
        return y

    qx = torch.randint(-127, 128, (1, 64, 5, 10, 18), generator=g, dtype=torch.int8)
    qx[:, :, :2] = 0                                            # the producer's two causal zero planes
    qx = qx.contiguous(memory_format=CL3)
    qw = torch.randint(-127, 128, (64, 27 * 64), generator=g, dtype=torch.int8)
    xs = torch.tensor(0.0123, dtype=torch.float32)
    ws = (torch.rand(64, generator=g) * 1e-3 + 1e-4).float()
    cb = (0.02 * randn(64)).half()
    out["cv_qx"], out["cv_qw"], out["cv_xs"], out["cv_ws"], out["cv_b"] = (
        qx.numpy(), qw.numpy(), xs.numpy().reshape(1), ws.numpy(), cb.numpy())
    out["cv_y_bias"] = conv(qx, qw, xs, ws, cb, (3, 3, 3), (1, 1, 1), "128x128x64_pipeline4", True).numpy()
    out["cv_y_nobias"] = conv(qx, qw, xs, ws, None, (3, 3, 3), (1, 1, 1), "128x128x64_pipeline4", True).numpy()
    qx2 = torch.randint(-127, 128, (1, 32, 5, 9, 12), generator=g, dtype=torch.int8).contiguous(memory_format=CL3)
    qw2 = torch.randint(-127, 128, (40, 9 * 32), generator=g, dtype=torch.int8)
    ws2 = (torch.rand(40, generator=g) * 1e-3 + 1e-4).float()
    cb2 = (0.02 * randn(40)).half()
    out["cv2_qx"], out["cv2_qw"], out["cv2_ws"], out["cv2_b"] = qx2.numpy(), qw2.numpy(), ws2.numpy(), cb2.numpy()
    out["cv2_y"] = conv(qx2, qw2, xs, ws2, cb2, (1, 3, 3), (2, 1, 2), "64x64x64", False).numpy()

    # ------------------------------------------------------------------ decoder producers
    qk = mods["decoder_fused_qk_rope"]
    b, n, heads, rot = 2, 6, 4, 48
    X = randn(b, n, 3 * 64 * heads, std=1.3).half()
    ang = torch.rand(b, n, 1, rot, generator=g) * 6.3
    C, S = ang.cos().half(), ang.sin().half()
    Q = torch.empty((b, n, heads, 64), dtype=torch.float16)
    Kt = torch.empty_like(Q)
    qk._qk_rope[(triton.cdiv(b * n * heads, 8),)](X, C, S, Q, Kt, b * n, heads, 64, rot, 1e-6, 8, num_warps=4,
                                                  enable_fp_fusion=False)
    out["qk_x"], out["qk_cos"], out["qk_sin"], out["qk_q"], out["qk_k"] = (X.numpy(), C.numpy(), S.numpy(),
                                                                            Q.numpy(), Kt.numpy())

    swq = mods["opt.int8_swiglu_fused"]._kernel()
    xs_ = randn(6, 2 * 96, std=2.5).half()
    xs_[3] = 0                                                   # zero row: scale 1e-30 -> fp16 0 -> -128
    qs = torch.empty((6, 96), dtype=torch.int8)
    ss = torch.empty((6, 1), dtype=torch.float32)
    swq[(6,)](xs_, qs, ss, 96, 128, num_warps=8, enable_fp_fusion=False)
    out["sw_x"], out["sw_q"], out["sw_s"] = xs_.numpy(), qs.numpy(), ss.numpy()

    rqk = mods["opt.int8_norm_quant"]._kernel()
    for kk, width in ((0, 1024), (1, 2048)):
        xr = randn(5, width).half()
        ar = randn(5, width, std=0.7).half()
        gr = (0.5 + 0.1 * randn(width)).half()
        wr = (1.0 + 0.1 * randn(width)).half()
        out[f"rq{kk}_x"], out[f"rq{kk}_a"], out[f"rq{kk}_g"], out[f"rq{kk}_w"] = (xr.numpy(), ar.numpy(), gr.numpy(),
                                                                                  wr.numpy())
        for rs in (False, True):
            h = torch.empty_like(xr)
            q = torch.empty((5, width), dtype=torch.int8)
            s = torch.empty((5, 1), dtype=torch.float32)
            rqk[(5,)](xr, ar, gr, wr, h, q, s, 1e-5, width, rs, num_warps=8, enable_fp_fusion=False)
            tag = "r" if rs else "u"
            out[f"rq{kk}_{tag}_h"], out[f"rq{kk}_{tag}_q"], out[f"rq{kk}_{tag}_s"] = h.numpy(), q.numpy(), s.numpy()

    lnk = mods["opt.decoder_final_norm"].kernel_for_inspection()
    m_, k_ = 4, 2048
    hl, ol = randn(m_, k_).half(), randn(m_, k_, std=0.8).half()
    gate, gam, bet = (0.5 + 0.1 * randn(k_)).half(), (1.0 + 0.1 * randn(k_)).half(), (0.1 * randn(k_)).half()
    yl = torch.empty_like(hl)
    lnk[(m_,)](hl, ol, gate, gam, bet, yl, m_, k_, 1e-5, num_warps=8, num_stages=1, enable_fp_fusion=True)
    out["ln_h"], out["ln_o"], out["ln_gate"], out["ln_gamma"], out["ln_beta"], out["ln_y"] = (
        hl.numpy(), ol.numpy(), gate.numpy(), gam.numpy(), bet.numpy(), yl.numpy())

    up_swiglu, quant_act = mods["opt.int8_ffn_up_fused"]._kernels()
    m_, n_, k_ = 70, 128, 128
    qa = torch.randint(-127, 128, (m_, k_), generator=g, dtype=torch.int8)
    sa = (torch.rand(m_, 1, generator=g) * 0.02 + 0.001).float()
    wq = torch.randint(-127, 128, (2 * n_, k_), generator=g, dtype=torch.int8)
    wsf = (torch.rand(2 * n_, generator=g) * 0.002 + 1e-4).float()
    bu = (0.05 * randn(2 * n_)).half()
    act = torch.empty((m_, n_), dtype=torch.float16)
    qo = torch.empty((m_, n_), dtype=torch.int8)
    so = torch.empty((m_, 1), dtype=torch.float32)
    bm, bn, bk, warps, stages = mods["opt.int8_ffn_up_fused"].CONFIG
    up_swiglu[(triton.cdiv(m_, bm) * triton.cdiv(n_, bn),)](qa, wq, sa, wsf, bu, act, m_, n_, k_, bm, bn, bk, True,
                                                            num_warps=warps, num_stages=stages,
                                                            enable_fp_fusion=False)
    quant_act[(m_,)](act, qo, so, n_, triton.next_power_of_2(n_), num_warps=8, enable_fp_fusion=False)
    out["fu_q"], out["fu_s"], out["fu_w"], out["fu_ws"], out["fu_b"] = (qa.numpy(), sa.numpy(), wq.numpy(),
                                                                         wsf.numpy(), bu.numpy())
    out["fu_act"], out["fu_qo"], out["fu_so"] = act.numpy(), qo.numpy(), so.numpy()

    b0 = mods["opt.decoder_block0_norm"]
    xb = randn(4, 2048, std=1.2).half()
    gb = (1.0 + 0.1 * randn(2048)).half()
    yb = torch.empty_like(xb)
    b0.kernel_for_inspection()[(2,)](xb, gb, yb, 4, 2, 2048, b0._EPS_F32, num_warps=16, num_stages=1,
                                     enable_fp_fusion=True)
    out["b0_x"], out["b0_g"], out["b0_y"] = xb.numpy(), gb.numpy(), yb.numpy()

    fin = mods["opt.fp16_finalize"].kernel()
    std = torch.tensor([0.229, 0.224, 0.225], dtype=torch.float32)
    mean = torch.tensor([0.485, 0.456, 0.406], dtype=torch.float32)
    xf = randn(1, 3, 2, 5, 7, std=3.0).half()
    xf.view(-1)[:4] = torch.tensor([float("nan"), float("inf"), -float("inf"), -0.0]).half()
    yf = torch.empty(xf.shape, dtype=torch.float32)
    fin[(triton.cdiv(xf.numel(), 1024),)](xf, std, mean, yf, xf.numel(), 2, 5, 7, *xf.stride(), True, 1024,
                                          num_warps=4, enable_fp_fusion=False)
    base = randn(1, 2, 5, 3, 7, std=3.0)
    xs32 = base.permute(0, 3, 1, 2, 4)                           # strided [1,3,2,5,7] fp32 view
    ys = torch.empty(xs32.shape, dtype=torch.float32)
    fin[(triton.cdiv(xs32.numel(), 1024),)](xs32, std, mean, ys, xs32.numel(), 2, 5, 7, *xs32.stride(), False,
                                            1024, num_warps=4, enable_fp_fusion=False)
    out["fp_x16"], out["fp_y16"] = xf.numpy(), yf.numpy()
    out["fp_x32"], out["fp_y32"] = xs32.contiguous().numpy(), ys.numpy()
    out["fp_std"], out["fp_mean"] = std.numpy(), mean.numpy()

    dest = Path(__file__).resolve().parent / "golden_v2.npz"
    np.savez_compressed(dest, **out)
    print(f"wrote {dest} ({dest.stat().st_size} bytes, {len(out)} arrays)")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden_triton.py <path-to-reference-checkout>")
    main(sys.argv[1])
