"""End-to-end runtime on the B200: a small H3-structured encoder/decoder, tiled encode/decode round
trip through the public first_stage_model API, and the INT8 path against the fp16 path of the same
weights (quality criterion: PSNR of INT8 vs fp16), and the fp16 profile's block chain against the
oracle composition."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _small_runtime(int8, **kw):
    from h3vae_b200.model import DecoderConfig, EncoderConfig
    from h3vae_b200.runtime import H3VAEPyOptRuntime
    enc = EncoderConfig(channels=(128, 256), blocks_per_stage=1, spatial_down=(True, False),
                        temporal_down=(True, False))
    dec = DecoderConfig(hidden=256, heads=4, blocks=2, ffn=512, up_channels=(128,), up_spatial=(True,),
                        up_temporal=(True,))
    return H3VAEPyOptRuntime(int8_encode=int8, int8_decode=int8, decode_fusions=int8, compile_decoder=False,
                             compile_encoder=False, log_calls=False, encoder_config=enc, decoder_config=dec,
                             encoder_tile_size=64, decoder_tile_size=64, tile_overlap_min=16, tile_batch=3, **kw)


def _psnr(a, b):
    mse = torch.mean((a.double() - b.double()) ** 2).item()
    return 10 * math.log10(1.0 / max(mse, 1e-20))


def test_round_trip_shapes_and_int8_vs_fp16():
    torch.manual_seed(0)
    video = (torch.rand(1, 3, 20, 96, 160) * 2 - 1).half()
    rt8 = _small_runtime(True)
    rt16 = _small_runtime(False)
    lat8 = rt8.encode(video.cuda())
    lat16 = rt16.encode(video.cuda())
    # 20 frames -> 2 clips of 9 tokens, minus the 6 tokens of the last clip's padding frames (toy
    # temporal ratio 2: a 5-frame tail keeps 3 tokens)
    assert lat8.shape == (1, 16, 12, 48, 80) and lat8.dtype == torch.float32
    assert torch.isfinite(lat8).all()
    rel = ((lat8 - lat16).norm() / lat16.norm()).item()
    assert rel < 0.05, rel
    out8 = rt8.decode(lat16.half())
    out16 = rt16.decode(lat16.half())
    assert out8.shape == rt8.decode_output_shape(lat16.shape) == (1, 3, 22, 96, 160)
    assert out8.dtype == torch.float32 and float(out8.min()) >= 0.0 and float(out8.max()) <= 1.0
    psnr = _psnr(out8, out16)
    print(f"INT8 vs fp16 decode PSNR {psnr:.2f} dB, encode latent rel err {rel:.4f}")
    assert psnr > 35.0, psnr
    # output_buffer contract (ref: h3vae_runtime.py:544-562)
    buf = torch.empty_like(out8)
    res = rt8.decode(lat16.half(), output_buffer=buf)
    assert res is buf and torch.equal(buf, out8)


def test_tiled_equals_untiled_blend_weights_sum_to_one():
    # a constant latent decodes to the same pixels with or without tiling where tiles agree
    from h3vae_b200 import tiling
    plan = tiling.TilePlan.build(96, 160, 64, 16, 2)
    canvas = torch.zeros(96, 160, dtype=torch.float64)
    for i, j in plan.tiles():
        tiling.accumulate_tile(canvas, torch.ones(plan.hs[i], plan.ws[j], dtype=torch.float64), plan, i, j)
    assert torch.allclose(canvas, torch.ones_like(canvas))


def _oracle_fp16_chain(dec, x, grid):
    """The fp16 block chain composed from the oracle's restatements (rms_norm_f16, linear_f16,
    qk_rope, attention, ffn_up_swiglu_f16), with the model's fp32 residual adds and final LayerNorm."""
    import numpy as np
    from oracle import h3vae_oracle as O
    cfg = dec.cfg
    b, n, d = x.shape
    cos, sin = (t.cpu().numpy() for t in dec._rope(b, *grid))
    npy = lambda t: t.detach().cpu().numpy()  # noqa: E731
    xs = x.reshape(b * n, d).numpy()
    for blk in dec.blocks:
        n1 = O.rms_norm_f16(xs, npy(blk.norm1_w), cfg.eps)
        qkv = O.linear_f16(n1, npy(blk.qkv_w), npy(blk.qkv_b)).reshape(b, n, 3 * d)
        q, k, v = O.qk_rope(qkv, cos, sin, cfg.heads, cfg.qk_eps)
        att = O.attention(q.transpose(0, 2, 1, 3), k.transpose(0, 2, 1, 3), v.transpose(0, 2, 1, 3), 1.0 / 8.0)
        y = att.transpose(0, 2, 1, 3).reshape(b * n, d).astype(np.float16)
        a = O.linear_f16(y, npy(blk.out_w), npy(blk.out_b))
        h = (xs.astype(np.float32) + a.astype(np.float32) * npy(blk.scale1).astype(np.float32)).astype(np.float16)
        n2 = O.rms_norm_f16(h, npy(blk.norm2_w), cfg.eps)
        act = O.ffn_up_swiglu_f16(n2, npy(blk.up_w), npy(blk.up_b))
        o = O.linear_f16(act, npy(blk.down_w), npy(blk.down_b))
        xs = (h.astype(np.float32) + o.astype(np.float32) * npy(blk.scale2).astype(np.float32)).astype(np.float16)
    xf = xs.astype(np.float64)
    mean, var = xf.mean(-1, keepdims=True), xf.var(-1, keepdims=True)
    ln = (xf - mean) / np.sqrt(var + cfg.eps) * npy(dec.ln_w).astype(np.float64) + npy(dec.ln_b).astype(np.float64)
    return ln.reshape(b, n, d)


def test_fp16_block_chain_matches_oracle():
    """The fp16 decoder profile's block chain (tcgen05 fp16 linears, fused FFN-up + SwiGLU, QK-norm +
    RoPE, tcgen05 attention) against the oracle composition: relative L2 error below 1e-2 after two
    blocks and the final LayerNorm (fp16 rounding points differ only by accumulation order)."""
    from h3vae_b200.model import DecoderConfig, H3Decoder
    cfg = DecoderConfig(hidden=256, heads=4, blocks=2, ffn=512, up_channels=(128,), up_spatial=(True,),
                        up_temporal=(True,))
    dec = H3Decoder(cfg, device="cuda", seed=3, int8=False)
    grid = (2, 8, 16)
    g = torch.Generator().manual_seed(9)
    x = torch.randn(2, 2 * 8 * 16, cfg.hidden, generator=g).half()
    got = dec.transformer(x.cuda(), grid).double().cpu()
    ref = torch.from_numpy(_oracle_fp16_chain(dec, x, grid))
    rel = ((got - ref).norm() / ref.norm()).item()
    assert rel < 1e-2, rel


def test_decode_into_pinned_host_buffer_streams_chunks():
    """decode(output_buffer=<pinned host tensor>) finalizes and copies each temporal chunk on a side
    stream while later chunks decode; the result equals the device-side decode bit for bit."""
    torch.manual_seed(1)
    rt = _small_runtime(True)
    lat = torch.randn(1, 16, 2 * 9, 40, 72).half()   # 2 temporal chunks x 2x3 tiles, 3 tiles per call
    ref = rt.decode(lat.cuda()).cpu()
    buf = torch.empty(ref.shape, dtype=torch.float32).pin_memory()
    res = rt.decode(lat, output_buffer=buf)
    assert res is buf
    assert torch.equal(buf, ref)


def test_encode_from_pinned_host_video_streams_clip_batches():
    """encode(<pinned host video>) uploads clip batch by clip batch on a side stream while earlier
    batches encode; the latents equal the encode of the same video already on the device."""
    torch.manual_seed(2)
    rt = _small_runtime(True, encoder_staged_batch=1)
    video = (torch.rand(1, 3, 40, 96, 160) * 2 - 1).half()   # 3 clips, the last one padded
    ref = rt.encode(video.cuda())
    got = rt.encode(video.pin_memory())
    assert torch.equal(got, ref)
