"""End-to-end runtime on the B200: a small H3-structured encoder/decoder, tiled encode/decode round
trip through the public first_stage_model API, and the INT8 path against the fp16 path of the same
weights (quality criterion: PSNR of INT8 vs fp16)."""
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
    assert lat8.shape == (1, 16, 2 * 9, 48, 80) and lat8.dtype == torch.float32
    assert torch.isfinite(lat8).all()
    rel = ((lat8 - lat16).norm() / lat16.norm()).item()
    assert rel < 0.05, rel
    out8 = rt8.decode(lat16.half())
    out16 = rt16.decode(lat16.half())
    assert out8.shape == rt8.decode_output_shape(lat16.shape) == (1, 3, 34, 96, 160)
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
