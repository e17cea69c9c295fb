"""Memory-bound producers on the B200 vs the CPU oracle: encoder GroupNorm/SiLU/pad (INT8 and
fp16), residual pack, per-tensor quantization, pixel finalization, decoder row producers,
standalone QK-RoPE and attention.  Cases follow tests/test_encoder_int8_norm.py:39-69 and
tests/test_int8_ffn_up_fused_gpu.py:21-46 of the reference."""
import numpy as np
import pytest
import torch

from oracle import h3vae_oracle as O

pytestmark = pytest.mark.gpu


def _close(got, ref, atol=1e-2, rtol=1e-3):
    got = np.asarray(got, np.float32)
    ref = np.asarray(ref, np.float32)
    diff = np.abs(got - ref)
    assert np.all(diff <= atol + rtol * np.abs(ref)), (diff.max(), np.unravel_index(diff.argmax(), diff.shape))


def _q_close(got, ref, frac=1e-3):
    d = np.abs(got.astype(np.int32) - ref.astype(np.int32))
    assert d.max() <= 1 and np.count_nonzero(d) <= max(2, frac * d.size), (d.max(), np.count_nonzero(d))


NORM_CASES = [(41, 1, 128, 1, 2, 3), (42, 1, 256, 3, 13, 19), (43, 1, 128, 17, 64, 64), (44, 4, 512, 3, 8, 8),
              (45, 2, 64, 2, 5, 7)]


@pytest.mark.parametrize("seed,b,c,d,h,w", NORM_CASES)
@pytest.mark.parametrize("with_pre_bias", [False, True])
def test_norm_pad_quant_and_f16(cuda_lib, seed, b, c, d, h, w, with_pre_bias):
    from h3vae_b200 import kernels as K
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(b, c, d, h, w, generator=g).half()
    gamma = torch.randn(c, generator=g).half()
    beta = torch.randn(c, generator=g).half()
    pre = torch.randn(c, generator=g).half() if with_pre_bias else None
    eps = 1e-6
    xc = x.cuda()
    for layout in (xc, xc.contiguous(memory_format=torch.channels_last_3d)):
        y = K.norm_pad_f16(layout, gamma.cuda(), beta.cuda(), eps, None if pre is None else pre.cuda())
        ref_y = O.norm_pad_f16(x.numpy(), gamma.numpy(), beta.numpy(), eps, None if pre is None else pre.numpy())
        assert y.is_contiguous(memory_format=torch.channels_last_3d)
        _close(y.cpu().numpy(), ref_y)
        q, s = K.norm_pad_quant(layout, gamma.cuda(), beta.cuda(), eps, None if pre is None else pre.cuda())
        ref_q, ref_s = O.norm_pad_quant(x.numpy(), gamma.numpy(), beta.numpy(), eps,
                                        None if pre is None else pre.numpy())
        assert abs(float(s) - float(ref_s)) <= 1e-3 * float(ref_s)
        _q_close(q.cpu().numpy(), ref_q)


@pytest.mark.parametrize("b,c,d,h,w,sp,tp", [(1, 128, 3, 4, 6, True, True), (2, 256, 5, 8, 8, True, False),
                                             (1, 64, 1, 3, 5, True, True), (1, 128, 4, 6, 6, False, True)])
def test_upsample_norm_pad_f16(cuda_lib, b, c, d, h, w, sp, tp):
    from h3vae_b200 import kernels as K
    g = torch.Generator().manual_seed(b * 7 + c + d)
    x = torch.randn(b, c, d, h, w, generator=g).half()
    gamma = torch.randn(c, generator=g).half()
    beta = torch.randn(c, generator=g).half()
    pre = torch.randn(c, generator=g).half()
    up = x
    if tp and d > 1:
        up = torch.cat([up[:, :, :1], up[:, :, 1:].repeat_interleave(2, dim=2)], dim=2)
    if sp:
        up = up.repeat_interleave(2, dim=3).repeat_interleave(2, dim=4)
    y = K.upsample_norm_pad_f16(x.cuda(), gamma.cuda(), beta.cuda(), 1e-6, spatial=sp, temporal=tp,
                                pre_bias=pre.cuda())
    ref = O.norm_pad_f16(up.numpy(), gamma.numpy(), beta.numpy(), 1e-6, pre.numpy())
    assert tuple(y.shape) == ref.shape
    _close(y.cpu().numpy(), ref)


def test_constant_norm_outputs(cuda_lib):
    # ref: tests/test_encoder_int8_norm.py:62-69 -- zero input, constant bias incl. subnormals
    from h3vae_b200 import kernels as K
    x = torch.zeros((1, 128, 1, 3, 5), dtype=torch.float16)
    gamma = torch.ones(128, dtype=torch.float16)
    for value in (0.0, 2**-24, 2**-14, -10.0, 2.0):
        beta = torch.full((128,), value, dtype=torch.float16)
        q, s = K.norm_pad_quant(x.cuda(), gamma.cuda(), beta.cuda(), 1e-6)
        ref_q, ref_s = O.norm_pad_quant(x.numpy(), gamma.numpy(), beta.numpy(), 1e-6)
        # the kernel's SiLU uses the fast exp/divide (the reference's Triton lowering): one fp16 ulp
        assert abs(float(s) - float(ref_s)) <= 2e-3 * float(ref_s)
        _q_close(q.cpu().numpy(), ref_q)


@pytest.mark.parametrize("shape", [(1, 256, 3, 6, 8), (2, 256, 17, 16, 16), (1, 128, 2, 2, 2)])
def test_residual_pack(cuda_lib, shape):
    from h3vae_b200 import kernels as K
    g = torch.Generator().manual_seed(3)
    x = torch.randn(*shape, generator=g).half()
    r = torch.randn(*shape, generator=g).half()
    bias = torch.randn(shape[1], generator=g).half()
    y = K.residual_pack(x.cuda(), r.cuda(), bias.cuda())
    assert np.array_equal(y.cpu().numpy(), O.residual_pack(x.numpy(), r.numpy(), bias.numpy()))


def test_quantize_tensor_layouts_and_known_answers(cuda_lib):
    # ref: tests/test_encoder_int8_gpu.py:42-72
    from h3vae_b200 import kernels as K
    torch.manual_seed(20261002)
    for shape in [(2, 3, 5, 7, 11), (1, 128, 19, 66, 66)]:
        x = torch.randn(shape, dtype=torch.float16)
        xc = x.cuda()
        layouts = [xc, xc.contiguous(memory_format=torch.channels_last_3d)]
        if shape[1] == 3:
            layouts.append(xc[..., ::2])
        for value in layouts:
            q, s = K.quantize_tensor_i8(value)
            rq, rs = O.quantize_activation_tensor(value.cpu().numpy())
            assert float(s) == float(rs)
            assert np.array_equal(q.cpu().numpy(), rq)
            assert q.is_contiguous(memory_format=torch.channels_last_3d)
    for maximum in [0.0, 2**-24, 2**-14, 0.5, 127.0, 65504.0]:
        x = torch.full((1, 1, 1, 1, 9), maximum, dtype=torch.float16)
        x[..., 0] = -maximum
        q, s = K.quantize_tensor_i8(x.cuda())
        rq, rs = O.quantize_activation_tensor(x.numpy())
        assert float(s) == float(rs) and np.array_equal(q.cpu().numpy(), rq)
    x = torch.tensor([-127.0, -0.5, -1.5, 0.0, 0.5, 1.5, 127.0], dtype=torch.float16).view(1, 1, 1, 1, 7)
    q, s = K.quantize_tensor_i8(x.cuda())
    assert float(s) == 1.0 and q.flatten().tolist() == [-127, -1, -2, 0, 1, 2, 127]
    with pytest.raises(ValueError, match="nonempty"):
        K.quantize_tensor_i8(torch.empty((1, 1, 0, 1, 1), dtype=torch.float16, device="cuda"))


def test_finalize_pixels(cuda_lib):
    from h3vae_b200 import kernels as K
    g = torch.Generator().manual_seed(5)
    x = (torch.randn(1, 3, 5, 16, 24, generator=g) * 3).half()
    x[0, 0, 0, 0, 0] = float("nan")
    std = torch.tensor((0.229, 0.224, 0.225), dtype=torch.float32)
    mean = torch.tensor((0.485, 0.456, 0.406), dtype=torch.float32)
    ref = O.finalize_pixels(x.numpy(), std.numpy(), mean.numpy())
    for xv in (x.cuda(), x.cuda().float(), x.cuda().transpose(3, 4).contiguous().transpose(3, 4)):
        out = K.finalize_pixels(xv, std.cuda(), mean.cuda())
        got = out.cpu().numpy()
        assert np.array_equal(np.isnan(got), np.isnan(ref))
        assert np.array_equal(np.nan_to_num(got), np.nan_to_num(ref))
    # a frame-major fp32 canvas ([b, t, c, h, w] storage viewed as [b, c, t, h, w]), two batch
    # entries, rows wider than one pass of the block's threads
    fm = (torch.randn(2, 5, 3, 7, 300, generator=g) * 3).permute(0, 2, 1, 3, 4)
    out = K.finalize_pixels(fm.cuda(), std.cuda(), mean.cuda())
    assert out.is_contiguous()
    assert np.array_equal(out.cpu().numpy(), O.finalize_pixels(fm.numpy(), std.numpy(), mean.numpy()))


@pytest.mark.parametrize("m,k", [(1, 2048), (17, 1024), (129, 2048), (7188, 2048), (64, 8192), (3, 16384),
                                 (300, 4096), (9, 1000)])
def test_row_quant_and_swiglu_quant(cuda_lib, m, k):
    from h3vae_b200 import kernels as K
    g = torch.Generator().manual_seed(m + k)
    x = torch.randn(m, k, generator=g).half()
    x[0, :] = 0
    if m > 2:
        x[1, :] *= 1e-5   # row scale below the fp16 normal range: every element takes the exact path
        x[2, :] = torch.round(x[2, :] * 8) / 8   # many quotients on fp16 midpoints
    q, s = K.row_quant(x.cuda())
    rq, rs = O.row_quant_ck(x.float().numpy())
    assert np.array_equal(s.cpu().numpy(), rs)
    assert np.array_equal(q.cpu().numpy(), rq)
    if k <= 16384:
        xx = torch.randn(m, 2 * k, generator=g).half() if k <= 8192 else torch.randn(m, k, generator=g).half()
        kk = xx.shape[1] // 2
        q2, s2 = K.swiglu_quant(xx.cuda())
        rq2, rs2 = O.quantize_swiglu(xx.numpy())
        np.testing.assert_allclose(s2.cpu().numpy(), rs2, rtol=1e-5)
        _q_close(q2.cpu().numpy(), rq2)
        assert q2.shape == (m, kk)


@pytest.mark.parametrize("m,k", [(1, 2048), (129, 1024), (7188, 2048), (33, 4096)])
@pytest.mark.parametrize("round_stats", [False, True])
def test_residual_rms_quant(cuda_lib, m, k, round_stats):
    from h3vae_b200 import kernels as K
    g = torch.Generator().manual_seed(m * 3 + k)
    x = torch.randn(m, k, generator=g).half()
    a = torch.randn(m, k, generator=g).half()
    gv = (torch.rand(k, generator=g) * 0.2).half()
    w = (torch.rand(k, generator=g) + 0.5).half()
    h, q, s, norm = K.residual_rms_quant(x.cuda(), a.cuda(), gv.cuda(), w.cuda(), 1e-5, round_stats=round_stats,
                                         return_norm=True)
    rh, rq, rs, rnorm = O.residual_rms_quant(x.numpy(), a.numpy(), gv.numpy(), w.numpy(), 1e-5, round_stats)
    assert np.array_equal(h.cpu().numpy(), rh)
    _close(norm.cpu().numpy(), rnorm)
    np.testing.assert_allclose(s.cpu().numpy(), rs, rtol=1e-3)
    _q_close(q.cpu().numpy(), rq, frac=2e-3)
    # in-place residual (the norm1 producer contract: h is updated in place)
    xc = x.cuda()
    h2, q2, s2 = K.residual_rms_quant(xc, a.cuda(), gv.cuda(), w.cuda(), 1e-5, h_out=xc)
    assert h2.data_ptr() == xc.data_ptr() and np.array_equal(xc.cpu().numpy(), rh)


@pytest.mark.parametrize("m,k", [(7188, 2048), (5, 1024)])
def test_rms_and_final_layernorm(cuda_lib, m, k):
    from h3vae_b200 import kernels as K
    g = torch.Generator().manual_seed(11)
    x = torch.randn(m, k, generator=g).half()
    o = torch.randn(m, k, generator=g).half()
    gamma = torch.randn(k, generator=g).half()
    beta = torch.randn(k, generator=g).half()
    gate = (torch.rand(k, generator=g) * 0.3).half()
    _close(K.rms_norm_f16(x.cuda(), gamma.cuda(), 1e-5).cpu().numpy(), O.rms_norm_f16(x.numpy(), gamma.numpy(), 1e-5))
    q, s = K.rms_quant(x.cuda(), gamma.cuda(), 1e-5)
    rq, rs = O.row_quant_ck(O.rms_norm_f16(x.numpy(), gamma.numpy(), 1e-5).astype(np.float32))
    _q_close(q.cpu().numpy(), rq, frac=2e-3)
    y = K.final_residual_layernorm(x.cuda(), o.cuda(), gate.cuda(), gamma.cuda(), beta.cuda(), 1e-5)
    _close(y.cpu().numpy(), O.final_residual_layernorm(x.numpy(), o.numpy(), gate.numpy(), gamma.numpy(),
                                                       beta.numpy(), 1e-5), atol=2e-2)


def test_qk_rope_standalone(cuda_lib):
    from h3vae_b200 import kernels as K
    rng = np.random.default_rng(2)
    b, n, heads, r = 2, 77, 4, 48
    qkv = (rng.standard_normal((b, n, heads * 192)) * 3).astype(np.float16)
    ang = rng.random((b, n, 1, r)).astype(np.float32) * 6.28
    cos, sin = np.cos(ang).astype(np.float16), np.sin(ang).astype(np.float16)
    q, k = K.qk_rope(torch.from_numpy(qkv).cuda(), torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda(),
                     heads, 1e-6)
    rq, rk, _ = O.qk_rope(qkv, cos, sin, heads, 1e-6)
    _close(q.cpu().numpy(), rq)
    _close(k.cpu().numpy(), rk)


@pytest.mark.parametrize("mode", ["self", "rising"])
def test_attention_running_max_moves(cuda_lib, mode):
    """Rows whose running max jumps by a lot in a later key block (the diagonal of q = k = v, or keys
    growing along the sequence) take the O rescale path while their warp neighbours may not."""
    from h3vae_b200 import kernels as K
    g = torch.Generator().manual_seed(11)
    q = torch.randn(1, 2, 1024, 64, generator=g).half()
    if mode == "self":
        k = v = q
    else:
        k = (torch.randn(1, 2, 1024, 64, generator=g) * torch.linspace(0.2, 3.0, 1024).view(1, 1, -1, 1)).half()
        v = torch.randn(1, 2, 1024, 64, generator=g).half()
    out = K.attention_f16(q.cuda(), k.cuda(), v.cuda(), 0.125)
    ref = O.attention(q.numpy(), k.numpy(), v.numpy(), 0.125)
    _close(out.cpu().numpy(), ref, atol=4e-3, rtol=4e-3)


@pytest.mark.parametrize("b,h,sq,skv", [(1, 2, 64, 64), (2, 3, 100, 77), (4, 16, 1024, 1024), (1, 2, 1797, 1797)])
def test_attention(cuda_lib, b, h, sq, skv):
    from h3vae_b200 import kernels as K
    g = torch.Generator().manual_seed(b + h + sq)
    q = torch.randn(b, h, sq, 64, generator=g).half()
    k = torch.randn(b, h, skv, 64, generator=g).half()
    v = torch.randn(b, h, skv, 64, generator=g).half()
    out = K.attention_f16(q.cuda(), k.cuda(), v.cuda(), 0.125)
    ref = O.attention(q.numpy(), k.numpy(), v.numpy(), 0.125)
    _close(out.cpu().numpy(), ref, atol=4e-3, rtol=4e-3)


@pytest.mark.parametrize("h,w,tile,ov,tile_dtype", [(96, 200, 64, 16, torch.float16), (40, 300, 256, 32, torch.float32),
                                                    (130, 130, 64, 8, torch.float16), (50, 200, 200, 16, torch.float16)])
def test_blend_accumulate(cuda_lib, h, w, tile, ov, tile_dtype):
    """Every tile of a split accumulated on the GPU equals the CPU weighted accumulation bit for
    bit and the reference's sequential blend-and-trim restatement within fp32 rounding; the
    canvas windows are strided views, the tiles strided channel slices of a larger tensor and the
    widths ragged against the kernel's 128-wide pieces."""
    from h3vae_b200 import kernels as K
    from h3vae_b200 import tiling
    plan = tiling.TilePlan.build(h, w, tile, ov, 1)
    g = torch.Generator().manual_seed(h * w)
    c, t = 3, 5
    tiles, dev_tiles = {}, {}
    for (i, j) in plan.tiles():
        moments = (torch.randn(2 * c, t, plan.hs[i], plan.ws[j], generator=g) * 2).to(tile_dtype)
        tiles[(i, j)] = moments[::2]
        dev_tiles[(i, j)] = moments.cuda()[::2]   # strided: every other channel
    ref = torch.zeros(2, c, t, plan.height, plan.width)
    for (i, j), v in tiles.items():
        tiling.accumulate_tile(ref[1], v, plan, i, j)
    canvas = torch.zeros(2, c, t, plan.height, plan.width, device="cuda")
    for (i, j), v in tiles.items():
        y, x = plan.ys[i], plan.xs[j]
        wmap = tiling.tile_weight_map(plan, i, j, torch.float32, "cuda")
        K.blend_accumulate(canvas[1, :, :, y:y + plan.hs[i], x:x + plan.ws[j]], dev_tiles[(i, j)], wmap)
    got = canvas.cpu()
    assert torch.equal(got[0], torch.zeros_like(got[0]))
    assert torch.equal(got[1], ref[1])
    seq = tiling.blend_sequential({k: v.double() for k, v in tiles.items()}, plan)
    assert torch.allclose(got[1].double(), seq, atol=1e-5, rtol=1e-5)


def test_blend_accumulate_rejects_bad_arguments(cuda_lib):
    from h3vae_b200 import kernels as K
    canvas = torch.zeros(3, 2, 8, 8, device="cuda")
    with pytest.raises(ValueError):
        K.blend_accumulate(canvas, torch.zeros(3, 2, 8, 7, device="cuda"), torch.ones(8, 8, device="cuda"))
    with pytest.raises(ValueError):
        K.blend_accumulate(canvas, torch.zeros(3, 2, 8, 8, device="cuda"), torch.ones(8, 16, device="cuda")[:, ::2])
    with pytest.raises(ValueError):
        K.blend_accumulate(canvas.half(), torch.zeros(3, 2, 8, 8, device="cuda"), torch.ones(8, 8, device="cuda"))
