"""fp16 implicit-GEMM conv3d (tcgen05 kind::f16, fp32 accumulate) on the B200 vs a plain PyTorch
fp32 reference of the same op (CPU F.conv3d on the fp16 inputs, rounded to fp16).  Tolerance:
max-abs 1e-2 / rel 1e-3 on the fp16 outputs.  Covers the convolutions of the fp16 encoder/decoder
path: stride-2 downsample convs after the residual pack, 1x1x1 shortcuts, narrow conv_out (O=32),
the decoder's upsampling convs, fused bias and residual, the causal-zero tap skip."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _ref(x, w, b, stride, residual=None):
    y = F.conv3d(x.float(), w.float(), None if b is None else b.float(), stride=stride)
    if residual is not None:
        y = y.half().float() + residual.float()
    return y.half().float()


def _close(got, ref, atol=1e-2, rtol=1e-3):
    diff = (got.float() - ref).abs()
    bad = diff > atol + rtol * ref.abs()
    assert not bool(bad.any()), (float(diff.max()), int(bad.sum()))


CASES = [
    # (shape [B,C,D,H,W] of the padded input, O, kernel, stride)
    ((1, 128, 5, 19, 23), 128, (3, 3, 3), (1, 1, 1)),
    ((2, 64, 4, 10, 18), 128, (3, 3, 3), (1, 1, 1)),
    ((1, 128, 19, 65, 65), 128, (3, 3, 3), (1, 2, 2)),       # stage-0 downsample after the residual pack
    ((1, 256, 11, 33, 33), 256, (3, 3, 3), (2, 2, 2)),       # stage-1 downsample
    ((1, 512, 7, 17, 17), 512, (3, 3, 3), (2, 2, 2)),        # stage-2 downsample
    ((2, 128, 9, 16, 16), 256, (1, 1, 1), (1, 1, 1)),        # 1x1x1 shortcut
    ((1, 512, 7, 10, 12), 32, (3, 3, 3), (1, 1, 1)),         # encoder conv_out (BN=64 tile)
    ((1, 1024, 7, 10, 10), 512, (3, 3, 3), (1, 1, 1)),       # decoder upsampling conv
    ((1, 256, 5, 131, 130), 128, (3, 3, 3), (1, 1, 1)),      # two M tiles per CTA, odd tile count (kw-strip)
    ((1, 128, 5, 9, 200), 192, (3, 3, 3), (1, 1, 1)),        # O not a multiple of the tile, W > 128
    ((1, 128, 4, 150, 130), 256, (3, 3, 3), (1, 1, 1)),      # kw-strip kernel, 256 output columns
    ((1, 128, 4, 76, 258), 192, (3, 3, 3), (1, 1, 1)),       # kw-strip, 192 of 256 columns, 2 M tiles per row
]


def test_conv3d_f16_kw_strip_residual_causal(cuda_lib):
    """The decoder's 3x3x3 up-conv shape class (128-column rows, enough tiles for the kw-strip
    mainloop) with the two causal zero frames skipped and a fused residual."""
    from h3vae_b200 import kernels as K
    g = torch.Generator().manual_seed(11)
    x = torch.randn((1, 256, 5, 131, 130), generator=g).half()
    x[:, :, :2] = 0
    w = (torch.randn((128, 256, 3, 3, 3), generator=g) / (256 * 27) ** 0.5).half()
    b = (torch.randn(128, generator=g) * 0.1).half()
    r = torch.randn((1, 128, 3, 129, 128), generator=g).half()
    y = K.conv3d_f16(x.cuda().contiguous(memory_format=torch.channels_last_3d), K.pack_conv_weight_f16(w).cuda(),
                     b.cuda(), (3, 3, 3), (1, 1, 1), causal_zero_frames=2,
                     residual=r.cuda().contiguous(memory_format=torch.channels_last_3d))
    _close(y.cpu(), _ref(x, w, b, (1, 1, 1), residual=r))


@pytest.mark.parametrize("shape,o,kernel,stride", CASES)
@pytest.mark.parametrize("with_bias", [False, True])
def test_conv3d_f16_matches_fp32_reference(cuda_lib, shape, o, kernel, stride, with_bias):
    from h3vae_b200 import kernels as K
    g = torch.Generator().manual_seed(sum(shape) * 7 + o)
    c = shape[1]
    x = torch.randn(shape, generator=g).half()
    w = (torch.randn((o, c, *kernel), generator=g) / (c * kernel[0] * kernel[1] * kernel[2]) ** 0.5).half()
    b = (torch.randn(o, generator=g) * 0.1).half() if with_bias else None
    y = K.conv3d_f16(x.cuda().contiguous(memory_format=torch.channels_last_3d), K.pack_conv_weight_f16(w).cuda(),
                     None if b is None else b.cuda(), kernel, stride)
    assert y.is_contiguous(memory_format=torch.channels_last_3d)
    _close(y.cpu(), _ref(x, w, b, stride))


def test_conv3d_f16_residual_and_causal_skip(cuda_lib):
    from h3vae_b200 import kernels as K
    g = torch.Generator().manual_seed(3)
    x = torch.randn((2, 128, 7, 12, 20), generator=g).half()
    x[:, :, :2] = 0                                   # the causal zero pad
    w = (torch.randn((128, 128, 3, 3, 3), generator=g) / 3456 ** 0.5).half()
    b = (torch.randn(128, generator=g) * 0.1).half()
    ref = _ref(x, w, b, (1, 1, 1))
    r = torch.randn(ref.shape, generator=g).half()
    xc = x.cuda().contiguous(memory_format=torch.channels_last_3d)
    wp = K.pack_conv_weight_f16(w).cuda()
    rc = r.cuda().contiguous(memory_format=torch.channels_last_3d)
    full = K.conv3d_f16(xc, wp, b.cuda(), (3, 3, 3), residual=rc)
    skip = K.conv3d_f16(xc, wp, b.cuda(), (3, 3, 3), causal_zero_frames=2, residual=rc)
    assert torch.equal(full, skip)
    _close(full.cpu(), _ref(x, w, b, (1, 1, 1), residual=r))
    # stride-2 temporal with the causal skip: od*2 + kd < 2 only for od = 0
    x2 = torch.randn((1, 256, 9, 17, 17), generator=g).half()
    x2[:, :, :2] = 0
    w2 = (torch.randn((256, 256, 3, 3, 3), generator=g) / 6912 ** 0.5).half()
    x2c = x2.cuda().contiguous(memory_format=torch.channels_last_3d)
    a = K.conv3d_f16(x2c, K.pack_conv_weight_f16(w2).cuda(), None, (3, 3, 3), (2, 2, 2))
    s = K.conv3d_f16(x2c, K.pack_conv_weight_f16(w2).cuda(), None, (3, 3, 3), (2, 2, 2), causal_zero_frames=2)
    assert torch.equal(a, s)
    _close(a.cpu(), _ref(x2, w2, None, (2, 2, 2)))


def test_conv3d_f16_rejects_unsupported(cuda_lib):
    from h3vae_b200 import kernels as K
    x = torch.zeros((1, 48, 3, 8, 8), dtype=torch.float16, device="cuda").contiguous(
        memory_format=torch.channels_last_3d)
    w = torch.zeros((16, 27 * 48), dtype=torch.float16, device="cuda")
    with pytest.raises(ValueError, match="multiple of 64"):
        K.conv3d_f16(x, w, None, (3, 3, 3))


@pytest.mark.parametrize("shape", [(2, 3, 5, 20, 140), (1, 3, 17, 33, 17), (1, 3, 3, 1, 5), (1, 1, 2, 6, 9)])
@pytest.mark.parametrize("normalize", [False, True])
def test_conv_in_matches_fp32_reference(cuda_lib, shape, normalize):
    """Fused pixel normalization + causal/reflect pad + 3x3x3 input conv (ref: h3vae_runtime.py:566-570
    and the encoder's first causal conv) vs the same steps in PyTorch fp32 on the CPU."""
    from h3vae_b200 import kernels as K
    from h3vae_b200.model import causal_reflect_pad
    g = torch.Generator().manual_seed(sum(shape))
    cin = shape[1]
    x = (torch.rand(shape, generator=g) * 2 - 1).half()
    w = (torch.randn((128, cin, 3, 3, 3), generator=g) / (27 * cin) ** 0.5).half()
    b = (torch.randn(128, generator=g) * 0.1).half()
    mean = torch.rand(cin, generator=g) * 0.5
    std = 0.2 + torch.rand(cin, generator=g) * 0.1
    n = x
    if normalize:
        n = (((x.float() + 1.0) * 0.5 - mean.view(1, -1, 1, 1, 1)) / std.view(1, -1, 1, 1, 1)).half()
    ref = F.conv3d(causal_reflect_pad(n.float()), w.float(), b.float()).half().float()
    y = K.conv_in_f16(x.cuda(), w.cuda(), b.cuda(), (mean.cuda(), std.cuda()) if normalize else None)
    assert y.is_contiguous(memory_format=torch.channels_last_3d)
    _close(y.cpu(), ref)


@pytest.mark.parametrize("shape", [(1, 128, 7, 18, 258), (2, 64, 5, 11, 40), (1, 256, 3, 9, 131), (1, 128, 19, 34, 130)])
@pytest.mark.parametrize("with_bias", [False, True])
def test_conv_rgb_matches_fp32_reference(cuda_lib, shape, with_bias):
    """Decoder RGB output conv (taps packed into N, kw shift across TMEM lanes) vs PyTorch fp32."""
    from h3vae_b200 import kernels as K
    g = torch.Generator().manual_seed(sum(shape) + int(with_bias))
    c = shape[1]
    x = torch.randn(shape, generator=g).half()
    w = (torch.randn((3, c, 3, 3, 3), generator=g) / (27 * c) ** 0.5).half()
    b = (torch.randn(3, generator=g) * 0.1).half() if with_bias else None
    y = K.conv3d_rgb_f16(x.cuda().contiguous(memory_format=torch.channels_last_3d), K.pack_rgb_weight(w).cuda(),
                         None if b is None else b.cuda())
    assert y.is_contiguous()
    _close(y.cpu(), _ref(x, w, b, (1, 1, 1)))


@pytest.mark.parametrize("shape,channels_last", [((1, 16, 5, 8, 8), False), ((2, 16, 7, 12, 20), True),
                                                 ((1, 8, 1, 9, 6), False), ((1, 16, 3, 1, 7), True)])
def test_latent_conv_in_rows_match_fp32_reference(cuda_lib, shape, channels_last):
    """The decoder's 16-channel latent conv-in as unrolled rows (h3b_im2col_causal_f16: two causal
    zero frames, reflect pad 1 in H/W, zero pad when H or W is 1) times the weight rows on the
    tcgen05 fp16 GEMM vs PyTorch fp32 on the padded input; also the unrolled rows themselves against
    the padded tensor, bit for bit."""
    from h3vae_b200 import kernels as K
    from h3vae_b200.model import causal_conv3_rows_f16, causal_reflect_pad
    g = torch.Generator().manual_seed(sum(shape))
    b_, c, t, h, w_ = shape
    z = torch.randn(shape, generator=g).half()
    wt = (torch.randn((256, c, 3, 3, 3), generator=g) / (27 * c) ** 0.5).half()
    bias = (torch.randn(256, generator=g) * 0.1).half()
    zc = z.cuda().contiguous(memory_format=torch.channels_last_3d) if channels_last else z.cuda()
    cols = K.im2col_causal_f16(zc).cpu()
    padded = causal_reflect_pad(z.float())                                   # [B, C, T+2, H+2, W+2]
    unfold = padded.unfold(2, 3, 1).unfold(3, 3, 1).unfold(4, 3, 1)        # [B, C, T, H, W, 3, 3, 3]
    ref_cols = unfold.permute(0, 2, 3, 4, 5, 6, 7, 1).reshape(b_ * t * h * w_, 27 * c)
    assert torch.equal(cols.float(), ref_cols)
    rows = causal_conv3_rows_f16(zc, K.conv_weight_rows(wt.cuda()), bias.cuda())
    got = rows.view(b_, t, h, w_, 256).permute(0, 4, 1, 2, 3).cpu()
    ref = F.conv3d(padded, wt.float(), bias.float()).half().float()
    _close(got, ref)


def test_quant_conv_1x1_matches_fp32_reference(cuda_lib):
    """The encoder's 32-channel 1x1x1 quant conv as one tcgen05 fp16 GEMM on the channels-last moments
    (a [positions, 32] matrix as stored) vs PyTorch fp32."""
    from h3vae_b200.model import conv1x1_f16
    g = torch.Generator().manual_seed(5)
    x = torch.randn((2, 32, 5, 9, 13), generator=g).half()
    w = (torch.randn((32, 32, 1, 1, 1), generator=g) / 32 ** 0.5).half()
    b = (torch.randn(32, generator=g) * 0.1).half()
    y = conv1x1_f16(x.cuda().contiguous(memory_format=torch.channels_last_3d), w.cuda(), b.cuda())
    assert y.shape == x.shape and y.is_contiguous(memory_format=torch.channels_last_3d)
    _close(y.cpu(), F.conv3d(x.float(), w.float(), b.float()).half().float())
