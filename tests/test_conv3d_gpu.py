"""INT8 implicit-GEMM conv3d on the B200 vs the CPU oracle.

int32 accumulators must be bit-exact; fp16 outputs (same accumulators, same scales) must agree
within max-abs 1e-2 / rel 1e-3.  Cases follow the reference's GPU tests
(tests/test_encoder_int8_gpu.py:84-165): channel tails, stride 2, (1,3,3) kernels, the causal-zero
skip on short clips, the all-ones 27*128 known answer, plus BASELINE config 1."""
import numpy as np
import pytest
import torch

from oracle import h3vae_oracle as O

pytestmark = pytest.mark.gpu


def _run(qx_np, qw, ws, bias, kernel, stride, causal, sx=0.01):
    from h3vae_b200 import kernels as K
    qx = torch.from_numpy(qx_np).cuda().contiguous(memory_format=torch.channels_last_3d)
    acc = None
    out = None
    b, c, d, h, w = qx_np.shape
    do, ho, wo = ((d - kernel[0]) // stride[0] + 1, (h - kernel[1]) // stride[1] + 1, (w - kernel[2]) // stride[2] + 1)
    acc = torch.empty((b, qw.shape[0], do, ho, wo), dtype=torch.int32, device="cuda",
                      memory_format=torch.channels_last_3d)
    scale = torch.tensor(sx, dtype=torch.float32, device="cuda")
    out = K.conv3d_i8(qx, scale, torch.from_numpy(qw).cuda(), torch.from_numpy(ws).cuda(),
                      None if bias is None else torch.from_numpy(bias).cuda(), kernel, stride,
                      causal_zero_frames=causal, acc_out=acc)
    torch.cuda.synchronize()
    return out.cpu().numpy(), acc.cpu().numpy()


def _check(qx, qw, ws, bias, kernel, stride, causal, sx=0.01):
    out, acc = _run(qx, qw, ws, bias, kernel, stride, causal, sx)
    ref_acc = O.conv3d_int_acc(qx, qw, kernel, stride)
    assert np.array_equal(acc, ref_acc), f"int32 mismatch: {np.count_nonzero(acc != ref_acc)} elements"
    ref = O.conv_epilogue(ref_acc, np.float32(sx), ws, bias).astype(np.float32)
    diff = np.abs(out.astype(np.float32) - ref)
    assert np.all(diff <= 1e-2 + 1e-3 * np.abs(ref)), diff.max()
    return out, acc


CASES = [
    # (ci, co, shape, kernel, stride)
    (128, 128, (1, 128, 3, 19, 23), (3, 3, 3), (1, 1, 1)),
    (128, 256, (1, 128, 19, 17, 19), (3, 3, 3), (1, 1, 1)),
    (256, 256, (1, 256, 19, 17, 19), (3, 3, 3), (1, 1, 1)),
    (256, 129, (1, 256, 19, 10, 18), (3, 3, 3), (1, 1, 1)),
    (128, 128, (1, 128, 3, 10, 18), (1, 3, 3), (1, 1, 1)),
    (512, 512, (2, 512, 4, 10, 12), (3, 3, 3), (1, 1, 1)),
    (128, 64, (1, 128, 5, 34, 130), (3, 3, 3), (1, 1, 1)),
    (7, 19, (2, 7, 5, 9, 11), (3, 3, 3), (1, 2, 2)),
    (128, 128, (1, 128, 5, 17, 33), (3, 3, 3), (1, 2, 2)),
    (256, 256, (1, 256, 11, 33, 35), (3, 3, 3), (2, 2, 2)),
    # two M tiles per CTA (O <= 128 with enough tiles to fill the SMs), an odd tile count; with
    # 128-column rows these take the kw-strip kernel (three kw taps from one input strip)
    (128, 128, (1, 128, 5, 131, 130), (3, 3, 3), (1, 1, 1)),
    # kw-strip kernel: two channel chunks, an output-channel tail, two M tiles per output row
    (256, 96, (1, 256, 5, 62, 258), (3, 3, 3), (1, 1, 1)),
    # kw-strip kernel with 256 output columns (one M tile per CTA), and with a tail of 200
    (128, 256, (1, 128, 4, 76, 130), (3, 3, 3), (1, 1, 1)),
    (256, 200, (1, 256, 4, 76, 130), (3, 3, 3), (1, 1, 1)),
]


@pytest.mark.parametrize("ci,co,shape,kernel,stride", CASES)
@pytest.mark.parametrize("with_bias", [False, True])
def test_conv_matches_oracle(cuda_lib, ci, co, shape, kernel, stride, with_bias):
    rng = np.random.default_rng(hash((ci, co, shape, kernel, stride)) % 2**32)
    qx = rng.integers(-127, 128, size=shape, dtype=np.int8)
    taps = kernel[0] * kernel[1] * kernel[2]
    qw = rng.integers(-127, 128, size=(co, taps * ci), dtype=np.int8)
    ws = (rng.random(co, dtype=np.float32) * 0.002 + 0.0005).astype(np.float32)
    bias = rng.standard_normal(co).astype(np.float16) if with_bias else None
    _check(qx, qw, ws, bias, kernel, stride, 0)


@pytest.mark.parametrize("ci,co,shape,kernel,stride", [
    (128, 128, (1, 128, 3, 10, 18), (3, 3, 3), (1, 1, 1)),
    (128, 256, (1, 128, 4, 10, 18), (3, 3, 3), (1, 1, 1)),
    (256, 129, (1, 256, 19, 10, 18), (3, 3, 3), (1, 1, 1)),
    (128, 128, (1, 128, 3, 7, 9), (3, 3, 3), (1, 1, 1)),
    (7, 19, (1, 7, 5, 10, 18), (3, 3, 3), (1, 1, 1)),
    (128, 128, (1, 128, 5, 17, 33), (3, 3, 3), (1, 2, 2)),
    (128, 128, (1, 128, 3, 10, 18), (1, 3, 3), (1, 1, 1)),
    (128, 128, (1, 128, 5, 130, 130), (3, 3, 3), (1, 1, 1)),
    (256, 256, (1, 256, 11, 17, 17), (3, 3, 3), (2, 2, 2)),
])
def test_causal_zero_skip_is_exact(cuda_lib, ci, co, shape, kernel, stride):
    # ref: tests/test_encoder_int8_gpu.py:119-151 -- a known-zero prefix skipped or not gives equal results
    rng = np.random.default_rng(7)
    qx = rng.integers(-127, 128, size=shape, dtype=np.int8)
    qx[:, :, :2] = 0
    taps = kernel[0] * kernel[1] * kernel[2]
    qw = rng.integers(-127, 128, size=(co, taps * ci), dtype=np.int8)
    ws = np.full(co, 0.001, np.float32)
    for with_bias in (False, True):
        bias = rng.standard_normal(co).astype(np.float16) if with_bias else None
        full, acc_full = _check(qx, qw, ws, bias, kernel, stride, 0)
        skip, acc_skip = _check(qx, qw, ws, bias, kernel, stride, 2)
        assert np.array_equal(full, skip) and np.array_equal(acc_full, acc_skip)


def test_all_ones_known_answer(cuda_lib):
    # ref: tests/test_encoder_int8_gpu.py:153-165 -- 27*128 everywhere, the temporal prefix is not skipped
    qx = np.ones((1, 128, 3, 10, 18), np.int8)
    qw = np.ones((128, 27 * 128), np.int8)
    ws = np.ones(128, np.float32)
    out, acc = _run(qx, qw, ws, None, (3, 3, 3), (1, 1, 1), 0, sx=1.0)
    assert np.all(acc == 27 * 128) and np.all(out == 27 * 128)


def test_config1_quantized_conv(cuda_lib):
    """x [1,128,9,64,64] ~N(0,1), causal pad 2, reflect pad 1, W ~N(0, 1/sqrt(3456)),
    bias ~N(0,0.02); per-tensor activation quant.  int32 bit-exact vs the oracle and the dequantized
    result close to the unquantized fp32 conv."""
    from h3vae_b200 import kernels as K
    g = torch.Generator().manual_seed(0)
    x = torch.randn(1, 128, 9, 64, 64, generator=g)
    w = torch.randn(128, 128, 3, 3, 3, generator=g) / 3456 ** 0.5
    b = torch.randn(128, generator=g) * 0.02
    xp = F_pad(x)
    xh = xp.half()
    qw, ws = O.prepare_int8_weight(w)
    qx, sx = K.quantize_tensor_i8(xh.cuda())
    qx_ref, sx_ref = O.quantize_activation_tensor(xh.numpy())
    assert float(sx) == float(sx_ref)
    assert np.array_equal(qx.cpu().numpy(), qx_ref)
    acc = torch.empty((1, 128, 9, 64, 64), dtype=torch.int32, device="cuda", memory_format=torch.channels_last_3d)
    out = K.conv3d_i8(qx, sx, qw.cuda(), ws.cuda(), b.half().cuda(), (3, 3, 3), causal_zero_frames=2, acc_out=acc)
    ref_acc = O.conv3d_int_acc(qx_ref, qw.numpy(), (3, 3, 3))
    assert np.array_equal(acc.cpu().numpy(), ref_acc)
    ref = O.conv_epilogue(ref_acc, sx_ref, ws.numpy(), b.half().numpy()).astype(np.float32)
    got = out.float().cpu().numpy()
    assert np.abs(got - ref).max() <= 1e-2
    fp32 = torch.nn.functional.conv3d(xh.float(), w, b).numpy()
    assert np.abs(got - fp32).max() < 0.2 and np.abs(got - fp32).mean() < 0.02


def F_pad(x):
    x = torch.nn.functional.pad(x, (1, 1, 1, 1, 0, 0), mode="reflect")
    return torch.nn.functional.pad(x, (0, 0, 0, 0, 2, 0))
