"""The reference-facing op layer (h3vae_b200.opt, mirroring the reference's opt/* modules and
torch.library ops) on the B200 vs the CPU oracle.  Each op is called through torch.ops so the
registration is exercised too.  int8 outputs within one step on at most 0.1% of elements (the
producer's reciprocal-vs-division rounding near ties), fp16 outputs within max-abs 1e-2 / rel 1e-3."""
import numpy as np
import pytest
import torch

from oracle import h3vae_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _inference():
    # the reference's ops are inference-only (they raise under autograd)
    with torch.no_grad():
        yield


def _close(got, ref, atol=1e-2, rtol=1e-3):
    got = np.asarray(got, np.float32)
    ref = np.asarray(ref, np.float32)
    diff = np.abs(got - ref)
    assert np.all(diff <= atol + rtol * np.abs(ref)), (diff.max(), np.unravel_index(diff.argmax(), diff.shape))


def _gen(seed):
    return torch.Generator().manual_seed(seed)


def test_int8_valid_conv3d_and_module(cuda_lib):
    from h3vae_b200.opt import encoder_int8 as E
    from h3vae_b200.opt import encoder_int8_integration  # noqa: F401 - registers the ops
    g = _gen(1)
    conv = torch.nn.Conv3d(128, 128, 3, bias=True).half()
    x = torch.randn(1, 128, 4, 10, 12, generator=g).half()
    q, s, cfg = E.prepare_int8_weight(conv.weight)
    q_ref, s_ref = O.prepare_int8_weight(conv.weight.detach())
    assert torch.equal(q, q_ref) and torch.equal(s, s_ref)
    mod = E.Int8Conv3d(conv).cuda()
    y = mod(x.cuda())
    ref = O.int8_valid_conv3d(x.numpy(), q_ref.numpy(), s_ref.numpy(), (3, 3, 3), (1, 1, 1),
                              conv.bias.detach().numpy())
    _close(y.cpu().numpy(), ref)
    y2 = torch.ops.h3vae_b200_encoder.int8_valid_conv3d_integration(
        x.cuda(), q.cuda(), s.cuda(), conv.bias.detach().cuda(), 3, 3, 3, 1, 1, 1, True, "tcgen05")
    _close(y2.cpu().numpy(), ref)
    with pytest.raises(ValueError, match="tile variant"):
        E.int8_valid_conv3d(x.cuda(), q.cuda(), s.cuda(), config=cfg, tile_variant="bogus")


def test_int8_norm_conv3d_op(cuda_lib):
    from h3vae_b200.opt import encoder_int8 as E
    from h3vae_b200.opt import encoder_int8_integration  # noqa: F401 - registers the ops
    g = _gen(2)
    c = 128
    x = torch.randn(1, c, 3, 9, 11, generator=g).half()
    gw, gb, pre = (torch.randn(c, generator=g).half() for _ in range(3))
    w = torch.randn(c, c, 3, 3, 3, generator=g) / 60
    bias = torch.randn(c, generator=g).half()
    qw, ws, _ = E.prepare_int8_weight(w)
    y = torch.ops.h3vae_b200_encoder.int8_norm_conv3d(x.cuda(), gw.cuda(), gb.cuda(), pre.cuda(), 1e-6,
                                                       qw.cuda(), ws.cuda(), bias.cuda())
    q_ref, s_ref = O.norm_pad_quant(x.numpy(), gw.numpy(), gb.numpy(), 1e-6, pre.numpy())
    acc = O.conv3d_int_acc(q_ref, qw.numpy(), (3, 3, 3))
    ref = O.conv_epilogue(acc, s_ref, ws.numpy(), bias.numpy())
    _close(y.cpu().numpy(), ref, atol=2e-2)


def test_encoder_norm_pack_ops(cuda_lib):
    from h3vae_b200.opt import encoder_fused_norm  # noqa: F401 - registers the ops
    g = _gen(3)
    c = 256
    x = torch.randn(2, c, 3, 6, 8, generator=g).half()
    gw, gb, pre = (torch.randn(c, generator=g).half() for _ in range(3))
    y = torch.ops.h3vae_b200_encoder.temporal_norm_pack(x.cuda(), gw.cuda(), gb.cuda(), 1e-6)
    _close(y.cpu().numpy(), O.norm_pad_f16(x.numpy(), gw.numpy(), gb.numpy(), 1e-6))
    y = torch.ops.h3vae_b200_encoder.bias_temporal_norm_pack(x.cuda(), pre.cuda(), gw.cuda(), gb.cuda(), 1e-6)
    _close(y.cpu().numpy(), O.norm_pad_f16(x.numpy(), gw.numpy(), gb.numpy(), 1e-6, pre.numpy()))
    r = torch.randn(2, c, 3, 6, 8, generator=g).half()
    y = torch.ops.h3vae_b200_encoder.residual_downsample_pack(x.cuda(), r.cuda(), pre.cuda())
    _close(y.cpu().numpy(), O.residual_pack(x.numpy(), r.numpy(), pre.numpy()))


def test_decoder_linear_ops(cuda_lib):
    from h3vae_b200.opt import int8_swiglu_fused  # noqa: F401 - registers the ops
    from h3vae_b200.opt.kitchen_int8 import KitchenInt8Linear
    g = _gen(4)
    lin = torch.nn.Linear(256, 192).half()
    x = torch.randn(3, 40, 256, generator=g).half()
    mod = KitchenInt8Linear(lin).cuda().eval()
    with torch.no_grad():
        y = mod(x.cuda())
    ref = O.int8_linear(x.reshape(-1, 256).numpy(), mod.qweight.cpu().numpy(), mod.weight_scale.cpu().numpy(),
                        lin.bias.detach().cpu().numpy())
    _close(y.reshape(-1, 192).cpu().numpy(), ref)
    # SwiGLU + INT8 down projection
    xs = torch.randn(50, 512, generator=g).half()
    qd, sd = O.quantize_rowwise_weight(torch.randn(128, 256, generator=g))
    y = torch.ops.h3vae_b200_exp.swiglu_int8_linear(xs.cuda(), qd.cuda(), sd.cuda(), None, 8)
    qa, sa = O.quantize_swiglu(xs.numpy())
    _close(y.cpu().numpy(), O.prequantized_linear(qa, sa, qd.numpy(), sd.numpy()))


def test_residual_norm_ops(cuda_lib):
    from h3vae_b200.opt import int8_ffn_up_fused, int8_norm1_quant, int8_norm_quant  # noqa: F401
    g = _gen(5)
    m, k, f = 96, 256, 384
    x, a = (torch.randn(m, k, generator=g).half() for _ in range(2))
    gate, w = (torch.randn(k, generator=g).half() for _ in range(2))
    qw, ws = O.quantize_rowwise_weight(torch.randn(3 * 64, k, generator=g))
    h, out = torch.ops.h3vae_b200_norm_exp.residual_rms_linear(x.cuda(), a.cuda(), gate.cuda(), w.cuda(), qw.cuda(),
                                                               ws.cuda(), None, 1e-5, 8)
    h_ref, q_ref, s_ref, _ = O.residual_rms_quant(x.numpy(), a.numpy(), gate.numpy(), w.numpy(), 1e-5)
    assert np.array_equal(h.cpu().numpy(), h_ref)
    _close(out.cpu().numpy(), O.prequantized_linear(q_ref, s_ref, qw.numpy(), ws.numpy()), atol=2e-2)
    # residual FFN: up [2F, K] with SwiGLU, down [K, F]
    qu, su = O.quantize_rowwise_weight(torch.randn(2 * f, k, generator=g) / 8)
    qdn, sdn = O.quantize_rowwise_weight(torch.randn(k, f, generator=g) / 8)
    h2, y = torch.ops.h3vae_b200_int8_ffn.residual_ffn(x.cuda(), a.cuda(), gate.cuda(), w.cuda(), qu.cuda(),
                                                       su.cuda(), None, qdn.cuda(), sdn.cuda(), None, 1e-5, 8)
    assert np.array_equal(h2.cpu().numpy(), h_ref)
    act = O.ffn_up_swiglu(q_ref, s_ref, qu.numpy(), su.numpy())
    qa, sa = O.row_quant_ck(act)
    _close(y.cpu().numpy(), O.prequantized_linear(qa, sa, qdn.numpy(), sdn.numpy()), atol=5e-2)
    # norm1: h updated in place
    hh = x.cuda().clone()
    qkv = torch.ops.h3vae_b200_norm1.residual_qkv(hh, a.cuda(), gate.cuda(), w.cuda(), qw.cuda(), ws.cuda(), None)
    assert np.array_equal(hh.cpu().numpy(), h_ref)
    _close(qkv.cpu().numpy(), O.prequantized_linear(q_ref, s_ref, qw.numpy(), ws.numpy()), atol=2e-2)


def test_qk_rope_and_norm_ops(cuda_lib):
    from h3vae_b200.opt import decoder_fused_qk_rope, decoder_norms  # noqa: F401
    g = _gen(6)
    b, n, heads, r = 2, 70, 3, 48
    qkv = torch.randn(b, n, heads * 192, generator=g).half()
    ang = torch.rand(b, n, 1, r, generator=g) * 6.28
    cos, sin = ang.cos().half(), ang.sin().half()
    q, k = torch.ops.h3vae_b200_decoder.qk_rope(qkv.cuda(), cos.cuda(), sin.cuda(), heads, 1e-6, 8)
    rq, rk, _ = O.qk_rope(qkv.numpy(), cos.numpy(), sin.numpy(), heads, 1e-6)
    _close(q.cpu().numpy(), rq)
    _close(k.cpu().numpy(), rk)
    x = torch.randn(77, 1024, generator=g).half()
    gamma, beta, gate = (torch.randn(1024, generator=g).half() for _ in range(3))
    y = torch.ops.h3vae_b200_norm1_block0.rms_fp16_x2_w16(x.cuda(), gamma.cuda())
    _close(y.cpu().numpy(), O.rms_norm_f16(x.numpy(), gamma.numpy(), decoder_norms.EPS))
    o = torch.randn(77, 1024, generator=g).half()
    y = torch.ops.h3vae_b200_final_ln.residual_ln_w8(x.cuda(), o.cuda(), gate.cuda(), gamma.cuda(), beta.cuda())
    _close(y.cpu().numpy(), O.final_residual_layernorm(x.numpy(), o.numpy(), gate.numpy(), gamma.numpy(),
                                                       beta.numpy(), decoder_norms.EPS))


def test_finalize_pixels_mirror(cuda_lib):
    from h3vae_b200.opt.fp16_finalize import finalize_pixels
    g = _gen(7)
    x = torch.randn(1, 3, 5, 16, 24, generator=g).half()
    x[0, 0, 0, 0, 0] = float("nan")
    std = torch.tensor([0.229, 0.224, 0.225])
    mean = torch.tensor([0.485, 0.456, 0.406])
    with torch.no_grad():
        y = finalize_pixels(x.cuda(), std.cuda(), mean.cuda())
    ref = O.finalize_pixels(x.numpy(), std.numpy(), mean.numpy())
    np.testing.assert_array_equal(y.cpu().numpy(), ref)


def test_fp16_swiglu_gemm_mirror(cuda_lib):
    """torch.ops.h3vae_b200_fp16_exp.w1_swiglu (ref: opt/fp16_swiglu_gemm.py:83-86) on a 3-D
    activation with a ragged F, and the FusedFP16FFN module swap (fused w1 + SwiGLU, the model's own
    w2) against the oracle composition."""
    from h3vae_b200.opt import fp16_swiglu_gemm as M
    g = _gen(12)
    x = torch.randn(3, 40, 256, generator=g).half()
    w = (torch.randn(2 * 192, 256, generator=g) / 16).half()
    b = (torch.randn(2 * 192, generator=g) * 0.5).half()
    y = torch.ops.h3vae_b200_fp16_exp.w1_swiglu(x.cuda(), w.cuda(), b.cuda(), 64, 64, 64, 4, 3)
    assert tuple(y.shape) == (3, 40, 192)
    ref = O.ffn_up_swiglu_f16(x.reshape(-1, 256).numpy(), w.numpy(), b.numpy())
    _close(y.reshape(-1, 192).cpu().numpy(), ref, atol=2e-2)
    ff = torch.nn.Module()
    ff.use_gated, ff.act_fn = True, torch.nn.SiLU()
    ff.w1 = torch.nn.Linear(256, 384).half()
    ff.w2 = torch.nn.Linear(192, 256).half()
    fused = M.FusedFP16FFN(ff.eval(), (64, 64, 64, 4, 3)).cuda()
    out = fused(x.cuda()).float().cpu()
    act = O.ffn_up_swiglu_f16(x.reshape(-1, 256).numpy(), ff.w1.weight.detach().cpu().numpy(),
                              ff.w1.bias.detach().cpu().numpy())
    ref2 = torch.from_numpy(O.linear_f16(act, ff.w2.weight.detach().cpu().numpy(),
                                         ff.w2.bias.detach().cpu().numpy()).astype(np.float32)).reshape(3, 40, 256)
    assert ((out - ref2).norm() / ref2.norm()).item() < 1e-2
