"""Decoder GEMM family on the B200 vs the CPU oracle: INT8 (CK contract restated from
opt/int8_ffn_up_fused.py:76-90 and opt/decoder_fused_qk_rope.py:13-35) and the fp16 profile
(opt/fp16_swiglu_gemm.py:20-47).  int32 accumulators are
bit-exact; fp16 outputs within max-abs 1e-2 / rel 1e-3."""
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


def _rand_operands(rng, m, n, k):
    q = rng.integers(-127, 128, size=(m, k), dtype=np.int8)
    s = (rng.random((m, 1), dtype=np.float32) * 0.02 + 0.001).astype(np.float32)
    w = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
    ws = (rng.random(n, dtype=np.float32) * 0.001 + 0.0001).astype(np.float32)
    b = (rng.standard_normal(n) * 0.5).astype(np.float16)
    return q, s, w, ws, b


@pytest.mark.parametrize("m,n,k", [(1, 1024, 1024), (17, 3072, 1024), (129, 2048, 2048), (300, 136, 256),
                                   (4096, 1024, 1024), (4096, 1024, 4096), (7188, 2048, 2048)])
@pytest.mark.parametrize("with_bias", [False, True])
def test_gemm_i8(cuda_lib, m, n, k, with_bias):
    from h3vae_b200 import kernels as K
    rng = np.random.default_rng(m * 31 + n + k)
    q, s, w, ws, b = _rand_operands(rng, m, n, k)
    bias = b if with_bias else None
    acc = torch.empty((m, n), dtype=torch.int32, device="cuda")
    out = K.gemm_i8(torch.from_numpy(q).cuda(), torch.from_numpy(s).cuda(), torch.from_numpy(w).cuda(),
                    torch.from_numpy(ws).cuda(), None if bias is None else torch.from_numpy(bias).cuda(), acc_out=acc)
    ref_acc = O.linear_acc(q, w)
    assert np.array_equal(acc.cpu().numpy(), ref_acc)
    _close(out.cpu().numpy(), O.linear_epilogue(ref_acc, s, ws, bias))


@pytest.mark.parametrize("m,f,k", [(1, 4096, 1024), (17, 4096, 1024), (129, 8192, 2048), (4096, 4096, 1024),
                                   (200, 136, 256)])
@pytest.mark.parametrize("with_bias", [False, True])
def test_ffn_up_swiglu(cuda_lib, m, f, k, with_bias):
    from h3vae_b200 import kernels as K
    rng = np.random.default_rng(m + f + k)
    q, s, w, ws, b = _rand_operands(rng, m, 2 * f, k)
    bias = b if with_bias else None
    act = K.gemm_i8_swiglu(torch.from_numpy(q).cuda(), torch.from_numpy(s).cuda(), torch.from_numpy(w).cuda(),
                           torch.from_numpy(ws).cuda(), None if bias is None else torch.from_numpy(bias).cuda())
    _close(act.cpu().numpy(), O.ffn_up_swiglu(q, s, w, ws, bias))          # max-abs 1e-2, rel 1e-3


@pytest.mark.parametrize("batch,tokens,heads,k,r", [(4, 1024, 16, 1024, 48), (2, 300, 4, 256, 48),
                                                    (1, 129, 2, 512, 64), (1, 64, 1, 128, 0)])
def test_qkv_rope(cuda_lib, batch, tokens, heads, k, r):
    from h3vae_b200 import kernels as K
    rng = np.random.default_rng(batch * tokens + heads)
    m = batch * tokens
    q, s, w, ws, b = _rand_operands(rng, m, heads * 192, k)
    ang = rng.random((batch, tokens, 1, max(r, 2)), dtype=np.float32)[..., :r] * 6.28
    cos = np.cos(ang).astype(np.float16)
    sin = np.sin(ang).astype(np.float16)
    eps = 1e-6
    qo, ko, vo = K.gemm_i8_qkv_rope(torch.from_numpy(q).cuda(), torch.from_numpy(s).cuda(),
                                    torch.from_numpy(w).cuda(), torch.from_numpy(ws).cuda(),
                                    torch.from_numpy(b).cuda(), batch, tokens, heads,
                                    torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda(), eps)
    qkv = O.prequantized_linear(q, s, w, ws, b).reshape(batch, tokens, heads * 192)
    rq, rk, rv = O.qk_rope(qkv, cos, sin, heads, eps)
    # kernel layout is [b, H, n, 64]; oracle returns [b, n, H, 64]
    _close(qo.permute(0, 2, 1, 3).cpu().numpy(), rq, atol=1e-2)
    _close(ko.permute(0, 2, 1, 3).cpu().numpy(), rk, atol=1e-2)
    _close(vo.permute(0, 2, 1, 3).cpu().numpy(), rv, atol=1e-2)


def _f16_operands(rng, m, n, k):
    a = rng.standard_normal((m, k)).astype(np.float16)
    w = (rng.standard_normal((n, k)) / np.sqrt(k)).astype(np.float16)
    b = (rng.standard_normal(n) * 0.5).astype(np.float16)
    return a, w, b


@pytest.mark.parametrize("m,n,k", [(1, 1024, 1024), (17, 3072, 1024), (129, 2048, 2048), (300, 136, 256),
                                   (4096, 1024, 4096), (200, 1000, 1000), (2048, 3072, 1024)])
@pytest.mark.parametrize("with_bias", [False, True])
def test_gemm_f16(cuda_lib, m, n, k, with_bias):
    """fp16 decoder-profile linear: fp16 outputs within max-abs 1e-2 / rel 1e-3 of the oracle (the
    fp32 accumulation order differs); K and N ragged against the 64-element k-blocks and tiles."""
    from h3vae_b200 import kernels as K
    rng = np.random.default_rng(m * 7 + n + k)
    a, w, b = _f16_operands(rng, m, n, k)
    bias = b if with_bias else None
    out = K.gemm_f16(torch.from_numpy(a).cuda(), torch.from_numpy(w).cuda(),
                     None if bias is None else torch.from_numpy(bias).cuda())
    _close(out.cpu().numpy(), O.linear_f16(a, w, bias))


@pytest.mark.parametrize("m,f,k", [(1, 4096, 1024), (129, 8192, 2048), (4096, 4096, 1024), (200, 136, 256),
                                   (33, 200, 1000)])
@pytest.mark.parametrize("with_bias", [False, True])
def test_ffn_up_swiglu_f16(cuda_lib, m, f, k, with_bias):
    from h3vae_b200 import kernels as K
    rng = np.random.default_rng(m + f * 3 + k)
    a, w, b = _f16_operands(rng, m, 2 * f, k)
    bias = b if with_bias else None
    act = K.gemm_f16_swiglu(torch.from_numpy(a).cuda(), torch.from_numpy(w).cuda(),
                            None if bias is None else torch.from_numpy(bias).cuda())
    # fp32 accumulation order differs from the oracle's float64 dot product, so a gate or up value can
    # round to the neighbouring fp16 value; through silu(g) * u that moves act by up to ~2.3 fp16 ulps
    # (2.3 * 2^-10 relative), hence rel 3e-3 here; the INT8 path above has exact sums and meets 1e-3
    _close(act.cpu().numpy(), O.ffn_up_swiglu_f16(a, w, bias), atol=1e-2, rtol=3e-3)


def test_gemm_f16_rejects_bad_arguments(cuda_lib):
    from h3vae_b200 import kernels as K
    a = torch.zeros(4, 36, dtype=torch.float16, device="cuda")
    with pytest.raises(ValueError):   # K not a multiple of 8
        K.gemm_f16(a, torch.zeros(8, 36, dtype=torch.float16, device="cuda"))
    with pytest.raises(ValueError):   # odd number of gate/up rows
        K.gemm_f16_swiglu(torch.zeros(4, 64, dtype=torch.float16, device="cuda"),
                          torch.zeros(7, 64, dtype=torch.float16, device="cuda"))
    with pytest.raises(ValueError):   # int8 operand
        K.gemm_f16(torch.zeros(4, 64, dtype=torch.int8, device="cuda"),
                   torch.zeros(8, 64, dtype=torch.float16, device="cuda"))


@pytest.mark.parametrize("m,n,k", [(4096, 1024, 1024), (300, 1024, 1024), (129, 2048, 2048), (200, 256, 256),
                                   (77, 200, 512)])
@pytest.mark.parametrize("round_stats", [False, True])
def test_gemm_i8_residual_then_rms_quant(cuda_lib, m, n, k, round_stats):
    """Attention-out GEMM with the residual in its epilogue (h = fp16(fma(fp16(linear), g, x)) and the
    row's partial sums of squares), then norm2 + row quantization from those sums, against the oracle's
    prequantized_linear followed by residual_rms_quant (ref opt/int8_norm_quant.py:23-44)."""
    from h3vae_b200 import kernels as K
    rng = np.random.default_rng(m * 7 + n + k)
    q, s, w, ws, b = _rand_operands(rng, m, n, k)
    x = rng.standard_normal((m, n)).astype(np.float16)
    g = (0.5 + 0.1 * rng.standard_normal(n)).astype(np.float16)
    nw = (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float16)
    cu = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    h, sums = K.gemm_i8_residual(cu(q), cu(s), cu(w), cu(ws), cu(b), cu(x), cu(g), round_stats=round_stats)
    qq, ss, act = K.rms_quant_parts(h, sums, cu(nw), 1e-5, return_norm=True)
    a = O.prequantized_linear(q, s, w, ws, b)
    ref_h, ref_q, ref_s, ref_act = O.residual_rms_quant(x, a, g, nw, 1e-5, round_stats=round_stats)
    got_h = h.cpu().numpy()
    _close(got_h, ref_h)
    assert np.count_nonzero(got_h != ref_h) <= max(2, 1e-3 * got_h.size)
    _close(act.cpu().numpy(), ref_act)
    dq = np.abs(qq.cpu().numpy().astype(np.int32) - ref_q.astype(np.int32))
    assert dq.max() <= 1 and np.count_nonzero(dq) <= max(2, 1e-3 * dq.size)
    # the row scale follows the row's largest |act|, which can sit one fp16 ulp away when the partial sums
    # (added in another order than the oracle's) move inv by a last-bit rounding
    assert np.allclose(ss.cpu().numpy(), ref_s, rtol=1e-3, atol=0)
    # in place: h written over x
    xin = cu(x)
    h2, _ = K.gemm_i8_residual(cu(q), cu(s), cu(w), cu(ws), cu(b), xin, cu(g), round_stats=round_stats, h_out=xin)
    assert h2 is xin and torch.equal(h2, h)
