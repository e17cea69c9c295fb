"""Pin the oracle's restatements of the reference's Triton kernels to those kernels' own output.

tests/golden/golden_v2.npz was written by tests/golden/make_golden_triton.py, which runs the
reference's @triton.jit kernels (launched with their wrappers' grids and arguments) under Triton's
CPU interpreter.  Integer results (INT8 codes, int32 conv sums) and the fp32 finalize must match
exactly; fp16 values that come after a reduction the oracle takes in float64 (GroupNorm / RMS /
LayerNorm statistics) may differ by an fp16 ulp or two on a few elements.
"""
import numpy as np
import pytest

from oracle import h3vae_oracle as O


@pytest.fixture(scope="module")
def g2():
    from pathlib import Path
    return dict(np.load(Path(__file__).resolve().parent / "golden" / "golden_v2.npz"))


def _ulps16(a, b):
    a = np.asarray(a, np.float16).view(np.int16).astype(np.int32)
    b = np.asarray(b, np.float16).view(np.int16).astype(np.int32)
    return np.abs(a - b)


def _few_ulps(a, b, max_ulps=2, frac=1e-3):
    d = _ulps16(a, b)
    assert d.max() <= max_ulps and np.count_nonzero(d) <= max(2, frac * d.size), (d.max(), np.count_nonzero(d))


@pytest.mark.parametrize("k", [0, 1])
def test_norm_producer_matches_reference_kernels(g2, k):
    # opt/encoder_int8_norm.py:16-110 (statistics, recompute pack, absmax/scale), k=1 with pre_bias
    x, w, b, pre = g2[f"np{k}_x"], g2[f"np{k}_w"], g2[f"np{k}_b"], g2.get(f"np{k}_pre")
    q, s = O.norm_pad_quant(x, w, b, 1e-6, pre)
    assert np.array_equal(q, g2[f"np{k}_q"])
    assert s == g2[f"np{k}_scale"][0]
    mean, rstd, _ = O.gn_stats(x, 1e-6, pre)
    st = g2[f"np{k}_stats"]                                     # [D, 32, (mean, rstd)]
    assert np.abs(mean[0] - st[..., 0]).max() <= 1e-6
    assert np.abs(rstd[0] / st[..., 1] - 1).max() <= 1e-6
    _few_ulps(O.norm_pad_f16(x, w, b, 1e-6, pre), g2[f"np{k}_y16"])


def test_residual_pack_matches_reference_kernel(g2):
    # opt/encoder_fused_residual_pack.py:12-32
    assert np.array_equal(O.residual_pack(g2["rp_x"], g2["rp_r"], g2["rp_b"]), g2["rp_y"])


def test_activation_quant_matches_reference_kernels(g2):
    # opt/encoder_int8.py:343-378 (partial_absmax, merge_scale, quantize_contiguous)
    q, s = O.quantize_activation_tensor(g2["aq_x"])
    assert np.array_equal(q, g2["aq_q"]) and s == g2["aq_scale"][0]


def test_conv_matches_reference_kernels(g2):
    # pipelined kernel with the causal skip (opt/encoder_int8_pipeline.py:16-121): exact int32 sums,
    # the bias-free epilogue bit-exact; with bias the oracle contracts the add into an fma
    acc = O.conv3d_int_acc(g2["cv_qx"], g2["cv_qw"], (3, 3, 3))
    xs = g2["cv_xs"][0]
    assert np.array_equal(O.conv_epilogue(acc, xs, g2["cv_ws"], None), g2["cv_y_nobias"])
    _few_ulps(O.conv_epilogue(acc, xs, g2["cv_ws"], g2["cv_b"]), g2["cv_y_bias"], max_ulps=1)
    # default 64x64x64 kernel, (1,3,3) kernel, stride (2,1,2) (opt/encoder_int8.py:157-269)
    acc2 = O.conv3d_int_acc(g2["cv2_qx"], g2["cv2_qw"], (1, 3, 3), (2, 1, 2))
    _few_ulps(O.conv_epilogue(acc2, xs, g2["cv2_ws"], g2["cv2_b"]), g2["cv2_y"], max_ulps=1)


def test_qk_rope_matches_reference_kernel(g2):
    # opt/decoder_fused_qk_rope.py:12-35
    q, k, _ = O.qk_rope(g2["qk_x"], g2["qk_cos"], g2["qk_sin"], 4, 1e-6)
    _few_ulps(q, g2["qk_q"], max_ulps=1)
    _few_ulps(k, g2["qk_k"], max_ulps=1)


def test_swiglu_quant_matches_reference_kernel(g2):
    # opt/int8_swiglu_fused.py:21-40, including the all-zero row (scale 1e-30 -> codes -128)
    q, s = O.quantize_swiglu(g2["sw_x"])
    assert np.array_equal(q, g2["sw_q"]) and np.array_equal(s, g2["sw_s"])
    assert (g2["sw_q"][3] == -128).all()


@pytest.mark.parametrize("k", [0, 1])
@pytest.mark.parametrize("tag,round_stats", [("u", False), ("r", True)])
def test_residual_quant_matches_reference_kernel(g2, k, tag, round_stats):
    # opt/int8_norm_quant.py:22-44
    h, q, s, _ = O.residual_rms_quant(g2[f"rq{k}_x"], g2[f"rq{k}_a"], g2[f"rq{k}_g"], g2[f"rq{k}_w"], 1e-5,
                                      round_stats=round_stats)
    assert np.array_equal(h, g2[f"rq{k}_{tag}_h"])
    assert np.array_equal(q, g2[f"rq{k}_{tag}_q"])
    assert np.abs(s / g2[f"rq{k}_{tag}_s"] - 1).max() <= 1e-6


def test_final_layernorm_matches_reference_kernel(g2):
    # opt/decoder_final_norm.py:34-56 (Welford in fp32; the oracle's float64 stats differ by rounding)
    y = O.final_residual_layernorm(g2["ln_h"], g2["ln_o"], g2["ln_gate"], g2["ln_gamma"], g2["ln_beta"], 1e-5)
    _few_ulps(y, g2["ln_y"], max_ulps=1)


def test_ffn_up_swiglu_matches_reference_kernels(g2):
    # opt/int8_ffn_up_fused.py:51-105: INT8 GEMM, fma epilogue, fp16 linear values, SwiGLU, row quant
    act = O.ffn_up_swiglu(g2["fu_q"], g2["fu_s"], g2["fu_w"], g2["fu_ws"], g2["fu_b"])
    _few_ulps(act, g2["fu_act"], max_ulps=1)
    q, s = O.row_quant_ck(g2["fu_act"].astype(np.float32))
    assert np.array_equal(q, g2["fu_qo"]) and np.array_equal(s, g2["fu_so"])


def test_block0_rms_matches_reference_kernel(g2):
    # opt/decoder_block0_norm.py:39-59
    y = O.rms_norm_f16(g2["b0_x"], g2["b0_g"], 9.999999747378752e-06)
    _few_ulps(y, g2["b0_y"], max_ulps=1)


def test_finalize_matches_reference_kernel(g2):
    # opt/fp16_finalize.py:23-41: NaN kept, infinities clamped, no FMA; strided fp32 input too
    for k in ("16", "32"):
        y = O.finalize_pixels(g2[f"fp_x{k}"], g2["fp_std"], g2["fp_mean"])
        assert np.array_equal(y, g2[f"fp_y{k}"], equal_nan=True)
