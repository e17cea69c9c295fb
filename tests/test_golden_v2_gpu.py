"""The CUDA kernels against the reference's own Triton kernels' output (tests/golden/golden_v2.npz,
written by tests/golden/make_golden_triton.py from the reference's kernels run under Triton's
interpreter).  Same bars as against the oracle: integer codes of the exact paths (residual pack,
per-tensor quantization, conv int32 sums, row quantization of given activations, finalize) are
bit-exact; fp16 outputs are within max-abs 1e-2 / rel 1e-3; INT8 codes that follow the kernels'
SFU SiLU / exp are within +-1 on at most 0.1 % of the elements."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import h3vae_oracle as O

pytestmark = pytest.mark.gpu
CL3 = torch.channels_last_3d


@pytest.fixture(scope="module")
def g2():
    return dict(np.load(Path(__file__).resolve().parent / "golden" / "golden_v2.npz"))


def _close(got, ref, atol=1e-2, rtol=1e-3):
    got, ref = np.asarray(got, np.float32), np.asarray(ref, np.float32)
    diff = np.abs(got - ref)
    assert np.all(diff <= atol + rtol * np.abs(ref)), (diff.max(), np.unravel_index(diff.argmax(), diff.shape))


def _q_close(got, ref, frac=1e-3):
    d = np.abs(np.asarray(got, np.int32) - np.asarray(ref, np.int32))
    assert d.max() <= 1 and np.count_nonzero(d) <= max(2, frac * d.size), (d.max(), np.count_nonzero(d))


def _cu(a, cl3=False):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t.contiguous(memory_format=CL3) if cl3 else t


@pytest.mark.parametrize("k", [0, 1])
def test_norm_producer(cuda_lib, g2, k):
    from h3vae_b200 import kernels as K
    pre = _cu(g2[f"np{k}_pre"]) if f"np{k}_pre" in g2 else None
    x, w, b = _cu(g2[f"np{k}_x"], cl3=True), _cu(g2[f"np{k}_w"]), _cu(g2[f"np{k}_b"])
    q, s = K.norm_pad_quant(x, w, b, 1e-6, pre)
    ref_s = float(g2[f"np{k}_scale"][0])
    assert abs(float(s) - ref_s) <= 1e-3 * ref_s
    _q_close(q.cpu().numpy(), g2[f"np{k}_q"])
    _close(K.norm_pad_f16(x, w, b, 1e-6, pre).cpu().numpy(), g2[f"np{k}_y16"])


def test_residual_pack(cuda_lib, g2):
    from h3vae_b200 import kernels as K
    y = K.residual_pack(_cu(g2["rp_x"], True), _cu(g2["rp_r"], True), _cu(g2["rp_b"]))
    assert np.array_equal(y.cpu().numpy(), g2["rp_y"])


def test_activation_quant(cuda_lib, g2):
    from h3vae_b200 import kernels as K
    q, s = K.quantize_tensor_i8(_cu(g2["aq_x"], True))
    assert np.array_equal(q.cpu().numpy(), g2["aq_q"]) and float(s) == float(g2["aq_scale"][0])


@pytest.mark.parametrize("case", ["bias", "nobias", "strided"])
def test_conv(cuda_lib, g2, case):
    from h3vae_b200 import kernels as K
    pre = "cv2" if case == "strided" else "cv"
    kernel, stride, causal = ((1, 3, 3), (2, 1, 2), 0) if case == "strided" else ((3, 3, 3), (1, 1, 1), 2)
    qx, qw = g2[f"{pre}_qx"], g2[f"{pre}_qw"]
    bias = None if case == "nobias" else g2[f"{pre}_b"]
    ref = g2["cv_y_nobias" if case == "nobias" else ("cv2_y" if case == "strided" else "cv_y_bias")]
    acc = torch.empty((1, qw.shape[0], *ref.shape[2:]), dtype=torch.int32, device="cuda", memory_format=CL3)
    out = K.conv3d_i8(_cu(qx, True), torch.tensor(float(g2["cv_xs"][0]), device="cuda"), _cu(qw), _cu(g2[f"{pre}_ws"]),
                      None if bias is None else _cu(bias), kernel, stride, causal_zero_frames=causal, acc_out=acc)
    assert np.array_equal(acc.cpu().numpy(), O.conv3d_int_acc(qx, qw, kernel, stride))
    got = out.cpu().numpy()
    if case == "nobias":
        assert np.array_equal(got, ref)          # fp16((acc * sx) * sw): the reference's own order
    _close(got, ref)


def test_qk_rope(cuda_lib, g2):
    from h3vae_b200 import kernels as K
    q, k = K.qk_rope(_cu(g2["qk_x"]), _cu(g2["qk_cos"]), _cu(g2["qk_sin"]), 4, 1e-6)
    _close(q.cpu().numpy(), g2["qk_q"])
    _close(k.cpu().numpy(), g2["qk_k"])


def test_swiglu_quant(cuda_lib, g2):
    from h3vae_b200 import kernels as K
    q, s = K.swiglu_quant(_cu(g2["sw_x"]))
    _q_close(q.cpu().numpy(), g2["sw_q"])
    assert np.allclose(s.cpu().numpy(), g2["sw_s"], rtol=1e-3, atol=0)


@pytest.mark.parametrize("k", [0, 1])
@pytest.mark.parametrize("tag,round_stats", [("u", False), ("r", True)])
def test_residual_quant(cuda_lib, g2, k, tag, round_stats):
    from h3vae_b200 import kernels as K
    h, q, s = K.residual_rms_quant(_cu(g2[f"rq{k}_x"]), _cu(g2[f"rq{k}_a"]), _cu(g2[f"rq{k}_g"]), _cu(g2[f"rq{k}_w"]),
                                   1e-5, round_stats=round_stats)
    assert np.array_equal(h.cpu().numpy(), g2[f"rq{k}_{tag}_h"])
    _q_close(q.cpu().numpy(), g2[f"rq{k}_{tag}_q"])
    assert np.allclose(s.cpu().numpy(), g2[f"rq{k}_{tag}_s"], rtol=1e-5, atol=0)


def test_final_layernorm(cuda_lib, g2):
    from h3vae_b200 import kernels as K
    y = K.final_residual_layernorm(_cu(g2["ln_h"]), _cu(g2["ln_o"]), _cu(g2["ln_gate"]), _cu(g2["ln_gamma"]),
                                   _cu(g2["ln_beta"]), 1e-5)
    _close(y.cpu().numpy(), g2["ln_y"])


def test_ffn_up_swiglu_and_row_quant(cuda_lib, g2):
    from h3vae_b200 import kernels as K
    act = K.gemm_i8_swiglu(_cu(g2["fu_q"]), _cu(g2["fu_s"]), _cu(g2["fu_w"]), _cu(g2["fu_ws"]), _cu(g2["fu_b"]))
    _close(act.cpu().numpy(), g2["fu_act"])
    q, s = K.row_quant(_cu(g2["fu_act"]))                     # the reference's own activations
    assert np.array_equal(q.cpu().numpy(), g2["fu_qo"]) and np.array_equal(s.cpu().numpy(), g2["fu_so"])


def test_block0_rms(cuda_lib, g2):
    from h3vae_b200 import kernels as K
    y = K.rms_norm_f16(_cu(g2["b0_x"]), _cu(g2["b0_g"]), 9.999999747378752e-06)
    _close(y.cpu().numpy(), g2["b0_y"])


def test_finalize(cuda_lib, g2):
    from h3vae_b200 import kernels as K
    std, mean = _cu(g2["fp_std"]), _cu(g2["fp_mean"])
    y = K.finalize_pixels(_cu(g2["fp_x16"]), std, mean)
    assert np.array_equal(y.cpu().numpy(), g2["fp_y16"], equal_nan=True)
    base = torch.from_numpy(np.ascontiguousarray(g2["fp_x32"].transpose(0, 2, 3, 1, 4))).cuda()
    y = K.finalize_pixels(base.permute(0, 3, 1, 2, 4), std, mean)      # strided fp32 input
    assert np.array_equal(y.cpu().numpy(), g2["fp_y32"], equal_nan=True)
