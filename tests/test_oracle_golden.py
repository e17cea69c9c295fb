"""Pin the CPU oracle to vectors produced by the reference's own CPU functions
(tests/golden/make_golden.py) and to the known-answer vectors of its tests."""
import json

import numpy as np
import torch

from oracle import h3vae_oracle as O


def test_weight_pack_matches_reference(golden):
    for k in ("wpack1", "wpack2"):
        q, s = O.prepare_int8_weight(torch.from_numpy(golden[f"{k}_w"]))
        assert np.array_equal(q.numpy(), golden[f"{k}_q"])
        assert np.array_equal(s.numpy(), golden[f"{k}_s"])
    # the all-zero output channel keeps scale 1 and q 0
    assert golden["wpack1_s"][3] == 1.0 and not golden["wpack1_q"][3].any()


def test_dequant_conv_matches_reference_cpu_oracle(golden):
    for k, stride in (("conv1", (1, 1, 1)), ("conv2", (2, 1, 2)), ("conv3", (1, 1, 1))):
        got = O.int8_valid_conv3d_dequant_fp32(golden[f"{k}_x"], torch.from_numpy(golden[f"{k}_w"]),
                                               golden[f"{k}_b"], stride)
        assert got.shape == golden[f"{k}_y"].shape
        assert np.array_equal(got, golden[f"{k}_y"]), np.abs(got - golden[f"{k}_y"]).max()


def test_integer_conv_equals_dequant_conv(golden):
    # exact int32 accumulation, dequantized in fp64, agrees with the reference's fp32 conv
    for k, stride in (("conv1", (1, 1, 1)), ("conv2", (2, 1, 2))):
        x, w, b = golden[f"{k}_x"], torch.from_numpy(golden[f"{k}_w"]), golden[f"{k}_b"]
        qw, ws = O.prepare_int8_weight(w)
        qx, sx = O.quantize_activation_tensor(x, true_division=True)
        acc = O.conv3d_int_acc(qx, qw.numpy(), tuple(w.shape[-3:]), stride)
        y = acc.astype(np.float64) * float(sx) * ws.numpy().astype(np.float64).reshape(1, -1, 1, 1, 1)
        y += b.astype(np.float64).reshape(1, -1, 1, 1, 1)
        ref = golden[f"{k}_y"]
        assert np.abs(y - ref).max() <= 1e-4 * max(1.0, np.abs(ref).max())


def test_accumulator_bounds(golden):
    got = [O.int32_accumulator_bound(c, k) for c, k in ((128, (3, 3, 3)), (256, (3, 3, 3)), (512, (3, 3, 3)),
                                                        (7, (1, 3, 3)))]
    assert got == golden["acc_bounds"].tolist()


def test_split_tiles_match_reference(golden):
    cases = json.loads(bytes(golden["split_tiles_json"]).decode())
    for c in cases:
        starts, sizes, overlaps = O.split_tiles(*c["case"])
        assert (starts, sizes, overlaps) == (c["starts"], c["sizes"], c["overlaps"]), c["case"]


def test_ck_rowwise_weight_quant_matches_reference(golden):
    q, s = O.quantize_rowwise_weight(torch.from_numpy(golden["ckw_w"]))
    assert np.array_equal(q.numpy(), golden["ckw_q"])
    assert np.array_equal(s.numpy(), golden["ckw_s"])
    assert golden["ckw_s"][2] == 1.0 and not golden["ckw_q"][2].any()


def test_half_away_known_answer():
    # ref: tests/test_encoder_int8_gpu.py:65-72
    x = np.array([-127.0, -0.5, -1.5, 0.0, 0.5, 1.5, 127.0], dtype=np.float16).reshape(1, 1, 1, 1, 7)
    q, s = O.quantize_activation_tensor(x)
    assert s == 1.0
    assert q.ravel().tolist() == [-127, -1, -2, 0, 1, 2, 127]


def test_scale_edge_cases():
    # ref: tests/test_encoder_int8_gpu.py:57-64 -- zero, subnormal, extremes
    for m in (0.0, 2**-24, 2**-14, 0.5, 127.0, 65504.0):
        x = np.full((1, 1, 1, 1, 9), m, dtype=np.float16)
        x[..., 0] = -m
        q, s = O.quantize_activation_tensor(x)
        expect = np.float32(m) * O.RECIP_127 if m > 0 else np.float32(1.0)
        assert s == expect
        assert np.all(np.abs(q) <= 127)
        if m > 0:
            assert q.ravel()[0] == -127 and q.ravel()[1] == 127


def test_row_quant_ck_rules():
    act = np.array([[0.0, 0.0, 0.0, 0.0], [1.0, -2.0, 0.5, 127.0], [np.nan, 1.0, 0.0, -1.0]], np.float32)
    q, s = O.row_quant_ck(act)
    # an all-zero row: scale 1e-30 rounds to fp16 zero, 0/0 is NaN -> -128 (the CK behaviour the
    # reference documents at opt/kitchen_int8.py:131-134)
    assert s[0, 0] == np.float32(1e-30)
    assert q[0].tolist() == [-128, -128, -128, -128]
    assert q[1].tolist() == [1, -2, 0, 127]          # 0.5 rounds half-to-even
    assert s[2, 0] == np.float32(1.0) * O.RECIP_127  # NaN ignored by the row max
    assert q[2].tolist() == [-128, 127, 0, -127]     # NaN -> -128
