"""Generate tests/golden/golden_v1.npz from the reference's own CPU functions.

Run once in a container where the reference checkout (fishelegs/ComfyUI-H3VAE-PyOpt 0.2.0) is
available; the checkout path is a required argument:  python tests/golden/make_golden.py <checkout>
The GPU box never runs this script; the tests read only the committed .npz.

Vectors produced (all seeded):
  * prepare_int8_weight: packed int8 weights + fp32 scales (opt/encoder_int8.py:303-327), including
    an all-zero output channel and the non-cubic (3,1,3) kernel of the reference's own CPU test.
  * int8_valid_conv3d_cpu_reference: fp32 outputs for a 3x3x3 stride-1 case with bias, the
    reference test's rectangular stride (2,1,2) case, and a zero-weight case (opt/encoder_int8.py:591-619).
  * int32_accumulator_bound values (opt/encoder_int8.py:54-58).
  * H3VAEPyOptRuntime._split_encoder_tiles for the reference test lengths plus extra lengths
    (h3vae_runtime.py:584-603) and _select_encoder_tile (h3vae_runtime.py:605-607).
  * quantize_static_weight with the reference test's CK stand-in quantizer, including a zero row
    (opt/kitchen_int8.py:88-145, tests/test_kitchen_int8.py:19-26).
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import torch


def main(ref_root: str) -> None:
    ref = Path(ref_root)
    sys.path.insert(0, str(ref))
    sys.path.insert(0, str(ref / "tests"))
    from opt.encoder_int8 import (Int8Conv3DConfig, int32_accumulator_bound, int8_valid_conv3d_cpu_reference,
                                  prepare_int8_weight)
    from h3vae_runtime import H3VAEPyOptRuntime
    import opt.kitchen_int8 as kitchen_int8
    from test_kitchen_int8 import _fake_quantize_rowwise

    out: dict[str, np.ndarray] = {}

    torch.manual_seed(20261201)
    w1 = torch.randn(6, 16, 3, 3, 3)
    w1[3].zero_()
    q1, s1, _ = prepare_int8_weight(w1)
    out["wpack1_w"], out["wpack1_q"], out["wpack1_s"] = w1.numpy(), q1.numpy(), s1.numpy()

    w2 = torch.randn(5, 3, 3, 1, 3) * 7.0
    q2, s2, _ = prepare_int8_weight(w2, stride=(2, 1, 2))
    out["wpack2_w"], out["wpack2_q"], out["wpack2_s"] = w2.numpy(), q2.numpy(), s2.numpy()

    x1 = torch.randn(1, 16, 5, 7, 9)
    cw1 = torch.randn(8, 16, 3, 3, 3) / (16 * 27) ** 0.5
    cb1 = torch.randn(8) * 0.02
    out["conv1_x"], out["conv1_w"], out["conv1_b"] = x1.numpy(), cw1.numpy(), cb1.numpy()
    out["conv1_y"] = int8_valid_conv3d_cpu_reference(x1, cw1, cb1).numpy()

    x2 = torch.randn(1, 3, 5, 8, 10)
    cw2 = torch.randn(4, 3, 3, 1, 3)
    cb2 = torch.randn(4)
    out["conv2_x"], out["conv2_w"], out["conv2_b"] = x2.numpy(), cw2.numpy(), cb2.numpy()
    out["conv2_y"] = int8_valid_conv3d_cpu_reference(x2, cw2, cb2, stride=(2, 1, 2)).numpy()

    x3 = torch.randn(1, 2, 3, 4, 5)
    cw3 = torch.zeros(3, 2, 1, 1, 1)
    cb3 = torch.tensor([1.0, -2.0, 0.5])
    out["conv3_x"], out["conv3_w"], out["conv3_b"] = x3.numpy(), cw3.numpy(), cb3.numpy()
    out["conv3_y"] = int8_valid_conv3d_cpu_reference(x3, cw3, cb3).numpy()

    bounds = []
    for c, k in ((128, (3, 3, 3)), (256, (3, 3, 3)), (512, (3, 3, 3)), (7, (1, 3, 3))):
        bounds.append(int32_accumulator_bound(Int8Conv3DConfig(c, c, k, (1, 1, 1))))
    out["acc_bounds"] = np.array(bounds, dtype=np.int64)

    split = H3VAEPyOptRuntime._split_encoder_tiles
    cases = [(672, 672, 64, 16), (768, 256, 64, 16), (1344, 256, 64, 16), (768, 256, 32, 16),
             (1344, 256, 32, 16), (1000, 256, 64, 16), (300, 256, 64, 16), (2048, 512, 64, 16)]
    split_json = []
    for case in cases:
        starts, sizes, overlaps = split(*case)
        split_json.append({"case": list(case), "starts": starts, "sizes": sizes, "overlaps": overlaps})
    out["split_tiles_json"] = np.frombuffer(json.dumps(split_json).encode(), dtype=np.uint8)
    sel = [(c, h, w, H3VAEPyOptRuntime._select_encoder_tile(c, h, w))
           for c, h, w in ((0, 672, 672), (0, 768, 1344), (672, 768, 1344), (0, 256, 256), (512, 100, 100))]
    out["select_tile"] = np.array(sel, dtype=np.int64)

    lin = torch.nn.Linear(32, 7)
    with torch.no_grad():
        lin.weight.copy_(torch.randn(7, 32) * 0.05)
        lin.weight[2].zero_()
    qk, sk = kitchen_int8.quantize_static_weight(lin, quantize_fn=_fake_quantize_rowwise)
    out["ckw_w"], out["ckw_q"], out["ckw_s"] = lin.weight.detach().numpy(), qk.numpy(), sk.numpy()

    dest = Path(__file__).resolve().parent / "golden_v1.npz"
    np.savez_compressed(dest, **out)
    print(f"wrote {dest} ({dest.stat().st_size} bytes, {len(out)} arrays)")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden.py <path-to-reference-checkout>")
    main(sys.argv[1])
