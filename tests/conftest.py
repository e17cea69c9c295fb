"""Shared pytest setup: the `gpu` marker, import paths, seeded helpers.

Tests marked `gpu` call the CUDA library through its C ABI and need a B200;
everything else runs on CPU (oracle vs golden vectors, host logic, gloo ranks,
library symbol exports).
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG_PARENT = ROOT / "comfyui-h3vae-pyopt_b200"
for p in (ROOT, PKG_PARENT):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

os.environ.setdefault("MINIMAX_H3_TORCH_SDPA_BACKEND", "auto")
os.environ.setdefault("MINIMAX_H3_VAE_DECODER_VIT_FP32_NORM", "1")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (calls the sm_100a kernels)")


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return dict(np.load(ROOT / "tests" / "golden" / "golden_v1.npz"))


@pytest.fixture(scope="session")
def cuda_lib():
    """Build (if stale) and load the CUDA library; used by GPU tests."""
    import torch
    from h3vae_b200 import build_lib, _lib
    build_lib.build()
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    lib = _lib.load()
    yield lib
    assert _lib.device_error(clear=True) == 0, "a kernel reported a device-side error"
