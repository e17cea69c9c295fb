"""The tile-parallel runtime on two GPUs (one process per GPU, NCCL broadcast of the request and
one reduce of the blend canvases) must give the single-GPU result: the tile kernels are
deterministic and only the order of the canvas sums differs.  Skipped with fewer than two GPUs."""
from __future__ import annotations

import os
import socket
import subprocess
import sys

import pytest
import torch

from conftest import ROOT

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_round_trip_matches_one_gpu(cuda_lib, tmp_path):
    out = tmp_path / "rank0.pt"
    env = {**os.environ, "NCCL_NVLS_ENABLE": "0"}
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           str(ROOT / "tests" / "multigpu_worker.py"), str(out)]
    proc = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    got = torch.load(out)
    sys.path.insert(0, str(ROOT / "tests"))
    import multigpu_worker as W
    run = W.make_runtime(torch.device("cuda", 0), None)
    lat = run.encode(W.make_video(torch.device("cuda", 0)))
    pix = run.decode(lat.half())
    torch.testing.assert_close(got["lat"], lat.cpu(), rtol=0, atol=1e-4)
    torch.testing.assert_close(got["pix"], pix.cpu(), rtol=0, atol=1e-5)
