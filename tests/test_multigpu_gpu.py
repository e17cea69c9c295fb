"""The tile-parallel runtime on several GPUs (one process per GPU; rank 0 sends each rank its pixel
window and gathers the ranks' canvas slabs over NCCL point to point) must give the single-GPU result:
the tile kernels are deterministic and only the order of the canvas sums differs.  Run with 2 GPUs (the
shards own whole temporal chunks) and with 4 (slabs of one chunk overlap and are summed); also through
pinned host buffers.  Skipped with fewer than two GPUs."""
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


@pytest.mark.parametrize("nproc", [2, 4])
def test_multi_gpu_round_trip_matches_one_gpu(cuda_lib, tmp_path, nproc):
    if not torch.cuda.is_available() or torch.cuda.device_count() < nproc:
        pytest.skip(f"needs {nproc} GPUs")
    out = tmp_path / "rank0.pt"
    env = {**os.environ, "NCCL_NVLS_ENABLE": "0"}
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", str(nproc), "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           str(ROOT / "tests" / "multigpu_worker.py"), str(out)]
    proc = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    got = torch.load(out)
    sys.path.insert(0, str(ROOT / "tests"))
    import multigpu_worker as W
    run = W.make_runtime(torch.device("cuda", 0), None)
    lat = run.encode(W.make_video(torch.device("cuda", 0)))
    pix = run.decode(lat.half())
    for key, ref, atol in (("lat", lat, 1e-4), ("lat_host", lat, 1e-4), ("pix", pix, 1e-5), ("pix_host", pix, 1e-5)):
        torch.testing.assert_close(got[key], ref.cpu(), rtol=0, atol=atol, msg=key)
