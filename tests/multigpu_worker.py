"""torchrun worker for tests/test_multigpu_gpu.py: every rank builds the same seeded runtime, runs
one encode + decode of a seeded video with the tile work split over the ranks (device-resident, then
through pinned host buffers on rank 0), and rank 0 saves the latents and pixels.  Not collected by
pytest (no test_ prefix)."""
from __future__ import annotations

import datetime
import os
import sys
from pathlib import Path

import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "comfyui-h3vae-pyopt_b200"))

from h3vae_b200.runtime import H3VAEPyOptRuntime  # noqa: E402


def make_runtime(device, pg):
    return H3VAEPyOptRuntime(device=str(device), int8_encode=True, int8_decode=True, decode_fusions=True,
                             tile_batch=2, encoder_staged_batch=2, log_calls=False, compile_decoder=False,
                             compile_encoder=False, decoder_tile_size=256, encoder_tile_size=256,
                             process_group=pg)


def make_video(device):
    g = torch.Generator(device="cpu").manual_seed(5)
    return (torch.rand((1, 3, 34, 384, 448), generator=g) * 2 - 1).half().to(device)


def main():
    out = sys.argv[1]
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    try:
        run = make_runtime(dev, dist.group.WORLD)
        video = make_video(dev) if dist.get_rank() == 0 else None
        lat = run.encode(video)
        pix = run.decode(None if lat is None else lat.half())
        # the host-buffer path: a pinned host video in, pixels into a pinned host buffer
        host_video = video.cpu().pin_memory() if dist.get_rank() == 0 else None
        lat_h = run.encode(host_video)
        buf = None
        if dist.get_rank() == 0:
            buf = torch.empty(run.decode_output_shape(lat_h.shape), dtype=torch.float32).pin_memory()
        res = run.decode(None if lat_h is None else lat_h.half(), output_buffer=buf)
        if dist.get_rank() == 0:
            assert res is buf
            torch.save({"lat": lat.cpu(), "pix": pix.cpu(), "lat_host": lat_h.cpu(), "pix_host": buf.clone()}, out)
        torch.cuda.synchronize()
        dist.barrier()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
