"""The N>1 runtime path on CPU: 2, 3 or 8 gloo ranks run the same encode/decode call, each takes
its contiguous block of (tile, clip) work items (at 8 ranks some ranks get none), rank 0 sends each
rank the pixel window its items read, and every rank sends rank 0 the canvas slab its items cover.

The encoder/decoder are replaced by small linear stand-ins (the sharding, blending, broadcast and
reduce logic is what is under test; the kernels have their own GPU tests).  The sharded result
must equal the single-process result.  A second test makes one rank fail before the first
collective and checks that the other rank's call ends with an error instead of waiting forever.
"""
from __future__ import annotations

import datetime
import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import multiprocessing as mp

from h3vae_b200 import runtime as rt
from h3vae_b200.model import DecoderConfig, EncoderConfig

TINY_ENC = EncoderConfig(channels=(32, 32, 32, 32), blocks_per_stage=1, int8_stages=())
TINY_DEC = DecoderConfig(hidden=64, heads=1, blocks=1, ffn=128, up_channels=(32, 32, 32))


class _FakeEncoder:
    """[n,3,17,h,w] -> moments [n, 2*16, 5, h/8, w/8]: 8x8 average pool, frames 0,4,..,16, a fixed
    3 -> 32 channel mix.  Linear, like the blend, so any split of the work gives the same sum."""

    def __init__(self):
        self.cfg = TINY_ENC
        self.int8_conv_count = 0
        self.mix = torch.randn(32, 3, generator=torch.Generator().manual_seed(3)).double()

    def __call__(self, x, norm=None):
        if norm is not None:
            mean, std = (v.float().view(1, -1, 1, 1, 1) for v in norm)
            x = (((x.float() + 1.0) * 0.5 - mean) / std).half()
        p = torch.nn.functional.avg_pool3d(x.double()[:, :, ::4], (1, 8, 8))
        return torch.einsum("oc,ncthw->nothw", self.mix, p).half()


class _FakeDecoder:
    spatial_ratio = 8

    def __init__(self):
        self.mix = torch.randn(3, 16, generator=torch.Generator().manual_seed(4)).double()

    def frames_for(self, tokens_t):
        return 1 + 4 * (tokens_t - 1)

    def __call__(self, lat):
        y = torch.einsum("oc,ncthw->nothw", self.mix, lat.double())
        y = y.repeat_interleave(4, dim=2)[:, :, 3:]
        return y.repeat_interleave(8, dim=3).repeat_interleave(8, dim=4).half()


def _make_runtime(pg):
    r = rt.H3VAEPyOptRuntime(device="cpu", decoder_tile_size=64, encoder_tile_size=64, tile_batch=1,
                             encoder_staged_batch=1, log_calls=False, compile_decoder=False,
                             compile_encoder=False, encoder_config=TINY_ENC, decoder_config=TINY_DEC,
                             process_group=pg)
    r.encoder, r.decoder = _FakeEncoder(), _FakeDecoder()
    return r


def _cpu_finalize(x, std, mean, out=None):
    y = torch.clamp(x.float() * std.view(1, 3, 1, 1, 1) + mean.view(1, 3, 1, 1, 1), 0.0, 1.0)
    if out is not None:
        out.copy_(y)
        return out
    return y


def _cpu_blend(canvas, tile, weight):
    canvas.add_(tile.float() * weight)


def _inputs():
    g = torch.Generator().manual_seed(11)
    video = (torch.rand((1, 3, 30, 96, 160), generator=g) * 2 - 1).half()
    lat = torch.randn((1, 16, 10, 12, 20), generator=g).half()
    return video, lat


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    rt.K.finalize_pixels = _cpu_finalize
    rt.K.blend_accumulate = _cpu_blend
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
        run = _make_runtime(dist.group.WORLD)
        video, lat = _inputs()
        if mode == "fail" and rank == 1:
            raise RuntimeError("planted failure on rank 1 before its first collective")
        enc = run.encode(video if rank == 0 else None)
        dec = run.decode(lat if rank == 0 else None)
        queue.put((rank, "ok", None if enc is None else (enc.numpy(), dec.numpy())))
    except Exception as exc:  # noqa: BLE001 - reported to the parent
        queue.put((rank, "error", f"{type(exc).__name__}: {exc}\n{traceback.format_exc(limit=2)}"))
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:  # noqa: BLE001
                pass


def _run(world, mode):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, status, payload = queue.get(timeout=120)
        results[rank] = (status, payload)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return results


@pytest.mark.parametrize("world", [2, 3, 8])
def test_multi_rank_encode_decode_equals_single_process(monkeypatch, world):
    """Rank 0 sends each rank only its pixel window and adds the ranks' canvas slabs; with 3 ranks
    the shard boundaries fall inside clip batches and temporal chunks, so slabs overlap and are
    summed."""
    # CPU stand-ins for this test only (the spawned ranks set their own)
    monkeypatch.setattr(rt.K, "finalize_pixels", _cpu_finalize)
    monkeypatch.setattr(rt.K, "blend_accumulate", _cpu_blend)
    single = _make_runtime(None)
    video, lat = _inputs()
    enc_ref = single.encode(video)
    dec_ref = single.decode(lat)
    results = _run(world, "ok")
    assert results[0][0] == "ok", results[0][1]
    for r in range(1, world):
        assert results[r] == ("ok", None)       # non-zero ranks return None
    enc, dec = (torch.from_numpy(a) for a in results[0][1])
    assert enc.shape == enc_ref.shape and dec.shape == dec_ref.shape
    torch.testing.assert_close(enc, enc_ref, rtol=0, atol=1e-5)
    torch.testing.assert_close(dec, dec_ref, rtol=0, atol=1e-6)


def test_rank_failure_surfaces_as_error_on_peer():
    results = _run(2, "fail")
    assert results[1][0] == "error" and "planted failure" in results[1][1]
    assert results[0][0] == "error", "rank 0 must not wait forever for a rank that died"


def test_temporal_contract_matches_reference(monkeypatch):
    """Frames 17k+5 <-> latents 5k+2 and one frame <-> one latent, through encode and decode
    (ref: h3vae_runtime.py:483-491, 572-582, 524-537; opt/encoder_staged_batch.py:39-57)."""
    monkeypatch.setattr(rt.K, "finalize_pixels", _cpu_finalize)
    monkeypatch.setattr(rt.K, "blend_accumulate", _cpu_blend)
    run = _make_runtime(None)
    g = torch.Generator().manual_seed(5)
    video = (torch.rand((1, 3, 124, 64, 64), generator=g) * 2 - 1).half()
    lat = run.encode(video)
    assert lat.shape == (1, 16, 37, 8, 8)
    out = run.decode(lat.half())
    assert out.shape == run.decode_output_shape(lat.shape) == (1, 3, 124, 64, 64)
    # the kept tokens are the first 37 of the 8 clips' 40 (the dropped 3 encode padding frames)
    clips = torch.cat([video[:, :, :119], video[:, :, -1:].expand(-1, -1, 17, -1, -1)], dim=2)
    full = run.encode(clips)
    assert full.shape[2] == 8 * 5 - 3
    for k in range(4):
        v = video[:, :, :17 * k + 5]
        z = run.encode(v)
        assert z.shape[2] == 5 * k + 2 == run._tokens_from_frames(17 * k + 5)
        assert run.decode(z.half()).shape[2] == 17 * k + 5 == run._frames_from_tokens(5 * k + 2)
    img = video[:, :, 0]                      # a single image [B,3,H,W]
    z1 = run.encode(img)
    assert z1.shape == (1, 16, 1, 8, 8)
    assert run.decode(z1.half()).shape == (1, 3, 1, 64, 64)
