"""H3 video-VAE runtime: the ComfyUI first_stage_model interface over the B200 INT8 path.

Mirrors H3VAEPyOptRuntime of the reference (h3vae_runtime.py:283-717): option validation that
fails before any weight is built (no silent fallback), encode / decode / decode_output_shape /
*_tiled / warmup, spatial tile split + overlap blend, staged 17-frame clip encoding, batched
decoder tiles, latent (de)normalisation and pixel finalisation.  build_comfy_vae wraps it as a
comfy.sd.VAE exactly like the reference (h3vae_runtime.py:720-806).

B200 additions: the hot kernels are the sm_100a library (there is no torch.compile; the
compile_* options are accepted and ignored), and the tile work can be sharded over the GPUs of
one node: with a torch.distributed process group (one process per GPU) every rank runs the same
encode/decode call, takes a contiguous block of the (clip batch, tile) work items, accumulates its tiles'
blend contributions into a canvas, and one NCCL reduce sums the canvases on rank 0, which
returns the result (other ranks return None).

The real klvae model code and weights are not distributed with the reference; without them the
runtime builds the H3-structured synthetic model of h3vae_b200.model with seeded random weights.
"""
from __future__ import annotations

import logging
import os
import time

import torch

from . import kernels as K
from . import tiling
from .model import DecoderConfig, EncoderConfig, H3Decoder, H3Encoder

logger = logging.getLogger("ComfyUI_H3VAE_PyOpt")

DEFAULT_MODEL_CODE_DIR = os.environ.get("H3_VAE_MODEL_CODE_DIR", "")
DEFAULT_WEIGHTS_FALLBACK = os.environ.get("H3_VAE_WEIGHTS_PATH", "")

CLIP_LENGTH = 17          # frames per causal encoder clip (ref: opt/encoder_staged_batch.py:39-57)
IMG_MEAN = (0.485, 0.456, 0.406)
IMG_STD = (0.229, 0.224, 0.225)


# ---------------------------------------------------------------------------
# Option validation (ref: h3vae_runtime.py:50-181).  Pure functions with injectable probes so the
# policy is testable on CPU.
# ---------------------------------------------------------------------------
def _cuda_probe(device, cuda_available, capability, hip):
    try:
        device_type = torch.device(device).type
    except (TypeError, RuntimeError) as exc:
        raise RuntimeError(f"requires a CUDA device, got {device!r}") from exc
    if device_type != "cuda":
        raise RuntimeError(f"requires a CUDA device, got {device!r}")
    if (torch.version.hip if hip is None else hip) is not None:
        raise RuntimeError("is CUDA-only and does not support ROCm")
    if not (torch.cuda.is_available() if cuda_available is None else cuda_available):
        raise RuntimeError("requires an available CUDA GPU")
    capability = torch.cuda.get_device_capability(torch.device(device)) if capability is None else capability
    if tuple(capability) != (10, 0):
        raise RuntimeError(f"requires an sm_100 (B200) GPU; got SM{capability[0]}{capability[1]}")


def _validate_decode_fusions_options(*, enabled, device, dtype, fast_linear, compile_decoder=True,
                                     int8_encode=False, cuda_available=None, capability=None, hip=None):
    """ref: h3vae_runtime.py:50-74.  compile_decoder is accepted and ignored (no torch.compile)."""
    if not enabled:
        return
    if fast_linear:
        raise ValueError("decode_fusions and fast_linear are mutually exclusive")
    if dtype != torch.float16:
        raise RuntimeError("decode_fusions requires dtype=fp16")
    try:
        _cuda_probe(device, cuda_available, capability, hip)
    except RuntimeError as exc:
        raise RuntimeError(f"decode_fusions {exc}") from None
    if os.environ.get("MINIMAX_H3_VAE_DECODER_VIT_FP32_NORM", "1").lower() not in ("1", "true", "yes", "on"):
        raise ValueError("decode_fusions requires FP32 decoder normalization")


def _validate_int8_decode_options(*, enabled, fast_linear, device, dtype, cuda_available=None, hip=None,
                                  capability=None, library_available=None, check_dependencies=True):
    """ref: h3vae_runtime.py:77-141 (the comfy-kitchen check becomes a check of the sm_100a library)."""
    if not enabled:
        return
    if fast_linear:
        raise ValueError("int8_decode and fast_linear are mutually exclusive; choose one")
    try:
        torch.device(device)
    except (TypeError, RuntimeError) as exc:
        raise RuntimeError(f"int8_decode requires a CUDA device, got {device!r}") from exc
    if torch.device(device).type != "cuda":
        raise RuntimeError(f"int8_decode requires a CUDA device, got {device!r}")
    if dtype != torch.float16:
        raise RuntimeError("int8_decode requires dtype=fp16")
    try:
        _cuda_probe(device, cuda_available, capability, hip)
    except RuntimeError as exc:
        raise RuntimeError(f"int8_decode {exc}") from None
    if check_dependencies:
        _require_library(library_available, "int8_decode")


def _validate_int8_encode_options(*, enabled, device, dtype, cuda_available=None, hip=None, capability=None,
                                  library_available=None, check_dependencies=True):
    """ref: h3vae_runtime.py:144-181."""
    if not enabled:
        return
    try:
        torch.device(device)
    except (TypeError, RuntimeError) as exc:
        raise RuntimeError(f"int8_encode requires a CUDA device, got {device!r}") from exc
    if torch.device(device).type != "cuda":
        raise RuntimeError(f"int8_encode requires a CUDA device, got {device!r}")
    if dtype != torch.float16:
        raise RuntimeError("int8_encode requires dtype=fp16")
    try:
        _cuda_probe(device, cuda_available, capability, hip)
    except RuntimeError as exc:
        raise RuntimeError(f"int8_encode {exc}") from None
    if check_dependencies:
        _require_library(library_available, "int8_encode")


def _require_library(available, what):
    if available is None:
        from . import _lib
        try:
            _lib.load()
            available = True
        except (OSError, RuntimeError):
            available = False
    if not available:
        raise RuntimeError(f"{what} requires the h3vae_b200 sm_100a library; no fallback is available")


# ---------------------------------------------------------------------------
# The runtime
# ---------------------------------------------------------------------------
class H3VAEPyOptRuntime(torch.nn.Module):
    """comfy first_stage_model interface over the B200-native INT8 H3 VAE path."""

    comfy_has_chunked_io = True

    def __init__(self, model_code_dir: str = DEFAULT_MODEL_CODE_DIR, weights_path: str = DEFAULT_WEIGHTS_FALLBACK,
                 device: str = "cuda", dtype: torch.dtype = torch.float16, decoder_tile_size: int = 256,
                 tile_batch: int = 2, compile_decoder: bool = True, compile_encoder: bool = True, qk_rows: int = 8,
                 encoder_staged_batch: int = 4, log_calls: bool = True, encoder_tile_size: int = 0,
                 fast_linear: bool = False, int8_decode: bool = False, int8_encode: bool = False,
                 decode_fusions: bool = False, *, encoder_config: EncoderConfig | None = None,
                 decoder_config: DecoderConfig | None = None, tile_overlap_min: int = 32, seed: int = 0,
                 process_group=None, act_scale_mode: str = "tensor"):
        super().__init__()
        int8_decode, int8_encode = bool(int8_decode), bool(int8_encode)
        if fast_linear:
            raise ValueError("fast_linear (comfy-kitchen fp16 linears) is not available in the B200 build; "
                             "use int8_decode or the default path")
        _validate_decode_fusions_options(enabled=bool(decode_fusions), device=device, dtype=dtype,
                                         fast_linear=bool(fast_linear), compile_decoder=bool(compile_decoder),
                                         int8_encode=int8_encode)
        _validate_int8_decode_options(enabled=int8_decode, fast_linear=bool(fast_linear), device=device, dtype=dtype)
        _validate_int8_encode_options(enabled=int8_encode, device=device, dtype=dtype)
        if encoder_tile_size < 0 or encoder_tile_size % 16:
            raise ValueError("encoder_tile_size must be 0 (auto) or a positive multiple of 16")
        if int(tile_batch) < 0:
            raise ValueError("tile_batch must be non-negative")
        if int(encoder_staged_batch) not in (1, 2, 4):
            raise ValueError("encoder_staged_batch must be 1, 2 or 4")
        if encoder_tile_size and encoder_tile_size <= tile_overlap_min:
            raise ValueError("encoder_tile_size must exceed encoder tile overlap")
        if model_code_dir or weights_path:
            raise NotImplementedError(
                "loading the real klvae model code / H3 checkpoint is not implemented in the B200 build; "
                "leave model_code_dir and weights_path empty to run the H3-structured synthetic model")
        if compile_decoder or compile_encoder:
            logger.info("[H3VAE-B200] compile_* options ignored: kernels are precompiled sm_100a code")
        if dtype != torch.float16:
            raise RuntimeError("the B200 path runs fp16 activations (dtype=fp16)")
        if act_scale_mode not in ("tensor", "token"):
            raise ValueError("act_scale_mode must be 'tensor' (per-tensor, the reference's scheme) or 'token'")

        self.dev = torch.device(device)
        enc_cfg = EncoderConfig(**{**(encoder_config or EncoderConfig()).__dict__, "act_scale_mode": act_scale_mode})
        if not int8_encode:
            enc_cfg = EncoderConfig(**{**enc_cfg.__dict__, "int8_stages": ()})
        self.encoder = H3Encoder(enc_cfg, device=self.dev, seed=seed)
        self.decoder = H3Decoder(decoder_config or DecoderConfig(), device=self.dev, seed=seed + 1, int8=int8_decode)
        self.decoder_tile_size = int(decoder_tile_size)
        self.encoder_tile_size = int(encoder_tile_size)
        self.tile_batch = int(tile_batch)
        self.encoder_staged_batch = int(encoder_staged_batch)
        self.tile_overlap_min = int(tile_overlap_min)
        self.int8_decode, self.int8_encode = int8_decode, int8_encode
        self.decode_fusions = bool(decode_fusions)
        self.fast_linear = False
        self.process_group = process_group
        self.latent_channels = self.encoder.cfg.latent_channels
        g = torch.Generator().manual_seed(seed + 7)
        self.latents_mean = (0.1 * torch.randn(self.latent_channels, generator=g)).half().to(self.dev).view(1, -1, 1, 1, 1)
        self.latents_std = (1.0 + 0.1 * torch.rand(self.latent_channels, generator=g)).half().to(self.dev).view(1, -1, 1, 1, 1)
        self._img_mean = torch.tensor(IMG_MEAN, dtype=torch.float32, device=self.dev).view(1, 3, 1, 1, 1)
        self._img_std = torch.tensor(IMG_STD, dtype=torch.float32, device=self.dev).view(1, 3, 1, 1, 1)
        self._weight_cache: dict = {}
        self.log_calls = bool(log_calls)
        self._dec_calls = self._enc_calls = 0
        self._dec_total_ms = self._enc_total_ms = 0.0
        logger.info("[H3VAE-B200] runtime ready: decoder_tile=%d encoder_tile=%s tile_batch=%d staged_batch=%d "
                    "int8_decode=%s int8_encode=%s (%d INT8 convs) decode_fusions=%s world=%d",
                    self.decoder_tile_size, self.encoder_tile_size or "auto", self.tile_batch,
                    self.encoder_staged_batch, int8_decode, int8_encode, self.encoder.int8_conv_count,
                    self.decode_fusions, self.world)

    # -- distributed helpers -------------------------------------------------
    @property
    def world(self) -> int:
        if self.process_group is None:
            return 1
        import torch.distributed as dist
        return dist.get_world_size(self.process_group)

    @property
    def rank(self) -> int:
        if self.process_group is None:
            return 0
        import torch.distributed as dist
        return dist.get_rank(self.process_group)

    def _reduce_to_rank0(self, canvas: torch.Tensor) -> None:
        if self.world > 1:
            import torch.distributed as dist
            dist.reduce(canvas, dst=dist.get_global_rank(self.process_group, 0), op=dist.ReduceOp.SUM,
                        group=self.process_group)

    def _share_input(self, t: torch.Tensor | None) -> torch.Tensor:
        """Rank 0 owns the request tensor; the other ranks receive it (shape, then fp16 data)."""
        if self.world == 1:
            return t
        import torch.distributed as dist
        src = dist.get_global_rank(self.process_group, 0)
        shape = torch.tensor(list(t.shape) if self.rank == 0 else [0] * 5, dtype=torch.int64, device=self.dev)
        dist.broadcast(shape, src=src, group=self.process_group)
        if self.rank == 0:
            t = t.to(torch.float16).contiguous()
        else:
            t = torch.empty(tuple(int(v) for v in shape.tolist()), dtype=torch.float16, device=self.dev)
        dist.broadcast(t, src=src, group=self.process_group)
        return t

    # -- shapes ----------------------------------------------------------------
    def _device(self):
        return self.dev

    def _frames_from_tokens(self, t: int) -> int:
        return max(1, -(-t // self.tokens_per_clip) * CLIP_LENGTH)

    def _tokens_from_frames(self, frames: int) -> int:
        return -(-frames // CLIP_LENGTH) * self.tokens_per_clip

    @property
    def tokens_per_clip(self) -> int:
        t = CLIP_LENGTH
        for down in self.encoder.cfg.temporal_down:
            if down:
                t = (t - 1) // 2 + 1
        return t

    def decode_output_shape(self, input_shape):
        b, c, t, h, w = input_shape
        r = self.decoder.spatial_ratio
        return (b, 3, self._frames_from_tokens(t), h * r, w * r)

    def _log_call(self, kind: str, t0: float):
        if not self.log_calls:
            return
        torch.cuda.synchronize(self.dev)
        dt = (time.monotonic() - t0) * 1000.0
        if kind == "decode":
            self._dec_calls += 1
            self._dec_total_ms += dt
            logger.info("[H3VAE-B200] decode #%d: %.1f ms (running mean %.1f ms)", self._dec_calls, dt,
                        self._dec_total_ms / self._dec_calls)
        else:
            self._enc_calls += 1
            self._enc_total_ms += dt
            logger.info("[H3VAE-B200] encode #%d: %.1f ms (running mean %.1f ms)", self._enc_calls, dt,
                        self._enc_total_ms / self._enc_calls)

    def _weights(self, plan: tiling.TilePlan, i: int, j: int, dtype=torch.float32) -> torch.Tensor:
        key = (plan, i, j, dtype)
        w = self._weight_cache.get(key)
        if w is None:
            w = tiling.tile_weight_map(plan, i, j, dtype, self.dev)
            self._weight_cache[key] = w
        return w

    # -- encode ----------------------------------------------------------------
    def _normalize_pixels(self, x):
        """ref: h3vae_runtime.py:566-570."""
        x01 = (x.float() + 1.0) * 0.5
        return ((x01 - self._img_mean) / self._img_std).to(torch.float16)

    @torch.no_grad()
    def encode(self, x, device=None):
        """x: [B,3,T,H,W] (or [B,3,H,W]) in [-1,1] -> fp32 latents [B, C, t, H/r, W/r] (rank 0)."""
        t0 = time.monotonic()
        if self.int8_encode and x is not None and x.dtype != torch.float16:
            raise RuntimeError("int8_encode requires FP16 pixel input; use the FP16 VAE dtype")
        if self.rank == 0 and x.ndim == 4:
            x = x.unsqueeze(2)
        # A pinned host video on one GPU is uploaded clip batch by clip batch on a side stream, and
        # the work items run clip-major, so the host->device copy overlaps the encoding.
        streamed = (self.world == 1 and x.device.type == "cpu" and x.is_pinned() and x.is_contiguous())
        if self.rank == 0 and not streamed:
            x = x.to(device=self.dev)
        x = self._share_input(x)
        b, _, t, h, w = x.shape
        tile = tiling.select_encoder_tile(self.encoder_tile_size, h, w)
        r = self.encoder.cfg.spatial_ratio
        if h > tile or w > tile:
            plan = tiling.TilePlan.build(h, w, tile, self.tile_overlap_min, r)
        else:
            plan = tiling.TilePlan((0,), (h,), (), (0,), (w,), ())
        lplan = plan.scaled(r)
        clips = -(-t // CLIP_LENGTH)
        tpc = self.tokens_per_clip
        lat = torch.zeros((b, self.latent_channels, clips * tpc, lplan.height, lplan.width), dtype=torch.float32,
                          device=self.dev)
        # work items: (staged batch of clips, tile), clip-major; the clip batches write disjoint
        # latent frames, so each latent value still receives its tiles in row-major tile order
        cbatches = tiling.batches(list(range(clips)), self.encoder_staged_batch)
        items = [(g, i, j) for g in range(len(cbatches)) for (i, j) in plan.tiles()]
        arrived = None
        if streamed:
            x, arrived = self._upload_clip_batches(x, cbatches, t)
        for k in tiling.shard_range(len(items), self.world, self.rank):
            g, i, j = items[k]
            cs = cbatches[g]
            if arrived is not None and arrived[g] is not None:
                torch.cuda.current_stream(self.dev).wait_event(arrived[g])
                arrived[g] = None
            tile_px = x[..., plan.ys[i]:plan.ys[i] + plan.hs[i], plan.xs[j]:plan.xs[j] + plan.ws[j]]
            batch = []
            for bi in range(b):
                for c in cs:
                    clip = tile_px[bi:bi + 1, :, c * CLIP_LENGTH:(c + 1) * CLIP_LENGTH]
                    if clip.shape[2] < CLIP_LENGTH:   # pad the last clip by repeating its last frame
                        rep = clip[:, :, -1:].expand(-1, -1, CLIP_LENGTH - clip.shape[2], -1, -1)
                        clip = torch.cat([clip, rep], dim=2)
                    batch.append(clip)
            clips = torch.cat(batch, 0)
            if clips.dtype == torch.float16:
                # normalization fused into the encoder's input conv
                moments = self.encoder(clips, norm=(self._img_mean, self._img_std))
            else:
                moments = self.encoder(self._normalize_pixels(clips))
            mean = moments[:, : self.latent_channels]
            wmap = self._weights(lplan, i, j)
            for n, (bi, c) in enumerate((bi, c) for bi in range(b) for c in cs):
                ly, lx = lplan.ys[i], lplan.xs[j]
                K.blend_accumulate(lat[bi, :, c * tpc:(c + 1) * tpc, ly:ly + lplan.hs[i], lx:lx + lplan.ws[j]],
                                   mean[n], wmap)
        self._reduce_to_rank0(lat)
        self._log_call("encode", t0)
        if self.rank != 0:
            return None
        return (lat - self.latents_mean.float()) / self.latents_std.float()

    def _upload_clip_batches(self, x_host, cbatches, t):
        """Issue the host->device copy of each clip batch's frames on a side stream (one contiguous
        copy per (batch entry, channel) plane).  Returns the device video and one event per clip batch."""
        x_dev = torch.empty(x_host.shape, dtype=x_host.dtype, device=self.dev)
        copy_stream = torch.cuda.Stream(self.dev)
        copy_stream.wait_stream(torch.cuda.current_stream(self.dev))
        events = []
        with torch.cuda.stream(copy_stream):
            for cs in cbatches:
                f0, f1 = cs[0] * CLIP_LENGTH, min((cs[-1] + 1) * CLIP_LENGTH, t)
                for bi in range(x_host.shape[0]):
                    for ch in range(x_host.shape[1]):
                        x_dev[bi, ch, f0:f1].copy_(x_host[bi, ch, f0:f1], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(copy_stream)
                events.append(ev)
        # the allocator must not hand the block out again before the side-stream copies finish,
        # also when an exception ends the encode before every event was waited on
        x_dev.record_stream(copy_stream)
        return x_dev, events

    # -- decode ----------------------------------------------------------------
    @torch.no_grad()
    def decode(self, z, output_buffer=None, **kwargs):
        """z: [B, C, t, h, w] normalized latents -> fp32 pixels [B, 3, F, h*r, w*r] in [0, 1] (rank 0)."""
        t0 = time.monotonic()
        if self.int8_decode and z is not None and z.dtype != torch.float16:
            raise RuntimeError("int8_decode requires FP16 latent input; use the FP16 VAE dtype")
        z = self._share_input(z.to(device=self.dev) if self.rank == 0 else None)
        zn = (z * self.latents_std + self.latents_mean).to(torch.float16)
        b, _, t, h, w = zn.shape
        tpc = self.tokens_per_clip
        chunks = -(-t // tpc)
        if chunks * tpc != t:   # too few tokens for the last chunk: repeat the last latent frame
            zn = torch.cat([zn, zn[:, :, -1:].expand(-1, -1, chunks * tpc - t, -1, -1)], dim=2)
        r = self.decoder.spatial_ratio
        ltile = max(1, self.decoder_tile_size // r)
        lov = max(0, self.tile_overlap_min // r)
        if h > ltile or w > ltile:
            lplan = tiling.TilePlan.build(h, w, ltile, lov, 1)
        else:
            lplan = tiling.TilePlan((0,), (h,), (), (0,), (w,), ())
        pplan = tiling.TilePlan(*(tuple(v * r for v in seq) for seq in
                                  (lplan.ys, lplan.hs, lplan.oys, lplan.xs, lplan.ws, lplan.oxs)))
        fpc = self.decoder.frames_for(tpc)
        canvas = torch.zeros((b, 3, chunks * fpc, pplan.height, pplan.width), dtype=torch.float32, device=self.dev)
        tasks = [(bi, c, i, j) for bi in range(b) for c in range(chunks) for (i, j) in lplan.tiles()]
        per_call = max(1, self.tile_batch)
        groups = tiling.batches(tasks, per_call)
        frames = self._frames_from_tokens(t)
        # A pinned host output buffer on one GPU: each temporal chunk is finalized and copied to the
        # host on a side stream as soon as its last tile is blended (tasks run chunk by chunk), so the
        # device->host transfer overlaps the decoding of the later chunks.
        streamed = (output_buffer is not None and self.world == 1 and output_buffer.device.type == "cpu"
                    and output_buffer.is_pinned() and output_buffer.dtype == torch.float32
                    and output_buffer.is_contiguous()
                    and tuple(output_buffer.shape) == (b, 3, frames, pplan.height, pplan.width))
        copy_stream = torch.cuda.Stream(self.dev) if streamed else None
        pending = {}
        for (bi, c, _, _) in tasks:
            pending[(bi, c)] = pending.get((bi, c), 0) + 1
        for k in tiling.shard_range(len(groups), self.world, self.rank):
            group = groups[k]
            lat = torch.cat([zn[bi:bi + 1, :, c * tpc:(c + 1) * tpc, lplan.ys[i]:lplan.ys[i] + lplan.hs[i],
                                lplan.xs[j]:lplan.xs[j] + lplan.ws[j]] for (bi, c, i, j) in group], 0)
            pix = self.decoder(lat)
            for n, (bi, c, i, j) in enumerate(group):
                y0, x0 = pplan.ys[i], pplan.xs[j]
                K.blend_accumulate(canvas[bi, :, c * fpc:(c + 1) * fpc, y0:y0 + pplan.hs[i], x0:x0 + pplan.ws[j]],
                                   pix[n], self._weights(pplan, i, j))
                pending[(bi, c)] -= 1
                if streamed and pending[(bi, c)] == 0:
                    self._emit_chunk(canvas, bi, c * fpc, min((c + 1) * fpc, frames), output_buffer, copy_stream)
        if streamed:
            copy_stream.synchronize()
            self._log_call("decode", t0)
            return output_buffer
        self._reduce_to_rank0(canvas)
        if self.rank != 0:
            self._log_call("decode", t0)
            return None
        dec = canvas[:, :, :frames]
        direct = (output_buffer is not None and output_buffer.shape == dec.shape
                  and output_buffer.dtype == torch.float32 and output_buffer.device == dec.device
                  and output_buffer.is_contiguous())
        pixels = K.finalize_pixels(dec, self._img_std.reshape(3), self._img_mean.reshape(3),
                                   output_buffer if direct else None)
        if output_buffer is not None:
            if pixels is not output_buffer:
                output_buffer.copy_(pixels)
            out = output_buffer
        else:
            out = pixels
        self._log_call("decode", t0)
        return out

    def _emit_chunk(self, canvas, bi, f0, f1, host_out, copy_stream):
        """Finalize frames [f0, f1) of batch entry bi into a device staging tensor and copy them to the
        pinned host output on copy_stream (one contiguous copy per channel plane)."""
        if f0 >= f1:
            return
        stage = K.finalize_pixels(canvas[bi:bi + 1, :, f0:f1], self._img_std.reshape(3), self._img_mean.reshape(3))
        ready = torch.cuda.Event()
        ready.record()
        copy_stream.wait_event(ready)
        with torch.cuda.stream(copy_stream):
            for ch in range(3):
                host_out[bi, ch, f0:f1].copy_(stage[0, ch], non_blocking=True)
        stage.record_stream(copy_stream)

    def decode_tiled(self, z, **kwargs):
        return self.decode(z)

    def encode_tiled(self, x, **kwargs):
        return self.encode(x)

    @torch.no_grad()
    def warmup(self, frames: int, width: int, height: int, mode: str = "both"):
        """Run one decode and/or encode of the given video shape (first-call costs: cuDNN
        algorithm search, allocator growth).  ref: h3vae_runtime.py:673-717."""
        results = {}
        if mode in ("decode", "both"):
            r = self.decoder.spatial_ratio
            z = torch.randn((1, self.latent_channels, self._tokens_from_frames(frames), height // r, width // r),
                            device=self.dev, dtype=torch.float16)
            torch.cuda.synchronize(self.dev)
            t0 = time.monotonic()
            self.decode(z)
            torch.cuda.synchronize(self.dev)
            results["decode_first_s"] = round(time.monotonic() - t0, 3)
        if mode in ("encode", "both"):
            x = torch.rand((1, 3, frames, height, width), device=self.dev, dtype=torch.float16) * 2.0 - 1.0
            torch.cuda.synchronize(self.dev)
            t0 = time.monotonic()
            self.encode(x)
            torch.cuda.synchronize(self.dev)
            results["encode_first_s"] = round(time.monotonic() - t0, 3)
        self._dec_calls = self._enc_calls = 0
        self._dec_total_ms = self._enc_total_ms = 0.0
        logger.info("[H3VAE-B200] warmup %s (%d frames, %dx%d): %s", mode, frames, width, height, results)
        return results


def build_comfy_vae(runtime: H3VAEPyOptRuntime, dtype=None):
    """Wrap the runtime in a comfy.sd.VAE configured like the reference's H3 branch
    (ref: h3vae_runtime.py:720-806); comfy is imported lazily."""
    import comfy.model_management as model_management
    import comfy.model_patcher
    import comfy.sd

    tpc, ratio = runtime.tokens_per_clip, runtime.decoder.spatial_ratio

    class H3VAEPyOptVAE(comfy.sd.VAE):
        def __init__(self, first_stage_model, device=None, dtype=None):
            self.first_stage_model = first_stage_model
            self.latent_channels = runtime.latent_channels
            self.latent_dim = 3
            self.output_channels = 3
            self.upscale_ratio = (lambda a: max(1, -(-a // tpc) * CLIP_LENGTH), ratio, ratio)
            self.upscale_index_formula = (CLIP_LENGTH // tpc, ratio, ratio)
            self.downscale_ratio = (lambda a: max(1, -(-a // CLIP_LENGTH) * tpc), ratio, ratio)
            self.downscale_index_formula = (CLIP_LENGTH // tpc, ratio, ratio)
            self.working_dtypes = [torch.float16]
            self.handles_tiling = True
            self.process_output = lambda image: image
            self.process_input = lambda image: image * 2.0 - 1.0
            self.pad_channel_value = None
            self.disable_offload = False
            self.not_video = False
            self.size = None
            self.extra_1d_channel = None
            self.crop_input = True
            self.format_encoded = None
            if device is None:
                device = model_management.vae_device()
            self.device = device
            offload_device = model_management.vae_offload_device()
            if dtype is None:
                dtype = model_management.vae_dtype(self.device, self.working_dtypes)
            if dtype != torch.float16:
                raise RuntimeError("INT8 VAE mode requires ComfyUI to select an FP16 VAE dtype")
            self.vae_dtype = dtype
            self.output_device = model_management.intermediate_device()

            def estimate_encode_memory(shape, dtype_):
                b, c, t, h, w = shape
                act = 1000 * min(t, CLIP_LENGTH) * h * w
                return int((self.size or 0) + (act + 1_100_000_000) * model_management.dtype_size(dtype_) / 2 * 1.15)

            def estimate_decode_memory(shape, dtype_):
                b, c, t, h, w = shape
                frames = self.upscale_ratio[0](t)
                out = 3 * frames * (h * ratio) * (w * ratio) * 4 * 2.5
                return int((self.size or 0) + (out + 1_100_000_000) * model_management.dtype_size(dtype_) / 2 * 1.1)

            self.memory_used_encode = estimate_encode_memory
            self.memory_used_decode = estimate_decode_memory
            self.patcher = comfy.model_patcher.CoreModelPatcher(first_stage_model, load_device=self.device,
                                                                offload_device=offload_device)
            self.model_size()

    return H3VAEPyOptVAE(runtime, dtype=dtype)
