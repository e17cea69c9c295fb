"""H3 video-VAE runtime: the ComfyUI first_stage_model interface over the B200 INT8 path.

Mirrors H3VAEPyOptRuntime of the reference (h3vae_runtime.py:283-717): option validation that
fails before any weight is built (no silent fallback), encode / decode / decode_output_shape /
*_tiled / warmup, spatial tile split + overlap blend, staged 17-frame clip encoding, batched
decoder tiles, latent (de)normalisation and pixel finalisation.  build_comfy_vae wraps it as a
comfy.sd.VAE exactly like the reference (h3vae_runtime.py:720-806).

B200 additions: the hot kernels are the sm_100a library (there is no torch.compile; the
compile_* options are accepted and ignored), and the tile work can be sharded over the GPUs of
one node: with a torch.distributed process group (one process per GPU) every rank runs the same
encode/decode call and takes a contiguous block of the (clip batch, tile) work items.  Rank 0 holds
the request; it sends every other rank only the pixel window its encoder items read (point to
point, NCCL over NVLink; a decode request is the small latent tensor and is broadcast).  Each rank
accumulates its tiles' blend contributions into the slab of the canvas its items cover (frame range
x row band x column band), and rank 0 receives every slab and adds it into its canvas, then
finalizes and returns the result (other ranks return None).  No full-size canvas is reduced.

The real klvae model code and weights are not distributed with the reference; without them the
runtime builds the H3-structured synthetic model of h3vae_b200.model with seeded random weights.
"""
from __future__ import annotations

import logging
import os
import time
from contextlib import nullcontext as _nullcontext

import torch

from . import kernels as K
from . import tiling
from .model import DecoderConfig, EncoderConfig, H3Decoder, H3Encoder

logger = logging.getLogger("ComfyUI_H3VAE_PyOpt")

DEFAULT_MODEL_CODE_DIR = os.environ.get("H3_VAE_MODEL_CODE_DIR", "")
DEFAULT_WEIGHTS_FALLBACK = os.environ.get("H3_VAE_WEIGHTS_PATH", "")

CLIP_LENGTH = 17          # frames per causal encoder clip (ref: opt/encoder_staged_batch.py:39-57)
TAIL_FRAMES = 5           # frames 17k+5 <-> tokens 5k+2 (ref: h3vae_runtime.py:483-491, :739-742)
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
        if dtype not in (torch.float16, torch.float32):
            raise RuntimeError("dtype must be fp16 or fp32")
        if dtype == torch.float32:
            # the reference allows an fp32 VAE outside the INT8 / fused modes (h3vae_runtime.py:743-748);
            # here fp32 pixels and latents are accepted and returned, the arithmetic runs on the fp16
            # tensor-core path with fp32 accumulation
            logger.info("[H3VAE-B200] dtype=fp32: fp32 inputs accepted, activations computed in fp16")
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

    def _src(self) -> int:
        import torch.distributed as dist
        return dist.get_global_rank(self.process_group, 0)

    _DTYPES = (torch.float16, torch.float32, torch.bfloat16)

    def _share_meta(self, t: torch.Tensor | None) -> tuple[tuple[int, ...], torch.dtype]:
        """Rank 0 owns the request tensor; every rank learns its shape and dtype (one broadcast)."""
        if self.world == 1:
            return tuple(t.shape), t.dtype
        import torch.distributed as dist
        meta = torch.zeros(7, dtype=torch.int64, device=self.dev)
        if self.rank == 0:
            if t.dtype not in self._DTYPES:
                raise ValueError(f"unsupported request dtype {t.dtype}")
            meta[0], meta[1] = t.ndim, self._DTYPES.index(t.dtype)
            meta[2:2 + t.ndim] = torch.tensor(list(t.shape), dtype=torch.int64)
        dist.broadcast(meta, src=self._src(), group=self.process_group)
        m = [int(v) for v in meta.tolist()]
        return tuple(m[2:2 + m[0]]), self._DTYPES[m[1]]

    def _broadcast_tensor(self, t: torch.Tensor | None, shape, dtype) -> torch.Tensor:
        """The whole (small) request tensor on every rank: the latents of a decode call."""
        if self.world == 1:
            return t
        import torch.distributed as dist
        if self.rank == 0:
            t = t.to(device=self.dev).contiguous()
        else:
            t = torch.empty(shape, dtype=dtype, device=self.dev)
        dist.broadcast(t, src=self._src(), group=self.process_group)
        return t

    def _p2p(self, op, tensor, peer_group_rank: int) -> list:
        """One point-to-point send or receive, always posted through batch_isend_irecv so that every
        transfer of the runtime goes through the group's own communicator (PyTorch gives lone
        send/recv calls separate two-rank communicators and batched ones the group's; mixing the two
        styles between a sender and its receiver would never match)."""
        import torch.distributed as dist
        peer = dist.get_global_rank(self.process_group, peer_group_rank)
        return dist.batch_isend_irecv([dist.P2POp(op, tensor, peer, self.process_group)])

    @staticmethod
    def _frame_major(shape5, device, dtype=torch.float32):
        """A zeroed blend canvas with frames outermost after the batch ([B, T, C, H, W] storage),
        returned as its logical [B, C, T, H, W] view: one rank's frame range is then one contiguous
        block, and a slab of frames, rows and columns ships as one buffer."""
        b, c, t, h, w = shape5
        return torch.zeros((b, t, c, h, w), dtype=dtype, device=device).permute(0, 2, 1, 3, 4)

    def _aux_stream(self, role: str):
        """The runtime's side stream for one role ("copy": host uploads and chunk downloads;
        "scatter": window cut-outs sent to the other ranks), created once: the caching allocator
        reuses a freed block only on the stream it was allocated on, so a fresh stream per call
        would make every call allocate its windows and staging anew.  Separate roles keep a window
        from queueing behind the upload of frames it does not read."""
        streams = getattr(self, "_aux", None)
        if streams is None:
            streams = self._aux = {}
        if role not in streams:
            streams[role] = torch.cuda.Stream(self.dev)
        return streams[role]

    def _gather_slabs(self, canvas, slab, boxes, on_slab=None) -> list:
        """Bring every rank's blend slab to rank 0.  Rank r > 0 accumulated its work items into
        `slab`, the zero-initialised box boxes[r] = (t0, t1, y0, y1, x0, x1) of the canvas; rank 0
        accumulated its own items straight into `canvas`.  Rank 0 receives the other slabs (one
        point-to-point receive per rank, posted together) and adds each into its box, calling
        on_slab(r) after each add.  Returns the pending send works on ranks > 0."""
        if self.world == 1:
            return []
        import torch.distributed as dist
        if self.rank != 0:
            # frame-major contiguous storage of the slab is what crosses the link
            return self._p2p(dist.isend, slab.permute(0, 2, 1, 3, 4).contiguous(), 0)
        ops, bufs = [], {}
        for r in range(1, self.world):
            t0, t1, y0, y1, x0, x1 = boxes[r]
            if t1 <= t0:
                continue
            buf = torch.empty((canvas.shape[0], t1 - t0, canvas.shape[1], y1 - y0, x1 - x0), dtype=canvas.dtype,
                              device=canvas.device)
            bufs[r] = buf
            ops.append(dist.P2POp(dist.irecv, buf, dist.get_global_rank(self.process_group, r), self.process_group))
        works = dist.batch_isend_irecv(ops) if ops else []
        for w in works:
            w.wait()
        for r, buf in bufs.items():
            t0, t1, y0, y1, x0, x1 = boxes[r]
            canvas[:, :, t0:t1, y0:y1, x0:x1].add_(buf.permute(0, 2, 1, 3, 4))
            if on_slab is not None:
                on_slab(r)
        return []

    # -- shapes ----------------------------------------------------------------
    def _device(self):
        return self.dev

    def _frames_from_tokens(self, t: int) -> int:
        """Frame count of a decoded latent of t tokens: 17k+5 frames for 5k+2 tokens, one frame for
        one token (ref: h3vae_runtime.py:483-486).  For an encoder whose temporal ratio is not 4 the
        same rule holds with its own clip and tail token counts."""
        if t <= 1:
            return 1
        return max(1, (t - self.tail_tokens) // self.tokens_per_clip * CLIP_LENGTH + TAIL_FRAMES)

    def _tokens_from_frames(self, frames: int) -> int:
        """ref: h3vae_runtime.py:488-491."""
        if frames <= 1:
            return 1
        return max(1, (frames - TAIL_FRAMES) // CLIP_LENGTH * self.tokens_per_clip + self.tail_tokens)

    @staticmethod
    def _causal_tokens(frames: int, temporal_down) -> int:
        t = frames
        for down in temporal_down:
            if down:
                t = (t - 1) // 2 + 1
        return t

    @property
    def tokens_per_clip(self) -> int:
        """Tokens of one 17-frame clip (5 for the H3 temporal ratio 4)."""
        return self._causal_tokens(CLIP_LENGTH, self.encoder.cfg.temporal_down)

    @property
    def tail_tokens(self) -> int:
        """Tokens of the first 5 frames of a clip (2 for the H3 temporal ratio 4)."""
        return self._causal_tokens(TAIL_FRAMES, self.encoder.cfg.temporal_down)

    @property
    def token_drop(self) -> int:
        """Tokens dropped from the end of a staged encode (3 for H3: each clip gives 5 tokens, the
        trailing 3 belong to the repeated padding frames; ref: opt/encoder_staged_batch.py:57)."""
        return self.tokens_per_clip - self.tail_tokens

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

    @staticmethod
    def _box(boxes):
        """Bounding box (t0, t1, y0, y1, x0, x1) of several boxes; an empty list gives an empty box."""
        if not boxes:
            return (0, 0, 0, 0, 0, 0)
        return (min(b[0] for b in boxes), max(b[1] for b in boxes), min(b[2] for b in boxes),
                max(b[3] for b in boxes), min(b[4] for b in boxes), max(b[5] for b in boxes))

    @torch.no_grad()
    def encode(self, x, device=None):
        """x: [B,3,T,H,W] (or [B,3,H,W]) in [-1,1] -> fp32 latents [B, C, t, H/r, W/r] (rank 0).

        T frames are cut into causal 17-frame clips (the last one padded by repeating its final
        frame), each clip gives tokens_per_clip tokens, and the trailing token_drop tokens are
        dropped: 17k+5 frames -> 5k+2 tokens.  A single frame is encoded on its own and gives one
        token.  ref: h3vae_runtime.py:572-582, 641-661; opt/encoder_staged_batch.py:39-57."""
        t_start = time.monotonic()
        if self.rank == 0:
            if self.int8_encode and x.dtype != torch.float16:
                raise RuntimeError("int8_encode requires FP16 pixel input; use the FP16 VAE dtype")
            if x.ndim == 4:
                x = x.unsqueeze(2)
            if x.ndim != 5 or x.shape[1] != 3:
                raise ValueError("encode expects [B,3,T,H,W] or [B,3,H,W] pixels")
        shape, dtype = self._share_meta(x)
        b, _, t, h, w = shape
        tile = tiling.select_encoder_tile(self.encoder_tile_size, h, w)
        r = self.encoder.cfg.spatial_ratio
        if h > tile or w > tile:
            plan = tiling.TilePlan.build(h, w, tile, self.tile_overlap_min, r)
        else:
            plan = tiling.TilePlan((0,), (h,), (), (0,), (w,), ())
        lplan = plan.scaled(r)
        clip_len = 1 if t == 1 else CLIP_LENGTH
        tpc = 1 if t == 1 else self.tokens_per_clip
        clips = -(-t // clip_len)
        # work items: (staged batch of clips, tile), clip-major; the clip batches write disjoint
        # latent frames, so each latent value still receives its tiles in row-major tile order
        cbatches = tiling.batches(list(range(clips)), self.encoder_staged_batch)
        items = [(g, i, j) for g in range(len(cbatches)) for (i, j) in plan.tiles()]

        def px_box(k):
            g, i, j = items[k]
            cs = cbatches[g]
            return (cs[0] * clip_len, min((cs[-1] + 1) * clip_len, t), plan.ys[i], plan.ys[i] + plan.hs[i],
                    plan.xs[j], plan.xs[j] + plan.ws[j])

        def lat_box(k):
            g, i, j = items[k]
            cs = cbatches[g]
            return (cs[0] * tpc, (cs[-1] + 1) * tpc, lplan.ys[i], lplan.ys[i] + lplan.hs[i],
                    lplan.xs[j], lplan.xs[j] + lplan.ws[j])

        shards = [tiling.shard_range(len(items), self.world, q) for q in range(self.world)]
        px_boxes = [self._box([px_box(k) for k in sh]) for sh in shards]
        lat_boxes = [self._box([lat_box(k) for k in sh]) for sh in shards]
        mine = shards[self.rank]
        # -- input: rank 0 holds the video; every other rank receives only its pixel window
        xv, origin, arrived, sends = self._scatter_video(x, shape, dtype, cbatches, clip_len, px_boxes)
        # -- latent canvas (rank 0: all tokens; other ranks: their latent slab)
        lshape = (b, self.latent_channels, clips * tpc, lplan.height, lplan.width)
        if self.rank == 0:
            canvas = self._frame_major(lshape, self.dev)
            lorigin = (0, 0, 0)
        else:
            t0, t1, y0, y1, x0, x1 = lat_boxes[self.rank]
            canvas = self._frame_major((b, self.latent_channels, t1 - t0, y1 - y0, x1 - x0), self.dev)
            lorigin = (t0, y0, x0)
        for k in mine:
            g, i, j = items[k]
            cs = cbatches[g]
            if arrived is not None and arrived[g] is not None:
                torch.cuda.current_stream(self.dev).wait_event(arrived[g])
                arrived[g] = None
            py, px = plan.ys[i] - origin[1], plan.xs[j] - origin[2]
            tile_px = xv[..., py:py + plan.hs[i], px:px + plan.ws[j]]
            f_first = cs[0] * clip_len - origin[0]
            if b == 1 and tile_px.shape[2] - f_first >= len(cs) * clip_len:
                # whole consecutive clips of one video: a strided view [clips, 3, clip, h, w] of the
                # tile (batch stride = one clip of frames), no copy
                v = tile_px[0, :, f_first:f_first + len(cs) * clip_len]
                clip_batch = v.unflatten(1, (len(cs), clip_len)).transpose(0, 1)
            else:
                batch = []
                for bi in range(b):
                    for c in cs:
                        f0 = c * clip_len - origin[0]
                        clip = tile_px[bi:bi + 1, :, f0:f0 + clip_len]
                        if clip.shape[2] < clip_len:   # pad the last clip by repeating its last frame
                            rep = clip[:, :, -1:].expand(-1, -1, clip_len - clip.shape[2], -1, -1)
                            clip = torch.cat([clip, rep], dim=2)
                        batch.append(clip)
                clip_batch = torch.cat(batch, 0)
            if clip_batch.dtype == torch.float16:
                # normalization fused into the encoder's input conv
                moments = self.encoder(clip_batch, norm=(self._img_mean, self._img_std))
            else:
                moments = self.encoder(self._normalize_pixels(clip_batch))
            mean = moments[:, : self.latent_channels]
            wmap = self._weights(lplan, i, j)
            ly, lx = lplan.ys[i] - lorigin[1], lplan.xs[j] - lorigin[2]
            for n, (bi, c) in enumerate((bi, c) for bi in range(b) for c in cs):
                c0 = c * tpc - lorigin[0]
                K.blend_accumulate(canvas[bi, :, c0:c0 + tpc, ly:ly + lplan.hs[i], lx:lx + lplan.ws[j]],
                                   mean[n], wmap)
        sends += self._gather_slabs(canvas, canvas, lat_boxes)
        for work in sends:
            work.wait()
        self._log_call("encode", t_start)
        if self.rank != 0:
            return None
        tokens = clips * tpc - (self.token_drop if t > 1 else 0)
        lat = canvas[:, :, :tokens]
        return ((lat - self.latents_mean.float()) / self.latents_std.float()).contiguous()

    def _scatter_video(self, x, shape, dtype, cbatches, clip_len, px_boxes):
        """Place the request video for this rank's work items.

        Returns (video, origin, arrived, sends): `video` holds this rank's pixel window, whose
        (frame, row, column) origin in the full video is `origin`; `arrived` is one CUDA event per
        clip batch when the frames are still being uploaded (else None); `sends` are rank 0's
        pending sends.  A pinned host video on rank 0 is uploaded clip batch by clip batch on a
        side stream, so the host->device copy overlaps the encoding of the earlier batches.  At
        N > 1 rank 0 cuts every other rank's window out of its copy on that side stream and sends
        it point to point (NCCL over NVLink); the other ranks receive only their window."""
        b, c, t = shape[0], shape[1], shape[2]
        if self.rank == 0:
            streamed = (x.device.type == "cpu" and x.is_pinned() and x.is_contiguous()
                        and self.dev.type == "cuda")
            arrived = None
            if streamed:
                x, arrived = self._upload_clip_batches(x, cbatches, t, clip_len)
            else:
                x = x.to(device=self.dev)
            sends = []
            if self.world > 1:
                import torch.distributed as dist
                side = self._aux_stream("scatter") if self.dev.type == "cuda" else None
                if side is not None:
                    side.wait_stream(torch.cuda.current_stream(self.dev))
                for q in range(1, self.world):
                    t0, t1, y0, y1, x0, x1 = px_boxes[q]
                    if t1 <= t0:
                        continue
                    ctx = torch.cuda.stream(side) if side is not None else _nullcontext()
                    with ctx:
                        if arrived is not None:
                            for g, cs in enumerate(cbatches):
                                if cs[0] * clip_len < t1 and min((cs[-1] + 1) * clip_len, t) > t0:
                                    side.wait_event(arrived[g])
                        win = x[:, :, t0:t1, y0:y1, x0:x1].contiguous()
                        sends += self._p2p(dist.isend, win, q)
                if side is not None:
                    x.record_stream(side)
            return x, (0, 0, 0), arrived, sends
        import torch.distributed as dist
        t0, t1, y0, y1, x0, x1 = px_boxes[self.rank]
        win = torch.empty((b, c, t1 - t0, y1 - y0, x1 - x0), dtype=dtype, device=self.dev)
        if t1 > t0:
            for work in self._p2p(dist.irecv, win, 0):
                work.wait()
        return win, (t0, y0, x0), None, []

    def _upload_clip_batches(self, x_host, cbatches, t, clip_len=CLIP_LENGTH):
        """Issue the host->device copy of each clip batch's frames on a side stream (one contiguous
        copy per (batch entry, channel) plane).  Returns the device video and one event per clip batch."""
        x_dev = torch.empty(x_host.shape, dtype=x_host.dtype, device=self.dev)
        copy_stream = self._aux_stream("copy")
        copy_stream.wait_stream(torch.cuda.current_stream(self.dev))
        events = []
        with torch.cuda.stream(copy_stream):
            for cs in cbatches:
                f0, f1 = cs[0] * clip_len, min((cs[-1] + 1) * clip_len, t)
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
        """z: [B, C, t, h, w] normalized latents -> fp32 pixels [B, 3, F, h*r, w*r] in [0, 1] (rank 0).

        F = 17k+5 for t = 5k+2 tokens (one frame for one token).  The tokens are decoded in chunks
        of tokens_per_clip (the last chunk padded by repeating the final token) and the output is
        trimmed to F frames.  ref: h3vae_runtime.py:524-564."""
        t_start = time.monotonic()
        if self.rank == 0:
            if self.int8_decode and z.dtype != torch.float16:
                raise RuntimeError("int8_decode requires FP16 latent input; use the FP16 VAE dtype")
            if z.ndim != 5:
                raise ValueError("decode expects [B,C,t,h,w] latents")
            z = z.to(device=self.dev)
        shape, dtype = self._share_meta(z)
        z = self._broadcast_tensor(z, shape, dtype)
        zn = (z * self.latents_std + self.latents_mean).to(torch.float16)
        b, _, t, h, w = zn.shape
        tpc = 1 if t == 1 else self.tokens_per_clip
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
        frames = self._frames_from_tokens(t)
        tasks = [(bi, c, i, j) for bi in range(b) for c in range(chunks) for (i, j) in lplan.tiles()]
        groups = tiling.batches(tasks, max(1, self.tile_batch))
        shards = [tiling.shard_range(len(groups), self.world, q) for q in range(self.world)]

        def px_box(task):
            _, c, i, j = task
            return (c * fpc, (c + 1) * fpc, pplan.ys[i], pplan.ys[i] + pplan.hs[i], pplan.xs[j],
                    pplan.xs[j] + pplan.ws[j])

        boxes = [self._box([px_box(tk) for k in sh for tk in groups[k]]) for sh in shards]
        if self.rank == 0:
            canvas = self._frame_major((b, 3, chunks * fpc, pplan.height, pplan.width), self.dev)
            origin = (0, 0, 0)
        else:
            t0, t1, y0, y1, x0, x1 = boxes[self.rank]
            canvas = self._frame_major((b, 3, t1 - t0, y1 - y0, x1 - x0), self.dev)
            origin = (t0, y0, x0)
        # A pinned host output buffer on rank 0: each temporal chunk is finalized and copied to the
        # host on a side stream as soon as its last tile is blended (tasks run chunk by chunk, and
        # another rank's tiles count once its slab has been added), so the device->host transfer
        # overlaps the decoding of the later chunks.
        streamed = (self.rank == 0 and output_buffer is not None and output_buffer.device.type == "cpu"
                    and self.dev.type == "cuda" and output_buffer.is_pinned()
                    and output_buffer.dtype == torch.float32 and output_buffer.is_contiguous()
                    and tuple(output_buffer.shape) == (b, 3, frames, pplan.height, pplan.width))
        copy_stream = self._aux_stream("copy") if streamed else None
        pending = {}
        for (bi, c, _, _) in tasks:
            pending[(bi, c)] = pending.get((bi, c), 0) + 1

        def done(bi, c, n=1):
            pending[(bi, c)] -= n
            if streamed and pending[(bi, c)] == 0:
                self._emit_chunk(canvas, bi, c * fpc, min((c + 1) * fpc, frames), output_buffer, copy_stream)

        for k in shards[self.rank]:
            group = groups[k]
            lat = torch.cat([zn[bi:bi + 1, :, c * tpc:(c + 1) * tpc, lplan.ys[i]:lplan.ys[i] + lplan.hs[i],
                                lplan.xs[j]:lplan.xs[j] + lplan.ws[j]] for (bi, c, i, j) in group], 0)
            pix = self.decoder(lat)
            for n, (bi, c, i, j) in enumerate(group):
                f0, y0, x0 = c * fpc - origin[0], pplan.ys[i] - origin[1], pplan.xs[j] - origin[2]
                K.blend_accumulate(canvas[bi, :, f0:f0 + fpc, y0:y0 + pplan.hs[i], x0:x0 + pplan.ws[j]],
                                   pix[n], self._weights(pplan, i, j))
                if self.rank == 0:
                    done(bi, c)

        def slab_added(q):
            counts = {}
            for k in shards[q]:
                for (bi, c, _, _) in groups[k]:
                    counts[(bi, c)] = counts.get((bi, c), 0) + 1
            for key, n in counts.items():
                done(*key, n=n)

        sends = self._gather_slabs(canvas, canvas, boxes, on_slab=slab_added)
        for work in sends:
            work.wait()
        if self.rank != 0:
            self._log_call("decode", t_start)
            return None
        if streamed:
            copy_stream.synchronize()
            self._log_call("decode", t_start)
            return output_buffer
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
        self._log_call("decode", t_start)
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

    ratio = runtime.decoder.spatial_ratio

    class H3VAEPyOptVAE(comfy.sd.VAE):
        def __init__(self, first_stage_model, device=None, dtype=None):
            self.first_stage_model = first_stage_model
            self.latent_channels = runtime.latent_channels
            self.latent_dim = 3
            self.output_channels = 3
            # frames 17k+5 <-> latents 5k+2 (ref: h3vae_runtime.py:739-742)
            self.upscale_ratio = (lambda a: runtime._frames_from_tokens(a), ratio, ratio)
            self.upscale_index_formula = (4, ratio, ratio)
            self.downscale_ratio = (lambda a: runtime._tokens_from_frames(a), ratio, ratio)
            self.downscale_index_formula = (4, ratio, ratio)
            self.working_dtypes = ([torch.float16] if runtime.int8_decode or runtime.int8_encode
                                   else [torch.float16, torch.float32])
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
            if dtype not in self.working_dtypes:
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
