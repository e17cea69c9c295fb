"""Benchmark: BASELINE config 5, the full-video INT8 round trip (768x1344x124, tile256).

One step = encode + decode of the synthetic video through H3VAEPyOptRuntime (the reference's
first_stage_model API): 24 spatial tiles (tile 256, 32-px minimum overlap) x 8 causal 17-frame
clips, encoded 4 clips per call (config 3 shape [4,3,17,256,256], every 3x3x3 residual conv on the
INT8 tcgen05 kernel) and decoded 4 tiles per call (config 4 shape [4,16,5,32,32], 6 INT8
transformer blocks), blended linearly and finalized to fp32 RGB.  124 frames encode to 37 latent
frames and decode back to 124 (the reference's 17k+5 <-> 5k+2 contract).  With torchrun (one process
per GPU) the tile batches are sharded over the ranks: rank 0 sends each rank the pixel window its
encoder items read, and gathers every rank's latent / pixel canvas slab (NCCL point-to-point over
NVLink).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Prints one JSON line (rank 0).  `value` is seconds per round trip with the input already in HBM
(device-timed with CUDA events, max over ranks); `e2e` is the same call with the video in pinned
host memory, the host->device copy and the device->host copy of the fp32 result inside the
timed region.  Inputs (768 MB video, 1.7 GB canvas) are larger than L2.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (ROOT, ROOT / "comfyui-h3vae-pyopt_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

import torch  # noqa: E402

VIDEO_SHAPE = (1, 3, 124, 768, 1344)
TILE = 256
OVERLAP = 32
METRIC = "768x1344x124 tile256 encode+decode round-trip seconds"
# DRAM bytes (read + write) per INT8 conv launch at encoder batch 4: ncu dram__bytes_read.sum +
# dram__bytes_write.sum summed over the 16 INT8 conv launches of one tile-batch-1 encoder call
# (2.84 GB: kw-strip kernels for stages 1-2, the generic implicit-GEMM kernel for stages 3-4), times 4
# for batch 4 (activation traffic scales with the batch), divided by the 16 launches.
CONV_DRAM_BYTES_PER_LAUNCH = 2.84e9 * 4 / 16
UNIT = "s"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", choices=("video", "tile", "kernels"), default="video",
                    help="video: the config-5 round trip (the bench line); tile: one config-3 encoder call and "
                         "one config-4 decoder call per step (small enough for ncu captures); kernels: the "
                         "decoder GEMMs and attention at the real H3 shapes and the encoder conv calls the "
                         "reference publishes, each timed alone with CUDA events")
    ap.add_argument("--no-quality", action="store_true",
                    help="skip the INT8-vs-fp16 round-trip PSNR measured after the timed region (N=1)")
    ap.add_argument("--tile-batch", type=int, default=4,
                    help="tile workload: clips per encoder call and tiles per decoder call (4 = configs 3/4)")
    ap.add_argument("--tile-part", choices=("both", "encoder", "decoder"), default="both",
                    help="tile workload: run the encoder call, the decoder call or both per step")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# Synthetic input: smooth low-frequency noise (Gaussian-blurred N(0,1), sigma 8 px / 2 frames),
# renormalized and clipped to [-1, 1].  Generated on the GPU, seeded.
# ---------------------------------------------------------------------------
def _gauss(sigma: float, device) -> torch.Tensor:
    r = int(3 * sigma)
    x = torch.arange(-r, r + 1, dtype=torch.float32, device=device)
    k = torch.exp(-0.5 * (x / sigma) ** 2)
    return k / k.sum()


def synthetic_video(device, seed: int = 0) -> torch.Tensor:
    g = torch.Generator(device=device).manual_seed(seed)
    b, c, t, h, w = VIDEO_SHAPE
    out = torch.empty(VIDEO_SHAPE, dtype=torch.float16, device=device)
    ks, kt = _gauss(8.0, device), _gauss(2.0, device)
    for ci in range(c):
        v = torch.randn((t, h, w), generator=g, device=device)
        v = torch.nn.functional.conv1d(v.reshape(-1, 1, w), ks.view(1, 1, -1), padding=ks.numel() // 2).view(t, h, w)
        v = torch.nn.functional.conv1d(v.transpose(1, 2).reshape(-1, 1, h), ks.view(1, 1, -1),
                                       padding=ks.numel() // 2).view(t, w, h).transpose(1, 2)
        v = torch.nn.functional.conv1d(v.permute(1, 2, 0).reshape(-1, 1, t), kt.view(1, 1, -1),
                                       padding=kt.numel() // 2).view(h, w, t).permute(2, 0, 1)
        v = v / v.std()
        out[0, ci] = v.clamp(-1, 1).half()
    return out


# ---------------------------------------------------------------------------
# Clock sampling during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        if self.proc is None or self.path is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        os.unlink(self.path)
        load = [s for s in sm if smax and s > 0.5 * smax] or sm
        return {"sm_mhz": statistics.median(load) if load else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# CPU baseline: the oracle port on the host cores, on a bounded sample
# ---------------------------------------------------------------------------
def int8_ops_per_round_trip(cfg=None, dcfg=None) -> tuple[float, float]:
    """(INT8 ops, fp16 attention flops) of one round trip on the config-5 video, from the tile and
    clip counts and the per-call algorithmic counts of configs 3 and 4 (causal taps skipped)."""
    from h3vae_b200 import tiling
    from h3vae_b200.model import DecoderConfig, EncoderConfig
    cfg = cfg or EncoderConfig()
    dcfg = dcfg or DecoderConfig()
    b, c, t, h, w = VIDEO_SHAPE
    plan = tiling.TilePlan.build(h, w, TILE, OVERLAP, cfg.spatial_ratio)
    tiles = plan.rows * plan.cols
    clips = -(-t // 17)
    enc = 0.0
    d, hh, ww = 17, TILE, TILE
    for s, ch in enumerate(cfg.channels):
        cin = cfg.channels[s - 1] if s else ch
        for j in range(cfg.blocks_per_stage):
            ci = cin if j == 0 else ch
            taps = sum(min(x + 1, 3) for x in range(d)) * 9
            if s in cfg.int8_stages:
                enc += 2 * hh * ww * taps * (ci * ch + ch * ch)
        if cfg.spatial_down[s]:
            hh, ww = hh // 2, ww // 2
        if cfg.temporal_down[s]:
            d = (d - 1) // 2 + 1
    enc *= tiles * clips
    ratio = 2 ** sum(dcfg.up_spatial)
    tokens_t = 17
    for down in cfg.temporal_down:
        if down:
            tokens_t = (tokens_t - 1) // 2 + 1
    tok = tokens_t * (TILE // ratio) ** 2
    per_tile = dcfg.blocks * 2 * tok * dcfg.hidden * (3 * dcfg.hidden + dcfg.hidden + 2 * dcfg.ffn + dcfg.ffn)
    attn = dcfg.blocks * 4 * tok * tok * dcfg.hidden
    lplan = plan.scaled(ratio)
    dec_tasks = lplan.rows * lplan.cols * clips
    return enc + per_tile * dec_tasks, attn * dec_tasks


def cpu_model_name() -> str:
    try:
        for line in subprocess.run(["lscpu"], capture_output=True, text=True, timeout=10).stdout.splitlines():
            if line.lower().startswith("model name"):
                return line.split(":", 1)[1].strip()
    except (OSError, subprocess.SubprocessError):
        pass
    return "unknown"


ENC_CROP = 64      # encoder work item sampled on a 64x64 window of its 256x256 tile (area ratio 16)
DEC_CROP = 16      # decoder tile task sampled on a 16x16 window of its 32x32 latent tile (area ratio 4)


def cpu_round_trip_sample(enc, dec, tiles: int, clips: int, dec_tasks: int, seed: int = 0) -> dict:
    """The CPU restatement of the path (oracle.cpu_model: the reference's CPU arithmetic -- dequantized
    fp32 INT8 convs as its CPU oracle computes them, the producers with their fp16 rounding points, fp32
    convs rounded to fp16, the INT8 decoder block chain, torch SDPA on the CPU) on the host cores, per
    the CPU-baseline plan: one encoder work item (one tile x one 17-frame clip) and one decoder tile task
    (one tile x one 5-token chunk), each timed on a spatial crop and scaled to the full item by op count
    (work linear in the positions x area ratio, attention x area ratio squared), then multiplied by the
    item counts of the round trip.  Labelled "extrapolated"."""
    from oracle import cpu_model as C
    torch.set_num_threads(os.cpu_count() or 1)
    mean = torch.tensor([0.485, 0.456, 0.406])
    std = torch.tensor([0.229, 0.224, 0.225])
    t0 = time.perf_counter()
    enc_s, enc_info = C.encoder_item_seconds(enc, 17, ENC_CROP, TILE, mean, std, seed)
    dec_s, dec_info = C.decoder_task_seconds(dec, 5, DEC_CROP, TILE // 8, seed)
    wall = time.perf_counter() - t0
    total = enc_s * tiles * clips + dec_s * dec_tasks
    return {"seconds": total, "encoder_item_s": enc_s, "decoder_task_s": dec_s, "sample_wall_s": wall,
            "encoder_sample": enc_info, "decoder_sample": dec_info, "cores": torch.get_num_threads(),
            "items": {"encoder": tiles * clips, "decoder": dec_tasks}}


def cpu_models():
    """Host copies of the bench runtime's encoder and decoder (same configs and seeds, so the same
    random-init weights)."""
    from h3vae_b200.model import DecoderConfig, EncoderConfig, H3Decoder, H3Encoder
    return (H3Encoder(EncoderConfig(), device="cpu", seed=0),
            H3Decoder(DecoderConfig(), device="cpu", seed=1, int8=True))


def _round_trip_items(cfg=None, dcfg=None) -> tuple[int, int, int]:
    from h3vae_b200 import tiling
    from h3vae_b200.model import DecoderConfig, EncoderConfig
    cfg = cfg or EncoderConfig()
    dcfg = dcfg or DecoderConfig()
    b, c, t, h, w = VIDEO_SHAPE
    plan = tiling.TilePlan.build(h, w, TILE, OVERLAP, cfg.spatial_ratio)
    clips = -(-t // 17)
    lplan = plan.scaled(2 ** sum(dcfg.up_spatial))
    return plan.rows * plan.cols, clips, lplan.rows * lplan.cols * clips


def _cpu_baseline_line(sample: dict) -> dict:
    return {"value": sample["seconds"], "unit": UNIT, "cores": sample["cores"], "kind": "port",
            "cpu": cpu_model_name(),
            "sample": (f"extrapolated: one encoder work item (1 tile x 1 17-frame clip, timed on a {ENC_CROP}x{ENC_CROP} "
                       f"crop, {sample['encoder_item_s']:.2f} s scaled) x {sample['items']['encoder']} + one decoder "
                       f"tile task (timed on a {DEC_CROP}x{DEC_CROP} latent crop, {sample['decoder_task_s']:.2f} s "
                       f"scaled) x {sample['items']['decoder']}, oracle.cpu_model (reference CPU arithmetic) on "
                       f"{sample['cores']} threads; {sample['sample_wall_s']:.1f} s of CPU work per sample")}


# ---------------------------------------------------------------------------
def init_dist(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
        return dist.group.WORLD, dist.get_rank(), world, local
    torch.cuda.set_device(0)
    return None, 0, 1, 0


def max_over_ranks(v: float, pg) -> float:
    if pg is None:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=pg)
    return float(t.item())


def barrier(pg):
    if pg is not None:
        import torch.distributed as dist
        dist.barrier(group=pg)
    torch.cuda.synchronize()


def run_reference(args):
    """The reference arm.  The reference's own implementation of this path is Triton/CK GPU code with no
    CPU implementation, and its model code is not distributed, so the arm times the CPU restatement of its
    arithmetic (oracle.cpu_model) on the host cores, on the same config-5 workload, model config and
    weights as the b200 arm: every step is one encoder work item and one decoder tile task (bounded
    spatial samples, scaled by op count) extrapolated to the round trip's item counts.  Under torchrun
    rank 0 alone runs it."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    enc, dec = cpu_models()
    tiles, clips, dec_tasks = _round_trip_items()
    for _ in range(args.warmup):
        cpu_round_trip_sample(enc, dec, tiles, clips, dec_tasks)
    samples = [cpu_round_trip_sample(enc, dec, tiles, clips, dec_tasks, seed=k) for k in range(args.steps)]
    value = statistics.mean(sm["seconds"] for sm in samples)
    cpu = _cpu_baseline_line(samples[0])
    cpu["value"] = value
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": value * 1e3, "higher_is_better": False,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8 (dequantized fp32 CPU arithmetic), fp16",
            "data": "synthetic (random-init H3-structured weights, seeded)",
            "config": {"workload": "config5 full-video round trip (encode config3 tiles + decode config4 tiles), "
                                   "extrapolated from one encoder work item and one decoder tile task per step",
                       "video": list(VIDEO_SHAPE), "tile": TILE, "overlap_min": OVERLAP, "clip": 17,
                       "encoder_items": tiles * clips, "decoder_tasks": dec_tasks},
            "samples_s": [sm["seconds"] for sm in samples],
            "cpu_baseline": cpu,
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_tile(args):
    """One config-3 encoder call ([4,3,17,256,256]) + one config-4 decoder call ([4,16,5,32,32]) per
    step through the model objects (no tiling / blend); prints per-call milliseconds."""
    from h3vae_b200.runtime import H3VAEPyOptRuntime
    torch.cuda.set_device(0)
    rt = H3VAEPyOptRuntime(int8_encode=True, int8_decode=True, decode_fusions=True, log_calls=False,
                           compile_decoder=False, compile_encoder=False)
    g = torch.Generator(device="cuda").manual_seed(0)
    tb = args.tile_batch
    x = (torch.rand((tb, 3, 17, 256, 256), generator=g, device="cuda") * 2 - 1).half()
    z = torch.randn((tb, 16, 5, 32, 32), generator=g, device="cuda").half()
    run_enc, run_dec = args.tile_part in ("both", "encoder"), args.tile_part in ("both", "decoder")
    for _ in range(args.warmup):
        if run_enc:
            rt.encoder(x)
        if run_dec:
            rt.decoder(z)
    torch.cuda.synchronize()
    enc, dec = [], []
    for _ in range(args.steps):
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record()
        if run_enc:
            rt.encoder(x)
        e1.record()
        if run_dec:
            rt.decoder(z)
        e2.record()
        torch.cuda.synchronize()
        enc.append(e0.elapsed_time(e1))
        dec.append(e1.elapsed_time(e2))
    print(json.dumps({"workload": "tile", "tile_batch": tb, "encoder_tile_ms": statistics.mean(enc),
                      "decoder_tile_ms": statistics.mean(dec), "steps": args.steps, "warmup": args.warmup}))


# Reference timings (RTX PRO 5000, SM120) of the same operations, from the reference's own notes:
# docs/int8_norm_producer_2026-10-02.md:94-97 (CK INT8 GEMMs at M = 7188),
# docs/encoder_int8_analysis_2026-10-02.md:40-41 (INT8 conv op including its activation quantization).
REF_SM120_MS = {"gemm_qkv": 0.398, "gemm_attn_out": 0.143, "gemm_ffn_up": 1.018, "gemm_ffn_down": 0.473,
                "conv_c128": 4.222, "conv_c256": 3.403}


def _time_launches(fn, steps: int, warmup: int, flush: torch.Tensor) -> list[float]:
    """Milliseconds of each launch, CUDA events around the launch only; the L2 is flushed (a write
    larger than its 126 MB) before every launch."""
    for _ in range(warmup):
        fn()
    out = []
    for _ in range(steps):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        out.append(e0.elapsed_time(e1))
    return out


def run_kernels(args):
    """The decoder GEMMs and attention at the real H3 shapes (4 tiles x 1797 tokens = 7188 rows, hidden
    2048, 32 heads x 64, FFN 2 x 8192) and the encoder conv calls at the reference's published shapes,
    beside the reference's SM120 timings of the same operations."""
    from h3vae_b200 import kernels as K
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    flush = torch.empty(256 * 2 ** 20, dtype=torch.uint8, device=dev)
    steps, warmup = max(args.steps, 5), max(args.warmup, 3)
    m, d, heads, ffn, tokens = 7188, 2048, 32, 8192, 1797
    rows = []

    def record(name, shape, ms_list, ops, unit="TOPS"):
        ms = statistics.median(ms_list)
        row = {"name": name, "shape": shape, "ms": ms, unit.lower(): ops / (ms * 1e-3) / 1e12}
        if name in REF_SM120_MS:
            row["ref_sm120_ms"] = REF_SM120_MS[name]
        rows.append(row)

    def i8(*shape):
        return torch.randint(-127, 128, shape, generator=g, device=dev, dtype=torch.int8)

    q = i8(m, d)
    s = torch.rand((m, 1), generator=g, device=dev) * 0.02 + 0.001
    for name, n, k, kind in (("gemm_qkv", 3 * d, d, "linear"), ("gemm_attn_out", d, d, "linear"),
                             ("gemm_ffn_up", 2 * ffn, d, "linear"), ("gemm_ffn_down", d, ffn, "linear"),
                             ("gemm_ffn_up_swiglu", 2 * ffn, d, "swiglu"), ("gemm_qkv_qknorm_rope", 3 * d, d, "qkv"),
                             ("gemm_attn_out_residual", d, d, "residual")):
        a = q if k == d else i8(m, k)
        w = i8(n, k)
        ws = torch.rand(n, generator=g, device=dev) * 1e-3 + 1e-4
        b = (torch.randn(n, generator=g, device=dev) * 0.02).half()
        if kind == "linear":
            fn = lambda a=a, w=w, ws=ws, b=b: K.gemm_i8(a, s, w, ws, b)          # noqa: E731
        elif kind == "swiglu":
            fn = lambda a=a, w=w, ws=ws, b=b: K.gemm_i8_swiglu(a, s, w, ws, b)   # noqa: E731
        elif kind == "residual":
            xres = torch.randn((m, n), generator=g, device=dev).half()
            gate = (0.5 + 0.1 * torch.randn(n, generator=g, device=dev)).half()
            fn = lambda a=a, w=w, ws=ws, b=b, xres=xres, gate=gate: K.gemm_i8_residual(a, s, w, ws, b, xres, gate)  # noqa: E731
        else:
            ang = torch.rand((4, tokens, 1, 48), generator=g, device=dev) * 6.28
            cos, sin = ang.cos().half(), ang.sin().half()
            fn = lambda a=a, w=w, ws=ws, b=b: K.gemm_i8_qkv_rope(a, s, w, ws, b, 4, tokens, heads, cos, sin, 1e-6)  # noqa: E731
        record(name, [m, n, k], _time_launches(fn, steps, warmup, flush), 2.0 * m * n * k)
    qa, ka, va = (torch.randn((4, heads, tokens, 64), generator=g, device=dev).half() for _ in range(3))
    flops = 4.0 * 4 * heads * tokens * tokens * 64
    record("attention_tc", [4, heads, tokens, 64], _time_launches(lambda: K.attention_f16(qa, ka, va, 0.125), steps,
                                                                  warmup, flush), flops, "TFLOPS")
    sdpa = torch.nn.functional.scaled_dot_product_attention
    record("attention_torch_sdpa", [4, heads, tokens, 64],
           _time_launches(lambda: sdpa(qa, ka, va, scale=0.125), steps, warmup, flush), flops, "TFLOPS")
    # encoder INT8 conv calls incl. their activation quantization (the norm producer), reference shapes
    for name, c, hw in (("conv_c128", 128, 256), ("conv_c256", 256, 128)):
        x = (torch.randn((1, c, 17, hw, hw), generator=g, device=dev)).half().contiguous(
            memory_format=torch.channels_last_3d)
        gam = torch.ones(c, device=dev, dtype=torch.float16)
        bet = torch.zeros(c, device=dev, dtype=torch.float16)
        w = i8(c, 27 * c)
        ws = torch.rand(c, generator=g, device=dev) * 1e-3 + 1e-4

        def conv_call(x=x, gam=gam, bet=bet, w=w, ws=ws):
            qx, sx = K.norm_pad_quant(x, gam, bet, 1e-6)
            return K.conv3d_i8(qx, sx, w, ws, None, (3, 3, 3), causal_zero_frames=2)
        ops = 2.0 * hw * hw * c * c * 9 * sum(min(t + 1, 3) for t in range(17))
        record(name, [1, c, 17, hw, hw], _time_launches(conv_call, steps, warmup, flush), ops)
    print(json.dumps({"workload": "kernels", "device": torch.cuda.get_device_name(dev), "steps": steps,
                      "warmup": warmup, "l2": "flushed (256 MB write) before every timed launch",
                      "ref_source": "RTX PRO 5000 (SM120): docs/int8_norm_producer_2026-10-02.md:94-97, "
                                    "docs/encoder_int8_analysis_2026-10-02.md:40-41",
                      "kernels": rows}), flush=True)


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
        return
    if args.workload == "tile":
        run_tile(args)
        return
    if args.workload == "kernels":
        run_kernels(args)
        return
    from h3vae_b200 import kernels as K
    from h3vae_b200.runtime import H3VAEPyOptRuntime

    pg, rank, world, local = init_dist(args)
    dev = torch.device("cuda", local)
    runtime = H3VAEPyOptRuntime(device=str(dev), int8_encode=True, int8_decode=True, decode_fusions=True,
                                tile_batch=4, encoder_staged_batch=4, log_calls=False, compile_decoder=False,
                                compile_encoder=False, decoder_tile_size=TILE, tile_overlap_min=OVERLAP,
                                process_group=pg)
    video = synthetic_video(dev) if rank == 0 else None
    torch.cuda.synchronize()

    def fp16(lat):
        # ComfyUI hands latents to the VAE in its working dtype (fp16 for the INT8 modes)
        return None if lat is None else lat.half()

    def step(x):
        lat = runtime.encode(x)
        return lat, runtime.decode(fp16(lat))

    for _ in range(args.warmup):
        step(video)
    barrier(pg)

    # ---- timed region (inputs resident in HBM) ----
    stream = torch.cuda.current_stream()
    enc_ms, dec_ms, tot_ms = [], [], []
    K.CONV_TIMING = []
    launches0 = K.LAUNCHES["count"]
    with ClockSampler(local) as clocks:
        barrier(pg)
        for _ in range(args.steps):
            e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
            e0.record(stream)
            lat = runtime.encode(video)
            e1.record(stream)
            runtime.decode(fp16(lat))
            e2.record(stream)
            torch.cuda.synchronize()
            enc_ms.append(e0.elapsed_time(e1))
            dec_ms.append(e1.elapsed_time(e2))
            tot_ms.append(e0.elapsed_time(e2))
        barrier(pg)
    launches = K.LAUNCHES["count"] - launches0
    conv_events = K.CONV_TIMING
    K.CONV_TIMING = None
    step_s = max_over_ranks(statistics.mean(tot_ms) / 1e3, pg)
    enc_s = max_over_ranks(statistics.mean(enc_ms) / 1e3, pg)
    dec_s = max_over_ranks(statistics.mean(dec_ms) / 1e3, pg)

    # roofline of the dominant INT8 kernel (the tcgen05 implicit-GEMM conv), live CUDA events
    conv_ms = sum(a.elapsed_time(b) for a, b, _ in conv_events)
    conv_ops = sum(o for _, _, o in conv_events)
    conv_launches = len(conv_events)
    a_ = torch.randint(-127, 127, (8192, 8192), dtype=torch.int8, device=dev)
    for _ in range(3):
        torch._int_mm(a_, a_.t())
    torch.cuda.synchronize()
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record()
    for _ in range(10):
        torch._int_mm(a_, a_.t())
    p1.record()
    torch.cuda.synchronize()
    int8_peak = 2 * 8192 ** 3 * 10 / (p0.elapsed_time(p1) * 1e-3) / 1e12
    del a_
    conv_tops = conv_ops / (conv_ms * 1e-3) / 1e12 if conv_ms > 0 else 0.0

    # ---- end-to-end through the public API with host buffers ----
    e2e = None
    if not args.no_e2e:
        host_video = video.cpu().pin_memory() if rank == 0 else None
        out_shape = runtime.decode_output_shape((1, runtime.latent_channels, runtime._tokens_from_frames(124),
                                                 VIDEO_SHAPE[3] // 8, VIDEO_SHAPE[4] // 8))
        host_out = torch.empty(out_shape, dtype=torch.float32).pin_memory() if rank == 0 else None
        e2e_ms = []
        # one untimed pass through the host-buffer path first (its staging buffers and streams)
        lat = runtime.encode(host_video)
        runtime.decode(fp16(lat), output_buffer=host_out)
        torch.cuda.synchronize()
        barrier(pg)
        for _ in range(max(1, args.steps)):
            t0 = torch.cuda.Event(enable_timing=True)
            t1 = torch.cuda.Event(enable_timing=True)
            t0.record(stream)
            lat = runtime.encode(host_video)
            # the ComfyUI chunked-IO call: pixels land in the caller's pinned host buffer
            runtime.decode(fp16(lat), output_buffer=host_out)
            t1.record(stream)
            torch.cuda.synchronize()
            e2e_ms.append(t0.elapsed_time(t1))
        barrier(pg)
        e2e_s = max_over_ranks(statistics.mean(e2e_ms) / 1e3, pg)
        e2e = {"value": e2e_s, "unit": UNIT, "step_s": [round(t / 1e3, 4) for t in e2e_ms],
               "h2d_bytes_per_step": int(video.numel() * video.element_size()) if rank == 0 else 0,
               "d2h_bytes_per_step": int(host_out.numel() * 4) if rank == 0 else 0}

    # ---- quality (north_star): INT8 round trip against the fp16 round trip of the same weights ----
    quality = None
    if world == 1 and not args.no_quality:
        out8 = runtime.decode(fp16(runtime.encode(video)))
        rt16 = H3VAEPyOptRuntime(device=str(dev), tile_batch=4, encoder_staged_batch=4, log_calls=False,
                                 compile_decoder=False, compile_encoder=False, decoder_tile_size=TILE,
                                 tile_overlap_min=OVERLAP)
        out16 = rt16.decode(fp16(rt16.encode(video)))
        mse = float(((out8 - out16).double() ** 2).mean())
        quality = {"psnr_db": 10.0 * __import__("math").log10(1.0 / max(mse, 1e-20)),
                   "against": "fp16 encode + fp16 decode of the same weights (int8_encode / int8_decode off)",
                   "unclamped_fraction": float(((out16 > 0) & (out16 < 1)).float().mean()),
                   "frames": int(out8.shape[2])}
        del rt16, out8, out16
        torch.cuda.empty_cache()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tiles, clips, dec_tasks = _round_trip_items(runtime.encoder.cfg, runtime.decoder.cfg)
        enc_cpu, dec_cpu = cpu_models()
        cpu_round_trip_sample(enc_cpu, dec_cpu, tiles, clips, dec_tasks)     # warm-up
        cpu = _cpu_baseline_line(cpu_round_trip_sample(enc_cpu, dec_cpu, tiles, clips, dec_tasks))

    if rank == 0:
        cl = clocks.summary()
        int8_ops, attn = int8_ops_per_round_trip(runtime.encoder.cfg, runtime.decoder.cfg)
        line = {
            "metric": METRIC, "value": step_s, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_s * 1e3, "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None, "dtype": "int8 (conv/linear), fp16 (attention, fp16 convs)",
            "data": "synthetic (seeded Gaussian-blurred noise video; random-init H3-structured weights)",
            "config": {"workload": "config5 full-video round trip: encode (config3 tiles, all 3x3x3 residual convs "
                                   "INT8) + decode (config4 tiles, 6 INT8 blocks) + linear overlap blend",
                       "video": list(VIDEO_SHAPE), "tile": TILE, "overlap_min": OVERLAP, "clip": 17,
                       "encoder_batch": 4, "decoder_tile_batch": 4, "parallelism": f"tile-dp{world}",
                       "l2": "inputs larger than L2 (768 MB video, 1.7 GB canvas)"},
            "encode_s": enc_s, "decode_s": dec_s,
            "int8_ops_per_step": int8_ops, "attention_flops_per_step": attn,
            "roofline": {"bound": "tensor", "kernel": "h3b conv3d_i8 (tcgen05 kind::i8 implicit GEMM)",
                         "achieved": conv_tops, "peak": int8_peak, "unit": "TFLOP/s",
                         "peak_source": "INT8 ops/s of torch._int_mm 8192^3 measured live on this GPU "
                                        "(MEASURED_PEAKS.json has no INT8 entry)",
                         "frac": conv_tops / int8_peak if int8_peak else None,
                         "traffic": CONV_DRAM_BYTES_PER_LAUNCH,
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, conv launches of a "
                                           "tile-batch-1 encoder call scaled x4 (bytes per launch)",
                         "launches": conv_launches, "ms_total": conv_ms},
            "e2e": e2e, "cpu_baseline": cpu, "clocks": cl, "gpu_launches": launches, "quality": quality,
        }
        print(json.dumps(line), flush=True)
    if pg is not None:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
