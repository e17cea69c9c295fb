"""Spatial tile planning, overlap blending and the multi-GPU work split.

The reference encodes spatial tiles, then blends each tile with its upper and left neighbours
with `core.blend` and trims the overlaps (h3vae_runtime.py:609-639); the split itself is
`_split_encoder_tiles` (h3vae_runtime.py:584-603).  `core.blend` is external; the linear ramp
used here is b[k] = a[-o + k] * (1 - k/o) + b[k] * (k/o), k = 0..o-1 (the linear overlap blend
the benchmark configuration specifies).

That sequential blend-then-trim is linear in the raw tiles, so it can be written as
    canvas = sum over tiles t of  W_t * raw_t     (each W_t supported on t's footprint)
with per-tile weight maps W_t (tile_weight_map).  Accumulating tile contributions this way is
order-free, which makes the multi-GPU blend a plain sum: each rank accumulates its own tiles
into a canvas and one NCCL reduce adds the canvases on rank 0.  blend_sequential restates the
reference's procedure directly and the tests check that both agree.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch


def split_tiles(length: int, tile_size: int, overlap_min: int, ratio: int):
    """(starts, sizes, overlaps) of a 1-D tile split.  ref: h3vae_runtime.py:584-603."""
    if tile_size <= overlap_min:
        raise ValueError("encoder tile must exceed its minimum overlap")
    if tile_size >= length:
        return [0], [length], []
    count = math.ceil(length / tile_size)
    while True:
        overlaps = [overlap_min] * (count - 1)
        remaining = tile_size * count - sum(overlaps) - length
        if remaining >= 0:
            break
        count += 1
    for i in range(remaining // ratio):
        overlaps[i % (count - 1)] += ratio
    starts = [0]
    for overlap in overlaps:
        starts.append(starts[-1] + tile_size - overlap)
    return starts, [tile_size] * count, overlaps


def select_encoder_tile(configured: int, height: int, width: int) -> int:
    """0 = auto: 672 up to 672x672, else 256.  ref: h3vae_runtime.py:605-607."""
    return configured or (672 if max(height, width) <= 672 else 256)


@dataclass(frozen=True)
class TilePlan:
    """A 2-D tile grid: per axis the starts, sizes and overlaps of split_tiles."""
    ys: tuple[int, ...]
    hs: tuple[int, ...]
    oys: tuple[int, ...]
    xs: tuple[int, ...]
    ws: tuple[int, ...]
    oxs: tuple[int, ...]

    @classmethod
    def build(cls, height: int, width: int, tile: int, overlap_min: int, ratio: int) -> "TilePlan":
        ys, hs, oys = split_tiles(height, tile, overlap_min, ratio)
        xs, ws, oxs = split_tiles(width, tile, overlap_min, ratio)
        # When the leftover is not a multiple of `ratio` the last tile overhangs the image; the
        # reference's slicing x[..., pos:pos + size] then yields a shorter last tile.
        hs[-1] = min(hs[-1], height - ys[-1])
        ws[-1] = min(ws[-1], width - xs[-1])
        return cls(tuple(ys), tuple(hs), tuple(oys), tuple(xs), tuple(ws), tuple(oxs))

    @property
    def rows(self) -> int:
        return len(self.ys)

    @property
    def cols(self) -> int:
        return len(self.xs)

    @property
    def height(self) -> int:
        return self.ys[-1] + self.hs[-1]

    @property
    def width(self) -> int:
        return self.xs[-1] + self.ws[-1]

    def tiles(self):
        for i in range(self.rows):
            for j in range(self.cols):
                yield i, j

    def scaled(self, factor: int) -> "TilePlan":
        """The same grid in units `factor` times smaller (e.g. pixels -> latents)."""
        vals = (self.ys, self.hs, self.oys, self.xs, self.ws, self.oxs)
        if any(v % factor for seq in vals for v in seq):
            raise ValueError(f"tile grid is not divisible by {factor}")
        return TilePlan(*(tuple(v // factor for v in seq) for seq in vals))


def _ramp(o: int, dtype, device) -> torch.Tensor:
    return torch.arange(o, dtype=torch.float64, device=device).div(o).to(dtype)


def tile_weight_map(plan: TilePlan, i: int, j: int, dtype=torch.float32, device="cpu") -> torch.Tensor:
    """[h, w] weights of raw tile (i, j) such that sum_t W_t * raw_t equals the reference's
    sequential blend-and-trim canvas (see module docstring)."""
    h, w = plan.hs[i], plan.ws[j]
    o_up = plan.oys[i - 1] if i > 0 else 0
    o_left = plan.oxs[j - 1] if j > 0 else 0
    o_down = plan.oys[i] if i < plan.rows - 1 else 0
    o_right = plan.oxs[j] if j < plan.cols - 1 else 0
    own_h, own_w = h - o_down, w - o_right
    wy = torch.ones(h, dtype=dtype, device=device)
    wx = torch.ones(w, dtype=dtype, device=device)
    if o_up:
        wy[:o_up] = _ramp(o_up, dtype, device)
    if o_left:
        wx[:o_left] = _ramp(o_left, dtype, device)
    m = torch.zeros(h, w, dtype=dtype, device=device)
    # own region: the vertical ramp, then the horizontal ramp over the blended tile
    m[:own_h, :own_w] = wy[:own_h, None] * wx[None, :own_w]
    # A band reaches only as far as the neighbour's own trimmed part: when an overlap is larger
    # than that part, the rest of the overlap is trimmed from the neighbour and belongs to the
    # tile after it, which blends with the neighbour's raw tile, not with this one.
    # band below: this tile is the raw "upper" tile of (i+1, j)
    if o_down:
        next_h = plan.hs[i + 1] - (plan.oys[i + 1] if i + 1 < plan.rows - 1 else 0)
        nd = min(o_down, next_h)
        m[own_h:own_h + nd, :own_w] = (1 - _ramp(o_down, dtype, device))[:nd, None] * wx[None, :own_w]
    # band right: this tile is the raw "left" tile of (i, j+1), over that tile's whole trimmed height
    if o_right:
        next_w = plan.ws[j + 1] - (plan.oxs[j + 1] if j + 1 < plan.cols - 1 else 0)
        nr = min(o_right, next_w)
        m[:own_h, own_w:own_w + nr] = (1 - _ramp(o_right, dtype, device))[None, :nr]
    return m


def accumulate_tile(canvas: torch.Tensor, tile: torch.Tensor, plan: TilePlan, i: int, j: int,
                    weights: torch.Tensor | None = None) -> None:
    """canvas[..., y:y+h, x:x+w] += W_ij * tile (in the canvas dtype)."""
    if weights is None:
        weights = tile_weight_map(plan, i, j, canvas.dtype, canvas.device)
    y, x = plan.ys[i], plan.xs[j]
    h, w = plan.hs[i], plan.ws[j]
    canvas[..., y:y + h, x:x + w].add_(tile.to(canvas.dtype) * weights)


def blend_sequential(tiles: dict, plan: TilePlan) -> torch.Tensor:
    """Direct restatement of the reference's blend + trim + concatenate
    (h3vae_runtime.py:623-639) with the linear ramp blend; tiles[(i, j)] -> canvas."""
    def blend(a, b, o, dim):
        if o <= 0:
            return b
        b = b.clone()
        r = _ramp(o, b.dtype, b.device)
        shape = [1] * b.ndim
        shape[dim] = o
        r = r.view(shape)
        n = a.shape[dim]
        b_head = b.narrow(dim, 0, o)
        b_head.copy_(a.narrow(dim, n - o, o) * (1 - r) + b_head * r)
        return b

    rows = []
    for i in range(plan.rows):
        row = []
        for j in range(plan.cols):
            t = tiles[(i, j)]
            if i:
                t = blend(tiles[(i - 1, j)], t, plan.oys[i - 1], t.ndim - 2)
            if j:
                t = blend(tiles[(i, j - 1)], t, plan.oxs[j - 1], t.ndim - 1)
            if i < plan.rows - 1:
                t = t[..., : t.shape[-2] - plan.oys[i], :]
            if j < plan.cols - 1:
                t = t[..., : t.shape[-1] - plan.oxs[j]]
            row.append(t)
        rows.append(torch.cat(row, dim=-1))
    return torch.cat(rows, dim=-2)


# ---------------------------------------------------------------------------
# Work split across GPUs (one process per GPU)
# ---------------------------------------------------------------------------
def shard_range(num_items: int, world: int, rank: int) -> range:
    """Contiguous block of work items for `rank`: spatially adjacent tiles stay on one GPU and
    the per-rank counts differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    base, extra = divmod(num_items, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def batches(items: list, size: int) -> list[list]:
    if size <= 0:
        raise ValueError("batch size must be positive")
    return [items[k:k + size] for k in range(0, len(items), size)]
