"""Tile planner, overlap blend and GPU work split (CPU)."""
import json

import pytest
import torch

from h3vae_b200 import tiling


def test_split_matches_reference_goldens(golden):
    for c in json.loads(bytes(golden["split_tiles_json"]).decode()):
        assert tiling.split_tiles(*c["case"]) == (c["starts"], c["sizes"], c["overlaps"])
    for conf, h, w, expect in golden["select_tile"].tolist():
        assert tiling.select_encoder_tile(conf, h, w) == expect


def test_split_rejects_tile_not_larger_than_overlap():
    with pytest.raises(ValueError):
        tiling.split_tiles(768, 64, 64, 16)


@pytest.mark.parametrize("h,w,tile,ov,ratio", [(768, 1344, 256, 32, 8), (96, 160, 64, 16, 2), (300, 257, 128, 24, 4),
                                               (64, 64, 64, 16, 2)])
def test_weighted_accumulation_equals_sequential_blend(h, w, tile, ov, ratio):
    plan = tiling.TilePlan.build(h, w, tile, ov, ratio)
    g = torch.Generator().manual_seed(h + w)
    tiles = {(i, j): torch.randn(2, plan.hs[i], plan.ws[j], generator=g, dtype=torch.float64) for i, j in plan.tiles()}
    ref = tiling.blend_sequential(tiles, plan)
    canvas = torch.zeros(2, plan.height, plan.width, dtype=torch.float64)
    for (i, j), t in tiles.items():
        tiling.accumulate_tile(canvas, t, plan, i, j)
    assert ref.shape == canvas.shape == (2, h, w)
    assert torch.allclose(ref, canvas, atol=1e-12)


def test_weights_partition_unity():
    plan = tiling.TilePlan.build(768, 1344, 256, 32, 8)
    canvas = torch.zeros(768, 1344, dtype=torch.float64)
    for i, j in plan.tiles():
        tiling.accumulate_tile(canvas, torch.ones(plan.hs[i], plan.ws[j], dtype=torch.float64), plan, i, j)
    assert torch.allclose(canvas, torch.ones_like(canvas))
    assert (plan.rows, plan.cols) == (4, 6)


def test_scaled_plan_in_latent_units():
    plan = tiling.TilePlan.build(768, 1344, 256, 32, 8)
    lp = plan.scaled(8)
    assert lp.height == 96 and lp.width == 168 and lp.hs[0] == 32
    with pytest.raises(ValueError):
        tiling.TilePlan.build(768, 1344, 256, 32, 8).scaled(7)


@pytest.mark.parametrize("n,world", [(48, 1), (48, 2), (48, 8), (49, 4), (3, 8), (0, 2)])
def test_shard_range_partitions(n, world):
    seen = []
    sizes = []
    for r in range(world):
        rr = tiling.shard_range(n, world, r)
        seen.extend(rr)
        sizes.append(len(rr))
    assert seen == list(range(n))
    assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("seed", range(40))
def test_random_plans_partition_unity_and_match_sequential_blend(seed):
    """Randomized plans (tile, overlap, ratio, ragged sizes): the per-tile weights sum to one on every
    canvas pixel and the weighted accumulation equals the reference's sequential blend-and-trim."""
    rng = torch.Generator().manual_seed(1000 + seed)
    ratio = [1, 2, 4, 8][int(torch.randint(0, 4, (1,), generator=rng))]
    tile = ratio * int(torch.randint(8, 40, (1,), generator=rng))
    ov = ratio * int(torch.randint(1, tile // ratio // 2 + 1, (1,), generator=rng))
    h = ratio * int(torch.randint(1, 3 * tile // ratio, (1,), generator=rng))
    w = ratio * int(torch.randint(1, 3 * tile // ratio, (1,), generator=rng))
    if tile <= ov:
        pytest.skip("tile must exceed the overlap")
    plan = tiling.TilePlan.build(h, w, tile, ov, ratio) if (h > tile or w > tile) else \
        tiling.TilePlan((0,), (h,), (), (0,), (w,), ())
    assert plan.height == h and plan.width == w
    ones = torch.zeros(h, w, dtype=torch.float64)
    tiles = {}
    for i, j in plan.tiles():
        tiling.accumulate_tile(ones, torch.ones(plan.hs[i], plan.ws[j], dtype=torch.float64), plan, i, j)
        tiles[(i, j)] = torch.randn(plan.hs[i], plan.ws[j], generator=rng, dtype=torch.float64)
    assert torch.allclose(ones, torch.ones_like(ones), atol=1e-12)
    canvas = torch.zeros(h, w, dtype=torch.float64)
    for (i, j), t in tiles.items():
        tiling.accumulate_tile(canvas, t, plan, i, j)
    assert torch.allclose(canvas, tiling.blend_sequential(tiles, plan), atol=1e-12)


@pytest.mark.parametrize("seed", range(20))
def test_weighted_accumulation_matches_oracle_blend(seed):
    """The weighted per-tile accumulation (the product's blend, done on the device by
    h3b_blend_accumulate) against the oracle's restatement of the reference's blend + trim on
    random splits from the oracle's split_tiles."""
    import numpy as np
    from oracle import h3vae_oracle as O
    rng = np.random.default_rng(seed)
    tile = int(rng.integers(8, 96))
    ov = int(rng.integers(1, tile))
    h, w = int(rng.integers(tile + 1, 4 * tile)), int(rng.integers(1, 4 * tile))
    ys, hs, oys = O.split_tiles(h, tile, ov, 1)
    xs, ws, oxs = O.split_tiles(w, tile, ov, 1) if w > tile else ([0], [w], [])
    assert [list(ys), list(hs), list(oys)] == [list(v) for v in tiling.split_tiles(h, tile, ov, 1)]
    plan = tiling.TilePlan(tuple(ys), tuple(hs), tuple(oys), tuple(xs), tuple(ws), tuple(oxs))
    raw = [[rng.standard_normal((2, hs[i], ws[j])) for j in range(len(xs))] for i in range(len(ys))]
    ref = O.blend_tiles_sequential(raw, oys, oxs)
    canvas = torch.zeros(2, plan.height, plan.width, dtype=torch.float64)
    for i, j in plan.tiles():
        tiling.accumulate_tile(canvas, torch.from_numpy(raw[i][j]), plan, i, j)
    assert ref.shape == tuple(canvas.shape)
    assert np.allclose(canvas.numpy(), ref, atol=1e-12)
