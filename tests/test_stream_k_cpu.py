"""The 2-CTA kernel's work split (whole tiles, then a split tail), restated in Python and
checked over a sweep of shapes: each k-block of each tile is computed by exactly one unit,
a tail tile's k-slices are contiguous and in k order, partial slots are distinct and inside
the workspace the planner sizes, and the k-slice-major numbering keeps one wave's clusters on
at most two neighbouring k-slices.

The restatement follows pair_plan (skeletons/gemm_sm100/launch.cuh) and PairSegIter
(skeletons/gemm_sm100/kernel.cuh) step for step, and the shipped select.py carries the same
plan (checked equal here); the GPU tests check the compiled code's results against the
oracle on shapes from each regime."""
import importlib.util
import math
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def plan(M, N, K, bn, sms=148):
    tiles = -(-M // 256) * -(-N // bn)
    num_kb = -(-K // 64)
    P = sms // 2
    out = dict(tiles=tiles, num_kb=num_kb, clusters=min(tiles, P), sk_tile0=tiles, sk_tiles=0,
               sk_splits=0, cost=float(-(-tiles // P)))
    if tiles % P == 0:
        return out
    R = tiles % P if tiles >= P else tiles
    full = (tiles - R) // P
    best, best_s = out["cost"] * 0.97, 0
    for S in range(2, 17):
        if S * 4 > num_kb or R * S > 3 * P:
            break
        c = full + math.ceil(R * S / P) / S + S * 20000.0 / (num_kb * 2.0 * bn)
        if c < best:
            best, best_s = c, S
    if best_s:
        out.update(clusters=P, sk_tile0=tiles - R, sk_tiles=R, sk_splits=best_s, cost=best)
    return out


def units(pl, c):
    t = c
    while t < pl["sk_tile0"]:
        yield dict(tile=t, kb0=0, kb1=pl["num_kb"], slot=0, contrib=1, t=0)
        t += pl["clusters"]
    if not pl["sk_splits"]:
        return
    u = c
    while u < pl["sk_tiles"] * pl["sk_splits"]:
        sl = u // pl["sk_tiles"]
        tt = u - sl * pl["sk_tiles"]
        yield dict(tile=pl["sk_tile0"] + tt, kb0=pl["num_kb"] * sl // pl["sk_splits"],
                   kb1=pl["num_kb"] * (sl + 1) // pl["sk_splits"], slot=sl,
                   contrib=pl["sk_splits"], t=tt, u=u)
        u += pl["clusters"]


SHAPES = [(M, N, K) for M in (256, 512, 1000, 1024, 2048, 4096, 8192)
          for N in (136, 1000, 3840, 8192, 15360, 30720) for K in (64, 1000, 4096, 15360)]


def _check_sweep(bn):
    n_tail = 0
    for M, N, K in SHAPES:
        pl = plan(M, N, K, bn)
        seen = set()
        slots = set()
        for c in range(pl["clusters"]):
            for s in units(pl, c):
                assert 0 <= s["kb0"] < s["kb1"] <= pl["num_kb"], (M, N, K, s)
                for kb in range(s["kb0"], s["kb1"]):
                    assert (s["tile"], kb) not in seen, (M, N, K, s)
                    seen.add((s["tile"], kb))
                if s["contrib"] > 1:
                    slot = s["slot"] * pl["sk_tiles"] + s["t"]
                    assert slot < pl["sk_tiles"] * pl["sk_splits"] and slot not in slots
                    slots.add(slot)
        assert len(seen) == pl["tiles"] * pl["num_kb"], (M, N, K)
        if pl["sk_splits"]:
            n_tail += 1
            assert pl["sk_tiles"] * pl["sk_splits"] <= 3 * (148 // 2)
            # one wave of tail units spans at most two neighbouring k-slices
            P = pl["clusters"]
            for w in range(0, pl["sk_tiles"] * pl["sk_splits"], P):
                sl = {u // pl["sk_tiles"] for u in range(w, min(w + P, pl["sk_tiles"] * pl["sk_splits"]))}
                assert max(sl) - min(sl) <= 1 + P // max(1, pl["sk_tiles"])
    return n_tail


@pytest.mark.parametrize("bn", [128, 160, 192, 224, 256])
def test_split_tail_covers_every_k_block_once(bn):
    _check_sweep(bn)


def test_sweep_exercises_the_split_tail():
    assert sum(_check_sweep(bn) for bn in (224, 256)) > 10


def test_split_tail_only_for_ragged_waves():
    assert plan(4096, 30720, 3840, 256)["sk_splits"] == 0   # 1920 tiles: 25.9 waves, kept
    pl = plan(4096, 3840, 15360, 256)                      # 240 tiles: 3.24 waves
    assert (pl["sk_tile0"], pl["sk_tiles"], pl["sk_splits"]) == (222, 18, 3)
    # 30 tiles < 74 clusters with 64 k-blocks each: at the measured fix-up cost (~20000 cycles
    # per slice) no cut pays; one whole wave
    assert plan(512, 3840, 4096, 256)["sk_splits"] == 0
    assert plan(1024, 3840, 15360, 256)["sk_splits"] == 0   # 60 tiles: no cut gains 3 %


def test_shipped_select_mirrors_the_plan():
    p = os.path.join(ROOT, "cuda_tempiler_b200", "kernels", "shipped", "gemm_fp16", "sm_100a",
                     "select.py")
    spec = importlib.util.spec_from_file_location("tempo_select_fp16", p)
    sel = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(sel)
    for M, N, K in SHAPES:
        for bn in (256, 224, 128):
            cost, R, S = sel.pair_plan(M, N, K, bn)
            pl = plan(M, N, K, bn)
            assert (R, S) == (pl["sk_tiles"], pl["sk_splits"]) and abs(cost - pl["cost"]) < 1e-9
