"""The 2-CTA kernel's stream-K work split, restated in Python and checked for every shape of
a sweep: each k-block of each tile is computed by exactly one cluster, the clusters sharing a
tile see the same contributor count, their partial slots are distinct, consecutive per tile and
inside the workspace the planner sizes, and no cluster's run is shorter than the minimum.

The restatement follows pair_plan (skeletons/gemm_sm100/launch.cuh) and PairSegIter
(skeletons/gemm_sm100/kernel.cuh) step for step; the GPU tests check the compiled code's
results against the oracle on shapes from each regime."""
import math

import pytest

MIN_RUN = 8  # kPairMinSkRun


def plan(M, N, K, bn, sms=148):
    tiles = -(-M // 256) * -(-N // bn)
    num_kb = -(-K // 64)
    P = sms // 2
    out = dict(tiles=tiles, num_kb=num_kb, clusters=min(tiles, P), sk_tile0=tiles, sk_clusters=0,
               sk_iters=0, slots=0)
    if tiles % P == 0:
        return out
    waves = tiles / P
    if math.ceil(waves) - waves < 0.15:
        return out
    full = tiles // P
    sk_tiles = tiles % P + (P if full >= 1 else 0)
    iters = sk_tiles * num_kb
    out.update(clusters=P, sk_tile0=tiles - sk_tiles, sk_iters=iters,
               sk_clusters=max(1, min(P, iters // MIN_RUN)))
    out["slots"] = sk_tiles + out["sk_clusters"]
    return out


def owner(pl, i):
    return ((i + 1) * pl["sk_clusters"] - 1) // pl["sk_iters"]


def segments(pl, c):
    t = c
    while t < pl["sk_tile0"]:
        yield dict(tile=t, kb0=0, kb1=pl["num_kb"], slot=0, contrib=1, slot0=0)
        t += pl["clusters"]
    if c >= pl["sk_clusters"]:
        return
    it = pl["sk_iters"] * c // pl["sk_clusters"]
    end = pl["sk_iters"] * (c + 1) // pl["sk_clusters"]
    nkb = pl["num_kb"]
    while it < end:
        tt = it // nkb
        kb0 = it - tt * nkb
        kb1 = min(nkb, kb0 + (end - it))
        cf, cl = owner(pl, tt * nkb), owner(pl, tt * nkb + nkb - 1)
        yield dict(tile=pl["sk_tile0"] + tt, kb0=kb0, kb1=kb1, slot=owner(pl, it) - cf,
                   contrib=cl - cf + 1, slot0=tt + cf)
        it += kb1 - kb0


SHAPES = [(M, N, K) for M in (256, 1000, 1024, 2048, 4096, 8192)
          for N in (136, 1000, 3840, 8192, 15360) for K in (64, 1000, 4096, 15360)]


@pytest.mark.parametrize("bn", [128, 256])
def test_stream_k_split_covers_every_k_block_once(bn):
    n_sk = 0
    for M, N, K in SHAPES:
        pl = plan(M, N, K, bn)
        seen = {}
        slots = {}
        for c in range(pl["clusters"]):
            runs = 0
            for s in segments(pl, c):
                assert 0 <= s["kb0"] < s["kb1"] <= pl["num_kb"]
                for kb in range(s["kb0"], s["kb1"]):
                    key = (s["tile"], kb)
                    assert key not in seen, (M, N, K, key)
                    seen[key] = c
                if s["tile"] >= pl["sk_tile0"]:
                    runs += s["kb1"] - s["kb0"]
                    if s["contrib"] > 1:
                        slot = s["slot0"] + s["slot"]
                        assert 0 <= s["slot"] < s["contrib"]
                        assert slot < pl["slots"]
                        assert slot not in slots, (M, N, K, slot)
                        slots[slot] = (s["tile"], s["contrib"], s["slot0"])
            if c < pl["sk_clusters"] and pl["sk_iters"] >= MIN_RUN:
                assert runs >= MIN_RUN
        assert len(seen) == pl["tiles"] * pl["num_kb"], (M, N, K)
        # every shared tile has exactly `contrib` pieces, in consecutive slots from slot0
        per_tile = {}
        for slot, (t, contrib, slot0) in slots.items():
            per_tile.setdefault(t, []).append((slot, contrib, slot0))
        for t, lst in per_tile.items():
            contrib, slot0 = lst[0][1], lst[0][2]
            assert all(x[1] == contrib and x[2] == slot0 for x in lst)
            assert sorted(x[0] for x in lst) == list(range(slot0, slot0 + contrib))
        n_sk += pl["sk_clusters"] > 0
    assert n_sk > 10  # the sweep exercises the stream-K region


def test_stream_k_only_for_ragged_waves():
    assert plan(4096, 30720, 3840, 256)["sk_clusters"] == 0   # 1920 tiles: 25.9 waves
    assert plan(4096, 3840, 15360, 256)["sk_clusters"] == 74  # 240 tiles: 3.24 waves
    pl = plan(4096, 3840, 15360, 256)
    assert pl["sk_tile0"] == 240 - (240 % 74) - 74
    assert plan(1024, 3840, 15360, 256)["sk_tile0"] == 0      # 60 tiles < 74 clusters
