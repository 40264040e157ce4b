"""Measured search over the skeleton family's launch axes (the ``measure`` stage's engine).

For each problem (kind, M, N, K) every instantiated hyperform (bn, swap) is timed with the
k-split the run-time cost model picks and with no split, alternating with cuBLAS (torch
``F.linear`` on a dequantised copy for W8A16) in paired rounds; an L2 flush (a 256 MB write)
precedes every timed launch so weights come from HBM.  The result rows feed ``select.py`` /
``dispatch.inc`` generation.  Correctness is gated before the stopwatch: a hyperform whose
output misses relL2 <= 3e-3 against cuBLAS on the same inputs is recorded as FAILGATE and
never timed (reference discipline: tempo/core/measure/correctness.py:21-39).
"""
from __future__ import annotations

import json
import statistics
import sys

import torch

from . import ops
from ._lib import NotCovered

HYPER = {"swap": [16, 32, 64, 128], "noswap": [64, 128, 256], "swap_sdq": [32, 64, 128]}


def model_splits(kind, M, N, K, bn, swap):
    """The k-split the shipped run-time cycle model picks for this hyperform."""
    import importlib.util
    import os
    op = "gemm_fp16" if kind == 0 else "gemm_w8a16"
    p = os.path.join(os.path.dirname(os.path.abspath(__file__)), "kernels", "shipped", op,
                     "sm_100a", "select.py")
    spec = importlib.util.spec_from_file_location("tune_sel_" + op, p)
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m.choose_splits(M, N, K, bn, int(swap), 2 if kind == 0 else 1)


class L2Flush:
    """Evict L2 by READING a 256 MB buffer (written once at set-up): L2 ends up full of clean
    lines, so the timed kernel never pays for writing back someone else's dirty data."""

    def __init__(self, dev, nbytes=256 << 20):
        self.buf = torch.ones(nbytes // 4, dtype=torch.int32, device=dev)
        self.out = torch.empty((), dtype=torch.int64, device=dev)

    def __call__(self):
        self.out = self.buf.sum()


def time_paired(fa, fb, flush, rounds=7):
    """Median of per-round times (ms) of fa and fb, interleaved, each after an L2 flush."""
    ta, tb = [], []
    for _ in range(2):
        fa(); fb()
    for _ in range(rounds):
        for f, acc in ((fa, ta), (fb, tb)):
            flush()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            f()
            e1.record()
            torch.cuda.synchronize()
            acc.append(e0.elapsed_time(e1))
    return statistics.median(ta), statistics.median(tb)


def make_problem(kind, M, N, K, dev, g, group=128):
    A = torch.randn(M, K, generator=g, device=dev).half()
    if kind == 0:
        W = (torch.randn(N, K, generator=g, device=dev) * 0.02).half()
        return dict(A=A, W=W, scale=None, zero=None, group=0, Wref=W)
    if kind == 1:
        W = torch.randint(-127, 128, (N, K), generator=g, device=dev, dtype=torch.int8)
        s = (torch.rand(N, generator=g, device=dev) * 3e-4 + 1e-4).half()
        return dict(A=A, W=W, scale=s, zero=None, group=0,
                    Wref=(W.float() * s.float()[:, None]).half())
    W = torch.randint(0, 256, (N, K), generator=g, device=dev, dtype=torch.uint8)
    s = (torch.rand(K // group, N, generator=g, device=dev) * 0.019 + 1e-3).half()
    z = torch.randint(100, 157, (K // group, N), generator=g, device=dev, dtype=torch.uint8)
    Wd = ((W.float() - z.float().repeat_interleave(group, 0).T) * s.float().repeat_interleave(group, 0).T).half()
    return dict(A=A, W=W, scale=s, zero=z, group=group, Wref=Wd)


def tune_problem(kind, M, N, K, dev, flush, g, rounds=7, quick=False, kinds_bn=None):
    p = make_problem(kind, M, N, K, dev, g)
    ref = torch.nn.functional.linear(p["A"], p["Wref"])
    cublas = lambda: torch.nn.functional.linear(p["A"], p["Wref"])
    rows = []
    cands = [(bn, True) for bn in HYPER["swap"] if M <= 256 or kind != 0] + \
        [(bn, False) for bn in HYPER["noswap"]]
    if kind != 0:  # swapped 8-bit weights dequantised in shared memory (swap code 2)
        cands += [(bn, 2) for bn in HYPER["swap_sdq"]]
    if M <= 16:
        cands = [(0, False)] + cands  # the streaming GEMV
    if quick:  # only the tiles that can win at this M
        cands = [(bn, sw) for bn, sw in cands
                 if bn == 0 or (sw and bn >= min(M, 128) and bn <= max(16, 2 * M))
                 or (sw == 2 and bn >= min(M, 128) // 2 and bn <= max(32, 2 * M))
                 or (not sw and M >= 128)]
    pair = [(bn, sk) for bn in (256, 224, 192, 160, 128) for sk in (1, 2)] \
        if kind == 0 and M >= 512 else []
    for bn, sk in pair:
        f = lambda: ops.gemm_hyperform(p["A"], p["W"], bn=bn, swap=False, cta_group=2, group_m=16,
                                       splits=sk)
        try:
            out = f()
        except NotCovered:
            continue
        torch.cuda.synchronize()
        rel = ((out.float() - ref.float()).norm() / ref.float().norm()).item()
        if not rel <= 3e-3:
            rows.append(dict(bn=bn, swap=0, splits=sk, cg=2, status="FAILGATE", rel=rel))
            continue
        t, tc = time_paired(f, cublas, flush, rounds)
        rows.append(dict(bn=bn, swap=0, splits=sk, cg=2, us=t * 1e3, cublas_us=tc * 1e3,
                         x_cublas=tc / t, rel=rel, status="CAND"))
    for bn, swap in cands:
        model = ops.select(kind, M, N, K)
        rows_p, rows_q = (N, M) if swap else (M, N)
        tiles = -(-rows_p // 128) * -(-rows_q // max(bn, 1))
        splits_set = {1}
        if bn == 0:
            pass
        elif quick:
            # the run-time model's k-split for this hyperform
            splits_set.add(model_splits(kind, M, N, K, bn, swap))
        else:
            for s in (2, 3, 4, 6, 8):
                if tiles * s <= 4 * 148 and s <= K // 128:
                    splits_set.add(s)
        for splits in sorted(splits_set):
            f = lambda: ops.gemm_hyperform(p["A"], p["W"], bn=bn, swap=swap, splits=splits,
                                           scale=p["scale"], zero=p["zero"], group_size=p["group"])
            try:
                out = f()
            except NotCovered:
                continue
            torch.cuda.synchronize()
            rel = ((out.float() - ref.float()).norm() / ref.float().norm()).item()
            if not rel <= 3e-3:
                rows.append(dict(bn=bn, swap=int(swap), splits=splits, status="FAILGATE", rel=rel))
                continue
            t, tc = time_paired(f, cublas, flush, rounds)
            rows.append(dict(bn=bn, swap=int(swap), splits=splits, us=t * 1e3, cublas_us=tc * 1e3,
                             x_cublas=tc / t, rel=rel, status="CAND"))
    disp = lambda: (ops.gemm_fp16(p["A"], p["W"]) if kind == 0 else
                    ops.gemm_w8a16(p["A"], p["W"], p["scale"], p["zero"], p["group"]))
    td, tc = time_paired(disp, cublas, flush, rounds)
    ok = [r for r in rows if r["status"] == "CAND"]
    best = min(ok, key=lambda r: r["us"]) if ok else None
    return dict(kind=kind, M=M, N=N, K=K, rows=rows, best=best,
                dispatch=dict(us=td * 1e3, cublas_us=tc * 1e3, x_cublas=tc / td,
                              cfg=ops.select(kind, M, N, K)))


def main(argv=None):
    import argparse
    from . import workloads as WL
    ap = argparse.ArgumentParser()
    ap.add_argument("--set", default="fp16", choices=["fp16", "w8pc", "w8g", "all"])
    ap.add_argument("--ms", default=None, help="comma-separated M values")
    ap.add_argument("--rounds", type=int, default=5)
    ap.add_argument("--out", default=None)
    ap.add_argument("--quick", action="store_true", help="model k-split only, plausible tiles only")
    ap.add_argument("--budget-s", type=float, default=600.0, help="stop after this many seconds")
    ap.add_argument("--shapes", default=None, help="comma-separated shape names")
    a = ap.parse_args(argv)
    import time
    t_start = time.time()
    dev = torch.device("cuda", 0)
    flush = L2Flush(dev)
    g = torch.Generator(device=dev)
    g.manual_seed(11)
    sets = ["fp16", "w8pc", "w8g"] if a.set == "all" else [a.set]
    res = []
    for st in sets:
        kind = {"fp16": 0, "w8pc": 1, "w8g": 2}[st]
        shapes = WL.LAYER_FP16 if kind == 0 else WL.LAYER_W8
        ms = ([int(x) for x in a.ms.split(",")] if a.ms else
              list(WL.LAYER_FP16_M) if kind == 0 else
              list(WL.W8_PER_CHANNEL_M) if kind == 1 else list(WL.W8_GROUP_M))
        for s in shapes:
            if a.shapes and s.name not in a.shapes.split(","):
                continue
            for M in ms:
                if time.time() - t_start > a.budget_s:
                    print("time budget reached", flush=True)
                    break
                r = tune_problem(kind, M, s.N, s.K, dev, flush, g, a.rounds, a.quick)
                r["name"] = s.name
                res.append(r)
                b = r["best"]
                print(f"{st:5s} {s.name:8s} M={M:5d} best bn={b['bn']:3d} swap={b['swap']} "
                      f"splits={b['splits']} {b['us']:8.1f}us x{b['x_cublas']:.2f} | dispatch "
                      f"{r['dispatch']['us']:8.1f}us x{r['dispatch']['x_cublas']:.2f} {r['dispatch']['cfg']}",
                      flush=True)
    if a.out:
        with open(a.out, "w") as f:
            json.dump(res, f, indent=1)
    return 0


if __name__ == "__main__":
    sys.exit(main())
