"""The measure stage on a GPU: correctness gate before the stopwatch (relL2 against an
fp32-accumulated reference + coverage by poison fill + an independent fp64 spot check), then
paired interleaved timing against the two mandatory bars -- the naive INPUT kernel and cuBLAS
(torch F.linear) -- reported as medians of per-round ratios (reference
tempo/core/measure/{correctness,ratio,baseline}.py, harness.cu:214-250)."""
from __future__ import annotations

import statistics

from .core.measure.baseline import Baseline, Comparison
from .core.measure.correctness import must_pass_before_timing
from .core.measure.ratio import median_ci, median_ratio
from .core.op.coverage import Coverage
from .core.op.oracle import OracleResult
from .core.report import Report
from .plugins.base import CardState


def _card(torch):
    import datetime
    import subprocess
    mhz = 0
    try:
        out = subprocess.run(["nvidia-smi", "-i", "0", "--query-gpu=clocks.sm", "--format=csv,noheader,nounits"],
                             capture_output=True, text=True, timeout=10).stdout.strip()
        mhz = int(float(out.splitlines()[0]))
    except Exception:
        pass
    procs = 0
    try:
        out = subprocess.run(["nvidia-smi", "--query-compute-apps=pid", "--format=csv,noheader"],
                             capture_output=True, text=True, timeout=10).stdout
        import os
        procs = len([l for l in out.splitlines() if l.strip() and int(l.strip()) != os.getpid()])
    except Exception:
        pass
    return CardState(index=0, clock_mhz=mhz, foreign_procs=procs,
                     date=datetime.datetime.now(datetime.timezone.utc).isoformat(timespec="seconds"))


def measure(plugin, op, rounds: int = 9) -> int:
    import torch

    from .. import ops
    from ..tune import L2Flush, make_problem
    if not torch.cuda.is_available():
        print("measure needs a GPU")
        return 2
    dev = torch.device("cuda", 0)
    s = op.shapes
    M, N, K = s["M"], s["N"], s["K"]
    kind = {"fp16": 0, "int8": 1, "uint8": 2}[op.dtype_b]
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    p = make_problem(kind, M, N, K, dev, g)
    ours = (lambda: ops.gemm_fp16(p["A"], p["W"])) if kind == 0 else \
        (lambda: ops.gemm_w8a16(p["A"], p["W"], p["scale"], p["zero"], p["group"]))
    lib = lambda: torch.nn.functional.linear(p["A"], p["Wref"])
    naive = (lambda: ops.naive_gemm_fp16(p["A"], p["W"])) if kind == 0 else \
        (lambda: ops.naive_gemm_w8a16(p["A"], p["W"], p["scale"], p["zero"], p["group"]))
    # ---- gate before the stopwatch
    out = torch.empty(M, N, dtype=torch.float16, device=dev)
    out.view(torch.int16).fill_(0x7F7F)
    if kind == 0:
        ops.gemm_fp16(p["A"], p["W"], out=out)
    else:
        ops.gemm_w8a16(p["A"], p["W"], p["scale"], p["zero"], p["group"], out=out)
    ref = p["A"].float() @ p["Wref"].float().T
    rel = ((out.float() - ref).norm() / ref.norm()).item()
    zero = int((out.view(torch.int16) == 0x7F7F).sum().item())
    idx_m = torch.randint(0, M, (2048,), generator=g, device=dev)
    idx_n = torch.randint(0, N, (2048,), generator=g, device=dev)
    spot_ref = (p["A"][idx_m].double() * p["Wref"][idx_n].double()).sum(1)
    spot_got = out[idx_m, idx_n].double()
    spot = ((spot_got - spot_ref).norm() / spot_ref.norm()).item()
    res = OracleResult(rel_l2=rel, tol=op.tol_rel_l2 or 3e-3,
                       coverage=Coverage(total=M * N, zero=zero, over=0, max_hits=1),
                       independent_rel_l2=spot,
                       independent_path="fp64 dot products on 2048 sampled cells (no tensor cores)")
    print(res.render())
    must_pass_before_timing(res)
    # ---- paired interleaved rounds, L2 flushed before every timed launch
    flush = L2Flush(dev)
    arms = {"ours": ours, "cublas": lib, "naive": naive}
    times = {k: [] for k in arms}
    for f in arms.values():
        f()
    torch.cuda.synchronize()
    for _ in range(rounds):
        for k, f in arms.items():
            flush()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            f()
            e1.record()
            torch.cuda.synchronize()
            times[k].append(e0.elapsed_time(e1))
    rep = Report(title=f"measure {op.kind} {M}x{N}x{K} {op.dtype_a}*{op.dtype_b} on {plugin.id}",
                 plugin_id=plugin.id, card=_card(torch))
    for k, kind_b, what in (("naive", "INPUT", "one thread per output, fp32 accumulate"),
                            ("cublas", "LIBRARY", "torch F.linear (cuBLAS) on dequantised fp16 weights")):
        pairs = list(zip(times[k], times["ours"]))
        ratios = [a / b for a, b in pairs]
        rep.compare(Comparison(Baseline(kind_b, k, what), median_ratio(pairs), median_ci(ratios),
                               rounds))
    t = statistics.median(times["ours"]) * 1e-3
    sec = rep.section("THROUGHPUT (median of rounds, L2 flushed)")
    sec.add(f"ours {t * 1e6:.1f} us: {2 * M * N * K / t / 1e12:.1f} TFLOP/s, "
            f"{(2 * M * K + (2 if kind == 0 else 1) * N * K + 2 * M * N) / t / 1e9:.0f} GB/s")
    sec.add(f"dispatch: {ops.select(kind, M, N, K)}")
    print(rep.render())
    return 0
