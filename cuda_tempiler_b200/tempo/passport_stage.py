"""The passport of a ship directory, taken on a GPU: the card it was gated on and the gate
over every production point of BASELINE's configurations.

The reference's shipped manifest carries a ``card`` (index, name, clock, foreign processes
before and after) and a ``gate`` summary (kernels/shipped/gemm_fp16/sm_70/manifest.json:107-126),
and its report refuses measured numbers without a card (tempo/core/report/provenance.py:25-48).
``passport()`` gathers both for the shipped dispatch of this library:

* card: device index and name, the SM clock sampled while the gate runs (median, max), the
  driver's max clock, and the number of other processes on the GPU before and after;
* gate, per op: every (shape, M) of the op's configurations through the public dispatcher
  with the output poisoned (0x7f7f), coverage, relL2 against an fp32-accumulated product of
  the same fp16 / dequantised inputs (<= 3e-3, the BASELINE gate) and relL2 of 256 sampled
  cells against an fp64 product (the independent path).

``ship --passport FILE`` writes the result into each manifest.
"""
from __future__ import annotations

import datetime as _dt
import json
import os
import statistics
import subprocess
import threading
import time

GATE = 3e-3

FP16_SHAPES = [("qkv", 8192, 3840), ("o_proj", 3840, 4096), ("gate_up", 30720, 3840),
               ("down", 3840, 15360)]
FP16_M = [1, 16, 128, 1024, 4096]
W8_SHAPES = [("qkv", 10240, 5120), ("o_proj", 5120, 8192), ("gate_up", 34816, 5120),
             ("down", 5120, 17408)]
W8_PC_M = [1, 2, 4, 8, 16, 64, 512]
W8_GRP_M = [1, 16, 256, 4096]


def _smi(args):
    try:
        return subprocess.run(["nvidia-smi", *args], capture_output=True, text=True,
                              timeout=15).stdout
    except (OSError, subprocess.TimeoutExpired):
        return ""


def foreign_procs(index: int) -> int:
    out = _smi(["-i", str(index), "--query-compute-apps=pid", "--format=csv,noheader"])
    own = os.getpid()
    return sum(1 for line in out.splitlines() if line.strip() and int(line.strip()) != own)


class _Clocks:
    def __init__(self, index):
        self.index, self.samples, self._stop = index, [], threading.Event()
        self._t = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        while not self._stop.is_set():
            out = _smi(["-i", str(self.index), "--query-gpu=clocks.sm", "--format=csv,noheader,nounits"])
            try:
                self.samples.append(float(out.strip().splitlines()[0]))
            except (ValueError, IndexError):
                pass
            time.sleep(0.2)

    def __enter__(self):
        self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        self._t.join(timeout=5)


def _gate_point(torch, run, A, Wf):
    """(relL2 vs fp32, relL2 of 256 cells vs fp64, uncovered cells) for one launch."""
    C = run()
    torch.cuda.synchronize()
    uncovered = int((C.view(torch.int16) == 0x7F7F).sum().item())
    ref = A.float() @ Wf.t()
    rel = float(((C.float() - ref).norm() / ref.norm()).item())
    g = torch.Generator(device=A.device).manual_seed(11)
    ms = torch.randint(0, A.shape[0], (256,), generator=g, device=A.device)
    ns = torch.randint(0, Wf.shape[0], (256,), generator=g, device=A.device)
    ref64 = (A[ms].double() * Wf[ns].double()).sum(1)
    got = C[ms, ns].double()
    spot = float(((got - ref64).norm() / ref64.norm()).item())
    return rel, spot, uncovered


def _poisoned(torch, M, N, dev):
    C = torch.empty(M, N, dtype=torch.float16, device=dev)
    C.view(torch.int16).fill_(0x7F7F)
    return C


def passport(index: int = 0) -> dict:
    import torch

    from .. import ops
    dev = torch.device("cuda", index)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev)
    g.manual_seed(2024)
    before = foreign_procs(index)
    gates = {}
    with _Clocks(index) as clocks:
        rows = []
        for name, N, K in FP16_SHAPES:
            W = (torch.randn(N, K, generator=g, device=dev) * 0.02).half()
            Wf = W.float()
            for M in FP16_M:
                A = torch.randn(M, K, generator=g, device=dev).half()
                rel, spot, unc = _gate_point(
                    torch, lambda: ops.gemm_fp16(A, W, out=_poisoned(torch, M, N, dev)), A, Wf)
                rows.append(dict(gemm=name, M=M, N=N, K=K, rel_l2=rel, spot_fp64=spot,
                                 uncovered=unc, sel=ops.select(0, M, N, K)))
            del W, Wf
        gates["gemm_fp16"] = rows
        rows = []
        for kind, ms in ((1, W8_PC_M), (2, W8_GRP_M)):
            for name, N, K in W8_SHAPES:
                if kind == 1:
                    W = torch.randint(-127, 128, (N, K), generator=g, device=dev, dtype=torch.int8)
                    s = (torch.rand(N, generator=g, device=dev) * 2e-4 + 5e-5).half()
                    z, G = None, 0
                    Wf = W.float() * s.float()[:, None]
                else:
                    G = 128
                    W = torch.randint(0, 256, (N, K), generator=g, device=dev, dtype=torch.uint8)
                    s = (torch.rand(K // G, N, generator=g, device=dev) * 0.019 + 1e-3).half()
                    z = torch.randint(100, 157, (K // G, N), generator=g, device=dev,
                                      dtype=torch.uint8)
                    Wf = (W.float() - z.float().repeat_interleave(G, 0).t()) * \
                        s.float().repeat_interleave(G, 0).t()
                for M in ms:
                    A = torch.randn(M, K, generator=g, device=dev).half()
                    rel, spot, unc = _gate_point(
                        torch, lambda: ops.gemm_w8a16(A, W, s, z, G,
                                                      out=_poisoned(torch, M, N, dev)), A, Wf)
                    rows.append(dict(gemm=name, scale="per_channel" if kind == 1 else "group:128",
                                     M=M, N=N, K=K, rel_l2=rel, spot_fp64=spot, uncovered=unc,
                                     sel=ops.select(kind, M, N, K)))
                del W, Wf
                torch.cuda.empty_cache()
        gates["gemm_w8a16"] = rows
    status = ops.device_status()
    after = foreign_procs(index)
    name = _smi(["-i", str(index), "--query-gpu=name", "--format=csv,noheader"]).strip()
    maxclk = _smi(["-i", str(index), "--query-gpu=clocks.max.sm", "--format=csv,noheader,nounits"])
    card = {"index": index, "name": name or torch.cuda.get_device_name(dev),
            "sm_clock_mhz_median": statistics.median(clocks.samples) if clocks.samples else None,
            "sm_clock_mhz_max_seen": max(clocks.samples) if clocks.samples else None,
            "sm_clock_mhz_max": float(maxclk.strip()) if maxclk.strip() else None,
            "clock_locked": False, "foreign_procs_before": before, "foreign_procs_after": after,
            "device_status": status,
            "date": _dt.datetime.now(_dt.timezone.utc).strftime("%Y-%m-%dT%H:%M:%SZ")}
    out = {"schema": "tempo/passport/1", "card": card, "gate": {}}
    for op, rows in gates.items():
        ok = [r for r in rows if r["rel_l2"] <= GATE and r["spot_fp64"] <= GATE
              and r["uncovered"] == 0]
        out["gate"][op] = {
            "tolerance_rel_l2": GATE, "points": len(rows), "passed": len(ok),
            "max_rel_l2": max(r["rel_l2"] for r in rows),
            "max_spot_fp64_rel_l2": max(r["spot_fp64"] for r in rows),
            "uncovered_cells": sum(r["uncovered"] for r in rows),
            "reference": "fp32-accumulated product of the same fp16 / dequantised inputs on the "
                         "device; fp64 on 256 sampled cells; output poisoned with 0x7f7f",
            "rows": rows}
    return out


def main(out_path: str | None, index: int = 0) -> int:
    import torch
    if not torch.cuda.is_available():
        print("passport needs a GPU")
        return 2
    p = passport(index)
    text = json.dumps(p, indent=1, sort_keys=True)
    if out_path:
        with open(out_path, "w") as f:
            f.write(text)
    for op, gt in p["gate"].items():
        print(f"{op}: {gt['passed']}/{gt['points']} points pass, max relL2 {gt['max_rel_l2']:.2e}")
    print("card:", json.dumps(p["card"]))
    return 0 if all(g["passed"] == g["points"] for g in p["gate"].values()) else 1
