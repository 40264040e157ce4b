"""The ``calibrate`` stage: measure the sm_100a plugin's NOT_MEASURED channel rates on the card
and record them as tempo/calib/2 records, which the plugin's machine table then loads as
MEASURED rates (the reference's calibration loop: tempo/core/calib/schema.py:1-33 for the
record, tools/probe.cu for its sm_70 measuring stand).

Probes (csrc/calib_probes.cu, one CTA per SM, clock64 periods):

  CAP.TMA_L2   cycles per byte of the bulk-copy feed into shared memory from an L2-resident
               buffer (16 MB), all SMs streaming at once -- the per-SM share the "sched"
               channel charges
  CAP.DEQ      cycles per element of the int8 -> fp16 shared-memory conversion by 4 warps
  CAP.EPI      cycles per byte of 16-byte fp16 stores by 4 warps (the epilogue's store side)
  LAT.TMA_L2   cycles per dependent L1-bypassing load from a ring inside L2
  LAT.HBM      cycles per dependent load from a ring of 1 GB (mostly L2 misses)

The HBM bulk feed (a 2 GB buffer) is recorded beside the binds as a cross-check of the
machine's CAP.HBM share (derived from the measured copy bandwidth), not bound.
"""
from __future__ import annotations

import datetime as _dt
import json
import os
import statistics
import subprocess

SYMBOL_UNITS = {"CAP.TMA_L2": "cycle/B", "CAP.DEQ": "cycle/element", "CAP.EPI": "cycle/B",
                "LAT.TMA_L2": "cycle", "LAT.HBM": "cycle"}


def foreign_processes(index: int) -> int:
    """Compute processes on GPU `index` other than this one (nvidia-smi); -1 when unknown."""
    try:
        out = subprocess.run(["nvidia-smi", "-i", str(index), "--query-compute-apps=pid",
                              "--format=csv,noheader"], capture_output=True, text=True,
                             timeout=30).stdout
    except (OSError, subprocess.TimeoutExpired):
        return -1
    pids = [int(x) for x in out.split() if x.strip().isdigit()]
    return sum(1 for p in pids if p != os.getpid())


def sm_clock(index: int) -> int:
    try:
        out = subprocess.run(["nvidia-smi", "-i", str(index), "--query-gpu=clocks.sm",
                              "--format=csv,noheader,nounits"], capture_output=True, text=True,
                             timeout=30).stdout.strip()
        return int(float(out.split()[0]))
    except (OSError, subprocess.TimeoutExpired, ValueError, IndexError):
        return 0


def _check(rc, what):
    if rc != 0:
        raise RuntimeError(f"{what}: CUDA error {rc}")


def _periods(t):
    v = [int(x) for x in t.cpu().tolist()]
    if any(x == (1 << 64) - 1 or x < 0 for x in v):
        raise RuntimeError("a probe's bounded wait gave up")
    return v


def chase_ring(torch, n_lines: int, dev, seed: int):
    """One random cycle through n_lines entries 128 bytes apart (one per cache line): entry
    i * 32 holds the index of the next; entry 0 is on the cycle (the probe starts there)."""
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    perm = torch.randperm(n_lines, generator=g, device=dev) * 32
    ring = torch.zeros(n_lines * 32, dtype=torch.int32, device=dev)
    ring[perm] = torch.roll(perm, -1).to(torch.int32)
    return ring


def run(dev_index: int = 0) -> dict:
    """Run every probe on GPU `dev_index`; returns the tempo/calib/2 record."""
    import torch

    from .. import _lib
    lib = _lib.load()
    dev = torch.device("cuda", dev_index)
    torch.cuda.set_device(dev)
    st = torch.cuda.current_stream(dev).cuda_stream
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    out = torch.zeros(2 * sms, dtype=torch.int64, device=dev)
    meas = {}

    # bulk feed from L2 (16 MB buffer, touched once first) and from HBM (2 GB)
    def feed(nbytes, chunks):
        buf = torch.ones(nbytes, dtype=torch.uint8, device=dev)
        _check(lib.tempo_sm100_probe_bulk_feed(buf.data_ptr(), nbytes, sms, 8, out.data_ptr(),
                                               st), "bulk feed warm-up")
        _check(lib.tempo_sm100_probe_bulk_feed(buf.data_ptr(), nbytes, sms, chunks,
                                               out.data_ptr(), st), "bulk feed")
        per = _periods(out[:sms])
        del buf
        return chunks * 32768 / statistics.median(per), chunks * 32768 / max(per)

    l2_med, l2_min = feed(16 << 20, 256)
    hbm_med, hbm_min = feed(2 << 30, 256)
    meas["bulk_feed_l2_B_per_cycle_per_sm"] = round(l2_med, 2)
    meas["bulk_feed_hbm_B_per_cycle_per_sm"] = round(hbm_med, 2)

    # dequant: 16 KB int8 tile, 4 warps, 64 conversions per CTA
    src = torch.randint(-127, 128, (16384,), dtype=torch.int8, device=dev)
    iters = 64
    _check(lib.tempo_sm100_probe_dequant(src.data_ptr(), sms, iters, out.data_ptr(), st),
           "dequant")
    deq = statistics.median(_periods(out[:sms])) / (iters * 16384.0)
    meas["dequant_cycles_per_element"] = round(deq, 4)

    # stores: 4 MB per CTA
    per_cta = 4 << 20
    dst = torch.empty(per_cta * sms, dtype=torch.uint8, device=dev)
    _check(lib.tempo_sm100_probe_store(dst.data_ptr(), per_cta, sms, out.data_ptr(), st),
           "store")
    epi = statistics.median(_periods(out[:sms])) / per_cta
    meas["store_cycles_per_byte"] = round(epi, 4)
    del dst

    # latency: ring of 8 MB (inside L2) and 1 GB
    def chase(nbytes, steps, seed):
        ring = chase_ring(torch, nbytes // 128, dev, seed)
        _check(lib.tempo_sm100_probe_chase(ring.data_ptr(), 2000, out.data_ptr(), st), "chase")
        _check(lib.tempo_sm100_probe_chase(ring.data_ptr(), steps, out.data_ptr(), st), "chase")
        c = int(out[0].item()) / steps
        del ring
        return c

    lat_l2 = chase(8 << 20, 20000, 1)
    lat_hbm = chase(1 << 30, 20000, 2)
    meas["latency_l2_cycles"] = round(lat_l2, 1)
    meas["latency_1GB_ring_cycles"] = round(lat_hbm, 1)

    props = torch.cuda.get_device_properties(dev)
    now = _dt.datetime.now(_dt.timezone.utc).strftime("%Y-%m-%dT%H:%M:%SZ")
    binds = [
        {"symbol": "CAP.TMA_L2", "value": 1.0 / l2_med,
         "note": f"{l2_med:.1f} B/cycle per SM, bulk copies into shared memory from a 16 MB "
                 f"L2-resident buffer, all {sms} SMs at once (slowest SM {l2_min:.1f})"},
        {"symbol": "CAP.DEQ", "value": deq,
         "note": f"{1.0 / deq:.1f} int8 -> fp16 elements per cycle per SM (4 warps, shared "
                 f"memory to shared memory, byte-permute conversion)"},
        {"symbol": "CAP.EPI", "value": epi,
         "note": f"{1.0 / epi:.1f} B/cycle per SM of 16-byte fp16 stores by 4 warps, all SMs"},
        {"symbol": "LAT.TMA_L2", "value": lat_l2,
         "note": "dependent L1-bypassing load from an 8 MB ring (L2 hit), one thread"},
        {"symbol": "LAT.HBM", "value": lat_hbm,
         "note": "dependent L1-bypassing load from a 1 GB ring (mostly L2 misses), one thread"},
    ]
    return {
        "schema": "tempo/calib/2",
        "id": "sm100_probe_channels",
        "kind": "rate",
        "plugin": "sm_100a",
        "quantity": "channel capacities and latencies of the sm_100a machine table",
        "units": "per bind: " + ", ".join(f"{k} {v}" for k, v in SYMBOL_UNITS.items()),
        "taken_with": {"tool": "csrc/calib_probes.cu via `tempo calibrate`",
                       "counter": "clock64 period per CTA (median over SMs)",
                       "version": lib.tempo_sm100_version().decode()},
        "shape": {"ctas": sms, "bulk_chunk_bytes": 32768, "bulk_ring": 4, "dequant_tile": 16384,
                  "store_bytes_per_cta": per_cta, "l2_ring_bytes": 8 << 20,
                  "hbm_ring_bytes": 1 << 30},
        "card": {"index": dev_index, "name": props.name, "clock_mhz": sm_clock(dev_index),
                 "foreign_procs": foreign_processes(dev_index)},
        "observability": "clean",
        "provenance": {"date": now, "who": "tempo calibrate",
                       "source": ["cuda_tempiler_b200/csrc/calib_probes.cu"]},
        "measured": meas,
        "binds": binds,
    }


def write(rec: dict, out_dir: str) -> str:
    from .core.calib.schema import validate
    validate(rec)
    os.makedirs(out_dir, exist_ok=True)
    path = os.path.join(out_dir, rec["id"] + ".json")
    with open(path, "w", encoding="utf-8") as f:
        json.dump(rec, f, indent=1, sort_keys=True)
    return path
