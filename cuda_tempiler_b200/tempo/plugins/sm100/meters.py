"""Section 8b -- meters: Nsight Compute counter names per question, and a profile call that
runs ``ncu --clock-control none`` (never locking clocks).  This plugin never changes GPU
settings: ``clock_lock`` refuses."""
from __future__ import annotations

import csv
import io
import shutil
import subprocess
from pathlib import Path

from ..base import NotSupported

COUNTERS = {
    "time": ["gpu__time_duration.sum"],
    "tensor": ["sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_elapsed",
               "sm__inst_executed_pipe_tensor.sum"],
    "dram": ["dram__bytes_read.sum", "dram__bytes_write.sum",
             "gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed"],
    "l2": ["lts__throughput.avg.pct_of_peak_sustained_elapsed", "lts__t_sector_hit_rate.pct"],
    "tma": ["l1tex__m_xbar2l1tex_read_bytes.sum"],
    "occupancy": ["sm__warps_active.avg.pct_of_peak_sustained_active",
                  "launch__registers_per_thread"],
}


class Sm100Meters:
    def counters(self, kind: str):
        if kind not in COUNTERS:
            raise NotSupported(f"counter kind {kind!r}; known: {sorted(COUNTERS)}")
        return list(COUNTERS[kind])

    def profile(self, binary: Path, kernel: str, counters: list):
        ncu = shutil.which("ncu") or "/usr/local/cuda/bin/ncu"
        cmd = [ncu, "--clock-control", "none", "--csv", "--page", "raw", "-k", f"regex:{kernel}",
               "-c", "1", "--metrics", ",".join(counters), str(binary)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise NotSupported(f"ncu failed ({r.returncode}): {r.stderr[-300:]}")
        rows = [row for row in csv.reader(io.StringIO(r.stdout)) if row]
        head = next((i for i, row in enumerate(rows) if "Kernel Name" in row or "ID" in row), None)
        if head is None or head + 2 >= len(rows):
            return {}
        names, values = rows[head], rows[head + 2]
        out = {}
        for n, v in zip(names, values):
            if n in counters:
                try:
                    out[n] = float(v.replace(",", ""))
                except ValueError:
                    pass
        return out

    def clock_lock(self, card: int, mhz: int):
        raise NotSupported("GPU clocks are never locked or changed by this plugin; clocks are "
                           "sampled during the timed region instead")
