"""Section 1 -- the machine: NVIDIA B200 (sm_100a).

Structural facts (SM count, shared memory, TMEM, register file) are architectural constants
(status SPEC: never allowed in a time bound).  Time-bound capacities are derived from the
MEASURED peaks in data/rates.json (copy bandwidth and dense tensor throughput measured on this
pool's B200s with the card state recorded), converted to per-SM, per-cycle capacities at the
measured under-load clock; the shared-memory read port is an UPPER_BOUND (architectural
128 B/cycle/SM).  Channels use scope "sched": capacity = cycles per unit of load, the
skeleton's atoms carry whole-launch loads for the busiest SM, so the bound is in cycles.
"""
from __future__ import annotations

import json
import os

from ..base import (CardState, Channel, Provenance, Rate, UnknownSymbol, closed_table_get,
                    not_measured, rate)

_HERE = os.path.dirname(os.path.abspath(__file__))
ARCH = "sm_100a"


def _load_measured():
    with open(os.path.join(_HERE, "data", "rates.json"), encoding="utf-8") as f:
        doc = json.load(f)
    c = doc["card"]
    card = CardState(index=c["index"], clock_mhz=int(c["clock_mhz"]),
                     foreign_procs=int(c["foreign_procs"]), date=c["date"])
    out = {}
    for sym, r in doc["rates"].items():
        prov = Provenance(tool=r["tool"], counter=None, version="1", date=c["date"],
                          who="build driver", observability="clean", card=card)
        out[sym] = Rate(sym, float(r["value"]), r["units"], "MEASURED", prov, doc["source"])
    return out, card


CALIB_DIR = os.path.join(_HERE, "data", "calib")


def _apply_calibration(table):
    """Measured channel rates from the ``calibrate`` stage (tempo/calib/2 records under
    data/calib/) replace NOT_MEASURED / UPPER_BOUND entries.  Inside the reference's tree,
    whose calibration loader has another interface, the plugin keeps its own table."""
    try:
        from ...core.calib.load import apply, load_dir
    except ImportError:
        return table, []
    if not os.path.isdir(CALIB_DIR):
        return table, []
    recs = load_dir(CALIB_DIR, ARCH)
    return apply(table, recs, ARCH), [r["id"] for r in recs]


class Sm100Machine:
    SMS = 148
    SCHEDULERS = 4
    WARP_SLOTS = 64
    WARP = 32
    SMEM_PER_SM = 233472       # 228 KB
    SMEM_PER_CTA = 232448      # 227 KB opt-in maximum
    REGFILE_WORDS = 65536
    TMEM_COLS = 512            # x 128 lanes x 32 bit = 256 KB
    CLOCK_MAX_MHZ = 1965.0
    SMEM_BYTES_PER_CYCLE = 128.0

    def __init__(self):
        self._measured, self.card = _load_measured()
        m = self._measured
        clk = m["CLOCK.SM_UNDER_LOAD"].value * 1e6
        derived_prov = lambda sym: Provenance(tool="derived from " + sym, counter=None,
                                              version="1", date=self.card.date, who="plugin",
                                              observability="derived", card=self.card)
        umma_flop_per_cycle = m["PEAK.TENSOR_DENSE_F16_SUSTAINED"].value * 1e12 / (self.SMS * clk)
        hbm_b_per_cycle = m["PEAK.HBM_COPY"].value * 1e9 / (self.SMS * clk)
        t = {
            "SMS": rate("SMS", self.SMS, "SM", "SPEC"),
            "SCHEDULERS_PER_SM": rate("SCHEDULERS_PER_SM", self.SCHEDULERS, "scheduler", "SPEC"),
            "WARP_SLOTS_PER_SM": rate("WARP_SLOTS_PER_SM", self.WARP_SLOTS, "warp", "SPEC"),
            "THREADS_PER_WARP": rate("THREADS_PER_WARP", self.WARP, "thread", "SPEC"),
            "SMEM_PER_SM": rate("SMEM_PER_SM", self.SMEM_PER_SM, "B", "SPEC"),
            "SMEM_PER_CTA_MAX": rate("SMEM_PER_CTA_MAX", self.SMEM_PER_CTA, "B", "SPEC"),
            "REGFILE_WORDS_PER_SM": rate("REGFILE_WORDS_PER_SM", self.REGFILE_WORDS, "word", "SPEC"),
            "TMEM_COLS_PER_SM": rate("TMEM_COLS_PER_SM", self.TMEM_COLS, "column", "SPEC",
                                     note="128 lanes x 512 columns x 32 bit"),
            "CLOCK_MAX_MHZ": rate("CLOCK_MAX_MHZ", self.CLOCK_MAX_MHZ, "MHz", "SPEC"),
            "CAP.UMMA": Rate("CAP.UMMA", 1.0 / umma_flop_per_cycle, "cycle/FLOP", "MEASURED",
                             derived_prov("PEAK.TENSOR_DENSE_F16_SUSTAINED"),
                             f"{umma_flop_per_cycle:.0f} FLOP/cycle/SM at the under-load clock"),
            "CAP.HBM": Rate("CAP.HBM", 1.0 / hbm_b_per_cycle, "cycle/B", "MEASURED",
                            derived_prov("PEAK.HBM_COPY"),
                            f"{hbm_b_per_cycle:.1f} B/cycle per SM share of the copy bandwidth"),
            "CAP.SMEM_RD": rate("CAP.SMEM_RD", 1.0 / self.SMEM_BYTES_PER_CYCLE, "cycle/B",
                                "UPPER_BOUND", "architectural 128 B/cycle/SM shared-memory port"),
            "CAP.TMA_L2": not_measured("CAP.TMA_L2", "cycle/B", "L2 -> SM TMA feed per SM"),
            "CAP.EPI": not_measured("CAP.EPI", "cycle/B", "TMEM -> register -> global epilogue"),
            "CAP.DEQ": not_measured("CAP.DEQ", "cycle/element", "int8/uint8 -> fp16 smem dequant"),
            "LAT.TMA_L2": not_measured("LAT.TMA_L2", "cycle"),
            "LAT.HBM": not_measured("LAT.HBM", "cycle"),
            "LAT.UMMA_128x256x16": not_measured("LAT.UMMA_128x256x16", "cycle"),
        }
        t.update(self._measured)
        t, self.calibration = _apply_calibration(t)
        self._table = t
        self._channels = {
            "UMMA": Channel("UMMA", "sched", t["CAP.UMMA"]),
            "HBM": Channel("HBM", "sched", t["CAP.HBM"]),
            "SMEM_RD": Channel("SMEM_RD", "sched", t["CAP.SMEM_RD"]),
            "TMA_L2": Channel("TMA_L2", "sched", t["CAP.TMA_L2"]),
            "EPI": Channel("EPI", "sched", t["CAP.EPI"]),
            "DEQ": Channel("DEQ", "sched", t["CAP.DEQ"]),
        }

    def arch(self):
        return ARCH

    def symbols(self):
        return dict(self._table)

    def channels(self):
        return dict(self._channels)

    def latency(self, atom_class: str) -> Rate:
        return closed_table_get(self._table, "LAT." + atom_class)

    def sms(self):
        return self._table["SMS"]

    def schedulers_per_sm(self):
        return self._table["SCHEDULERS_PER_SM"]

    def warp_slots_per_sm(self):
        return self._table["WARP_SLOTS_PER_SM"]

    def threads_per_warp(self):
        return self._table["THREADS_PER_WARP"]

    def smem_per_sm(self):
        return self._table["SMEM_PER_SM"]

    def smem_per_cta_max(self):
        return self._table["SMEM_PER_CTA_MAX"]

    def regfile_words_per_sm(self):
        return self._table["REGFILE_WORDS_PER_SM"]

    def clock_mhz(self):
        return self._table["CLOCK.SM_UNDER_LOAD"]

    def peak(self, kind: str) -> Rate:
        key = {"tensor_dense": "PEAK.TENSOR_DENSE_F16", "tensor_dense_sustained":
               "PEAK.TENSOR_DENSE_F16_SUSTAINED", "hbm_copy": "PEAK.HBM_COPY",
               "hbm_read": "PEAK.HBM_COPY"}.get(kind)
        if key is None:
            raise UnknownSymbol(f"peak kind {kind!r} is not declared")
        return self._table[key]
