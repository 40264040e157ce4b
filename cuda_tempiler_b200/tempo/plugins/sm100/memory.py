"""Section 2 -- memory: HBM3e, L2, shared memory (32 banks x 4 B) and TMEM.

Operand tiles are staged by TMA with the 128-byte swizzle (bank-conflict free by
construction), so padding is never needed: ``pad_family`` yields 0 only.
"""
from __future__ import annotations

from ..base import Layout, MemLevel, WavefrontCost, not_measured, rate


class Sm100Memory:
    BANKS = 32
    BANK_BYTES = 4

    def __init__(self, machine):
        self.m = machine

    def levels(self):
        t = self.m.symbols()
        return (
            MemLevel("HBM3e", rate("HBM.BYTES", 180e9, "B", "SPEC"), t["PEAK.HBM_COPY"],
                     not_measured("LAT.HBM", "cycle")),
            MemLevel("L2", rate("L2.BYTES", 126 * 2 ** 20, "B", "SPEC"),
                     not_measured("BW.L2", "GB/s"), not_measured("LAT.L2", "cycle")),
            MemLevel("SMEM", t["SMEM_PER_SM"], t["CAP.SMEM_RD"], not_measured("LAT.SMEM", "cycle")),
            MemLevel("TMEM", rate("TMEM.BYTES", 256 * 1024, "B", "SPEC"),
                     not_measured("BW.TMEM", "B/cycle"), not_measured("LAT.TMEM", "cycle")),
        )

    def wavefronts(self, lane_words, width_bytes: int) -> WavefrontCost:
        """Bank-conflict law: per access of ``width_bytes`` per lane, the degree is the largest
        number of distinct 4-byte words that map to one bank; the floor is the bytes moved
        divided by the 128-byte port (at least one)."""
        per_bank: dict = {}
        words_per_lane = max(1, width_bytes // self.BANK_BYTES)
        for w in lane_words:
            for i in range(words_per_lane):
                word = int(w) + i
                per_bank.setdefault(word % self.BANKS, set()).add(word)
        degree = max((len(s) for s in per_bank.values()), default=1)
        floor = max(1.0, len(lane_words) * width_bytes / (self.BANKS * self.BANK_BYTES))
        return WavefrontCost(degree=float(degree), floor=floor, wavefronts=max(float(degree), floor))

    def alignment_rule(self, width_bytes: int) -> int:
        """TMA and vector accesses need 16-byte alignment; narrower accesses their own width."""
        return 16 if width_bytes >= 16 else max(1, width_bytes)

    def pad_family(self, layout: Layout):
        return (0,)

    def swizzle_family(self, layout: Layout):
        row_bytes = layout.row_words * 4
        fam = ["none"]
        for name, span in (("32B", 32), ("64B", 64), ("128B", 128)):
            if row_bytes % span == 0:
                fam.append(name)
        return tuple(fam)

    def residency_policy(self) -> str:
        return "lru+evict_first_hint"
