"""Section 4 -- resources and occupancy on sm_100a.

Walls: 227 KB dynamic shared memory per CTA (WALL_SMEM), 255 registers per thread and the
64 K register file (WALL_REG), 512 TMEM columns per SM shared by the resident CTAs (mapped to
NO_BUDGET: contract v1's verdict codes are closed).  The TMEM demand of a hyperform travels
with its shared-memory figure: ``resources_of`` returns an ``SmemBytes`` -- an int (so any
pipeline treats it as the byte count) that also carries ``tmem_cols``.
"""
from __future__ import annotations

from ..base import Occupancy, ResourceVerdict, not_measured


class SmemBytes(int):
    """Shared-memory bytes of a hyperform that also carries its TMEM column demand."""

    def __new__(cls, value, tmem_cols=0):
        obj = int.__new__(cls, value)
        obj.tmem_cols = int(tmem_cols)
        return obj


class Sm100Resources:
    MAX_REGS = 255
    MAX_THREADS_PER_SM = 2048
    MAX_CTAS_PER_SM = 32
    REG_GRANULE = 8

    def __init__(self, machine):
        self.m = machine

    def reg_budget(self, warps_per_sm: int) -> int:
        per = self.m.REGFILE_WORDS // max(1, warps_per_sm * 32)
        return max(0, min(self.MAX_REGS, per - per % self.REG_GRANULE))

    def spill_threshold(self, max_live: int) -> int:
        return self.MAX_REGS

    def free_spills(self) -> int:
        return 0

    def spill_cost(self, n: int):
        return not_measured("COST.SPILL", "cycle", "spills are rejected by the verify stage")

    def occupancy(self, regs: int, smem_bytes: int, threads: int) -> Occupancy:
        warps = -(-threads // 32)
        by_threads = self.MAX_THREADS_PER_SM // max(1, warps * 32)
        regs_r = -(-max(1, regs) // self.REG_GRANULE) * self.REG_GRANULE
        by_regs = self.m.REGFILE_WORDS // max(1, regs_r * warps * 32)
        by_smem = self.m.SMEM_PER_SM // max(1, int(smem_bytes) + 1024) if smem_bytes else self.MAX_CTAS_PER_SM
        tmem = getattr(smem_bytes, "tmem_cols", 0)
        by_tmem = self.m.TMEM_COLS // tmem if tmem else self.MAX_CTAS_PER_SM
        limits = {"threads": by_threads, "registers": by_regs, "smem": by_smem, "tmem": by_tmem,
                  "ctas": self.MAX_CTAS_PER_SM}
        limiter = min(limits, key=limits.get)
        ctas = max(0, limits[limiter])
        return Occupancy(warps_per_sm=ctas * warps, ctas_per_sm=ctas, regs_per_thread=regs,
                         limiter=limiter)

    def verdict(self, regs: int, max_live: int, smem_bytes: int, threads: int,
                min_ctas_per_sm: int = 1) -> ResourceVerdict:
        occ = self.occupancy(regs, smem_bytes, threads)
        if int(smem_bytes) > self.m.SMEM_PER_CTA:
            return ResourceVerdict(False, "WALL_SMEM", occ,
                                   f"{int(smem_bytes)} B dynamic shared memory > {self.m.SMEM_PER_CTA} B per CTA")
        tmem = getattr(smem_bytes, "tmem_cols", 0)
        if tmem > self.m.TMEM_COLS or tmem * max(1, min_ctas_per_sm) > self.m.TMEM_COLS:
            return ResourceVerdict(False, "NO_BUDGET", occ,
                                   f"TMEM: {tmem} columns x {max(1, min_ctas_per_sm)} CTA(s) > "
                                   f"{self.m.TMEM_COLS} columns per SM")
        if regs > self.MAX_REGS:
            return ResourceVerdict(False, "WALL_REG", occ, f"{regs} registers > {self.MAX_REGS}")
        if occ.ctas_per_sm < max(1, min_ctas_per_sm):
            return ResourceVerdict(False, "NO_BUDGET", occ,
                                   f"only {occ.ctas_per_sm} CTA(s)/SM fit (limit: {occ.limiter}); "
                                   f"{min_ctas_per_sm} declared")
        budget = self.reg_budget(max(1, min_ctas_per_sm) * (-(-threads // 32)))
        if max_live > budget:
            return ResourceVerdict(False, "SPILL", occ,
                                   f"estimated {max_live} live registers > budget {budget}")
        return ResourceVerdict(True, "FITS", occ,
                               f"{occ.ctas_per_sm} CTA/SM, limiter {occ.limiter}, TMEM {tmem} cols")

    def wave_quantum(self, occ: Occupancy) -> int:
        return self.m.SMS * max(1, occ.ctas_per_sm)

    def declared_bounds_required(self) -> bool:
        return True
