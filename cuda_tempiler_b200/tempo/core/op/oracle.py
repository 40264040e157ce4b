"""Correctness arithmetic: relative L2 and the gate (reference tempo/core/op/oracle.py:28-151).

A small relL2 is necessary, not sufficient: the reference is computed on the same inputs and
catches arithmetic only.  The gate passes only when an *independent*, *named* path (e.g. an
fp64 spot check on sampled cells) agrees as well, and coverage (every output cell written
exactly once) holds when it was measured.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field


@dataclass
class OracleResult:
    rel_l2: float
    tol: float
    coverage: object = None
    independent_rel_l2: float = float("nan")
    independent_path: str = ""
    notes: list = field(default_factory=list)

    @property
    def necessary_ok(self) -> bool:
        if self.rel_l2 != self.rel_l2 or self.rel_l2 > self.tol:
            return False
        return self.coverage is None or self.coverage.ok

    @property
    def sufficient_ok(self) -> bool:
        if not self.independent_path.strip():
            return False
        if self.independent_rel_l2 != self.independent_rel_l2:
            return False
        return self.independent_rel_l2 <= self.tol

    @property
    def ok(self) -> bool:
        return self.necessary_ok and self.sufficient_ok

    def render(self) -> str:
        out = [f"CORRECTNESS GATE: relL2 = {self.rel_l2:.3e} at tolerance {self.tol:.3e} -- "
               + ("PASSED" if self.ok else "NOT PASSED")]
        if self.coverage is not None:
            out.append("  " + self.coverage.render())
        if self.independent_rel_l2 == self.independent_rel_l2:
            out.append(f"  independent path: {self.independent_rel_l2:.3e}"
                       + (f" -- differs in: {self.independent_path}"
                          if self.independent_path.strip()
                          else " -- the independent path is not named: not counted"))
        if not self.sufficient_ok:
            out.append("  small relL2 is necessary, not sufficient: an independent named path "
                       "must agree too")
        out.extend("  " + n for n in self.notes)
        return "\n".join(out)


def rel_l2(got, ref) -> float:
    """sqrt(sum (got - ref)^2 / sum ref^2); NaN when the reference is all zero."""
    num = den = 0.0
    for a, b in zip(got, ref):
        d = float(a) - float(b)
        num += d * d
        den += float(b) * float(b)
    if den <= 0.0:
        return float("nan")
    return math.sqrt(num / den)


def gate(got, ref, tol: float, stamps=None, independent=None,
         independent_path: str = "") -> OracleResult:
    from .coverage import check
    cov = check(stamps) if stamps is not None else None
    res = OracleResult(rel_l2=rel_l2(got, ref), tol=tol, coverage=cov,
                       independent_rel_l2=(rel_l2(got, independent) if independent is not None
                                           else float("nan")),
                       independent_path=independent_path)
    if cov is not None and cov.zero:
        res.notes.append("uncovered cells with a passing value check: trust coverage")
    return res


def speedup_vs_input(t_input_s: float, t_output_s: float) -> float:
    """The compiler's own metric; only printable next to a second (library) bar."""
    return float("nan") if t_output_s <= 0 else t_input_s / t_output_s
