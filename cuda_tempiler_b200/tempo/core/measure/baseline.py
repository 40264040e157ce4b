"""A comparison arm as an object: a number without a named base is not a number (reference
tempo/core/measure/baseline.py:1-81).  Kinds: INPUT (the naive input kernel), LIBRARY (a tuned
library on the same machine), SHIPPED (our own shipped kernel), FORMAT (our path in another
data format).  Two bars are mandatory: INPUT plus a strong one."""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

KINDS = ("INPUT", "LIBRARY", "SHIPPED", "FORMAT")


@dataclass(frozen=True)
class Baseline:
    kind: str
    name: str
    what: str
    entry_proof: Optional[str] = None

    def __post_init__(self):
        if self.kind not in KINDS:
            raise ValueError(f"baseline kind {self.kind!r} not in {KINDS}")

    def label(self) -> str:
        return f"{self.name} ({self.kind})"


@dataclass(frozen=True)
class Comparison:
    baseline: Baseline
    ratio: float  # > 1: we are faster
    ci: tuple = ()
    rounds: int = 0
    note: str = ""

    def render(self) -> str:
        ci = f" [{self.ci[0]:.3f}..{self.ci[1]:.3f}]" if self.ci and len(self.ci) == 2 else ""
        return (f"vs {self.baseline.label():<30} x{self.ratio:.3f}{ci}  rounds {self.rounds}"
                + (f"  -- {self.note}" if self.note else ""))


def two_bars_required(comps) -> None:
    kinds = {c.baseline.kind for c in comps}
    if "INPUT" not in kinds:
        raise ValueError("no INPUT bar: unknown whether the compiler produced the result")
    if not kinds & {"LIBRARY", "SHIPPED", "FORMAT"}:
        raise ValueError("no second bar: 'x faster than the naive input' alone is trivially large")


def wall_share_required(share: Optional[float]) -> str:
    if share is None:
        return "share of the wall NOT MEASURED -- a kernel speed-up cannot be read as a task speed-up"
    return f"share of this kernel's work in the wall: {100.0 * share:.1f} % (ceiling of the end-to-end effect)"
