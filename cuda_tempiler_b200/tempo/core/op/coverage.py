"""Coverage by atomic stamp: every output cell written exactly once (reference
tempo/core/op/coverage.py:6-62).  A value check compares only what was computed; coverage
catches the quarter-tile that was never computed and the overlap that was computed twice.
On the GPU the same property is checked with a poison fill (0x7f7f) that must be gone."""
from __future__ import annotations

from dataclasses import dataclass

STAMP_MACRO = "TEMPO_COVERAGE_STAMP"


@dataclass
class Coverage:
    total: int
    zero: int
    over: int
    max_hits: int

    @property
    def ok(self) -> bool:
        return self.zero == 0 and self.over == 0

    def render(self) -> str:
        if self.ok:
            return f"coverage complete: {self.total} cells, each exactly once"
        return (f"coverage broken: {self.zero} uncovered, {self.over} written more than once "
                f"(max {self.max_hits}) of {self.total}")


def check(stamps) -> Coverage:
    total = zero = over = mx = 0
    for v in stamps:
        v = int(v)
        total += 1
        zero += v == 0
        over += v > 1
        mx = max(mx, v)
    return Coverage(total=total, zero=zero, over=over, max_hits=mx)


def from_poison(cells_u16, poison: int = 0x7F7F) -> Coverage:
    """Coverage from a poison-filled fp16 output viewed as uint16: a cell still equal to the
    poison was not written (a write of exactly 0x7f7f is astronomically unlikely)."""
    total = zero = 0
    for v in cells_u16:
        total += 1
        zero += int(v) == poison
    return Coverage(total=total, zero=zero, over=0, max_hits=1)
