"""Report: two bars always, the status of every rate, the card state, and the right to be
silent (reference tempo/core/report/__init__.py:1-114)."""
from __future__ import annotations

from dataclasses import dataclass, field

from ..measure.baseline import Comparison, two_bars_required, wall_share_required
from .provenance import require_provenance


@dataclass
class Section:
    title: str
    lines: list = field(default_factory=list)

    def add(self, s):
        self.lines.append(s)
        return self


@dataclass
class Report:
    title: str
    plugin_id: str
    card: object = None
    sections: list = field(default_factory=list)
    comparisons: list = field(default_factory=list)
    wall_share: float = None
    bound: object = None
    rates_used: list = field(default_factory=list)

    def section(self, title) -> Section:
        s = Section(title)
        self.sections.append(s)
        return s

    def compare(self, c: Comparison):
        self.comparisons.append(c)
        return self

    def render(self) -> str:
        require_provenance(self)
        two_bars_required(self.comparisons)
        rule = "=" * 100
        out = [rule, self.title, rule]
        if self.card is None:
            out.append("NO CARD GIVEN -- every number below is invalid as a measurement")
        else:
            out.append(f"card {self.card.index}, clock {self.card.clock_mhz} MHz, foreign "
                       f"processes {self.card.foreign_procs}, date {self.card.date}")
            if self.card.foreign_procs:
                out.append("A MEASUREMENT WITH A NEIGHBOUR ON THE CARD IS INVALID")
        out.append(f"plugin: {self.plugin_id}")
        nm = [r for r in self.rates_used if getattr(r, "status", "") == "NOT_MEASURED"]
        if nm:
            out.append("CONCLUSIONS REST ON UNMEASURED RATES: " + ", ".join(r.symbol for r in nm))
        if self.bound is not None:
            out += ["", self.bound.render()]
        out += ["", "BARS:"] + ["  " + c.render() for c in self.comparisons]
        out.append("  " + wall_share_required(self.wall_share))
        for s in self.sections:
            out += ["", s.title] + ["  " + str(x) for x in s.lines]
        return "\n".join(out)
