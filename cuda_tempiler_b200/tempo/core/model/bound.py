"""Lower bound of the period of a schedule, T >= max(ResMII, RecMII) -- the reference's
model (tempo/core/model/bound.py:61-162), computed here as follows:

* ResMII: each channel that carries load and has a usable capacity contributes a time; the
  largest is ResMII and names the binding channel.  A channel of scope "sm" has a capacity in
  units per cycle for the whole SM, and the per-warp load is multiplied by the resident warps;
  a channel of scope "sched" has a capacity in cycles per unit of load.
* RecMII: the maximum mean cycle of the loop-carried dependence graph (Karp, below).

The bound is a floor, not a prediction, and it may stay silent: when no loaded channel has a
usable (measured or upper-bound) rate it says so instead of inventing a number.  Datasheet
(SPEC) rates are refused outright.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

from ...plugins.base import spec_forbidden_in_time_bound
from ..ir.atom import channel_load


@dataclass
class Bound:
    T: float
    res_mii: float
    rec_mii: float
    binding: str
    per_channel: dict = field(default_factory=dict)
    silent: bool = False
    silent_reason: str = ""
    uses_not_measured: tuple = ()

    @classmethod
    def without_model(cls, unmeasured: tuple) -> "Bound":
        why = "none of the loaded channels has a usable rate"
        if unmeasured:
            why += " (unmeasured: " + ", ".join(unmeasured) + ")"
        nan = math.nan
        return cls(T=nan, res_mii=nan, rec_mii=nan, binding="", silent=True,
                   silent_reason=why, uses_not_measured=unmeasured)

    def render(self) -> str:
        if self.silent:
            return "MODEL SILENT: " + self.silent_reason
        text = (f"T >= {self.T:.2f} cycles, bound by {self.binding} "
                f"[ResMII {self.res_mii:.2f}, RecMII {self.rec_mii:.2f}]")
        if self.uses_not_measured:
            text += "\n  caution, unmeasured rates were skipped: " + ", ".join(self.uses_not_measured)
        return text


_TINY = 1e-12
# scope -> time of `load` on a channel of capacity `cap` with `warps` resident warps
_CHANNEL_TIME = {
    "sm": lambda load, cap, warps: load * max(1, warps) / max(cap, _TINY),
    "sched": lambda load, cap, warps: load * cap,
}


def res_mii(atoms, channels, warps_per_sm: int = 1, schedulers: int = 1):
    """(per-channel times, unmeasured rate symbols) for the channels the atoms load."""
    times, unmeasured = {}, []
    for name, load in channel_load(atoms).items():
        if name not in channels:
            continue
        ch = channels[name]
        spec_forbidden_in_time_bound(ch.capacity)
        if ch.capacity.status == "NOT_MEASURED":
            unmeasured.append(ch.capacity.symbol)
        else:
            times[name] = _CHANNEL_TIME[ch.scope](load, ch.capacity.value, warps_per_sm)
    return times, tuple(unmeasured)


def _max_mean_cycle(n, edges):
    """Karp's maximum mean cycle over edges (u, v, weight, distance>0), as weight/distance
    per cycle; distances are unrolled by adding chain nodes (small graphs only)."""
    nodes = n
    unit = []
    for u, v, w, d in edges:
        prev = u
        for i in range(d - 1):
            unit.append((prev, nodes, w if i == 0 else 0.0))
            prev = nodes
            nodes += 1
        unit.append((prev, v, w if d == 1 else 0.0))
    if not unit:
        return 0.0
    N = nodes
    NEG = float("-inf")
    D = [[NEG] * N for _ in range(N + 1)]
    for s in range(N):
        D[0][s] = 0.0
    for k in range(1, N + 1):
        for u, v, w in unit:
            if D[k - 1][u] != NEG and D[k - 1][u] + w > D[k][v]:
                D[k][v] = D[k - 1][u] + w
    best = NEG
    for v in range(N):
        if D[N][v] == NEG:
            continue
        worst = float("inf")
        for k in range(N):
            if D[k][v] != NEG:
                worst = min(worst, (D[N][v] - D[k][v]) / (N - k))
        best = max(best, worst)
    return 0.0 if best == NEG else best


def rec_mii(atoms) -> float:
    idx = {a.uid: i for i, a in enumerate(atoms)}
    edges = []
    for a in atoms:
        for d in a.deps:
            if d.src_uid in idx and d.distance > 0:
                src = atoms[idx[d.src_uid]]
                edges.append((idx[d.src_uid], idx[a.uid], float(src.latency) + float(d.min_gap),
                              int(d.distance)))
    if not edges or len(atoms) > 64:
        return 0.0
    return _max_mean_cycle(len(atoms), edges)


def bound(atoms, channels, warps_per_sm: int = 1, schedulers: int = 1) -> Bound:
    times, unmeasured = res_mii(atoms, channels, warps_per_sm, schedulers)
    if not times:
        return Bound.without_model(unmeasured)
    res_name, res = max(times.items(), key=lambda kv: kv[1])
    rec = rec_mii(atoms)
    return Bound(T=max(res, rec), res_mii=res, rec_mii=rec,
                 binding="RECURRENCE" if rec > res else res_name, per_channel=times,
                 uses_not_measured=unmeasured)


def headroom(measured_cycles: float, b: Bound) -> float:
    """measured / bound: how far a measurement sits above the floor (NaN without a model; a
    value below 1 means the model or the measurement has a unit error)."""
    if b.silent or not b.T > 0:
        return math.nan
    return measured_cycles / b.T
