"""Lower bound of the period (reference tempo/core/model/bound.py:61-162):

    ResMII = max over channels (load / capacity),  RecMII = max mean cycle of the dependence
    graph,  T >= max(ResMII, RecMII).

The bound is not a prediction.  It must be able to stay silent: when no channel with a usable
(non-NOT_MEASURED) rate carries load, it returns ``silent=True`` instead of a wrong number.
SPEC (datasheet) rates are refused in a time bound.
"""
from __future__ import annotations

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

    def render(self) -> str:
        if self.silent:
            return "MODEL SILENT: " + self.silent_reason
        s = (f"T >= {self.T:.2f} cycles (ResMII {self.res_mii:.2f}, RecMII {self.rec_mii:.2f}), "
             f"bound by {self.binding}")
        if self.uses_not_measured:
            s += "\n  WARNING: rests on unmeasured rates: " + ", ".join(self.uses_not_measured)
        return s


def res_mii(atoms, channels, warps_per_sm: int = 1, schedulers: int = 1):
    """scope "sm": capacity is units per cycle for the whole SM and the per-warp load scales
    with the resident warps; scope "sched": capacity is cycles per unit of load."""
    per, nm = {}, []
    for name, load in channel_load(atoms).items():
        ch = channels.get(name)
        if ch is None:
            continue
        cap = ch.capacity
        spec_forbidden_in_time_bound(cap)
        if cap.status == "NOT_MEASURED":
            nm.append(cap.symbol)
            continue
        if ch.scope == "sm":
            per[name] = load * max(1, warps_per_sm) / max(1e-12, cap.value)
        else:
            per[name] = load * cap.value
    return per, tuple(nm)


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
    per, nm = res_mii(atoms, channels, warps_per_sm, schedulers)
    if not per:
        return Bound(T=float("nan"), res_mii=float("nan"), rec_mii=float("nan"), binding="",
                     silent=True, uses_not_measured=nm,
                     silent_reason="no channel with a usable rate carries the binding load"
                     + (f" (not measured: {', '.join(nm)})" if nm else ""))
    binding = max(per, key=per.get)
    r = per[binding]
    rec = rec_mii(atoms)
    return Bound(T=max(r, rec), res_mii=r, rec_mii=rec,
                 binding=binding if r >= rec else "RECURRENCE", per_channel=per,
                 uses_not_measured=nm)


def headroom(measured_cycles: float, b: Bound) -> float:
    """How far above the bound a measurement sits; below 1 means a unit error."""
    if b.silent or not b.T or b.T != b.T:
        return float("nan")
    return measured_cycles / b.T
