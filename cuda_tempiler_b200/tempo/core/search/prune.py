"""Build-free pruning: the resource verdict first, then the model bound (reference
tempo/core/search/prune.py:52-171).

Only the hard verdict codes cut (WALL_SMEM, NO_BUDGET): a register estimate without a build has
no precision, so a SPILL suspicion is kept and flagged.  The bound is a lower bound, not a
prediction, so only variants worse than the best bound by ``bound_slack`` are cut, and a
variant on which the model is silent is never cut.
"""
from __future__ import annotations

from dataclasses import dataclass

from ..model.bound import bound

HARD_CODES = frozenset({"WALL_SMEM", "NO_BUDGET"})


@dataclass
class Candidate:
    hyper: object
    verdict: object
    bound: object
    kept: bool
    reason: str

    def render(self) -> str:
        return f"{'KEPT  ' if self.kept else 'PRUNED'} {getattr(self.hyper, 'key', '?'):<42} {self.reason}"


def prune(plugin, op, hyperforms, keep_silent: bool = True, bound_slack: float = 4.0):
    channels = plugin.machine.channels()
    out, rows, best = [], [], None
    for h in hyperforms:
        try:
            regs, max_live, smem = plugin.skeletons.resources_of(op, h)
            lau = plugin.skeletons.launch_of(op, h)
            v = plugin.resources.verdict(regs, max_live, smem, lau.threads, lau.min_ctas_per_sm)
        except Exception as e:
            out.append(Candidate(h, None, None, False, f"resource verdict unavailable: {e}"))
            continue
        if not v.ok and v.code in HARD_CODES:
            out.append(Candidate(h, v, None, False, f"{v.code}: {v.explain}"))
            continue
        advice = "" if v.ok else ("SPILL SUSPECTED (estimate without a build) -- kept, the build "
                                  "must show it; ")
        try:
            atoms = plugin.skeletons.estimate_atoms(op, h)
            b = bound(atoms, channels, warps_per_sm=v.occ.warps_per_sm)
        except Exception as e:
            out.append(Candidate(h, v, None, keep_silent,
                                 advice + f"bound unavailable ({e}) -- kept: no cut on ignorance"))
            continue
        rows.append((h, v, b, advice))
        if not b.silent and (best is None or b.T < best):
            best = b.T
    for h, v, b, advice in rows:
        if b.silent:
            out.append(Candidate(h, v, b, keep_silent, advice + "MODEL SILENT: " + b.silent_reason))
        elif best is not None and b.T > best * bound_slack:
            out.append(Candidate(h, v, b, False, advice + f"bound {b.T:.2f} worse than the best "
                                 f"({best:.2f}) by more than {bound_slack:.1f}x"))
        else:
            out.append(Candidate(h, v, b, True, advice + f"{v.code}; T >= {b.T:.2f}, bound by "
                                 f"{b.binding}"))
    return out


def kept(cands):
    return [c for c in cands if c.kept]


def ranked(cands):
    """Kept candidates, best model bound first (silent ones last, in enumeration order)."""
    k = kept(cands)
    return sorted(k, key=lambda c: (c.bound is None or c.bound.silent,
                                    c.bound.T if c.bound is not None and not c.bound.silent else 0))


def summary(cands) -> str:
    k = sum(1 for c in cands if c.kept)
    silent = sum(1 for c in cands if c.bound is not None and c.bound.silent)
    risky = sum(1 for c in cands if c.kept and c.verdict is not None and not c.verdict.ok)
    return (f"hyperforms {len(cands)}, kept {k} (spill-suspected {risky}), pruned {len(cands) - k} "
            f"(silent model: {silent}, never pruned)")
