"""Build-free pruning of a hyperform list.

Policy (the reference's, tempo/core/search/prune.py:52-171):
* only the hard resource codes cut (WALL_SMEM, NO_BUDGET); a SPILL verdict is an estimate
  without a build, so the hyperform is kept and flagged for the build to confirm;
* the model bound is a floor, not a prediction, so a hyperform is cut only when its floor is
  more than ``bound_slack`` times the best floor of the list;
* a hyperform on which the model is silent, or whose bound cannot be computed, is never cut
  for that (``keep_silent``).

Implementation: each hyperform is first *assessed* on its own (``assess``: resource verdict,
then bound), then every assessment is *decided* against the best floor of the list
(``decide``).  The two passes are needed because the best floor is known only at the end.
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
        mark = "KEPT  " if self.kept else "PRUNED"
        return f"{mark} {getattr(self.hyper, 'key', '?'):<42} {self.reason}"


@dataclass
class Assessment:
    hyper: object
    verdict: object = None
    bound: object = None
    failure: str = ""  # why the verdict or the bound could not be had
    stage: str = ""    # "verdict" | "bound" when failure is set

    @property
    def spill_note(self) -> str:
        if self.verdict is not None and not self.verdict.ok:
            return "spill suspected by the estimate (kept: only a build can confirm it); "
        return ""

    @property
    def floor(self):
        """The bound's T when it is usable for ranking, else None."""
        b = self.bound
        return None if b is None or b.silent else b.T


def assess(plugin, op, h, channels) -> Assessment:
    a = Assessment(h)
    try:
        regs, max_live, smem = plugin.skeletons.resources_of(op, h)
        launch = plugin.skeletons.launch_of(op, h)
        a.verdict = plugin.resources.verdict(regs, max_live, smem, launch.threads,
                                             launch.min_ctas_per_sm)
    except Exception as e:  # a plugin may refuse or fail on any hyperform
        a.failure, a.stage = str(e), "verdict"
        return a
    if not a.verdict.ok and a.verdict.code in HARD_CODES:
        return a
    try:
        atoms = plugin.skeletons.estimate_atoms(op, h)
        a.bound = bound(atoms, channels, warps_per_sm=a.verdict.occ.warps_per_sm)
    except Exception as e:
        a.failure, a.stage = str(e), "bound"
    return a


def decide(a: Assessment, best_floor, keep_silent: bool, bound_slack: float) -> Candidate:
    v, b = a.verdict, a.bound
    if a.stage == "verdict":
        return Candidate(a.hyper, None, None, False, f"no resource verdict: {a.failure}")
    if not v.ok and v.code in HARD_CODES:
        return Candidate(a.hyper, v, None, False, f"{v.code}: {v.explain}")
    note = a.spill_note
    if a.stage == "bound":
        return Candidate(a.hyper, v, None, keep_silent,
                         note + f"no bound ({a.failure}); kept, ignorance cuts nothing")
    if b.silent:
        return Candidate(a.hyper, v, b, keep_silent, note + "MODEL SILENT: " + b.silent_reason)
    if best_floor is not None and b.T > bound_slack * best_floor:
        return Candidate(a.hyper, v, b, False,
                         note + f"floor {b.T:.2f} is over {bound_slack:.1f}x the best floor "
                                f"{best_floor:.2f}")
    return Candidate(a.hyper, v, b, True,
                     note + f"{v.code}; T >= {b.T:.2f}, bound by {b.binding}")


def prune(plugin, op, hyperforms, keep_silent: bool = True, bound_slack: float = 4.0):
    channels = plugin.machine.channels()
    assessed = [assess(plugin, op, h, channels) for h in hyperforms]
    floors = [a.floor for a in assessed if a.floor is not None]
    best_floor = min(floors) if floors else None
    return [decide(a, best_floor, keep_silent, bound_slack) for a in assessed]


def kept(cands):
    return [c for c in cands if c.kept]


def ranked(cands):
    """Kept candidates with a usable floor first, lowest floor first; then the rest in
    enumeration order."""
    def key(c):
        usable = c.bound is not None and not c.bound.silent
        return (0, c.bound.T) if usable else (1, 0.0)
    return sorted(kept(cands), key=key)


def summary(cands) -> str:
    n_kept = len(kept(cands))
    n_silent = sum(1 for c in cands if c.bound is not None and c.bound.silent)
    n_spill = sum(1 for c in kept(cands) if c.verdict is not None and not c.verdict.ok)
    return (f"{len(cands)} hyperforms: {n_kept} kept ({n_spill} with a suspected spill), "
            f"{len(cands) - n_kept} pruned; the model was silent on {n_silent} (never a cut)")
