"""Atoms: the pipeline's only IR in v1.  An atom carries a footprint per channel; its op id is
opaque (reference tempo/core/ir/atom.py)."""
from __future__ import annotations

from ...plugins.base import Atom, AtomKind, Dep  # noqa: F401


def channel_load(atoms) -> dict:
    out: dict = {}
    for a in atoms:
        for ch, cyc in a.footprint.items():
            out[ch] = out.get(ch, 0.0) + float(cyc)
    return out


def region_of(atoms, region: str):
    return [a for a in atoms if a.region == region]


def summary(atoms) -> str:
    load = sorted(channel_load(atoms).items(), key=lambda kv: -kv[1])
    return f"{len(atoms)} atoms; channels: " + ", ".join(f"{k}={v:.1f}" for k, v in load)
