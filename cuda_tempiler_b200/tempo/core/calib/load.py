"""Loading calibration records into a plugin's rate table.

The substitution rule of the reference (tempo/core/calib/load.py:29-52): a MEASURED record
replaces MODEL / NOT_MEASURED / UPPER_BOUND rates, only in that direction (a model never
overwrites a measurement), only for the record's own plugin, and only for symbols the closed
table already declares -- a bind to an unknown symbol is a refusal, not an extension.
"""
from __future__ import annotations

import glob
import json
import os

from ...plugins.base import CardState, Provenance, Rate
from .schema import CalibError, validate


def load_dir(path: str, plugin: str) -> list:
    """Every valid tempo/calib/2 record of ``plugin`` under ``path`` (sorted by file name).
    Invalid records raise CalibError: a bad calibration file is an error, not a silence."""
    out = []
    for f in sorted(glob.glob(os.path.join(path, "*.json"))):
        with open(f, encoding="utf-8") as fh:
            rec = json.load(fh)
        try:
            validate(rec)
        except CalibError as e:
            raise CalibError(f"{os.path.basename(f)}: {e}") from None
        if rec["plugin"] == plugin:
            out.append(rec)
    return out


def apply(symbols: dict, records: list, plugin: str) -> dict:
    """A new rate table in which the records' binds replace non-measured rates."""
    out = dict(symbols)
    for rec in records:
        if rec.get("plugin") != plugin:
            raise CalibError(f"record {rec.get('id')!r} belongs to plugin {rec.get('plugin')!r}, "
                             f"not {plugin!r}")
        c = rec["card"]
        card = CardState(index=int(c.get("index", -1)), clock_mhz=int(c.get("clock_mhz", 0)),
                         foreign_procs=int(c["foreign_procs"]),
                         date=rec["provenance"].get("date", ""))
        tw = rec["taken_with"]
        prov = Provenance(tool=tw.get("tool", ""), counter=tw.get("counter"),
                          version=str(tw.get("version", "")),
                          date=rec["provenance"].get("date", ""),
                          who=rec["provenance"].get("who", ""),
                          observability=rec["observability"], card=card)
        for b in rec.get("binds") or []:
            sym = b["symbol"]
            if sym not in out:
                raise KeyError(f"calibration binds symbol {sym!r}, which the closed table does "
                               f"not declare: a refusal, not an extension")
            old = out[sym]
            if old.status in ("MEASURED", "SPEC") and rec.get("kind") != "rate":
                continue
            if old.status == "SPEC":
                continue  # architectural constants are not re-measured
            out[sym] = Rate(symbol=sym, value=float(b["value"]), units=old.units,
                            status="MEASURED", prov=prov, note=b.get("note", old.note))
    return out
