"""The calibration record schema ``tempo/calib/2``.

Restates the reference's schema (tempo/core/calib/schema.py:19-46): version 2 is version 1 plus
a mandatory ``plugin`` field, so a rate measured on one architecture can never stand in for
another's; the required fields, the record kinds and the observability classes are the same,
and a record taken while foreign processes ran on the card is invalid.
"""
from __future__ import annotations

SCHEMA = "tempo/calib/2"
REQUIRED = ("id", "kind", "quantity", "units", "taken_with", "shape", "card", "observability",
            "provenance", "plugin")
KINDS = ("padcurve", "phases", "law_points", "wf_per_inst", "conflict_share", "rate")
OBSERVABILITY = ("clean", "code_edit", "derived")


class CalibError(ValueError):
    """A calibration record that must not be used."""


def validate(rec: dict) -> None:
    """Raise CalibError unless ``rec`` is a usable tempo/calib/2 record."""
    if rec.get("schema") != SCHEMA:
        raise CalibError(f"schema {rec.get('schema')!r}: expected {SCHEMA}")
    for f in REQUIRED:
        if f not in rec:
            raise CalibError(f"record without field {f!r} (schema {SCHEMA})")
    if rec["kind"] not in KINDS:
        raise CalibError(f"kind {rec['kind']!r} not in {KINDS}")
    if rec["observability"] not in OBSERVABILITY:
        raise CalibError(f"observability {rec['observability']!r} not in {OBSERVABILITY}")
    card = rec.get("card") or {}
    if card.get("foreign_procs", 1) != 0:
        raise CalibError("taken while foreign processes ran on the card: invalid")
    for b in rec.get("binds") or []:
        if "symbol" not in b or "value" not in b:
            raise CalibError(f"bind without symbol/value: {b!r}")
        if not isinstance(b["value"], (int, float)) or b["value"] != b["value"]:
            raise CalibError(f"bind {b['symbol']}: value {b['value']!r} is not a number")
