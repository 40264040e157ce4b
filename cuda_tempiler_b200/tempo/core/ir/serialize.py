"""``tempo/atoms/1`` JSON and a stable hash (insensitive to dict order) used to name ship
directories.  The document's keys, the 6-digit rounding and the 16-hex sha256 prefix are the
reference's format (tempo/core/ir/serialize.py), kept so that hashes name the same atoms; the
pipeline only writes these documents, it never reads them back."""
from __future__ import annotations

import hashlib
import json

from ...plugins.base import AtomKind

SCHEMA = "tempo/atoms/1"


def to_json(atoms, meta=None) -> str:
    doc = {"schema": SCHEMA, "meta": meta or {}, "atoms": [{
        "uid": a.uid, "kind": a.kind.value if isinstance(a.kind, AtomKind) else str(a.kind),
        "op_id": a.op_id, "footprint": {k: round(float(v), 6) for k, v in sorted(a.footprint.items())},
        "latency": round(float(a.latency), 6), "token": a.token, "region": a.region,
        "deps": [{"src": d.src_uid, "type": d.type, "distance": d.distance,
                  "min_gap": round(float(d.min_gap), 6)} for d in a.deps]} for a in atoms]}
    return json.dumps(doc, ensure_ascii=False, sort_keys=True, indent=2)


def stable_hash(atoms, meta=None) -> str:
    return hashlib.sha256(to_json(atoms, meta).encode("utf-8")).hexdigest()[:16]
