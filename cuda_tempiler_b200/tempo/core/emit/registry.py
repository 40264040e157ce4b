"""Registry "shape -> variant -> fallback", serialisable, read by the ship dispatcher
(reference tempo/core/emit/registry.py:39-83).  A fallback is mandatory: predicate coverage is
never complete.  Predicate keys: ``x`` equality, ``x_max`` / ``x_min`` inclusive bounds,
``x_divides`` (x % v == 0)."""
from __future__ import annotations

import json
from dataclasses import dataclass, field


@dataclass
class Entry:
    predicate: dict
    kernel_id: str
    params: dict = field(default_factory=dict)
    note: str = ""


@dataclass
class Registry:
    op: str
    arch: str
    entries: list = field(default_factory=list)
    fallback: str = "the caller's own path"

    def select(self, **kw):
        for e in self.entries:
            if _match(e.predicate, kw):
                return e
        return None

    def to_json(self) -> str:
        return json.dumps({"schema": "tempo/registry/1", "op": self.op, "arch": self.arch,
                           "fallback": self.fallback,
                           "entries": [{"predicate": e.predicate, "kernel_id": e.kernel_id,
                                        "params": e.params, "note": e.note} for e in self.entries]},
                          ensure_ascii=False, indent=2, sort_keys=True)

    @classmethod
    def from_json(cls, text: str) -> "Registry":
        d = json.loads(text)
        if d.get("schema") != "tempo/registry/1":
            raise ValueError("not a tempo/registry/1 document")
        return cls(op=d["op"], arch=d["arch"], fallback=d["fallback"],
                   entries=[Entry(e["predicate"], e["kernel_id"], e.get("params", {}),
                                  e.get("note", "")) for e in d["entries"]])


def _match(pred, kw) -> bool:
    for k, v in pred.items():
        if k.endswith("_max"):
            x = kw.get(k[:-4])
            if x is None or x > v:
                return False
        elif k.endswith("_min"):
            x = kw.get(k[:-4])
            if x is None or x < v:
                return False
        elif k.endswith("_divides"):
            x = kw.get(k[:-8])
            if x is None or x % v:
                return False
        elif kw.get(k) != v:
            return False
    return True
