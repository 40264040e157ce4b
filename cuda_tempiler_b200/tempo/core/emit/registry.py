"""Shape registry: an ordered list of (predicate -> kernel) entries plus a mandatory fallback,
serialisable as a ``tempo/registry/1`` document (the reference's format,
tempo/core/emit/registry.py:39-83).  Predicate coverage is never complete, so a registry always
names what happens to a problem no entry matches: the caller's own path.

Predicate keys are the interface's: ``x`` equality, ``x_max`` / ``x_min`` inclusive bounds,
``x_divides`` (x % value == 0); a bound on a keyword the caller did not supply fails.  Each
predicate is compiled once into a list of checks (``compile_predicate``).
"""
from __future__ import annotations

import json
import operator
from dataclasses import asdict, dataclass, field
from typing import Callable

SCHEMA = "tempo/registry/1"

# suffix -> (how the keyword's value must relate to the predicate's value)
_RELATIONS = (
    ("_max", operator.le),
    ("_min", operator.ge),
    ("_divides", lambda x, v: x % v == 0),
)


def _check(key: str, want) -> Callable[[dict], bool]:
    for suffix, rel in _RELATIONS:
        if key.endswith(suffix):
            name = key[: -len(suffix)]
            return lambda kw: kw.get(name) is not None and bool(rel(kw[name], want))
    return lambda kw: kw.get(key) == want


def compile_predicate(pred: dict) -> Callable[[dict], bool]:
    checks = [_check(k, v) for k, v in pred.items()]
    return lambda kw: all(c(kw) for c in checks)


def _match(pred: dict, kw: dict) -> bool:
    return compile_predicate(pred)(kw)


@dataclass
class Entry:
    predicate: dict
    kernel_id: str
    params: dict = field(default_factory=dict)
    note: str = ""

    def __post_init__(self):
        self._test = compile_predicate(self.predicate)

    def covers(self, **kw) -> bool:
        return self._test(kw)


@dataclass
class Registry:
    op: str
    arch: str
    entries: list = field(default_factory=list)
    fallback: str = "the caller's own path"

    def select(self, **kw):
        """The first entry whose predicate holds, or None (= take ``fallback``)."""
        return next((e for e in self.entries if e.covers(**kw)), None)

    def to_json(self) -> str:
        doc = {"schema": SCHEMA, "op": self.op, "arch": self.arch, "fallback": self.fallback,
               "entries": [{k: v for k, v in asdict(e).items()} for e in self.entries]}
        return json.dumps(doc, ensure_ascii=False, indent=2, sort_keys=True)

    @classmethod
    def from_json(cls, text: str) -> "Registry":
        doc = json.loads(text)
        if doc.get("schema") != SCHEMA:
            raise ValueError(f"document schema {doc.get('schema')!r} is not {SCHEMA!r}")
        entries = [Entry(predicate=e["predicate"], kernel_id=e["kernel_id"],
                         params=e.get("params", {}), note=e.get("note", ""))
                   for e in doc["entries"]]
        return cls(op=doc["op"], arch=doc["arch"], entries=entries, fallback=doc["fallback"])
