"""Recognition: a naive source carrying an in-source ``TEMPO-OP`` block -> OpSpec.

The block grammar is the reference's interface (kernels/naive/gemm_fp16.cu:30-38; its parser
is tempo/core/op/recognize.py:41-141): comment lines of ``key: value`` after a
``TEMPO-OP: <kind>`` marker, in any order, ending at ``TEMPO-OP-END`` or after 40 lines:

    TEMPO-OP: gemm
    dtype: a=fp16 b=fp16 c=fp16 acc=fp32
    layout: a=k b=k c=n
    shape: M=* N=* K=*
    tol_rel_l2: 1e-3
    entry: naive_gemm_fp16
    signature: (const __half* A, const __half* B, __half* C, int M, int N, int K)
    scale: per_channel | group:128        (W8A16 only)

``*`` shapes are supplied at run time.  Text without a block is refused: only declared
operations are recognised, there is no C++ parser.  The entry the block names must have a
declaration in the source with as many parameters as the block's signature.

Implementation: every field has a value parser (``_FIELD_PARSERS``); the block is read as a
stream of (key, raw value) pairs, and unknown keys are ignored.
"""
from __future__ import annotations

import re

from ...plugins.base import OpSpec
from .spec import validate

_MARKER = re.compile(r"TEMPO-OP\s*:\s*(?P<kind>\w+)")
_FIELD = re.compile(r"^[\s/*#]*(?P<key>[A-Za-z_]\w*)\s*:\s*(?P<val>.*?\S)\s*$")
_END = "TEMPO-OP-END"
_SCAN_LINES = 40


class NotRecognised(Exception):
    """An unknown kernel gets a refusal, not bad code."""


def _assignments(raw: str) -> dict:
    """``a=fp16, b=fp16 c=n`` -> {'a': 'fp16', 'b': 'fp16', 'c': 'n'} (keys lower-cased)."""
    pairs = (tok.partition("=") for tok in re.split(r"[\s,]+", raw) if "=" in tok)
    return {k.strip().lower(): v.strip() for k, _, v in pairs}


def _as_is(raw: str) -> str:
    return raw


_FIELD_PARSERS = {
    "dtype": _assignments, "layout": _assignments, "shape": _assignments,
    "tol_rel_l2": _as_is, "entry": _as_is, "signature": _as_is, "coverage": _as_is,
    "scale": _as_is,
}


def _fields(text: str, start: int):
    """(key, raw value) pairs of the block that begins at ``start``."""
    for n, line in enumerate(text[start:].split("\n")):
        if n >= _SCAN_LINES or _END in line:
            return
        m = _FIELD.match(line)
        if m is not None:
            yield m.group("key").lower(), m.group("val")


def parse_block(text: str) -> dict:
    marker = _MARKER.search(text)
    if marker is None:
        raise NotRecognised("no TEMPO-OP block in the source: only operations declared by such "
                            "a block are recognised (there is no C++ parser)")
    block = {"kind": marker.group("kind")}
    block.update((key, _FIELD_PARSERS[key](raw)) for key, raw in _fields(text, marker.end())
                 if key in _FIELD_PARSERS)
    return block


def _shape(sym: str, given: dict, declared: dict) -> int:
    value = given.get(sym)
    if value is None:
        value = declared.get(sym, declared.get(sym.lower()))
    if value is None or str(value).strip() == "*":
        raise NotRecognised(f"shape {sym} is a run-time shape ('*') and no value was supplied")
    return int(value)


def to_spec(block: dict, shapes: dict | None = None) -> OpSpec:
    types = {"a": "fp16", "b": "fp16", "c": "fp16", "acc": "fp32", **block.get("dtype", {})}
    lays = {"a": "k", "b": "k", "c": "n", **block.get("layout", {})}
    given, declared = shapes or {}, block.get("shape", {})
    op = OpSpec(
        kind=block["kind"],
        dtype_a=types["a"], dtype_b=types["b"], dtype_c=types["c"], dtype_acc=types["acc"],
        layout_a=lays["a"], layout_b=lays["b"], layout_c=lays["c"],
        shapes={sym: _shape(sym, given, declared) for sym in ("M", "N", "K")},
        scale=block.get("scale"),
        tol_rel_l2=float(block.get("tol_rel_l2", 0.0)),
        coverage=block.get("coverage", "atomic_stamp"))
    validate(op)
    return op


def _arity(params: str) -> int:
    return sum(1 for p in params.split(",") if p.strip())


def check_signature(block: dict, text: str) -> None:
    """The named entry must be declared in the source -- a name followed by a parameter list;
    the block's own mention of the name does not count -- with the block's parameter count."""
    entry = block.get("entry")
    if not entry:
        raise NotRecognised("the TEMPO-OP block names no entry")
    decl = re.search(rf"{re.escape(entry)}\s*\(([^)]*)\)", text)
    if decl is None:
        raise NotRecognised(f"the block names entry {entry!r} but no function of that name is "
                            "declared in the source (a stale block)")
    declared_sig = block.get("signature")
    if declared_sig:
        want, have = _arity(declared_sig.strip().strip("()")), _arity(decl.group(1))
        if want != have:
            raise NotRecognised(f"entry {entry!r}: the block's signature has {want} parameters, "
                                f"the source's declaration {have}")


def from_text(text: str, shapes: dict | None = None) -> OpSpec:
    block = parse_block(text)
    check_signature(block, text)
    return to_spec(block, shapes)


def from_file(path: str, shapes: dict | None = None) -> OpSpec:
    with open(path, encoding="utf-8") as f:
        return from_text(f.read(), shapes)
