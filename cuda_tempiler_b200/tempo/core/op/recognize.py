"""Recognition: a naive source with an in-source ``TEMPO-OP`` block -> OpSpec.

The block (comment lines, any order; reference kernels/naive/gemm_fp16.cu:30-38 and
tempo/core/op/recognize.py:41-141):

    TEMPO-OP: gemm
    dtype: a=fp16 b=fp16 c=fp16 acc=fp32
    layout: a=k b=k c=n
    shape: M=* N=* K=*
    tol_rel_l2: 1e-3
    entry: naive_gemm_fp16
    signature: (const __half* A, const __half* B, __half* C, int M, int N, int K)
    scale: per_channel | group:128        (W8A16 only)

``*`` shapes are given at run time.  No block -> refusal (the product does not parse
arbitrary C++).  The declared entry must be *declared* in the text (name followed by an
argument list) and its argument count must match the signature.
"""
from __future__ import annotations

import re

from ...plugins.base import OpSpec
from .spec import validate

BLOCK_START = re.compile(r"TEMPO-OP\s*:\s*(\w+)")
KEY_VALUE = re.compile(r"^\s*(?://|#|\*)?\s*([A-Za-z_]\w*)\s*:\s*(.+?)\s*$")
_PAIRS = ("dtype", "layout", "shape")
_SCALARS = ("tol_rel_l2", "entry", "signature", "coverage", "scale")


class NotRecognised(Exception):
    """An unknown kernel gets a refusal, not bad code."""


def parse_block(text: str) -> dict:
    m = BLOCK_START.search(text)
    if not m:
        raise NotRecognised("the source has no TEMPO-OP block; only declared operations are "
                            "recognised (there is no C++ parser)")
    block = {"kind": m.group(1)}
    for line in text[m.end():].split("\n")[:40]:
        if "TEMPO-OP-END" in line:
            break
        kv = KEY_VALUE.match(line)
        if not kv:
            continue
        key, val = kv.group(1).lower(), kv.group(2)
        if key in _PAIRS:
            sub = {}
            for tok in val.replace(",", " ").split():
                if "=" in tok:
                    a, b = tok.split("=", 1)
                    sub[a.strip().lower()] = b.strip()
            block[key] = sub
        elif key in _SCALARS:
            block[key] = val
    return block


def to_spec(block: dict, shapes: dict | None = None) -> OpSpec:
    dt, lay = block.get("dtype", {}), block.get("layout", {})
    declared = dict(block.get("shape", {}))
    shapes = shapes or {}
    resolved = {}
    for k in ("M", "N", "K"):
        v = shapes.get(k, declared.get(k, declared.get(k.lower())))
        if v is None or str(v) == "*":
            raise NotRecognised(f"shape {k} is declared '*' (run-time) but was not given")
        resolved[k] = int(v)
    op = OpSpec(kind=block["kind"], dtype_a=dt.get("a", "fp16"), dtype_b=dt.get("b", "fp16"),
                dtype_c=dt.get("c", "fp16"), dtype_acc=dt.get("acc", "fp32"),
                layout_a=lay.get("a", "k"), layout_b=lay.get("b", "k"), layout_c=lay.get("c", "n"),
                shapes=resolved, scale=block.get("scale"),
                tol_rel_l2=float(block.get("tol_rel_l2", 0.0)),
                coverage=block.get("coverage", "atomic_stamp"))
    validate(op)
    return op


def check_signature(block: dict, text: str) -> None:
    """The declared entry must be declared in the source (not merely mentioned: the name
    also occurs inside the block itself), with the declared number of arguments."""
    entry = block.get("entry")
    if not entry:
        raise NotRecognised("the TEMPO-OP block declares no entry:")
    decl = re.search(re.escape(entry) + r"\s*\(([^)]*)\)", text)
    if not decl:
        raise NotRecognised(f"entry {entry!r} is declared in the TEMPO-OP block but the source "
                            "has no declaration with that name: the block is stale")
    sig = block.get("signature")
    if sig:
        want = [a for a in sig.strip().strip("()").split(",") if a.strip()]
        real = [a for a in decl.group(1).split(",") if a.strip()]
        if len(want) != len(real):
            raise NotRecognised(f"TEMPO-OP signature declares {len(want)} arguments, the "
                                f"source declares {len(real)}")


def from_text(text: str, shapes: dict | None = None) -> OpSpec:
    block = parse_block(text)
    check_signature(block, text)
    return to_spec(block, shapes)


def from_file(path: str, shapes: dict | None = None) -> OpSpec:
    with open(path, encoding="utf-8") as f:
        return from_text(f.read(), shapes)
