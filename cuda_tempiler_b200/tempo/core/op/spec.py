"""Declared operations: what a recognised OpSpec may contain and how much work it is.

The OpSpec type belongs to the contract (``tempo.plugins.base``).  The pipeline only accepts
operations it has a declaration for (the reference's rule, tempo/core/op/spec.py:19-46); each
declaration names the shape symbols the op needs and how its useful FLOPs are counted.  The
element-type vocabulary (``KNOWN_DTYPES``) is part of the interface and is kept as the
reference spells it.

``validate`` reports every problem of a spec at once (one ValueError listing them all), so a
TEMPO-OP block with several mistakes is fixed in one edit.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Mapping

from ...plugins.base import OpSpec  # noqa: F401

KNOWN_DTYPES = ("fp16", "fp32", "int8", "uint8", "q7", "bf16")
_TYPE_FIELDS = ("dtype_a", "dtype_b", "dtype_c", "dtype_acc")


@dataclass(frozen=True)
class Declaration:
    shape_symbols: tuple
    work: Callable[[Mapping], float]  # useful FLOPs from the resolved shapes


DECLARED = {
    # C[M,N] = A[M,K] * B[K,N]: one multiply and one add per (m, n, k)
    "gemm": Declaration(("M", "N", "K"), lambda s: 2.0 * s["M"] * s["N"] * s["K"]),
}
KNOWN_KINDS = tuple(DECLARED)


def _positive_int(v) -> bool:
    try:
        return int(v) > 0 and float(v) == int(v)
    except (TypeError, ValueError):
        return False


def problems(op: OpSpec) -> list:
    """Everything wrong with ``op``, as readable strings (empty when it is valid)."""
    found = []
    decl = DECLARED.get(op.kind)
    if decl is None:
        found.append(f"operation {op.kind!r} has no declaration (declared: "
                     f"{', '.join(KNOWN_KINDS)})")
    odd_types = [f"{f}={getattr(op, f)!r}" for f in _TYPE_FIELDS
                 if getattr(op, f) not in KNOWN_DTYPES]
    if odd_types:
        found.append("element types outside the declared set: " + ", ".join(odd_types))
    for sym in (decl.shape_symbols if decl else ()):
        if not _positive_int(op.shapes.get(sym)):
            found.append(f"shape symbol {sym} needs a positive integer, has "
                         f"{op.shapes.get(sym)!r}")
    if not op.tol_rel_l2 >= 0:
        found.append(f"tolerance tol_rel_l2={op.tol_rel_l2!r} is negative")
    return found


def validate(op: OpSpec) -> None:
    found = problems(op)
    if found:
        raise ValueError("; ".join(found))


def flops(op: OpSpec) -> float:
    decl = DECLARED.get(op.kind)
    if decl is None:
        raise ValueError(f"no work count for undeclared operation {op.kind!r}")
    return decl.work(op.shapes)


def describe(op: OpSpec) -> str:
    s = op.shapes
    dims = "x".join(str(s.get(k)) for k in ("M", "N", "K"))
    text = (f"{op.kind} {dims}: {op.dtype_a} x {op.dtype_b} -> {op.dtype_c}, "
            f"accumulate {op.dtype_acc}; layouts a={op.layout_a} b={op.layout_b} "
            f"c={op.layout_c}")
    return text + (f"; weight scale {op.scale}" if op.scale else "")
