"""Operation spec validation and work counting.  The OpSpec type itself is defined by the
contract (tempo.plugins.base); the pipeline recognises *declared* operations only (reference
tempo/core/op/spec.py:19-46)."""
from __future__ import annotations

from ...plugins.base import OpSpec  # noqa: F401

KNOWN_KINDS = ("gemm",)
KNOWN_DTYPES = ("fp16", "fp32", "int8", "uint8", "q7", "bf16")


def validate(op: OpSpec) -> None:
    if op.kind not in KNOWN_KINDS:
        raise ValueError(f"operation {op.kind!r} is not declared; known: {', '.join(KNOWN_KINDS)}")
    for name in ("dtype_a", "dtype_b", "dtype_c", "dtype_acc"):
        v = getattr(op, name)
        if v not in KNOWN_DTYPES:
            raise ValueError(f"type {name}={v!r} is not declared")
    if op.kind == "gemm":
        for k in ("M", "N", "K"):
            if k not in op.shapes:
                raise ValueError(f"'gemm' needs shape {k!r}")
            if int(op.shapes[k]) <= 0:
                raise ValueError(f"shape {k} = {op.shapes[k]!r}")
    if op.tol_rel_l2 < 0:
        raise ValueError("negative tolerance")


def flops(op: OpSpec) -> float:
    if op.kind != "gemm":
        raise ValueError("work is declared for 'gemm' only")
    s = op.shapes
    return 2.0 * s["M"] * s["N"] * s["K"]


def describe(op: OpSpec) -> str:
    s = op.shapes
    return (f"{op.kind} {s.get('M')}x{s.get('N')}x{s.get('K')}  {op.dtype_a}*{op.dtype_b}->"
            f"{op.dtype_c} (acc {op.dtype_acc}), layouts {op.layout_a}/{op.layout_b}/{op.layout_c}"
            + (f", scale {op.scale}" if op.scale else ""))
