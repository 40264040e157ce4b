"""Section 3 -- the tensor unit: 5th-generation tensor cores, ``tcgen05.mma.cta_group::1
.kind::f16`` (UMMA), M = 128, N = 16..256 step 16, K = 16, fp16/bf16 operands read straight
from shared memory through descriptors, fp32 accumulator in TMEM.

Fragment maps: A and B are never in registers (``smem_direct``), so their maps are empty;
the accumulator lives in TMEM, not in registers, so ``frag.c`` yields no register slots and
``acc_regs_per_thread`` derives 0 -- the register-budget law correctly sees no accumulator
pressure.  (The epilogue's tcgen05.ld 32x32b shape -- lane l of warp w reads TMEM lane
32*(w%4)+l -- is a load, not a fragment of the MMA.)
"""
from __future__ import annotations

from ..base import FragmentMap, PluginCapabilityError, TensorOp, not_measured

_EMPTY = lambda lane: ()

UMMA_NS = tuple(range(16, 257, 16))


def _op(n: int, dtype: str) -> TensorOp:
    return TensorOp(id=f"UMMA.{dtype.upper()}.F32.M128N{n}K16", m=128, n=n, k=16,
                    in_dtypes=(dtype, dtype), acc_dtype="fp32",
                    frag=FragmentMap(a=_EMPTY, b=_EMPTY, c=_EMPTY),
                    cost=not_measured(f"LAT.UMMA_128x{n}x16", "cycle"),
                    operand_source="smem_direct", loader=None,
                    exact_while="fp32 accumulate")


class Sm100TensorUnit:
    def __init__(self):
        self._ops = tuple(_op(n, d) for d in ("fp16", "bf16") for n in UMMA_NS)

    def ops(self):
        return self._ops

    def select(self, in_dtypes: tuple, acc_dtype: str) -> TensorOp:
        if acc_dtype != "fp32":
            raise PluginCapabilityError(f"accumulator {acc_dtype!r}: only fp32 accumulation is "
                                        "offered (an fp16 accumulator loses the gate)")
        a, b = in_dtypes
        if a == b and a in ("fp16", "bf16"):
            return next(o for o in self._ops if o.in_dtypes == (a, b) and o.n == 256)
        if a == "fp16" and b in ("int8", "uint8"):
            base = next(o for o in self._ops if o.in_dtypes == ("fp16", "fp16") and o.n == 256)
            return TensorOp(id=base.id + ".DEQ_" + b.upper(), m=base.m, n=base.n, k=base.k,
                            in_dtypes=(a, b), acc_dtype="fp32", frag=base.frag, cost=base.cost,
                            operand_source="smem_direct", loader="smem_dequant",
                            exact_while=base.exact_while)
        raise PluginCapabilityError(f"no tensor op for operands {in_dtypes!r}")
