"""The correctness gate comes before the stopwatch (reference
tempo/core/measure/correctness.py:21-39)."""
from __future__ import annotations

from ..op.coverage import check as coverage_check  # noqa: F401
from ..op.oracle import OracleResult, gate, rel_l2  # noqa: F401

ORDER = (
    "1. build the variant",
    "2. check coverage (poison fill / atomic stamp)",
    "3. check values against a higher-precision reference (fp32 accumulate or better)",
    "4. break the symmetry with an independent, named path (fp64 spot check)",
    "5. only now start the stopwatch",
)


class TimingForbidden(AssertionError):
    pass


def must_pass_before_timing(res: OracleResult) -> None:
    if not res.ok:
        raise TimingForbidden("stopwatch forbidden: the correctness gate did not pass\n" + res.render())
