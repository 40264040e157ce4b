"""Paired time ratios: arms alternate inside each round; the statistic is the median of the
per-round ratios, not the ratio of medians (reference tempo/core/measure/ratio.py:63-73)."""
from __future__ import annotations

DISCIPLINE = (
    "correctness gate before the stopwatch",
    "paired ratios, arms alternated inside each round",
    "median of the ratios, not the ratio of the medians",
    "GPU clocks are never locked or changed; they are sampled and reported",
    "L2 flushed (or inputs larger than L2) before every timed launch",
)


def median_ratio(pairs):
    vals = sorted(float(a) / float(b) for a, b in pairs if b)
    if not vals:
        return float("nan")
    n = len(vals)
    return vals[n // 2] if n % 2 else 0.5 * (vals[n // 2 - 1] + vals[n // 2])


def median_ci(values, z: float = 1.96):
    """Distribution-free CI of the median by order statistics (normal approximation)."""
    v = sorted(values)
    n = len(v)
    if n < 3:
        return ()
    half = z * (n ** 0.5) / 2.0
    lo = max(0, int(n / 2.0 - half))
    hi = min(n - 1, int(n / 2.0 + half))
    return (v[lo], v[hi])
