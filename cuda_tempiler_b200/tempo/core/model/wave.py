"""Wave and tail arithmetic; the SM count comes from the plugin (reference
tempo/core/model/wave.py)."""
from __future__ import annotations


def waves(ctas: int, quantum: int) -> float:
    return float("nan") if quantum <= 0 else ctas / float(quantum)


def efficiency(ctas: int, quantum: int) -> float:
    """ctas / (quantum * ceil(ctas / quantum)): the useful share of the launched waves."""
    if quantum <= 0 or ctas <= 0:
        return 0.0
    return ctas / float(quantum * -(-ctas // quantum))


def tail_share(ctas: int, quantum: int) -> float:
    return 1.0 - efficiency(ctas, quantum)


def nearest_quantised(ctas: int, quantum: int) -> int:
    return ctas if quantum <= 0 else quantum * -(-ctas // quantum)
