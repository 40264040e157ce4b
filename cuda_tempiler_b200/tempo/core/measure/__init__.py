"""Measurement stage: baselines (bars), gate-before-stopwatch, paired ratios."""
