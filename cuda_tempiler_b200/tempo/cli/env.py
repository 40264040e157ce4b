"""The single place that resolves tool paths (reference tempo/cli/env.py:6-30)."""
from __future__ import annotations

import os
import shutil


def tool(name: str) -> str | None:
    for c in (os.environ.get(name.upper()), shutil.which(name),
              os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", name)):
        if c and os.path.exists(c):
            return c
    return None


def report() -> list:
    rows = []
    for t in ("nvcc", "ncu", "nvidia-smi"):
        rows.append((t, tool(t) or "NOT FOUND"))
    try:
        import torch
        rows.append(("torch", torch.__version__))
        rows.append(("cuda device", torch.cuda.get_device_name(0) if torch.cuda.is_available()
                     else "none (CPU-only host: build/space/emit/verify work, measure needs a GPU)"))
    except Exception as e:  # torch is plumbing only; the pipeline stages do not need it
        rows.append(("torch", f"unavailable ({e})"))
    return rows


def main(argv=None) -> int:
    for k, v in report():
        print(f"  {k:<12} {v}")
    return 0
