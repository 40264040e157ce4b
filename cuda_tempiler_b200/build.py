"""Build the in-tree sm_100a shared library ``libtempo_sm100.so`` with nvcc.

The library compiles the SHIPPED artifacts: csrc/tempo_sm100.cu (the C-ABI shim) includes the
launch.cu of kernels/shipped/gemm_fp16/sm_100a and of kernels/shipped/gemm_w8a16/sm_100a, each
of which brings its POD ABI (launch.cuh), the frozen kernels (kernel.cuh) and its generated
dispatch body (dispatch.inc) -- the reference's launch.cu + dispatch.inc scheme.

The library is the product: the CUDA kernels plus the extern "C" entry points declared in
``include/tempo_sm100.h``.  It is built in-tree so that it travels with the repository to the
GPU box; there is no JIT cache and no CPU fallback.
"""
from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
SHIPPED = PKG / "kernels" / "shipped"
LIB = PKG / "libtempo_sm100.so"
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put CUDA's bin on PATH)")


def sources() -> list:
    return (sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh"))
            + sorted(SHIPPED.glob("*/sm_100a/*.cuh")) + sorted(SHIPPED.glob("*/sm_100a/*.cu"))
            + sorted(SHIPPED.glob("*/sm_100a/*.inc")) + [INCLUDE / "tempo_sm100.h"])


def stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in sources())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every .cu under csrc/ into one shared library (no-op when up to date)."""
    if not force and not stale():
        return LIB
    cmd = [
        nvcc(), *ARCH_FLAGS, "-O3", "-std=c++17", "-lineinfo", "-Xptxas", "-v",
        "-Xcompiler", "-fPIC", "-shared", f"-I{INCLUDE}", f"-I{CSRC}", f"-I{SHIPPED}",
        "-o", str(LIB) + ".tmp", *[str(p) for p in sorted(CSRC.glob("*.cu"))],
    ]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + res.stdout + res.stderr)
    os.replace(str(LIB) + ".tmp", LIB)
    (PKG / "libtempo_sm100.ptxas.log").write_text(res.stderr)
    if verbose:
        print(res.stderr)
    return LIB


if __name__ == "__main__":
    build(force=True)
    print(LIB)
