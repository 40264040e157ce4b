"""Section 8a -- toolchain: nvcc for sm_100a with ``-Xptxas -v``.

The verify facts are the ones the tools print: registers, spill stores/loads, stack frame and
static shared memory per entry (from ptxas), plus the CUDA runtime's local-memory size.  The
machine code of our own builds is never read (no SASS/PTX inspection), so
``ldl_stl_in_loops`` stays None and ``disasm`` refuses.
"""
from __future__ import annotations

import os
import re
import shutil
import subprocess
from pathlib import Path

from ..base import BuildResult, EnvReq, NotSupported

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
_ENTRY = re.compile(r"Compiling entry function '([^']+)' for 'sm_100a'")
_PROPS = re.compile(r"(\d+) bytes stack frame, (\d+) bytes spill stores, (\d+) bytes spill loads")
_USED = re.compile(r"Used (\d+) registers(?:, used \d+ barriers)?(?:, (\d+) bytes smem)?")


def nvcc_path() -> str | None:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    return None


def parse_ptxas(log: str) -> dict:
    """Per mangled entry: regs, spill_st, spill_ld, stack_frame, smem_static."""
    out, cur = {}, None
    for line in log.splitlines():
        m = _ENTRY.search(line)
        if m:
            cur = m.group(1)
            out[cur] = dict(regs=0, spill_st=0, spill_ld=0, stack_frame=0, smem_static=0)
            continue
        if cur is None:
            continue
        m = _PROPS.search(line)
        if m:
            out[cur].update(stack_frame=int(m.group(1)), spill_st=int(m.group(2)),
                            spill_ld=int(m.group(3)))
            continue
        m = _USED.search(line)
        if m:
            out[cur]["regs"] = int(m.group(1))
            if m.group(2):
                out[cur]["smem_static"] = int(m.group(2))
            cur = None
    return out


def demangle_family(mangled: str) -> str | None:
    """'_ZN11tempo_sm10012k_gemm_sm100ILi256ELi0ELb0EEEv...' -> 'tempo_sm100::k_gemm_sm100<256, 0, false>'."""
    m = re.search(r"k_gemm_sm100ILi(\d+)ELi(\d+)ELb([01])E", mangled)
    if not m:
        return None
    return (f"tempo_sm100::k_gemm_sm100<{m.group(1)}, {m.group(2)}, "
            f"{'true' if m.group(3) == '1' else 'false'}>")


class Sm100Toolchain:
    def arch_flags(self):
        return list(ARCH_FLAGS)

    def compile(self, source: Path, out: Path, mode: str, extra: list, build_dir: Path) -> BuildResult:
        nvcc = nvcc_path()
        if nvcc is None:
            return BuildResult(False, None, 0, 0, 0, 0, 0, 0, None, "nvcc not found")
        os.makedirs(build_dir, exist_ok=True)
        kind = {"obj": ["-c"], "shared": ["-shared", "-Xcompiler", "-fPIC"], "exe": []}.get(mode)
        if kind is None:
            raise NotSupported(f"build mode {mode!r}")
        cmd = [nvcc, *ARCH_FLAGS, "-O3", "-std=c++17", "-lineinfo", "-Xptxas", "-v", *kind,
               *extra, "-o", str(out), str(source)]
        r = subprocess.run(cmd, capture_output=True, text=True, cwd=str(build_dir))
        log = r.stdout + r.stderr
        facts = parse_ptxas(log)
        gemm = [v for k, v in facts.items() if "k_gemm_sm100" in k]
        worst = max(gemm, key=lambda v: (v["stack_frame"] + v["spill_st"] + v["spill_ld"], v["regs"]),
                    default=dict(regs=0, spill_st=0, spill_ld=0, stack_frame=0, smem_static=0))
        return BuildResult(ok=r.returncode == 0, binary=Path(out) if r.returncode == 0 else None,
                           regs=worst["regs"], spill_st=worst["spill_st"], spill_ld=worst["spill_ld"],
                           stack_frame=worst["stack_frame"], smem_static=worst["smem_static"],
                           smem_dynamic=0, ldl_stl_in_loops=None, log=log)

    def disasm(self, binary: Path) -> str:
        raise NotSupported("reading the machine code of our own builds is not done: verify uses "
                           "ptxas-reported facts and profiler counters only")

    def requirements(self):
        return [EnvReq("nvcc", nvcc_path(), "CUDA 12.9 compiler with sm_100a support"),
                EnvReq("ncu", shutil.which("ncu") or "/usr/local/cuda/bin/ncu",
                       "Nsight Compute for counter summaries (GPU box only)")]
