"""Each ship directory builds alone: a copy of kernels/shipped/<op>/sm_100a plus one host
program compiles and links with nvcc (cross-compiled for sm_100a; no GPU needed)."""
import os

from shipprobe import start_build


def test_ship_dirs_build_alone():
    jobs = {op: start_build(op) for op in ("gemm_fp16", "gemm_w8a16")}
    for op, (proc, exe) in jobs.items():
        out, _ = proc.communicate(timeout=900)
        assert proc.returncode == 0, f"{op}: {out[-3000:]}"
        assert os.path.exists(exe)
