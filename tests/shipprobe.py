"""Build a ship directory ALONE: copy kernels/shipped/<op>/sm_100a into a scratch directory
with one host program from tests/ship_probe/, and compile launch.cu + that program with nvcc
and nothing else of the repository on the include path -- what a host tree that vendors the
ship directory does (the reference's ship probe, kernels/shipped/gemm_fp16/sm_70/ship_probe.cu
and test_gate.py)."""
import os
import shutil
import subprocess
import tempfile

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SHIPPED = os.path.join(ROOT, "cuda_tempiler_b200", "kernels", "shipped")
PROBES = os.path.join(ROOT, "tests", "ship_probe")


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def start_build(op: str):
    """(Popen of the nvcc build, path of the binary it writes)."""
    d = tempfile.mkdtemp(prefix=f"ship_{op}_")
    src = os.path.join(SHIPPED, op, "sm_100a")
    for name in os.listdir(src):
        shutil.copy(os.path.join(src, name), d)
    probe = f"probe_{op}.cu"
    shutil.copy(os.path.join(PROBES, probe), d)
    exe = os.path.join(d, "probe")
    cmd = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17", "-O3",
           "-diag-suppress", "177", "launch.cu", probe, "-o", exe]
    return subprocess.Popen(cmd, cwd=d, stdout=subprocess.PIPE, stderr=subprocess.STDOUT,
                            text=True), exe
