"""The shipped path run from a ship directory built alone (a copy of
kernels/shipped/<op>/sm_100a + one host program, nothing else of the repository): the fp16
probe runs the reference ship probe's six shapes and patterned inputs against fp64 cells
(kernels/shipped/gemm_fp16/sm_70/ship_probe.cu:35-99); the W8A16 probe runs per-channel and
group-wise weights at decode, tile and prefill sizes."""
import subprocess

import pytest

from shipprobe import start_build

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("op", ["gemm_fp16", "gemm_w8a16"])
def test_ship_probe(dev, op):
    proc, exe = start_build(op)
    out, _ = proc.communicate(timeout=900)
    assert proc.returncode == 0, out[-3000:]
    run = subprocess.run([exe], capture_output=True, text=True, timeout=600)
    print(run.stdout)
    assert run.returncode == 0 and "SHIPPED PATH: PASS" in run.stdout, run.stdout + run.stderr
