"""Drop-in proof: the sm100 plugin directory, placed into a copy of the reference tree as
tempo/plugins/sm100/, is loaded and driven by the reference's own unmodified pipeline
(``python3 -m tempo.cli plugins/selftest/space/emit``) and the kernel it emits compiles for
sm_100a.  Runs when TEMPO_REFERENCE names a reference checkout (this is a CPU test; nothing on
the GPU side reads the reference)."""
import os
import shutil
import subprocess
import sys

import pytest

REF = os.environ.get("TEMPO_REFERENCE", "")
PLUGIN = os.path.join(os.path.dirname(os.path.dirname(__file__)), "cuda_tempiler_b200", "tempo",
                      "plugins", "sm100")

pytestmark = pytest.mark.skipif(not REF or not os.path.isdir(os.path.join(REF, "tempo")),
                                reason="set TEMPO_REFERENCE to a reference checkout")


@pytest.fixture(scope="module")
def tree(tmp_path_factory):
    d = tmp_path_factory.mktemp("ref")
    dst = d / "ref"
    shutil.copytree(REF, dst, ignore=shutil.ignore_patterns(".git", "profiled"))
    shutil.copytree(PLUGIN, dst / "tempo" / "plugins" / "sm100",
                    ignore=shutil.ignore_patterns("__pycache__"))
    return dst


def run(tree, *args):
    r = subprocess.run([sys.executable, "-m", "tempo.cli", *args], cwd=tree, capture_output=True,
                       text=True, timeout=300)
    return r.returncode, r.stdout + r.stderr


def test_reference_pipeline_loads_and_selftests_plugin(tree):
    rc, out = run(tree, "plugins")
    assert rc == 0 and "sm_100a" in out
    rc, out = run(tree, "selftest", "--arch", "sm100")
    assert rc == 0 and "15/15" in out, out[-2000:]


def test_reference_space_and_emit(tree, tmp_path):
    rc, out = run(tree, "space", "--arch", "sm100", "-M", "4096", "-N", "15360", "-K", "3840")
    assert rc == 0 and "gemm_sm100_bn256" in out
    rc, out = run(tree, "emit", "--arch", "sm100", "-M", "4096", "-N", "15360", "-K", "3840",
                  "--out", str(tmp_path))
    assert rc == 0, out
    cu = [f for f in os.listdir(tmp_path) if f.endswith(".cu")]
    assert cu and "bn256_sw0" in cu[0]
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if os.path.exists(nvcc):
        r = subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17", "-c",
                            str(tmp_path / cu[0]), "-o", str(tmp_path / "k.o")],
                           capture_output=True, text=True, timeout=600)
        assert r.returncode == 0, r.stderr[-2000:]
