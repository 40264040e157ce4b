"""CPU checks of the shipped artifacts (kernels/shipped/<op>/sm_100a): every file signed by the
manifest (md5), dispatch.inc equal to select.py's ladder, the frozen kernel equal to the current
skeleton, the ship gate the reference runs without a card (test_gate.py:78-203)."""
import importlib.util
import json
import os
import re

import pytest

from cuda_tempiler_b200.tempo.plugins.sm100 import ship
from cuda_tempiler_b200.tempo.plugins.sm100.skeletons_py import skeleton_source

ROOT = os.path.join(os.path.dirname(os.path.dirname(__file__)), "cuda_tempiler_b200", "kernels",
                    "shipped")
OPS = ("gemm_fp16", "gemm_w8a16")


def load_select(op):
    p = os.path.join(ROOT, op, "sm_100a", "select.py")
    spec = importlib.util.spec_from_file_location(f"sel_{op}", p)
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


@pytest.mark.parametrize("op", OPS)
def test_manifest_signs_every_file(op):
    assert ship.verify_ship(ROOT, op) == []
    m = json.load(open(os.path.join(ROOT, op, "sm_100a", "manifest.json")))
    assert m["schema"] == "tempo/shipped/1" and m["contract"] == "tempo/arch/1"
    assert set(m["md5"]) == {"kernel.cuh", "launch.cuh", "launch.cu", "dispatch.inc", "select.py"}


@pytest.mark.parametrize("op", OPS)
def test_dispatch_matches_select(op):
    sel = load_select(op)
    inc = open(os.path.join(ROOT, op, "sm_100a", "dispatch.inc")).read()
    table = inc[inc.index("kLadder[] = {"):]
    table = table[:table.index("};")]
    rows = re.findall(r"\{(0x7fffffff|\d+), (\d+), (\d+), (\d+), (\d+)\}", table)
    got = [[int(a, 0), int(b), int(c), int(d), int(e)] for a, b, c, d, e in rows]
    assert got == [list(r) for r in sel.LADDER]
    assert sel.LADDER[-1][0] >= 0x7FFFFFFF, "the last ladder row must cover every M"


@pytest.mark.parametrize("op", OPS)
def test_frozen_kernel_equals_skeleton(op):
    text = open(os.path.join(ROOT, op, "sm_100a", "kernel.cuh")).read()
    assert skeleton_source() in text, "skeleton changed since the last ship: re-run the ship stage"


def test_select_predicate_and_fallback():
    s16, s8 = load_select("gemm_fp16"), load_select("gemm_w8a16")
    assert s16.select("gemm_fp16", 1, 4096, 3840)["bn"] == 0           # streaming GEMV
    assert s16.select("gemm_fp16", 8, 4096, 3840)["bn"] == 0           # GEMV (tensor-core)
    assert s16.select("gemm_fp16", 16, 4096, 3840)["swap"] == 1
    assert s16.select("gemm_fp16", 4096, 15360, 3840)["bn"] == 256
    assert s16.select("gemm_fp16", 4, 4095, 3840) is None        # N % 8: not covered -> fallback
    assert s16.select("gemm_fp16", 4, 4096, 3840, arch="sm_70") is None
    assert s8.select("gemm_w8a16", 16, 5120, 17408, dtype_b="uint8") is not None
    assert s8.select("gemm_w8a16", 16, 5120, 17408, dtype_b="fp16") is None


def test_library_ladder_agrees_with_select_on_cpu():
    """bn/swap/group_m of the C++ dispatcher equal select.py's (the k-split needs the SM count,
    which a CPU host does not have)."""
    import ctypes as C
    from cuda_tempiler_b200 import _lib
    lib = _lib.load()
    sel = load_select("gemm_fp16")
    for M in (1, 16, 17, 64, 65, 128, 200, 256, 257, 4096):
        out = (C.c_int * 5)()
        assert lib.tempo_sm100_select(0, M, 4096, 4096, 0, out) == 0
        s = sel.select("gemm_fp16", M, 4096, 4096)
        if s["cta_group"] == 2:  # 2-CTA width: a wave model over the SM count (none here)
            assert out[0] >= s["bn"] and (out[1], out[3]) == (s["swap"], s["group_m"]), M
        else:
            assert (out[0], out[1], out[3]) == (s["bn"], s["swap"], s["group_m"]), M


def test_merge_ladder_partial_retune():
    """A tune that covers M <= 16 re-derives the bands up to 16 and keeps the shipped rows
    above; neighbouring rows with the same choice collapse; the last row reaches INF."""
    from cuda_tempiler_b200.tempo.plugins.sm100 import ship
    INF = ship.INF
    old = [(2, 0, 0, 0, 1), (16, 16, 1, 8, 1), (32, 64, 1, 8, 1), (64, 128, 1, 8, 1),
           (256, 128, 0, 16, 1), (INF, 256, 0, 16, 2)]
    lad, top = ship.merge_ladder([(4, 0, 0, 0, 1), (INF, 16, 1, 8, 1)], old, [1, 2, 4, 8, 16])
    assert top == 16
    assert lad == [(4, 0, 0, 0, 1), (16, 16, 1, 8, 1), (32, 64, 1, 8, 1), (64, 128, 1, 8, 1),
                   (256, 128, 0, 16, 1), (INF, 256, 0, 16, 2)]
    lad, top = ship.merge_ladder([(INF, 0, 0, 0, 1)], old, [1, 3])
    assert top == 4 and lad[0] == (4, 0, 0, 0, 1) and lad[1] == (16, 16, 1, 8, 1)
    assert ship.merge_ladder([], old, [1])[0] == old
