"""CPU checks of the drop-in boundary: the library loads and exports every function that
include/tempo_sm100.h declares, with the binding table in _lib matching the header."""
import ctypes as C
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def header_functions():
    text = (ROOT / "include" / "tempo_sm100.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(tempo_sm100_\w+)\s*\(", text)))


def test_header_declares_the_abi():
    fns = header_functions()
    for f in ("tempo_sm100_gemm_fp16", "tempo_sm100_gemm_fp16_applicable",
              "tempo_sm100_gemm_w8a16", "tempo_sm100_workspace_bytes"):
        assert f in fns


def test_library_exports_every_declared_symbol():
    from cuda_tempiler_b200 import _lib
    lib = _lib.load()
    for f in header_functions():
        assert hasattr(lib, f), f"{f} declared in the header but not exported"
        assert f in _lib.EXPORTS, f"{f} missing from the ctypes binding table"


def test_version_string_without_gpu():
    from cuda_tempiler_b200 import _lib
    assert b"sm_100a" in _lib.load().tempo_sm100_version()



def test_noalloc_scratch_size_matches_header():
    from cuda_tempiler_b200 import _lib
    text = (ROOT / "include" / "tempo_sm100.h").read_text()
    m = re.search(r"#define TEMPO_SM100_NOALLOC_SCRATCH_BYTES \((\d+)u \* 1024u \* 1024u\)", text)
    assert m and int(m.group(1)) * 1024 * 1024 == _lib.NOALLOC_SCRATCH_BYTES


def test_noalloc_scratch_covers_every_dispatched_plan():
    """The allocation-free entry's static scratch (64 MiB) is larger than any workspace the
    fp16 dispatcher can ask for on a B200 (74 two-CTA clusters): a 2-CTA split tail holds at
    most 3 x clusters k-slices of 2 x [128][256] fp32 after the 64 KiB counter prefix, and the
    1-CTA rows use in-cluster k-splits only (no workspace).  So its size check rejects nothing
    the shipped dispatch plans on this GPU; checked over a sweep with the shipped select.py."""
    import importlib.util
    import os
    from cuda_tempiler_b200 import _lib
    P = 148 // 2
    bound = 65536 + 3 * P * 2 * 128 * 256 * 4
    assert bound <= _lib.NOALLOC_SCRATCH_BYTES
    p = os.path.join(os.path.dirname(os.path.dirname(__file__)), "cuda_tempiler_b200", "kernels",
                     "shipped", "gemm_fp16", "sm_100a", "select.py")
    spec = importlib.util.spec_from_file_location("sel16", p)
    sel = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(sel)
    worst = 0
    for M in (257, 300, 512, 1024, 2048, 4096, 8192):
        for N in (256, 1024, 3840, 8192, 15360, 30720, 65536):
            for K in (1024, 4096, 15360, 65536):
                s = sel.select("gemm_fp16", M, N, K)
                if s["cta_group"] == 2:
                    _, R, S = sel.pair_plan(M, N, K, s["bn"])
                    if S:
                        worst = max(worst, 65536 + R * S * 2 * 128 * s["bn"] * 4)
    assert 0 < worst <= bound
