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
