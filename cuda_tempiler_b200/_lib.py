"""ctypes binding of ``libtempo_sm100.so`` (the C-ABI in ``include/tempo_sm100.h``).

Loading fails loudly: there is no CPU fallback for the product path.  ``EXPORTS`` lists
every symbol the header declares; tests check that the library exports all of them.
"""
from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

from . import build as _build

LIB_PATH = _build.LIB

CUDA_SUCCESS = 0
CUDA_ERROR_INVALID_CONFIGURATION = 9  # "not covered": caller takes its fallback

W8_INT8_PER_CHANNEL = 1
W8_UINT8_GROUP = 2
NOALLOC_SCRATCH_BYTES = 64 * 1024 * 1024  # TEMPO_SM100_NOALLOC_SCRATCH_BYTES

_vp, _i, _sz = C.c_void_p, C.c_int, C.c_size_t
_ip = C.POINTER(C.c_int)

EXPORTS = {
    "tempo_sm100_gemm_fp16_applicable": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i]),
    "tempo_sm100_gemm_fp16": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp, _sz, _vp]),
    "tempo_sm100_gemm_w8a16_applicable": (
        _i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i]),
    "tempo_sm100_gemm_w8a16": (
        _i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _vp, _sz, _vp]),
    "tempo_sm100_workspace_bytes": (_sz, [_i, _i, _i, _i]),
    "tempo_sm100_gemm_hyperform": (
        _i, [_i, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i,
             _vp, _sz, _vp]),
    "tempo_sm100_gemm_hyperform_cg": (
        _i, [_i, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i,
             _vp, _sz, _vp]),
    "tempo_sm100_pair_resources": (_i, [_i, _ip]),
    "tempo_sm100_select": (_i, [_i, _i, _i, _i, _sz, _ip]),
    "tempo_sm100_hyperform_resources": (_i, [_i, _i, _i, _ip]),
    "tempo_sm100_naive_gemm_fp16": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp]),
    "tempo_sm100_naive_gemm_w8a16": (
        _i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _vp]),
    "tempo_sm100_device_status": (_i, [_ip, _i]),
    "tempo_sm100_silu_mul": (_i, [_vp, _vp, _i, _i, _i, _i, _i, _vp]),
    "tempo_sm100_gemm_fp16_swiglu": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp]),
    "tempo_sm100_gemm_w8a16_swiglu": (
        _i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _vp, _sz, _vp]),
    "tempo_sm100_ipc_alloc": (_i, [_sz, C.POINTER(C.c_void_p)]),
    "tempo_sm100_ipc_free": (_i, [_vp]),
    "tempo_sm100_ipc_handle": (_i, [_vp, _vp]),
    "tempo_sm100_ipc_open": (_i, [_vp, C.POINTER(C.c_void_p)]),
    "tempo_sm100_ipc_close": (_i, [_vp]),
    "tempo_sm100_allreduce_oneshot": (
        _i, [_vp, _vp, C.c_longlong, C.c_longlong, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p),
             _i, _i, C.c_uint, _i, _vp]),
    "tempo_sm100_allreduce_oneshot_dev": (
        _i, [_vp, _vp, C.c_longlong, C.c_longlong, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p),
             _i, _i, _vp, _i, _vp]),
    "tempo_sm100_allreduce_oneshot_timed": (
        _i, [_vp, _vp, C.c_longlong, C.c_longlong, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p),
             _i, _i, C.c_uint, _i, C.c_ulonglong, _vp]),
    "tempo_sm100_version": (C.c_char_p, []),
    "tempo_sm100_probe_bulk_feed": (_i, [_vp, _sz, _i, _i, _vp, _vp]),
    "tempo_sm100_probe_chase": (_i, [_vp, _i, _vp, _vp]),
    "tempo_sm100_probe_dequant": (_i, [_vp, _i, _i, _vp, _vp]),
    "tempo_sm100_probe_store": (_i, [_vp, _sz, _i, _vp, _vp]),
    "tempo_sm100_gemm_fp16_noalloc": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp]),
}

_lock = threading.Lock()
_lib = None


class NotCovered(RuntimeError):
    """The dispatcher does not cover this problem (cudaErrorInvalidConfiguration)."""


def load(path: Path | str | None = None, build_if_missing: bool = True) -> C.CDLL:
    """Load (building first if absent or stale and nvcc exists) and bind every export."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path else LIB_PATH
        if path is None and build_if_missing:
            try:
                if _build.stale():
                    _build.build()
            except RuntimeError:
                if not p.exists():
                    raise
        if not p.exists():
            raise RuntimeError(f"{p} is missing: run `python -m cuda_tempiler_b200.build`")
        lib = C.CDLL(str(p))
        for name, (res, args) in EXPORTS.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if path is None:
            _lib = lib
        return lib


def check(rc: int, what: str) -> None:
    if rc == CUDA_SUCCESS:
        return
    if rc == CUDA_ERROR_INVALID_CONFIGURATION:
        raise NotCovered(f"{what}: not covered by the sm_100a dispatcher")
    raise RuntimeError(f"{what}: CUDA error {rc}")
