"""PyTorch-facing wrappers of the sm_100a kernels (device memory and streams come from torch;
the arithmetic runs only in ``libtempo_sm100.so``).

``gemm_fp16(A, B)`` computes ``A @ B.T`` for A [M,K], B [N,K] fp16 (the reference's k/k/n op,
kernels/shipped/gemm_fp16/sm_70/launch.cuh:20-26).  ``gemm_w8a16`` takes an 8-bit weight
[N,K] with per-channel or group-wise scales.  A problem the dispatcher does not cover raises
``NotCovered``; nothing falls back silently.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from ._lib import NotCovered, W8_INT8_PER_CHANNEL, W8_UINT8_GROUP  # noqa: F401

_ws_cache: dict = {}
# the W8A16 prefill's fp16 weight copy starts after the workspace's 64 KiB counter prefix
EXPAND_OFFSET = 65536


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def workspace(dev: torch.device, nbytes: int) -> torch.Tensor | None:
    """A zero-filled split-K workspace for (device, current stream), grown on demand.
    The kernels leave it zero-filled after every launch."""
    if nbytes <= 0:
        return None
    key = (dev.index, _stream(dev))
    ws = _ws_cache.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=dev)
        _ws_cache[key] = ws
    return ws


def _check_2d(t: torch.Tensor, name: str, dtype) -> None:
    if t.dim() != 2 or t.dtype != dtype or not t.is_cuda or t.stride(1) != 1:
        raise ValueError(f"{name}: expected a row-major 2-D {dtype} CUDA tensor, got "
                         f"{tuple(t.shape)} {t.dtype} stride {t.stride()} on {t.device}")


def gemm_fp16(A: torch.Tensor, B: torch.Tensor, out: torch.Tensor | None = None,
              use_workspace: bool = True) -> torch.Tensor:
    lib = _lib.load()
    _check_2d(A, "A", torch.float16)
    _check_2d(B, "B", torch.float16)
    M, K = A.shape
    N = B.shape[0]
    if B.shape[1] != K:
        raise ValueError(f"K mismatch: A {tuple(A.shape)} B {tuple(B.shape)}")
    if out is None:
        out = torch.empty((M, N), dtype=torch.float16, device=A.device)
    _check_2d(out, "C", torch.float16)
    nb = lib.tempo_sm100_workspace_bytes(M, N, K, 0) if use_workspace else 0
    ws = workspace(A.device, nb)
    rc = lib.tempo_sm100_gemm_fp16(
        _ptr(A), _ptr(B), _ptr(out), M, N, K, A.stride(0), B.stride(0), out.stride(0),
        _ptr(ws), 0 if ws is None else ws.numel(), _stream(A.device))
    _lib.check(rc, "tempo_sm100_gemm_fp16")
    return out


def gemm_w8a16(A: torch.Tensor, W: torch.Tensor, scale: torch.Tensor,
               zero: torch.Tensor | None = None, group_size: int = 0,
               out: torch.Tensor | None = None, use_workspace: bool = True) -> torch.Tensor:
    """kind: int8 W with scale [N] -> per-channel symmetric; uint8 W with scale/zero
    [K/group_size, N] (GPTQ orientation) -> group-wise asymmetric."""
    lib = _lib.load()
    _check_2d(A, "A", torch.float16)
    M, K = A.shape
    N = W.shape[0]
    if W.dtype == torch.int8:
        kind = W8_INT8_PER_CHANNEL
        _check_2d(W, "W", torch.int8)
    elif W.dtype == torch.uint8:
        kind = W8_UINT8_GROUP
        _check_2d(W, "W", torch.uint8)
        if zero is None or group_size <= 0:
            raise ValueError("uint8 group-wise weights need zero and group_size")
    else:
        raise ValueError(f"W dtype {W.dtype}: expected int8 or uint8")
    if out is None:
        out = torch.empty((M, N), dtype=torch.float16, device=A.device)
    nb = lib.tempo_sm100_workspace_bytes(M, N, K, kind) if use_workspace else 0
    ws = workspace(A.device, nb)
    rc = lib.tempo_sm100_gemm_w8a16(
        _ptr(A), _ptr(W), _ptr(scale.contiguous()), _ptr(zero.contiguous() if zero is not None else None),
        _ptr(out), M, N, K, A.stride(0), W.stride(0), out.stride(0), kind, group_size,
        _ptr(ws), 0 if ws is None else ws.numel(), _stream(A.device))
    _lib.check(rc, "tempo_sm100_gemm_w8a16")
    return out


def gemm_hyperform(A: torch.Tensor, W: torch.Tensor, *, bn: int, swap: bool, splits: int = 1,
                   group_m: int = 8, max_ctas: int = 0, cta_group: int = 1,
                   scale: torch.Tensor | None = None,
                   zero: torch.Tensor | None = None, group_size: int = 0,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    """Launch one explicit hyperform (search-space point) of the skeleton family; bn=0 is the
    decode GEMV (M <= 16), whose variant group_m selects: 1 CUDA-core FMAs, 2 warp tensor-core
    MMAs, anything else by M as the dispatcher does."""
    lib = _lib.load()
    M, K = A.shape
    N = W.shape[0]
    kind = 0 if W.dtype == torch.float16 else (W8_INT8_PER_CHANNEL if W.dtype == torch.int8
                                               else W8_UINT8_GROUP)
    if out is None:
        out = torch.empty((M, N), dtype=torch.float16, device=A.device)
    tiles = -(-(N if swap else M) // 128) * -(-(M if swap else N) // max(bn, 1))
    nb = 0
    if splits > 1 and cta_group == 2:
        # stream-K bound: 2 counters per tile of at most 2 waves, (3 x clusters) slot pairs
        P = torch.cuda.get_device_properties(A.device).multi_processor_count // 2
        nb = 65536 + 3 * P * 2 * 128 * bn * 4
    elif splits > 1:  # the fixed 64 KiB counter prefix, then the partials
        nb = 65536 + tiles * splits * 128 * bn * 4
    ws = workspace(A.device, nb)
    rc = lib.tempo_sm100_gemm_hyperform_cg(
        kind, _ptr(A), _ptr(W), _ptr(scale), _ptr(zero), _ptr(out), M, N, K, A.stride(0),
        W.stride(0), out.stride(0), group_size, bn, int(swap), splits, group_m, max_ctas,
        cta_group, _ptr(ws), 0 if ws is None else ws.numel(), _stream(A.device))
    _lib.check(rc, f"hyperform bn={bn} swap={swap} splits={splits}")
    return out


def naive_gemm_fp16(A: torch.Tensor, B: torch.Tensor) -> torch.Tensor:
    """The naive INPUT bar (one thread per output)."""
    lib = _lib.load()
    M, K = A.shape
    N = B.shape[0]
    out = torch.empty((M, N), dtype=torch.float16, device=A.device)
    rc = lib.tempo_sm100_naive_gemm_fp16(_ptr(A), _ptr(B), _ptr(out), M, N, K, A.stride(0),
                                         B.stride(0), out.stride(0), _stream(A.device))
    _lib.check(rc, "naive_gemm_fp16")
    return out


def naive_gemm_w8a16(A, W, scale, zero=None, group_size=0) -> torch.Tensor:
    lib = _lib.load()
    M, K = A.shape
    N = W.shape[0]
    kind = W8_INT8_PER_CHANNEL if W.dtype == torch.int8 else W8_UINT8_GROUP
    out = torch.empty((M, N), dtype=torch.float16, device=A.device)
    rc = lib.tempo_sm100_naive_gemm_w8a16(_ptr(A), _ptr(W), _ptr(scale), _ptr(zero), _ptr(out),
                                          M, N, K, A.stride(0), W.stride(0), out.stride(0), kind,
                                          group_size, _stream(A.device))
    _lib.check(rc, "naive_gemm_w8a16")
    return out


def select(kind: int, M: int, N: int, K: int, ws_bytes: int = 1 << 40) -> dict:
    lib = _lib.load()
    out = (C.c_int * 5)()
    rc = lib.tempo_sm100_select(kind, M, N, K, ws_bytes, out)
    _lib.check(rc, "select")
    return dict(bn=out[0], swap=out[1], splits=out[2], group_m=out[3], stages=out[4])


def device_status(reset: bool = True) -> list:
    lib = _lib.load()
    out = (C.c_int * 4)()
    rc = lib.tempo_sm100_device_status(out, int(reset))
    _lib.check(rc, "device_status")
    return list(out)


def silu_mul(gu: torch.Tensor, out: torch.Tensor | None = None, block: int = 0) -> torch.Tensor:
    """SwiGLU step: gu [M, 2I] holds [gate | up] (block 0) or gate and up alternating in blocks
    of `block` columns; returns silu(gate) * up as [M, I] fp16."""
    lib = _lib.load()
    _check_2d(gu, "gu", torch.float16)
    M, I2 = gu.shape
    I = I2 // 2
    if out is None:
        out = torch.empty((M, I), dtype=torch.float16, device=gu.device)
    rc = lib.tempo_sm100_silu_mul(_ptr(gu), _ptr(out), M, I, gu.stride(0), out.stride(0), block,
                                  _stream(gu.device))
    _lib.check(rc, "tempo_sm100_silu_mul")
    return out


def gemm_fp16_swiglu(A: torch.Tensor, W: torch.Tensor,
                     out: torch.Tensor | None = None) -> torch.Tensor:
    """silu(A Wg^T) * (A Wu^T) with gate/up rows of W interleaved in blocks of 64 (see
    ``tp.interleave_rows``); raises NotCovered for M <= 256."""
    lib = _lib.load()
    _check_2d(A, "A", torch.float16)
    _check_2d(W, "W", torch.float16)
    M, K = A.shape
    N = W.shape[0]
    if out is None:
        out = torch.empty((M, N // 2), dtype=torch.float16, device=A.device)
    rc = lib.tempo_sm100_gemm_fp16_swiglu(_ptr(A), _ptr(W), _ptr(out), M, N, K, A.stride(0),
                                          W.stride(0), out.stride(0), _stream(A.device))
    _lib.check(rc, "tempo_sm100_gemm_fp16_swiglu")
    return out


def gemm_w8a16_swiglu(A: torch.Tensor, W: torch.Tensor, scale: torch.Tensor,
                      zero: torch.Tensor | None = None, group_size: int = 0,
                      out: torch.Tensor | None = None) -> torch.Tensor:
    """The W8A16 form of ``gemm_fp16_swiglu`` (rows, scales and zero points interleaved alike);
    raises NotCovered below M = 512."""
    lib = _lib.load()
    _check_2d(A, "A", torch.float16)
    M, K = A.shape
    N = W.shape[0]
    kind = W8_INT8_PER_CHANNEL if W.dtype == torch.int8 else W8_UINT8_GROUP
    if out is None:
        out = torch.empty((M, N // 2), dtype=torch.float16, device=A.device)
    ws = workspace(A.device, EXPAND_OFFSET + N * K * 2)
    rc = lib.tempo_sm100_gemm_w8a16_swiglu(
        _ptr(A), _ptr(W), _ptr(scale.contiguous()),
        _ptr(zero.contiguous() if zero is not None else None), _ptr(out), M, N, K, A.stride(0),
        W.stride(0), out.stride(0), kind, group_size, _ptr(ws), 0 if ws is None else ws.numel(),
        _stream(A.device))
    _lib.check(rc, "tempo_sm100_gemm_w8a16_swiglu")
    return out
