"""Serving-side binding: torch custom ops over the sm_100a kernels and a gated linear layer.

The reference's host integration (kernels/shipped/gemm_fp16/sm_70/INTEGRATION.md:83-103) is
tensor -> POD -> launch(), with the framework's own path taken when the shipped dispatcher does
not cover a shape, and the whole thing behind an environment switch that is OFF by default
(``TEMPO_KERNELS=1`` turns it on).  This module is that template for PyTorch:

* ``torch.ops.tempo.gemm_fp16(A, B)`` and ``torch.ops.tempo.gemm_w8a16(A, W, scale, zero,
  group_size)`` are strict: they run the library's kernels or raise (``NotCovered`` for a shape
  the dispatcher does not cover, RuntimeError for a CUDA error or a missing library).  They have
  fake (meta) implementations, so they trace under torch.compile / export as opaque ops.
* ``linear_fp16`` / ``linear_w8a16`` are what a model's linear layer calls.  With the switch
  off they are the framework's stock path (``F.linear`` on the dequantised weight for W8A16);
  with it on they call the custom op when ``covered()`` says the shape is shipped and fall back
  to the stock path otherwise -- the caller's fallback, never a CPU path inside this library.
* ``route_counts()`` counts which way each call went (the reference's "entry proof": prove the
  kernels are entered before trusting an end-to-end number).
"""
from __future__ import annotations

import os
import threading

import torch
import torch.nn.functional as F

from . import ops
from ._lib import NotCovered

_lock = threading.Lock()
_routes = {"tempo": 0, "fallback": 0}


def enabled() -> bool:
    """The switch, read on every call: ``TEMPO_KERNELS=1`` turns the kernels on (default 0)."""
    return os.environ.get("TEMPO_KERNELS", "0") == "1"


def route_counts(reset: bool = False) -> dict:
    with _lock:
        out = dict(_routes)
        if reset:
            for k in _routes:
                _routes[k] = 0
    return out


def _count(route: str) -> None:
    with _lock:
        _routes[route] += 1


# ------------------------------------------------------------------------------ custom ops
@torch.library.custom_op("tempo::gemm_fp16", mutates_args=())
def gemm_fp16(A: torch.Tensor, B: torch.Tensor) -> torch.Tensor:
    """C[M, N] = A[M, K] @ B[N, K]^T on the tcgen05 kernels (fp16, fp32 accumulate)."""
    return ops.gemm_fp16(A, B)


@gemm_fp16.register_fake
def _(A, B):
    return A.new_empty((A.shape[0], B.shape[0]))


@torch.library.custom_op("tempo::gemm_w8a16", mutates_args=())
def gemm_w8a16(A: torch.Tensor, W: torch.Tensor, scale: torch.Tensor,
               zero: torch.Tensor | None, group_size: int) -> torch.Tensor:
    """C[M, N] = A[M, K] @ dequant(W)[N, K]^T; W int8 with scale [N] (per-channel) or uint8 with
    scale / zero [K / group_size, N] (group-wise, GPTQ orientation)."""
    return ops.gemm_w8a16(A, W, scale, zero, group_size)


@gemm_w8a16.register_fake
def _(A, W, scale, zero, group_size):
    return A.new_empty((A.shape[0], W.shape[0]))


# ------------------------------------------------------------------------------ coverage
def _aligned(t: torch.Tensor) -> bool:
    return t.data_ptr() % 16 == 0


def covered_fp16(x2: torch.Tensor, weight: torch.Tensor) -> bool:
    """Whether the shipped fp16 dispatcher takes this problem (the reference's applicable())."""
    if not (x2.is_cuda and weight.is_cuda and x2.dtype == weight.dtype == torch.float16):
        return False
    if x2.dim() != 2 or weight.dim() != 2 or x2.stride(1) != 1 or weight.stride(1) != 1:
        return False
    M, K = x2.shape
    N = weight.shape[0]
    if weight.shape[1] != K or M == 0:
        return False
    if K % 8 or N % 8 or x2.stride(0) % 8 or weight.stride(0) % 8:
        return False
    return _aligned(x2) and _aligned(weight)


def covered_w8a16(x2, W, scale, zero, group_size) -> bool:
    if not (x2.is_cuda and W.is_cuda and x2.dtype == torch.float16):
        return False
    if W.dtype not in (torch.int8, torch.uint8) or x2.dim() != 2 or W.dim() != 2:
        return False
    if x2.stride(1) != 1 or W.stride(1) != 1:
        return False
    M, K = x2.shape
    N = W.shape[0]
    if W.shape[1] != K or M == 0 or K % 16 or N % 8 or x2.stride(0) % 8 or W.stride(0) % 16:
        return False
    if W.dtype == torch.uint8:
        if zero is None or group_size <= 0 or group_size % 64 or K % group_size or N % 16:
            return False
    return _aligned(x2) and _aligned(W)


# ------------------------------------------------------------------------------ linear layers
def linear_fp16(x: torch.Tensor, weight: torch.Tensor,
                bias: torch.Tensor | None = None) -> torch.Tensor:
    """y = x @ weight^T (+ bias) for x [..., K], weight [N, K]."""
    if enabled():
        x2 = x.reshape(-1, x.shape[-1])
        if covered_fp16(x2, weight):
            try:
                y = torch.ops.tempo.gemm_fp16(x2, weight)
            except NotCovered:
                y = None
            if y is not None:
                _count("tempo")
                y = y.reshape(*x.shape[:-1], weight.shape[0])
                return y + bias if bias is not None else y
    _count("fallback")
    return F.linear(x, weight, bias)


def dequantize(W, scale, zero=None, group_size: int = 0) -> torch.Tensor:
    """The fp16 weight the W8A16 op multiplies by (the stock path's operand): q * s[n], or
    (q - z[g][n]) * s[g][n] with g = k // group_size (reference bench/gemm_baseline.py:214-231)."""
    if W.dtype == torch.int8:
        return (W.float() * scale.float()[:, None]).half()
    s = scale.float().repeat_interleave(group_size, 0).t()
    z = zero.float().repeat_interleave(group_size, 0).t()
    return ((W.float() - z) * s).half()


def linear_w8a16(x: torch.Tensor, W: torch.Tensor, scale: torch.Tensor,
                 zero: torch.Tensor | None = None, group_size: int = 0,
                 bias: torch.Tensor | None = None) -> torch.Tensor:
    if enabled():
        x2 = x.reshape(-1, x.shape[-1])
        if covered_w8a16(x2, W, scale, zero, group_size):
            try:
                y = torch.ops.tempo.gemm_w8a16(x2, W, scale, zero, group_size)
            except NotCovered:
                y = None
            if y is not None:
                _count("tempo")
                y = y.reshape(*x.shape[:-1], W.shape[0])
                return y + bias if bias is not None else y
    _count("fallback")
    return F.linear(x, dequantize(W, scale, zero, group_size), bias)
