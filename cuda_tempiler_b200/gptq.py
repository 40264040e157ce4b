"""GPTQ 8-bit checkpoint format -> the W8A16 kernel's layout.

GPTQ (bits=8) stores (reference bench/gemm_baseline.py:214-231): ``qweight`` int32 [K/4, N]
with byte j of qweight[k4, n] = q[4*k4 + j, n]; ``qzeros`` int32 [K/G, N/4] with byte j of
qzeros[g, n4] = z[g, 4*n4 + j]; ``scales`` fp16 [K/G, N]; W[k, n] = (q[k, n] - z[k//G, n]) *
s[k//G, n] (no +1 on the zero).

The kernel reads uint8 W [N][K] (K contiguous: TMA tiles of 128 rows x 64 k), fp16 scale
[K/G][N] and uint8 zero [K/G][N].  Scale is GPTQ's array as is, and zero is qzeros' memory
read as bytes (little-endian), so both are zero-copy views; only qweight is transposed once.
"""
from __future__ import annotations

import torch


def repack_gptq_int8(qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor,
                     group_size: int):
    """Returns (W uint8 [N, K] contiguous, scale fp16 [K/G, N], zero uint8 [K/G, N])."""
    if qweight.dtype != torch.int32 or qzeros.dtype != torch.int32:
        raise ValueError("qweight and qzeros must be int32")
    K4, N = qweight.shape
    K = 4 * K4
    G = group_size
    if K % G or scales.shape != (K // G, N) or qzeros.shape != (K // G, N // 4):
        raise ValueError(f"inconsistent GPTQ shapes: qweight {tuple(qweight.shape)}, qzeros "
                         f"{tuple(qzeros.shape)}, scales {tuple(scales.shape)}, G={G}")
    qb = qweight.contiguous().view(torch.uint8).view(K4, N, 4)      # [k4, n, j] = q[4 k4 + j, n]
    W = qb.permute(1, 0, 2).reshape(N, K).contiguous()               # [n, 4 k4 + j]
    zero = qzeros.contiguous().view(torch.uint8).view(K // G, N)     # byte j of [g, n4] = z[g, 4 n4 + j]
    return W, scales.contiguous(), zero


def dequantize(W: torch.Tensor, scale: torch.Tensor, zero: torch.Tensor, group_size: int):
    """fp32 [N, K] weights from the kernel layout (for checks; not on the hot path)."""
    N, K = W.shape
    s = scale.float().repeat_interleave(group_size, 0)[:K].T     # [N, K]
    z = zero.float().repeat_interleave(group_size, 0)[:K].T
    return (W.float() - z) * s
