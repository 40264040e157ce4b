"""The BASELINE.json GEMM configurations as data (shapes only; inputs are seeded synthetic).

The reference derives its shape sets from model headers (bench/shapes/*.json); these are
restated from BASELINE.json's configs, not read from the reference's data files.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class GemmShape:
    name: str
    N: int
    K: int


# Config 1: the naive TEMPO-OP example shape (kernels/naive/gemm_fp16.cu).
CONFIG1 = (4096, 15360, 3840)

# Config 2: fp16 transformer-layer GEMM set, hidden 3840, 16 q heads x 256, 8 kv heads, FFN 15360.
LAYER_FP16 = (
    GemmShape("qkv", 8192, 3840),
    GemmShape("o_proj", 3840, 4096),
    GemmShape("gate_up", 30720, 3840),
    GemmShape("down", 3840, 15360),
)
LAYER_FP16_M = (1, 16, 128, 1024, 4096)

# Configs 3-5: 27B-class dense layer (hidden 5120, 64 q heads x 128, 8 kv heads, FFN 17408).
LAYER_W8 = (
    GemmShape("qkv", 10240, 5120),
    GemmShape("o_proj", 5120, 8192),
    GemmShape("gate_up", 34816, 5120),
    GemmShape("down", 5120, 17408),
)
W8_PER_CHANNEL_M = (1, 2, 4, 8, 16, 64, 512)
W8_GROUP_M = (1, 16, 256, 4096)
W8_GROUP_SIZE = 128
TP_MLP_M = (1, 16, 1024, 4096)
TP_SIZES = (1, 2, 4, 8)


def flops(M: int, N: int, K: int) -> int:
    """Useful work 2*M*N*K (reference harness.cu:16)."""
    return 2 * M * N * K


def algorithmic_bytes(M: int, N: int, K: int, w_bytes: int = 2, aux: str = "none",
                      group: int = 128) -> int:
    """Compulsory HBM traffic: read A and W once, write C once, plus scale/zero metadata.
    aux: "none" | "per_channel" (2N bytes) | "group" (3 N K / group bytes)."""
    b = 2 * M * K + w_bytes * N * K + 2 * M * N
    if aux == "per_channel":
        b += 2 * N
    elif aux == "group":
        b += 3 * N * K // group
    return b
