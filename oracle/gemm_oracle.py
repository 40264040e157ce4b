"""TEST INFRASTRUCTURE ONLY -- CPU oracle for the sm_100a GEMM path (numpy, fp32 accumulate).

Restates, in numpy, the reference's correctness machinery for this path:

* ``rel_l2``: relative L2 error, reference tempo/core/op/oracle.py:114-124
  (sqrt(sum (got-ref)^2 / sum ref^2); NaN when the reference is all zero).
* ``gemm_fp16_ref``: C = A * B^T with fp32 accumulation on fp16 inputs -- the op of the
  naive INPUT kernel, reference kernels/naive/gemm_fp16.cu:60-68, and the fp32 numpy oracle
  BASELINE names.
* ``spot_fp64``: the independent fp64 spot check on sampled cells, reference
  tempo/plugins/sm70/skeletons/gemm_hmma884/harness.cu:59-72 (a different accumulation path,
  the "named independent path" of oracle.py:127-151).
* ``poison_count``: cells still holding the 0x7f7f poison after the kernel ran, reference
  harness.cu:50-57 (coverage: every output cell written).
* ``dequant_per_channel`` / ``dequant_group``: W = q * s[n] and W = (q - z[g]) * s[g], g = k // G,
  the GPTQ reconstruction of reference bench/gemm_baseline.py:214-231 (no +1 on the zero).
* ``ship_probe_inputs`` / ``ship_probe_cells``: the patterned inputs and sampled cells of the
  reference's ship probe, kernels/shipped/gemm_fp16/sm_70/ship_probe.cu:41-80.
"""
from __future__ import annotations

import numpy as np

GATE_REL_L2 = 3e-3  # BASELINE correctness gate; reference harness.cu:163 uses the same value


def rel_l2(got, ref) -> float:
    g = np.asarray(got, dtype=np.float64).ravel()
    r = np.asarray(ref, dtype=np.float64).ravel()
    den = float(np.dot(r, r))
    if den <= 0.0:
        return float("nan")
    d = g - r
    return float(np.sqrt(np.dot(d, d) / den))


def gemm_fp16_ref(A: np.ndarray, B: np.ndarray) -> np.ndarray:
    """fp32-accumulated C = A @ B.T for fp16 A [M,K], B [N,K]; returns fp32 [M,N]."""
    return A.astype(np.float32) @ B.astype(np.float32).T


def gemm_w_ref(A: np.ndarray, Wf32: np.ndarray) -> np.ndarray:
    """fp32 C = A @ W.T for an already dequantised fp32 weight W [N,K]."""
    return A.astype(np.float32) @ Wf32.T


def dequant_per_channel(q: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """int8 q [N,K], fp16 scale [N] -> fp32 W[n,k] = q[n,k] * s[n]."""
    return q.astype(np.float32) * scale.astype(np.float32)[:, None]


def dequant_group(q: np.ndarray, scale: np.ndarray, zero: np.ndarray, group: int) -> np.ndarray:
    """uint8 q [N,K], fp16 scale [K/G,N], uint8 zero [K/G,N] (GPTQ orientation) -> fp32
    (q[n,k] - z[k//G,n]) * s[k//G,n]."""
    N, K = q.shape
    s = np.repeat(scale.astype(np.float32), group, axis=0)[:K].T
    z = np.repeat(zero.astype(np.float32), group, axis=0)[:K].T
    return (q.astype(np.float32) - z) * s


def spot_fp64(A: np.ndarray, B: np.ndarray, C: np.ndarray, n_spots: int = 2048,
              seed: int = 7) -> float:
    """rel_l2 of C against an fp64 dot product on n_spots sampled (m, n) cells."""
    M, K = A.shape
    N = B.shape[0]
    rng = np.random.default_rng(seed)
    ms = rng.integers(0, M, n_spots)
    ns = rng.integers(0, N, n_spots)
    ref = np.einsum("ik,ik->i", A[ms].astype(np.float64), B[ns].astype(np.float64))
    return rel_l2(C[ms, ns].astype(np.float64), ref)


def poison_count(C: np.ndarray) -> int:
    """Number of fp16 cells still equal to the 0x7f7f poison pattern."""
    return int(np.count_nonzero(C.view(np.uint16) == 0x7F7F))


# ------------------------------------------------------------------ seeded input generators
def inputs_config1(M: int, N: int, K: int, seed: int = 0):
    """Config 1: A, B fp16 ~ U(-1,1)/sqrt(K), B stored [N,K]."""
    rng = np.random.default_rng(seed)
    a = (rng.uniform(-1, 1, (M, K)) / np.sqrt(K)).astype(np.float16)
    b = (rng.uniform(-1, 1, (N, K)) / np.sqrt(K)).astype(np.float16)
    return a, b


def inputs_layer(M: int, N: int, K: int, seed: int = 1):
    """Config 2: weights N(0, 0.02) fp16 [N,K], activations N(0,1) fp16 [M,K]."""
    rng = np.random.default_rng(seed)
    a = rng.standard_normal((M, K), dtype=np.float32).astype(np.float16)
    w = (rng.standard_normal((N, K), dtype=np.float32) * 0.02).astype(np.float16)
    return a, w


def inputs_w8_per_channel(M: int, N: int, K: int, seed: int = 2):
    """Config 3: int8 q U[-127,127] [N,K]; fp16 scale = absmax/127 of a notional fp16 weight
    drawn N(0, 0.02) (so scale ~ |N(0,0.02)|max/127); fp16 activations N(0,1)."""
    rng = np.random.default_rng(seed)
    a = rng.standard_normal((M, K), dtype=np.float32).astype(np.float16)
    q = rng.integers(-127, 128, (N, K), dtype=np.int16).astype(np.int8)
    absmax = np.abs(rng.standard_normal((N, 64), dtype=np.float32) * 0.02).max(axis=1)
    scale = (absmax / 127.0).astype(np.float16)
    return a, q, scale


def inputs_w8_group(M: int, N: int, K: int, group: int = 128, seed: int = 3):
    """Config 4: uint8 q U[0,255] [N,K], fp16 scale U(1e-3,2e-2) [K/G,N], uint8 zero U[100,156]
    [K/G,N] (GPTQ orientation)."""
    rng = np.random.default_rng(seed)
    a = rng.standard_normal((M, K), dtype=np.float32).astype(np.float16)
    q = rng.integers(0, 256, (N, K), dtype=np.int16).astype(np.uint8)
    scale = rng.uniform(1e-3, 2e-2, (K // group, N)).astype(np.float16)
    zero = rng.integers(100, 157, (K // group, N), dtype=np.int16).astype(np.uint8)
    return a, q, scale, zero


# ------------------------------------------------------------------ ship-probe known answers
SHIP_PROBE_SHAPES = [  # (M, N, K) of ship_probe.cu:42-46
    (1, 4096, 3840), (8, 4096, 3840), (32, 15360, 3840),
    (128, 4096, 3840), (512, 15360, 3840), (2048, 3840, 15360),
]


def ship_probe_inputs(M: int, N: int, K: int):
    ia = np.arange(M * K, dtype=np.int64)
    ib = np.arange(N * K, dtype=np.int64)
    a = (((ia % 7) - 3) * 0.125).astype(np.float16).reshape(M, K)
    b = (((ib % 5) - 2) * 0.125).astype(np.float16).reshape(N, K)
    return a, b


def ship_probe_cells(M: int, N: int):
    t = np.arange(64)
    return (t * 37) % M, (t * 53) % N


def ship_probe_expected(M: int, N: int, K: int) -> np.ndarray:
    """fp64 reference values on the 64 probe cells."""
    a, b = ship_probe_inputs(M, N, K)
    ms, ns = ship_probe_cells(M, N)
    return np.einsum("ik,ik->i", a[ms].astype(np.float64), b[ns].astype(np.float64))


def ship_probe_maxrel(got_cells: np.ndarray, expected: np.ndarray) -> float:
    """Max of |got - ref| / (|ref| + 1e-3) over the probe cells (ship_probe.cu:75-78)."""
    return float(np.max(np.abs(got_cells.astype(np.float64) - expected) / (np.abs(expected) + 1e-3)))
