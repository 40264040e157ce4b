"""Tensor-parallel W8A16 MLP: SwiGLU MLP of a dense layer split over the
ranks of a process group, one process per GPU.

    gate_up  column-parallel: rank r holds gate rows [r I/tp, (r+1) I/tp) and the matching up
             rows, stacked as one [2 I/tp, H] weight, so its GEMM output [M, 2 I/tp] is
             [gate_r | up_r] and SiLU(gate_r) * up_r needs no communication;
    down     row-parallel: rank r holds W_down[:, r I/tp : (r+1) I/tp] as a K-contiguous
             [H, I/tp] weight and produces a partial [M, H];
    reduce   one all-reduce (sum) of the fp16 [M, H] partial -- the only exchange step.

The reference is single-GPU (it has no multi-GPU code); this helper is new.  Each GEMM is the
sm_100a kernel (``ops.gemm_w8a16`` / ``ops.gemm_fp16``); the SwiGLU step is the library's
``silu_mul`` kernel; the all-reduce is ``torch.distributed.all_reduce`` (NCCL over NVLink on
B200).  ``gemm``/``swiglu`` are injectable so the sharding algebra can be checked on CPU ranks
(gloo) against an oracle.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


def shard_rows(n_total: int, world: int, rank: int) -> slice:
    if n_total % world:
        raise ValueError(f"{n_total} rows do not split over {world} ranks")
    per = n_total // world
    return slice(rank * per, (rank + 1) * per)


@dataclass
class MLPShard:
    """One rank's weights: W* are [rows, K] (K contiguous); scales per output row (int8) or
    None (fp16 weights)."""
    w_gate_up: torch.Tensor
    s_gate_up: torch.Tensor | None
    w_down: torch.Tensor
    s_down: torch.Tensor | None
    inter: int  # I / tp, the intermediate columns this rank owns


def shard_mlp(w_gate: torch.Tensor, w_up: torch.Tensor, w_down: torch.Tensor, world: int,
              rank: int, s_gate=None, s_up=None, s_down=None) -> MLPShard:
    """Cut full weights (gate/up [I, H], down [H, I]) into rank `rank`'s shard."""
    sl = shard_rows(w_gate.shape[0], world, rank)
    wgu = torch.cat([w_gate[sl], w_up[sl]], 0).contiguous()
    sgu = None if s_gate is None else torch.cat([s_gate[sl], s_up[sl]], 0).contiguous()
    return MLPShard(wgu, sgu, w_down[:, sl].contiguous(), s_down, sl.stop - sl.start)


def _default_gemm(x, w, s):
    from . import ops
    if w.dtype == torch.float16:
        return ops.gemm_fp16(x, w)
    return ops.gemm_w8a16(x, w, s)


def _default_swiglu(gu):
    from . import ops
    return ops.silu_mul(gu)


def mlp_forward(x: torch.Tensor, shard: MLPShard, group=None, gemm=None, swiglu=None,
                all_reduce=True) -> torch.Tensor:
    """y = down(silu(gate(x)) * up(x)) for this rank's shard, summed over the group."""
    gemm = gemm or _default_gemm
    swiglu = swiglu or _default_swiglu
    gu = gemm(x, shard.w_gate_up, shard.s_gate_up)       # [M, 2 I/tp]
    h = swiglu(gu)                                        # [M, I/tp]
    y = gemm(h, shard.w_down, shard.s_down)               # [M, H] partial
    if all_reduce:
        import torch.distributed as dist
        if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
            dist.all_reduce(y, op=dist.ReduceOp.SUM, group=group)
    return y
