"""Tensor-parallel W8A16 MLP: SwiGLU MLP of a dense layer split over the
ranks of a process group, one process per GPU.

    gate_up  column-parallel: rank r holds gate rows [r I/tp, (r+1) I/tp) and the matching up
             rows as one [2 I/tp, H] weight, interleaved in blocks of 64 rows (gate 64, up 64,
             ...) when I/tp is a multiple of 64, else stacked [gate_r | up_r], so SiLU(gate)
             * up needs no communication; with the interleaved layout the SwiGLU step runs in
             the gate_up GEMM's epilogue at prefill sizes (``ops.gemm_*_swiglu``);
    down     row-parallel: rank r holds W_down[:, r I/tp : (r+1) I/tp] as a K-contiguous
             [H, I/tp] weight and produces a partial [M, H];
    reduce   one all-reduce (sum) of the fp16 [M, H] partial -- the only exchange step: NCCL,
             or for decode-sized M the library's one-shot all-reduce over peer memory
             (``PeerAllReduce``).

The reference is single-GPU (it has no multi-GPU code); this helper is new.  Each GEMM is the
sm_100a kernel (``ops.gemm_w8a16`` / ``ops.gemm_fp16``); the SwiGLU step is the library's
``silu_mul`` kernel; the all-reduce is ``torch.distributed.all_reduce`` (NCCL over NVLink on
B200).  ``gemm``/``swiglu`` are injectable so the sharding algebra can be checked on CPU ranks
(gloo) against an oracle.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


GU_BLOCK = 64  # gate/up interleave block of the fused SwiGLU epilogue


def interleave_rows(a: torch.Tensor, b: torch.Tensor, block: int) -> torch.Tensor:
    """[a rows 0..block) | b rows 0..block) | a rows block..2 block) | ...] along dim 0."""
    n = a.shape[0]
    if n % block or b.shape != a.shape:
        raise ValueError(f"{tuple(a.shape)} / {tuple(b.shape)} do not interleave in blocks of {block}")
    rest = tuple(a.shape[1:])
    return torch.stack([a.reshape(n // block, block, *rest), b.reshape(n // block, block, *rest)],
                       1).reshape(2 * n, *rest)


def swiglu_ref(gu: torch.Tensor, block: int) -> torch.Tensor:
    """fp32 silu(gate) * up of a gate_up output in either layout (block 0: [gate | up])."""
    M, I2 = gu.shape
    I = I2 // 2
    if block:
        v = gu.float().reshape(M, I // block, 2, block)
        g, u = v[:, :, 0, :].reshape(M, I), v[:, :, 1, :].reshape(M, I)
    else:
        g, u = gu[:, :I].float(), gu[:, I:].float()
    return g * torch.sigmoid(g) * u


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
    gu_block: int = 0  # GU_BLOCK: gate/up rows interleaved in blocks of 64; 0: [gate | up]


def shard_mlp(w_gate: torch.Tensor, w_up: torch.Tensor, w_down: torch.Tensor, world: int,
              rank: int, s_gate=None, s_up=None, s_down=None) -> MLPShard:
    """Cut full weights (gate/up [I, H], down [H, I]) into rank `rank`'s shard."""
    sl = shard_rows(w_gate.shape[0], world, rank)
    inter = sl.stop - sl.start
    block = GU_BLOCK if inter % GU_BLOCK == 0 else 0
    if block:
        wgu = interleave_rows(w_gate[sl], w_up[sl], block).contiguous()
        sgu = None if s_gate is None else interleave_rows(s_gate[sl], s_up[sl], block).contiguous()
    else:
        wgu = torch.cat([w_gate[sl], w_up[sl]], 0).contiguous()
        sgu = None if s_gate is None else torch.cat([s_gate[sl], s_up[sl]], 0).contiguous()
    return MLPShard(wgu, sgu, w_down[:, sl].contiguous(), s_down, inter, block)


def _default_gemm(x, w, s):
    from . import ops
    if w.dtype == torch.float16:
        return ops.gemm_fp16(x, w)
    return ops.gemm_w8a16(x, w, s)


def _default_swiglu(gu, block):
    from . import ops
    return ops.silu_mul(gu, block=block)


def _default_fused(x, w, s):
    """The gate_up GEMM with SwiGLU in its epilogue, or None where it does not cover M."""
    from . import ops
    from ._lib import NotCovered
    try:
        if w.dtype == torch.float16:
            return ops.gemm_fp16_swiglu(x, w)
        return ops.gemm_w8a16_swiglu(x, w, s)
    except NotCovered:
        return None


class PeerAllReduce:
    """One-shot all-reduce (sum) of fp16 vectors up to `cap` values over the ranks of `group`
    through peer memory (``tempo_sm100_allreduce_oneshot``: every rank stores its vector into
    every rank's receive buffer, raises a flag there, waits for all flags and sums in rank
    order).  For the decode-sized down-projection partial; longer vectors fall back to
    ``torch.distributed.all_reduce``.  Buffers are exchanged once, by CUDA IPC handles
    all-gathered over the process group; all ranks must be on one node."""

    def __init__(self, cap: int, group=None, device=None, ctas: int = 16):
        import ctypes as C

        import torch.distributed as dist

        from . import _lib
        self._lib = _lib.load()
        self.group = group
        self.tp = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.tp > 8:
            raise ValueError("the one-shot all-reduce covers up to 8 ranks")
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.cap = -(-cap // 8) * 8
        self.ctas = ctas
        # whole allocations of their own (an IPC handle maps an allocation from its base)
        with torch.cuda.device(self.device):
            r, f = C.c_void_p(), C.c_void_p()
            _lib.check(self._lib.tempo_sm100_ipc_alloc(2 * self.tp * self.cap * 2, C.byref(r)),
                       "ipc_alloc")
            _lib.check(self._lib.tempo_sm100_ipc_alloc(self.tp * 32 * 4, C.byref(f)), "ipc_alloc")
        self._own = [r.value, f.value]
        hr, hf = (C.c_uint8 * 64)(), (C.c_uint8 * 64)()
        _lib.check(self._lib.tempo_sm100_ipc_handle(r.value, hr), "ipc_handle")
        _lib.check(self._lib.tempo_sm100_ipc_handle(f.value, hf), "ipc_handle")
        mine = torch.tensor(list(bytes(hr)) + list(bytes(hf)), dtype=torch.uint8,
                            device=self.device)
        every = [torch.empty_like(mine) for _ in range(self.tp)]
        dist.all_gather(every, mine, group=group)
        self._opened = []
        rp, fp = [], []
        for p, t in enumerate(every):
            if p == self.rank:
                rp.append(r.value)
                fp.append(f.value)
                continue
            raw = bytes(t.cpu().tolist())
            ptrs = []
            for h in (raw[:64], raw[64:]):
                out = C.c_void_p()
                buf = (C.c_uint8 * 64).from_buffer_copy(h)
                _lib.check(self._lib.tempo_sm100_ipc_open(buf, C.byref(out)), "ipc_open")
                self._opened.append(out.value)
                ptrs.append(out.value)
            rp.append(ptrs[0])
            fp.append(ptrs[1])
        self._recv_ptrs = (C.c_void_p * self.tp)(*rp)
        self._flag_ptrs = (C.c_void_p * self.tp)(*fp)
        self.epoch = 0
        # the device-side epoch of the graph-capturable form (``device_epoch=True`` calls)
        self._epoch_ctr = torch.zeros(2, dtype=torch.int32, device=self.device)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=group)

    def __call__(self, y: torch.Tensor) -> torch.Tensor:
        """In place: y <- sum of y over the ranks.  The epoch lives on the device, so the call
        can be captured in a CUDA graph (``MLPGraph``); all ranks make every call in step."""
        import torch.distributed as dist

        from . import _lib
        n = y.numel()
        if y.dtype != torch.float16 or not y.is_contiguous() or n % 8 or n > self.cap:
            dist.all_reduce(y, op=dist.ReduceOp.SUM, group=self.group)
            return y
        rc = self._lib.tempo_sm100_allreduce_oneshot_dev(
            y.data_ptr(), y.data_ptr(), n, self.cap, self._recv_ptrs, self._flag_ptrs, self.tp,
            self.rank, self._epoch_ctr.data_ptr(), self.ctas,
            torch.cuda.current_stream(self.device).cuda_stream)
        _lib.check(rc, "tempo_sm100_allreduce_oneshot_dev")
        return y

    def close(self):
        """Unmap the peers' buffers, then free this rank's (after a barrier, so no peer still
        maps them)."""
        import torch.distributed as dist
        for p in self._opened:
            self._lib.tempo_sm100_ipc_close(p)
        self._opened = []
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for p in self._own:
            self._lib.tempo_sm100_ipc_free(p)
        self._own = []


def mlp_forward(x: torch.Tensor, shard: MLPShard, group=None, gemm=None, swiglu=None,
                all_reduce=True, fused=None) -> torch.Tensor:
    """y = down(silu(gate(x)) * up(x)) for this rank's shard, summed over the group.  With the
    library's own GEMM (gemm None) and an interleaved shard the fused gate_up + SwiGLU kernel
    runs where it covers M; ``fused=False`` keeps the two-kernel path."""
    if fused is None:
        fused = _default_fused if gemm is None else False
    gemm = gemm or _default_gemm
    swiglu = swiglu or _default_swiglu
    h = fused(x, shard.w_gate_up, shard.s_gate_up) if (fused and shard.gu_block) else None
    if h is None:
        gu = gemm(x, shard.w_gate_up, shard.s_gate_up)   # [M, 2 I/tp]
        h = swiglu(gu, shard.gu_block)                    # [M, I/tp]
    y = gemm(h, shard.w_down, shard.s_down)               # [M, H] partial
    if callable(all_reduce):                              # e.g. a PeerAllReduce
        return all_reduce(y)
    if all_reduce:
        import torch.distributed as dist
        if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
            dist.all_reduce(y, op=dist.ReduceOp.SUM, group=group)
    return y


class MLPGraph:
    """One rank's MLP forward for a fixed M captured in a CUDA graph and replayed: at decode
    sizes the forward is a handful of short kernels (two GEMVs, SwiGLU, the all-reduce) whose
    host launch cost exceeds their device time once the weights are split over several GPUs,
    so each forward is one graph launch instead.  The all-reduce inside the graph is NCCL's
    (capturable) by default, or ``all_reduce=PeerAllReduce(...)``, the library's one-shot peer
    all-reduce, which keeps its epoch on the device and so replays correctly.  ``__call__(x)``
    copies x into the graph's input buffer, replays, and returns the
    graph's output buffer (overwritten by the next call)."""

    def __init__(self, shard: MLPShard, M: int, H: int, device, group=None, warmup: int = 2,
                 all_reduce=True):
        self.x = torch.zeros(M, H, dtype=torch.float16, device=device)
        self.stream = torch.cuda.Stream(device)
        self.stream.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(self.stream):
            # warm-up on the capture stream: cached workspaces and tensor maps exist before capture
            for _ in range(warmup):
                mlp_forward(self.x, shard, group, all_reduce=all_reduce)
        self.stream.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=self.stream):
            self.y = mlp_forward(self.x, shard, group, all_reduce=all_reduce)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        self.x.copy_(x)
        self.graph.replay()
        return self.y
