"""Tensor-parallel MLP sharding on CPU ranks (gloo, world 2 and 4): the sharded, all-reduced
output equals the unsharded oracle MLP.  GEMM and SwiGLU are the CPU oracle's here (the GPU
kernels are exercised by the GPU tests); what is tested is the sharding and the exchange."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _oracle_gemm(x, w, s):
    y = x.float() @ w.float().T
    if s is not None:
        y = y * s.float()[None, :]
    return y


def _oracle_swiglu(gu, block):
    from cuda_tempiler_b200 import tp
    return tp.swiglu_ref(gu, block)


def _weights(H, I, seed=0):
    g = torch.Generator().manual_seed(seed)
    wg = torch.randint(-127, 128, (I, H), generator=g, dtype=torch.int8)
    wu = torch.randint(-127, 128, (I, H), generator=g, dtype=torch.int8)
    wd = torch.randint(-127, 128, (H, I), generator=g, dtype=torch.int8)
    sg = torch.rand(I, generator=g) * 1e-3 + 1e-4
    su = torch.rand(I, generator=g) * 1e-3 + 1e-4
    sd = torch.rand(H, generator=g) * 1e-3 + 1e-4
    x = torch.randn(8, H, generator=g)
    return x, wg, wu, wd, sg, su, sd


def _worker(rank, world, port, H, I, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from cuda_tempiler_b200 import tp
    x, wg, wu, wd, sg, su, sd = _weights(H, I)
    sh = tp.shard_mlp(wg, wu, wd, world, rank, sg, su, sd)
    y = tp.mlp_forward(x, sh, gemm=_oracle_gemm, swiglu=_oracle_swiglu)
    if rank == 0:
        q.put(y.numpy())
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_tp_mlp_matches_unsharded(world):
    H, I = 64, 128
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, H, I, q)) for r in range(world)]
    for p in ps:
        p.start()
    y = q.get(timeout=120)
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0
    from cuda_tempiler_b200 import tp
    x, wg, wu, wd, sg, su, sd = _weights(H, I)
    full = tp.shard_mlp(wg, wu, wd, 1, 0, sg, su, sd)
    ref = tp.mlp_forward(x, full, gemm=_oracle_gemm, swiglu=_oracle_swiglu, all_reduce=False)
    rel = float(np.linalg.norm(y - ref.numpy()) / np.linalg.norm(ref.numpy()))
    assert rel < 1e-5, rel


def test_shard_layout():
    from cuda_tempiler_b200 import tp
    x, wg, wu, wd, sg, su, sd = _weights(16, 32)
    s1 = tp.shard_mlp(wg, wu, wd, 4, 1, sg, su, sd)
    assert s1.w_gate_up.shape == (16, 16) and s1.inter == 8
    assert torch.equal(s1.w_gate_up[:8], wg[8:16]) and torch.equal(s1.w_gate_up[8:], wu[8:16])
    assert torch.equal(s1.w_down, wd[:, 8:16]) and s1.w_down.is_contiguous()
    with pytest.raises(ValueError):
        tp.shard_rows(30, 4, 0)
