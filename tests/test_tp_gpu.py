"""Tensor-parallel MLP on the GPU: the SwiGLU kernel, the single-rank MLP through the sm_100a
kernels against the CPU oracle, and (when the box has >= 2 GPUs) the NCCL-sharded MLP."""
import os
import socket

import numpy as np
import pytest
import torch

from oracle import gemm_oracle as O

pytestmark = pytest.mark.gpu


def test_silu_mul_kernel(dev):
    from cuda_tempiler_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(0)
    gu = torch.randn(37, 2 * 264, generator=g, device="cuda").half()
    out = ops.silu_mul(gu)
    ref = torch.nn.functional.silu(gu[:, :264].float()) * gu[:, 264:].float()
    assert O.rel_l2(out.float().cpu().numpy(), ref.cpu().numpy()) < 1e-3


def _mlp_inputs(M, H, I, dev, seed=0):
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(M, H, generator=g, device=dev).half()
    wg = torch.randint(-127, 128, (I, H), generator=g, device=dev, dtype=torch.int8)
    wu = torch.randint(-127, 128, (I, H), generator=g, device=dev, dtype=torch.int8)
    wd = torch.randint(-127, 128, (H, I), generator=g, device=dev, dtype=torch.int8)
    sg = (torch.rand(I, generator=g, device=dev) * 2e-4 + 5e-5).half()
    su = (torch.rand(I, generator=g, device=dev) * 2e-4 + 5e-5).half()
    sd = (torch.rand(H, generator=g, device=dev) * 2e-4 + 5e-5).half()
    return x, wg, wu, wd, sg, su, sd


def _oracle_mlp(x, wg, wu, wd, sg, su, sd):
    xf = x.float().cpu().numpy()
    gate = xf @ (wg.float().cpu().numpy() * sg.float().cpu().numpy()[:, None]).T
    up = xf @ (wu.float().cpu().numpy() * su.float().cpu().numpy()[:, None]).T
    h = (gate / (1 + np.exp(-gate)) * up).astype(np.float16).astype(np.float32)
    return h @ (wd.float().cpu().numpy() * sd.float().cpu().numpy()[:, None]).T


@pytest.mark.parametrize("M", [1, 16, 256])
def test_mlp_single_rank(dev, M):
    from cuda_tempiler_b200 import tp
    x, wg, wu, wd, sg, su, sd = _mlp_inputs(M, 512, 1024, dev)
    sh = tp.shard_mlp(wg, wu, wd, 1, 0, sg, su, sd)
    y = tp.mlp_forward(x, sh)
    torch.cuda.synchronize()
    ref = _oracle_mlp(x, wg, wu, wd, sg, su, sd)
    assert O.rel_l2(y.float().cpu().numpy(), ref) <= O.GATE_REL_L2


def _nccl_worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank))
    from cuda_tempiler_b200 import tp
    x, wg, wu, wd, sg, su, sd = _mlp_inputs(16, 512, 1024, torch.device("cuda", rank))
    sh = tp.shard_mlp(wg, wu, wd, world, rank, sg, su, sd)
    y = tp.mlp_forward(x, sh)
    torch.cuda.synchronize()
    if rank == 0:
        q.put((y.float().cpu().numpy(), _oracle_mlp(x, wg, wu, wd, sg, su, sd)))
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_mlp_two_ranks_nccl():
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_nccl_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    y, ref = q.get(timeout=300)
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert O.rel_l2(y, ref) <= O.GATE_REL_L2
