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


def test_silu_mul_kernel_interleaved(dev):
    """The block-interleaved layout (gate 64 | up 64 | ...) of the fused entry points."""
    from cuda_tempiler_b200 import ops, tp
    g = torch.Generator(device="cuda").manual_seed(1)
    gu = torch.randn(19, 2 * 320, generator=g, device="cuda").half()
    out = ops.silu_mul(gu, block=64)
    ref = tp.swiglu_ref(gu, 64)
    assert O.rel_l2(out.float().cpu().numpy(), ref.cpu().numpy()) < 1e-3


def _swiglu_oracle(a, wg, wu):
    g = a.astype(np.float32) @ wg.astype(np.float32).T
    u = a.astype(np.float32) @ wu.astype(np.float32).T
    return g / (1 + np.exp(-g)) * u


@pytest.mark.parametrize("M,I,K", [(300, 512, 1024), (1024, 1536, 2048), (2048, 2176, 512)])
def test_fused_swiglu_fp16(dev, M, I, K):
    """gate_up GEMM with SwiGLU in the 2-CTA epilogue against silu(A Wg^T) * (A Wu^T)."""
    from cuda_tempiler_b200 import ops, tp
    a, wg = O.inputs_layer(M, I, K, seed=11)
    _, wu = O.inputs_layer(M, I, K, seed=12)
    W = tp.interleave_rows(torch.from_numpy(wg), torch.from_numpy(wu), 64).cuda()
    C = torch.empty((M, I), dtype=torch.float16, device="cuda")
    C.view(torch.int16).fill_(0x7F7F)
    ops.gemm_fp16_swiglu(torch.from_numpy(a).cuda(), W, out=C)
    torch.cuda.synchronize()
    c = C.cpu().numpy()
    assert O.poison_count(c) == 0
    assert O.rel_l2(c, _swiglu_oracle(a, wg, wu)) <= O.GATE_REL_L2
    assert ops.device_status() == [0, 0, 0, 0]


@pytest.mark.parametrize("M", [512, 1024])
def test_fused_swiglu_w8a16(dev, M):
    """The W8A16 form: per-channel weights and scales interleaved alike, expanded, fused."""
    from cuda_tempiler_b200 import ops, tp
    I, K = 1024, 1536
    a, qg, sg = O.inputs_w8_per_channel(M, I, K, 21)
    _, qu, su = O.inputs_w8_per_channel(M, I, K, 22)
    W = tp.interleave_rows(torch.from_numpy(qg), torch.from_numpy(qu), 64).cuda()
    S = tp.interleave_rows(torch.from_numpy(sg), torch.from_numpy(su), 64).cuda()
    C = ops.gemm_w8a16_swiglu(torch.from_numpy(a).cuda(), W, S)
    torch.cuda.synchronize()
    ref = _swiglu_oracle(a, O.dequant_per_channel(qg, sg), O.dequant_per_channel(qu, su))
    assert O.rel_l2(C.cpu().numpy(), ref) <= O.GATE_REL_L2
    from cuda_tempiler_b200._lib import NotCovered
    with pytest.raises(NotCovered):
        ops.gemm_w8a16_swiglu(torch.from_numpy(a[:16]).cuda(), W, S)


@pytest.mark.parametrize("M", [1, 16, 256, 1024])
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


def test_allreduce_oneshot_emulated_ranks(dev):
    """The one-shot all-reduce kernel's data path and flags for tp = 3 on one GPU: the other two
    ranks' slots and flags are filled beforehand (so the kernel waits on nothing another launch
    would have to provide), rank 0 pushes, flags, waits and sums; bit-identical to the rank-order
    fp32 sum, for both call parities."""
    import ctypes as C
    from cuda_tempiler_b200 import _lib
    lib = _lib.load()
    tp, cap, n, ctas = 3, 4096, 3000, 8
    g = torch.Generator(device="cuda").manual_seed(5)
    recv = [torch.zeros(2 * tp * cap, dtype=torch.float16, device="cuda") for _ in range(tp)]
    flags = [torch.zeros(tp * 32, dtype=torch.int32, device="cuda") for _ in range(tp)]
    rp = (C.c_void_p * tp)(*[t.data_ptr() for t in recv])
    fp = (C.c_void_p * tp)(*[t.data_ptr() for t in flags])
    for epoch in (1, 2):
        xs = [torch.randn(n, generator=g, device="cuda").half() for _ in range(tp)]
        half = (epoch & 1) * tp * cap
        for s in (1, 2):  # ranks 1 and 2 have already delivered into rank 0
            recv[0][half + s * cap: half + s * cap + n] = xs[s]
            flags[0][s * 32: s * 32 + ctas] = epoch
        y = xs[0].clone()
        rc = lib.tempo_sm100_allreduce_oneshot(y.data_ptr(), y.data_ptr(), n, cap, rp, fp, tp, 0,
                                               epoch, ctas, torch.cuda.current_stream().cuda_stream)
        assert rc == 0
        torch.cuda.synchronize()
        ref = (xs[0].float() + xs[1].float() + xs[2].float()).half()
        assert torch.equal(y, ref)
        for p in range(tp):  # rank 0's slice landed in every rank's slot 0, flags raised
            assert torch.equal(recv[p][half: half + n], xs[0])
            assert bool((flags[p][0:ctas] == epoch).all())
    assert ops_status() == [0, 0, 0, 0]


def test_allreduce_oneshot_wait_runs_out(dev):
    """A rank that never arrives: emulated tp = 3 on one GPU with rank 2's flags never raised and
    a 1 ms wait limit.  The kernel gives up, records status 1 / role 20 and returns (the launch
    succeeds and the context stays usable); the status is then cleared."""
    import ctypes as C
    from cuda_tempiler_b200 import _lib, ops
    lib = _lib.load()
    tp, cap, n, ctas, epoch = 3, 1024, 1024, 4, 1
    recv = [torch.zeros(2 * tp * cap, dtype=torch.float16, device="cuda") for _ in range(tp)]
    flags = [torch.zeros(tp * 32, dtype=torch.int32, device="cuda") for _ in range(tp)]
    rp = (C.c_void_p * tp)(*[t.data_ptr() for t in recv])
    fp = (C.c_void_p * tp)(*[t.data_ptr() for t in flags])
    flags[0][1 * 32: 1 * 32 + ctas] = epoch  # rank 1 has delivered, rank 2 never will
    y = torch.ones(n, dtype=torch.float16, device="cuda")
    assert ops.device_status(reset=True) == [0, 0, 0, 0]
    rc = lib.tempo_sm100_allreduce_oneshot_timed(y.data_ptr(), y.data_ptr(), n, cap, rp, fp, tp,
                                                 0, epoch, ctas, 1_000_000,
                                                 torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    st = ops.device_status(reset=True)
    assert st[0] == 1 and st[1] == 20 and 0 <= st[2] < ctas and st[3] == 2, st
    assert ops.device_status() == [0, 0, 0, 0]
    # the context is still usable: a normal GEMM afterwards passes the gate
    a, b = O.inputs_config1(64, 256, 256)
    c = ops.gemm_fp16(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda())
    assert O.rel_l2(c.cpu().numpy(), O.gemm_fp16_ref(a, b)) <= O.GATE_REL_L2
    # out-of-range limits are refused without a launch
    assert lib.tempo_sm100_allreduce_oneshot_timed(y.data_ptr(), y.data_ptr(), n, cap, rp, fp,
                                                   tp, 0, epoch, ctas, 0, None) == 1


def ops_status():
    from cuda_tempiler_b200 import ops
    return ops.device_status()


def _peer_worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank))
    from cuda_tempiler_b200 import ops, tp
    par = tp.PeerAllReduce(16 * 5120)
    ok = True
    for it in range(5):
        g = torch.Generator(device="cuda").manual_seed(100 * it + rank)
        y = torch.randn(16 * 5120, generator=g, device="cuda").half()
        ref = y.clone()
        dist.all_reduce(ref)
        par(y)
        torch.cuda.synchronize()
        ok &= bool(torch.allclose(y.float(), ref.float(), rtol=2e-3, atol=2e-3))
    # the MLP through the peer exchange equals the NCCL one
    x, wg, wu, wd, sg, su, sd = _mlp_inputs(16, 512, 1024, torch.device("cuda", rank))
    sh = tp.shard_mlp(wg, wu, wd, world, rank, sg, su, sd)
    y1 = tp.mlp_forward(x, sh, all_reduce=par)
    y2 = tp.mlp_forward(x, sh)
    torch.cuda.synchronize()
    ok &= bool(torch.allclose(y1.float(), y2.float(), rtol=2e-3, atol=2e-3))
    st = ops.device_status()
    par.close()
    dist.barrier()
    if rank == 0:
        q.put((ok, st))
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_peer_allreduce_two_ranks():
    """The one-shot all-reduce over CUDA IPC peer mappings on 2 GPUs against NCCL's."""
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_peer_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    ok, st = q.get(timeout=300)
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert ok and st == [0, 0, 0, 0]


@pytest.mark.parametrize("M", [1, 16, 1024])
def test_mlp_graph_replay_matches_eager(dev, M):
    """The MLP forward captured in a CUDA graph gives the eager forward's result, twice in a
    row with different inputs (the graph reads its input buffer on every replay)."""
    from cuda_tempiler_b200 import tp
    x, wg, wu, wd, sg, su, sd = _mlp_inputs(M, 512, 1024, dev)
    sh = tp.shard_mlp(wg, wu, wd, 1, 0, sg, su, sd)
    mg = tp.MLPGraph(sh, M, 512, dev)
    for seed in (1, 2):
        xs = _mlp_inputs(M, 512, 1024, dev, seed=seed)[0]
        y = mg(xs).clone()
        ref = tp.mlp_forward(xs, sh)
        torch.cuda.synchronize()
        assert torch.equal(y, ref)
        assert O.rel_l2(y.float().cpu().numpy(), _oracle_mlp(xs, wg, wu, wd, sg, su, sd)) <= O.GATE_REL_L2


def _graph_worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank))
    from cuda_tempiler_b200 import tp
    x, wg, wu, wd, sg, su, sd = _mlp_inputs(4, 512, 1024, torch.device("cuda", rank))
    sh = tp.shard_mlp(wg, wu, wd, world, rank, sg, su, sd)
    mg = tp.MLPGraph(sh, 4, 512, torch.device("cuda", rank))
    y = mg(x).clone()
    par = tp.PeerAllReduce(16 * 512)
    mp_ = tp.MLPGraph(sh, 4, 512, torch.device("cuda", rank), all_reduce=par)
    y2 = mp_(x).clone()
    y3 = mp_(x).clone()  # a second replay: a new device-side epoch
    torch.cuda.synchronize()
    del mg, mp_
    torch.cuda.synchronize()
    if rank == 0:
        q.put((y.float().cpu().numpy(), y2.float().cpu().numpy(), y3.float().cpu().numpy(),
               _oracle_mlp(x, wg, wu, wd, sg, su, sd)))
    par.close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_mlp_graph_two_ranks():
    """The graph-captured forward on 2 GPUs with NCCL's all-reduce inside the graph, and with
    the peer one-shot all-reduce (device-side epoch) inside it, replayed twice."""
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_graph_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    y, y2, y3, ref = q.get(timeout=300)
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0
    for got in (y, y2, y3):
        assert O.rel_l2(got, ref) <= O.GATE_REL_L2
