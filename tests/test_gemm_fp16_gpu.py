"""GPU parity of the fp16 tcgen05 GEMM against the CPU oracle (relL2 <= 3e-3, full poison
coverage, fp64 spot check), through the C-ABI (ctypes -> libtempo_sm100.so)."""
import numpy as np
import pytest
import torch

from oracle import gemm_oracle as O

pytestmark = pytest.mark.gpu

TOL = O.GATE_REL_L2  # relL2 <= 3e-3 (BASELINE gate)


def _run(fn, M, N, K, seed=0, **kw):
    a, b = O.inputs_config1(M, N, K, seed)
    A = torch.from_numpy(a).cuda()
    B = torch.from_numpy(b).cuda()
    C = torch.empty((M, N), dtype=torch.float16, device="cuda")
    C.view(torch.int16).fill_(0x7F7F)
    fn(A, B, out=C, **kw)
    torch.cuda.synchronize()
    c = C.cpu().numpy()
    return a, b, c


def _gate(a, b, c):
    assert O.poison_count(c) == 0, "uncovered output cells"
    ref = O.gemm_fp16_ref(a, b)
    r = O.rel_l2(c, ref)
    assert r <= TOL, f"relL2 {r:.3e}"
    s = O.spot_fp64(a, b, c)
    assert s <= TOL, f"fp64 spot relL2 {s:.3e}"
    return r


ODD = [(1, 64, 64), (3, 72, 136), (17, 200, 520), (100, 264, 200), (128, 256, 64),
       (129, 520, 1000), (300, 1000, 520), (640, 768, 4096)]


@pytest.mark.parametrize("M,N,K", ODD)
def test_dispatch_odd_shapes(dev, M, N, K):
    from cuda_tempiler_b200 import ops
    a, b, c = _run(ops.gemm_fp16, M, N, K)
    _gate(a, b, c)


HYPER = [(16, True), (32, True), (64, True), (128, True), (64, False), (128, False), (256, False)]


@pytest.mark.parametrize("bn,swap", HYPER)
@pytest.mark.parametrize("splits", [1, 3, 8, 10])
def test_every_hyperform(dev, bn, swap, splits):
    """splits 2..8 reduce inside a cluster through distributed shared memory, 10 through the
    global workspace."""
    from cuda_tempiler_b200 import ops
    M, N, K = (24, 776, 1032) if swap else (260, 776, 1032)
    a, b, c = _run(lambda A, B, out: ops.gemm_hyperform(A, B, bn=bn, swap=swap, splits=splits,
                                                         out=out), M, N, K)
    _gate(a, b, c)


def test_config1_full(dev):
    """Config 1: 4096 x 15360 x 3840 (the naive TEMPO-OP example)."""
    from cuda_tempiler_b200 import ops
    a, b, c = _run(ops.gemm_fp16, 4096, 15360, 3840, seed=0)
    _gate(a, b, c)


@pytest.mark.parametrize("M,N,K", O.SHIP_PROBE_SHAPES)
def test_ship_probe_kat(dev, M, N, K):
    """The reference ship probe's patterned inputs and 64 fp64 cells (ship_probe.cu:41-80)."""
    from cuda_tempiler_b200 import ops
    a, b = O.ship_probe_inputs(M, N, K)
    C = ops.gemm_fp16(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda())
    torch.cuda.synchronize()
    c = C.cpu().numpy()
    ms, ns = O.ship_probe_cells(M, N)
    exp = O.ship_probe_expected(M, N, K)
    assert O.ship_probe_maxrel(c[ms, ns], exp) <= 3e-3


def test_naive_input_bar(dev):
    from cuda_tempiler_b200 import ops
    a, b = O.inputs_config1(96, 136, 200)
    C = ops.naive_gemm_fp16(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda())
    assert O.rel_l2(C.cpu().numpy(), O.gemm_fp16_ref(a, b)) <= TOL


def test_workspace_left_zero(dev):
    """Split-K launches leave the workspace zero-filled (counters reset by the last CTA)."""
    from cuda_tempiler_b200 import ops
    a, b = O.inputs_config1(16, 3840, 4096)
    A, B = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    sel = ops.select(0, 16, 3840, 4096)
    assert sel["splits"] > 1
    for _ in range(3):
        C = ops.gemm_fp16(A, B)
    torch.cuda.synchronize()
    ws = ops._ws_cache[(0, torch.cuda.current_stream().cuda_stream)]
    tiles = (3840 // 128)
    assert int(ws[: tiles * 4].view(torch.int32).abs().sum()) == 0
    assert O.rel_l2(C.cpu().numpy(), O.gemm_fp16_ref(a, b)) <= TOL
    assert ops.device_status() == [0, 0, 0, 0]


def test_workspace_reuse_across_shapes(dev):
    """One workspace serves split-K problems of different tile counts in a row: a 30-tile
    problem leaves fp32 partials behind, then a 240-tile problem needs more counters than the
    first; the counters sit in a fixed prefix, so they never land on the old partials."""
    from cuda_tempiler_b200 import ops
    # k-splits above the cluster limit (8) take the global workspace path
    big = lambda: _run(lambda A, B, out: ops.gemm_hyperform(A, B, bn=16, swap=True, splits=10,
                                                            out=out), 16, 30720, 1024, seed=6)
    _gate(*big())  # sizes the cached workspace for both problems
    small = _run(lambda A, B, out: ops.gemm_hyperform(A, B, bn=16, swap=True, splits=12,
                                                       out=out), 16, 3840, 4096, seed=5)
    _gate(*small)
    _gate(*big())
    assert ops.device_status() == [0, 0, 0, 0]


@pytest.mark.parametrize("bn", [128, 160, 192, 224, 256])
@pytest.mark.parametrize("M,N,K", [(260, 784, 1032), (1000, 1000, 520), (640, 768, 4096),
                                   (4096, 15360, 3840)])
def test_pair_tiles_cta_group2(dev, bn, M, N, K):
    """256 x bn tiles on 2-CTA clusters (tcgen05.mma.cta_group::2)."""
    from cuda_tempiler_b200 import ops
    a, b, c = _run(lambda A, B, out: ops.gemm_hyperform(A, B, bn=bn, swap=False, cta_group=2,
                                                         out=out), M, N, K)
    _gate(a, b, c)
    assert ops.device_status() == [0, 0, 0, 0]


def test_pair_resources_match_python_plan(dev):
    import ctypes as C
    from cuda_tempiler_b200 import _lib
    from cuda_tempiler_b200.tempo.plugins.sm100.skeletons_py import pair_cfg
    lib = _lib.load()
    for bn in (128, 160, 192, 224, 256):
        out = (C.c_int * 6)()
        assert lib.tempo_sm100_pair_resources(bn, out) == 0
        c = pair_cfg(bn)
        assert (out[0], out[1], out[2], out[3]) == (c["threads"], c["smem"], c["stages"], c["tmem_cols"])
        assert out[5] == 0


# Split tails of the 2-CTA kernel: fewer tiles than clusters (every tile cut), a ragged last
# wave (the remainder cut), few tiles with many k-blocks (many k-slices), and odd edges.
SK_SHAPES = [(1000, 1000, 1000), (512, 3840, 4096), (4096, 3840, 1024), (2048, 3840, 2048),
             (520, 776, 8192), (264, 136, 4096)]


@pytest.mark.parametrize("bn", [128, 224, 256])
@pytest.mark.parametrize("M,N,K", SK_SHAPES)
def test_pair_split_tail(dev, bn, M, N, K):
    """Pair launches with a split tail pass the gate, are bit-identical run to run (partials
    are summed in k order) and leave their arrival counters at zero."""
    from cuda_tempiler_b200 import ops
    f = lambda A, B, out: ops.gemm_hyperform(A, B, bn=bn, swap=False, cta_group=2, splits=2,
                                             out=out)
    a, b, c = _run(f, M, N, K)
    _gate(a, b, c)
    _, _, c2 = _run(f, M, N, K)
    assert np.array_equal(c.view(np.int16), c2.view(np.int16))
    from test_stream_k_cpu import plan
    pl = plan(M, N, K, bn, torch.cuda.get_device_properties(0).multi_processor_count)
    n_ctr = 2 * pl["sk_tiles"]
    ws = ops._ws_cache[(0, torch.cuda.current_stream().cuda_stream)]
    assert int(ws[: 4 * n_ctr].view(torch.int32).abs().sum()) == 0
    assert ops.device_status() == [0, 0, 0, 0]


def test_dispatch_pair_width_by_waves(dev):
    """The dispatcher's 2-CTA row narrows the tile where 256 wide leaves a ragged last wave
    (down projection, M = 1024: 60 tiles of 256 on 74 clusters -> 72 tiles of 224), and the
    result passes the gate."""
    from cuda_tempiler_b200 import ops
    sel = ops.select(0, 1024, 3840, 15360)
    assert sel["bn"] == 224
    assert ops.select(0, 4096, 30720, 3840)["bn"] == 256
    a, b, c = _run(ops.gemm_fp16, 1024, 3840, 15360, seed=3)
    _gate(a, b, c)


@pytest.mark.parametrize("M,N,K", [(1, 248320, 512), (16, 248320, 512), (300, 248320, 256),
                                   (1, 96, 5120), (16, 96, 5120), (1024, 96, 5120)])
def test_lm_head_and_narrow_n(dev, M, N, K):
    """Shapes outside the layer set: an lm_head-class wide N (248320 rows; K cut to keep the
    CPU oracle's inputs small) and a narrow in-projection (N = 96), through the dispatcher."""
    from cuda_tempiler_b200 import ops
    a, b, c = _run(ops.gemm_fp16, M, N, K, seed=7)
    assert O.poison_count(c) == 0
    ref = O.gemm_fp16_ref(a, b)
    assert O.rel_l2(c, ref) <= TOL
    assert ops.device_status() == [0, 0, 0, 0]


def test_workspace_shared_with_w8a16_prefill(dev):
    """One cached workspace serves a W8A16 prefill (which writes an fp16 copy of its weights
    into the workspace) and then an fp16 launch with a split tail (which needs zeroed arrival
    counters at the workspace's start): the copy sits after the counter prefix, so the fp16
    result is right.  Before the copy moved there, the second launch read weight bytes as
    counters and returned garbage."""
    from cuda_tempiler_b200 import ops
    a8, q, s = O.inputs_w8_per_channel(1024, 5120, 4096, seed=9)
    sel = ops.select(1, 1024, 5120, 4096, 1 << 40)
    c8 = ops.gemm_w8a16(torch.from_numpy(a8).cuda(), torch.from_numpy(q).cuda(),
                        torch.from_numpy(s).cuda())
    M, N, K = 300, 1024, 15360  # a split-tail problem (the planner cuts its only wave)
    assert ops._lib.load().tempo_sm100_workspace_bytes(M, N, K, 0) > 0
    a, b, c = _run(ops.gemm_fp16, M, N, K, seed=4)
    _gate(a, b, c)
    torch.cuda.synchronize()
    assert O.rel_l2(c8.cpu().numpy(), O.gemm_w_ref(a8, O.dequant_per_channel(q, s))) <= TOL
    assert sel["bn"] > 0
    assert ops.device_status() == [0, 0, 0, 0]
