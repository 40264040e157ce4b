"""GPU parity of the W8A16 tcgen05 GEMM (smem dequant) against the CPU oracle."""
import numpy as np
import pytest
import torch

from oracle import gemm_oracle as O

pytestmark = pytest.mark.gpu
TOL = O.GATE_REL_L2


def _pc(M, N, K, fn, seed=2):
    a, q, s = O.inputs_w8_per_channel(M, N, K, seed)
    C = torch.empty((M, N), dtype=torch.float16, device="cuda")
    C.view(torch.int16).fill_(0x7F7F)
    fn(torch.from_numpy(a).cuda(), torch.from_numpy(q).cuda(), torch.from_numpy(s).cuda(), C)
    torch.cuda.synchronize()
    c = C.cpu().numpy()
    assert O.poison_count(c) == 0
    ref = O.gemm_w_ref(a, O.dequant_per_channel(q, s))
    return O.rel_l2(c, ref)


def _grp(M, N, K, fn, G=128, seed=3):
    a, q, s, z = O.inputs_w8_group(M, N, K, G, seed)
    C = torch.empty((M, N), dtype=torch.float16, device="cuda")
    C.view(torch.int16).fill_(0x7F7F)
    fn(torch.from_numpy(a).cuda(), torch.from_numpy(q).cuda(), torch.from_numpy(s).cuda(),
       torch.from_numpy(z).cuda(), G, C)
    torch.cuda.synchronize()
    c = C.cpu().numpy()
    assert O.poison_count(c) == 0
    ref = O.gemm_w_ref(a, O.dequant_group(q, s, z, G))
    return O.rel_l2(c, ref)


# N % 16 == 0: group-wise scale/zero rows are fetched by TMA (16-byte row strides)
SHAPES = [(1, 144, 256), (5, 528, 1024), (16, 1024, 512), (64, 272, 384), (200, 784, 1024),
          (512, 1040, 2048)]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_per_channel_dispatch(dev, M, N, K):
    from cuda_tempiler_b200 import ops
    r = _pc(M, N, K, lambda A, W, s, C: ops.gemm_w8a16(A, W, s, out=C))
    assert r <= TOL, r


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_group_dispatch(dev, M, N, K):
    from cuda_tempiler_b200 import ops
    r = _grp(M, N, K, lambda A, W, s, z, G, C: ops.gemm_w8a16(A, W, s, z, G, out=C))
    assert r <= TOL, r


# swap 2: swapped with the 8-bit weights dequantised in shared memory (W8A16 only)
HYPER = [(16, True), (32, True), (64, True), (128, True), (64, False), (128, False), (256, False),
         (32, 2), (64, 2), (128, 2)]


@pytest.mark.parametrize("bn,swap", HYPER)
@pytest.mark.parametrize("splits", [1, 2])
def test_every_hyperform(dev, bn, swap, splits):
    from cuda_tempiler_b200 import ops
    M = 24 if swap else 260
    if swap == 2:
        # shared-memory dequant: ragged M and N, splits through the cluster exchange
        r1 = _pc(37, 528, 2048, lambda A, W, s, C: ops.gemm_hyperform(
            A, W, bn=bn, swap=2, splits=splits, scale=s, out=C))
        r2 = _grp(37, 528, 2048, lambda A, W, s, z, G, C: ops.gemm_hyperform(
            A, W, bn=bn, swap=2, splits=splits, scale=s, zero=z, group_size=G, out=C))
        assert r1 <= TOL and r2 <= TOL, (r1, r2)
    r1 = _pc(M, 784, 1024, lambda A, W, s, C: ops.gemm_hyperform(
        A, W, bn=bn, swap=swap, splits=splits, scale=s, out=C))
    r2 = _grp(M, 784, 1024, lambda A, W, s, z, G, C: ops.gemm_hyperform(
        A, W, bn=bn, swap=swap, splits=splits, scale=s, zero=z, group_size=G, out=C))
    assert r1 <= TOL and r2 <= TOL, (r1, r2)


def test_naive_w8(dev):
    from cuda_tempiler_b200 import ops
    r = _pc(40, 144, 256, lambda A, W, s, C: C.copy_(ops.naive_gemm_w8a16(A, W, s)))
    assert r <= TOL
    r = _grp(40, 144, 256, lambda A, W, s, z, G, C: C.copy_(ops.naive_gemm_w8a16(A, W, s, z, G)))
    assert r <= TOL


def test_resources_match_python_plan(dev):
    """The plugin's Python shared-memory plan equals what the library launches with."""
    import ctypes as C
    from cuda_tempiler_b200 import _lib
    from cuda_tempiler_b200.tempo.plugins.sm100.skeletons_py import skel_cfg
    lib = _lib.load()
    for wq in (0, 1, 2):
        for bn, swap in HYPER:
            if wq == 0 and swap == 2:
                continue  # fp16 weights need no dequant: not instantiated
            out = (C.c_int * 6)()
            assert lib.tempo_sm100_hyperform_resources(wq, bn, int(swap), out) == 0
            c = skel_cfg(bn, wq, swap)
            assert (out[0], out[1], out[2], out[3]) == (c["threads"], c["smem"], c["stages"], c["tmem_cols"])
            assert out[5] == 0, "local memory (spills/stack) in an instantiation"


def test_gptq_checkpoint_layout_end_to_end(dev):
    """GPTQ arrays (reference generator output, golden fixture) -> repack -> kernel."""
    import os
    from cuda_tempiler_b200 import ops
    from cuda_tempiler_b200.gptq import dequantize, repack_gptq_int8
    d = np.load(os.path.join(os.path.dirname(__file__), "golden", "gptq_int8.npz"))
    W, s, z = repack_gptq_int8(torch.from_numpy(d["qweight"]), torch.from_numpy(d["qzeros"]),
                               torch.from_numpy(d["scales"]), 128)
    a = np.random.default_rng(9).standard_normal((24, 256)).astype(np.float16)
    C = ops.gemm_w8a16(torch.from_numpy(a).cuda(), W.cuda(), s.cuda(), z.cuda(), 128)
    torch.cuda.synchronize()
    ref = a.astype(np.float32) @ d["W"].astype(np.float32)
    assert O.rel_l2(C.cpu().numpy(), ref) <= TOL


@pytest.mark.parametrize("variant", [1, 2])
@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 8, 11, 16])
@pytest.mark.parametrize("N,K", [(272, 512), (10240, 1024), (9472, 2064), (264, 1040)])
def test_streaming_gemv(dev, M, N, K, variant):
    """The decode GEMV (hyperform bn=0, M <= 16) for all three weight kinds, both variants
    (group_m selects: 1 = CUDA-core FMAs, R rows per CTA; 2 = warp tensor-core MMAs, 16 rows
    per CTA with the k-slices of a row group on a cluster), ragged M and ragged N (264 rows:
    the last 16-row group is partly past N)."""
    from cuda_tempiler_b200 import ops
    r1 = _pc(M, N, K, lambda A, W, s, C: ops.gemm_hyperform(A, W, bn=0, swap=False, scale=s,
                                                             group_m=variant, out=C))
    if K % 64 == 0 and N % 16 == 0:
        r2 = _grp(M, N, K, lambda A, W, s, z, G, C: ops.gemm_hyperform(
            A, W, bn=0, swap=False, scale=s, zero=z, group_size=G, group_m=variant, out=C),
            G=128 if K % 128 == 0 else 64)
        assert r2 <= TOL, r2
    a, b = O.inputs_layer(M, N, K, seed=M)
    C = ops.gemm_hyperform(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda(), bn=0,
                           swap=False, group_m=variant)
    torch.cuda.synchronize()
    r3 = O.rel_l2(C.cpu().numpy(), O.gemm_fp16_ref(a, b))
    assert r1 <= TOL and r3 <= TOL, (r1, r3)
    assert ops.device_status() == [0, 0, 0, 0]


def test_gemv_variants_agree_and_repeat(dev):
    """Both GEMV variants on the same inputs: each deterministic over repeated launches (fixed
    reduction order, cluster k-split included), and the two within the gate of each other."""
    from cuda_tempiler_b200 import ops
    a, q, s = O.inputs_w8_per_channel(12, 3840, 15360, 4)
    A, Q, S = (torch.from_numpy(x).cuda() for x in (a, q, s))
    outs = {}
    for v in (1, 2):
        c1 = ops.gemm_hyperform(A, Q, bn=0, swap=False, scale=S, group_m=v)
        c2 = ops.gemm_hyperform(A, Q, bn=0, swap=False, scale=S, group_m=v)
        torch.cuda.synchronize()
        assert torch.equal(c1, c2), f"variant {v} not deterministic"
        outs[v] = c1.float().cpu().numpy()
    assert O.rel_l2(outs[2], outs[1]) <= TOL
    ref = O.gemm_w_ref(a, O.dequant_per_channel(q, s))
    assert O.rel_l2(outs[2], ref) <= TOL


@pytest.mark.parametrize("M,N,K", [(1024, 1040, 2048), (1100, 2064, 1024), (2048, 5120, 5120)])
def test_expand_path_prefill(dev, M, N, K):
    """M >= 1024 with a full workspace: the weights are expanded to fp16 in the workspace and
    the 2-CTA fp16 kernel runs on the copy (per-channel and group-wise); without workspace the
    same call takes the in-kernel dequant path (the W8A16 2-CTA tiles).  Both pass the gate."""
    from cuda_tempiler_b200 import ops
    sel = ops.select(1, M, N, K)
    assert sel["bn"] >= 128 and sel["swap"] == 0  # the fp16 2-CTA launch reports itself
    r = _pc(M, N, K, lambda A, W, s, C: ops.gemm_w8a16(A, W, s, out=C))
    assert r <= TOL, r
    r = _pc(M, N, K, lambda A, W, s, C: ops.gemm_w8a16(A, W, s, out=C, use_workspace=False))
    assert r <= TOL, r
    r = _grp(M, N, K, lambda A, W, s, z, G, C: ops.gemm_w8a16(A, W, s, z, G, out=C))
    assert r <= TOL, r
    assert ops.device_status() == [0, 0, 0, 0]


@pytest.mark.parametrize("bn", [128, 256])
@pytest.mark.parametrize("M,N,K", [(256, 1024, 1024), (300, 784, 2048), (77, 528, 512),
                                   (600, 2064, 1536)])
def test_pair_tiles_w8(dev, bn, M, N, K):
    """2-CTA W8A16 tiles (256 x bn, tcgen05.mma.cta_group::2): each CTA's 8 dequant warps turn
    its raw 8-bit B half into fp16 in shared memory; per-channel (scale in the epilogue) and
    group-wise (scale and zero point applied in the dequant), ragged M and N."""
    from cuda_tempiler_b200 import ops
    r1 = _pc(M, N, K, lambda A, W, s, C: ops.gemm_hyperform(
        A, W, bn=bn, swap=False, cta_group=2, scale=s, out=C))
    r2 = 0.0
    if N % 16 == 0:
        r2 = _grp(M, N, K, lambda A, W, s, z, G, C: ops.gemm_hyperform(
            A, W, bn=bn, swap=False, cta_group=2, scale=s, zero=z, group_size=G, out=C))
    assert r1 <= TOL and r2 <= TOL, (r1, r2)
    assert ops.device_status() == [0, 0, 0, 0]


@pytest.mark.parametrize("bn", [128, 256])
@pytest.mark.parametrize("M,N,K", [(256, 1024, 8192), (300, 784, 4096), (256, 5120, 17408)])
def test_pair_tiles_w8_split_tail(dev, bn, M, N, K):
    """W8A16 2-CTA tiles with the split tail (fewer tiles than clusters: every tile cut into
    k-slices, fp32 partials summed in k order by the last slice, per-channel scale applied
    there): gate passed, bit-identical run to run."""
    from cuda_tempiler_b200 import ops
    f = lambda A, W, s, C: ops.gemm_hyperform(A, W, bn=bn, swap=False, cta_group=2, splits=2,
                                              scale=s, out=C)
    assert _pc(M, N, K, f) <= TOL
    a, q, s = O.inputs_w8_per_channel(M, N, K, 2)
    A, Q, S = (torch.from_numpy(x).cuda() for x in (a, q, s))
    c1 = ops.gemm_hyperform(A, Q, bn=bn, swap=False, cta_group=2, splits=2, scale=S)
    c2 = ops.gemm_hyperform(A, Q, bn=bn, swap=False, cta_group=2, splits=2, scale=S)
    torch.cuda.synchronize()
    assert torch.equal(c1, c2)
    if N % 16 == 0:
        r = _grp(M, N, K, lambda A, W, s, z, G, C: ops.gemm_hyperform(
            A, W, bn=bn, swap=False, cta_group=2, splits=2, scale=s, zero=z, group_size=G, out=C))
        assert r <= TOL
    assert ops.device_status() == [0, 0, 0, 0]
