"""The allocation-free entry point tempo_sm100_gemm_fp16_noalloc, through the C-ABI.

It serves callers that cannot hand this library device memory (serving frameworks whose
allocator owns nearly all HBM, paths that must not let cudaMalloc synchronise the device,
FFI callers without a device allocator): its split-K scratch is a fixed device array inside
the library.  Checked against the workspace-taking entry point on two calls in a row, at the
tolerance every GEMM test here uses (relL2 <= 3e-3).  Collected last on purpose.
"""
import ctypes as C

import pytest
import torch

from oracle import gemm_oracle as O

pytestmark = pytest.mark.gpu

TOL = O.GATE_REL_L2


def _noalloc(lib, A, B, out):
    M, K = A.shape
    N = B.shape[0]
    return lib.tempo_sm100_gemm_fp16_noalloc(
        A.data_ptr(), B.data_ptr(), out.data_ptr(), M, N, K, A.stride(0), B.stride(0),
        out.stride(0), torch.cuda.current_stream().cuda_stream)


def test_noalloc_matches_workspace_entry_two_calls(dev):
    from cuda_tempiler_b200 import _lib, ops
    lib = _lib.load()
    # Two different problems back to back whose dispatched configuration is a 2-CTA launch
    # with a split tail, so both put fp32 partials and arrival counters in the scratch (the
    # in-cluster k-splits of small M need none and would leave the scratch untouched).
    cases = [(300, 1024, 15360), (257, 3840, 15360)]
    for M, N, K in cases:
        need = lib.tempo_sm100_workspace_bytes(M, N, K, 0)
        assert 0 < need <= _lib.NOALLOC_SCRATCH_BYTES, (M, N, K, need)
    outs = []
    for M, N, K in cases:
        a, b = O.inputs_layer(M, N, K, seed=M)
        A, B = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
        got = torch.empty((M, N), dtype=torch.float16, device="cuda")
        got.view(torch.int16).fill_(0x7F7F)
        assert _noalloc(lib, A, B, got) == 0
        ref = ops.gemm_fp16(A, B)
        torch.cuda.synchronize()
        outs.append((a, b, got.cpu().numpy(), ref.cpu().numpy()))
    for a, b, got, ref in outs:
        assert O.poison_count(got) == 0
        # the same configuration and the same k-order of the partial sums: bit-identical
        assert O.rel_l2(got, ref) <= TOL
        assert O.rel_l2(got, O.gemm_fp16_ref(a, b)) <= TOL
    # a repeat of the first problem after the second: the scratch now holds the second call's
    # partials and counters, which must not leak into the result
    M, N, K = cases[0]
    a, b = O.inputs_layer(M, N, K, seed=M)
    A, B = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    again = torch.empty((M, N), dtype=torch.float16, device="cuda")
    assert _noalloc(lib, A, B, again) == 0
    torch.cuda.synchronize()
    assert O.rel_l2(again.cpu().numpy(), outs[0][3]) <= TOL
    assert ops.device_status() == [0, 0, 0, 0]
