"""The serving binding on the GPU: with TEMPO_KERNELS=1 the linear layers enter the kernels
(route counter) and match the oracle; a shape outside the shipped predicate takes the stock
path; with the switch off nothing enters the kernels."""
import numpy as np
import pytest
import torch

from oracle import gemm_oracle as O

pytestmark = pytest.mark.gpu


def test_linear_fp16_routes(dev, monkeypatch):
    from cuda_tempiler_b200 import bind
    a, b = O.inputs_layer(40, 1024, 512, seed=3)
    x = torch.from_numpy(a).cuda().reshape(5, 8, 512)
    w = torch.from_numpy(b).cuda()
    monkeypatch.setenv("TEMPO_KERNELS", "1")
    bind.route_counts(reset=True)
    y = bind.linear_fp16(x, w)
    torch.cuda.synchronize()
    assert bind.route_counts() == {"tempo": 1, "fallback": 0}
    assert y.shape == (5, 8, 1024)
    assert O.rel_l2(y.reshape(40, 1024).cpu().numpy(), O.gemm_fp16_ref(a, b)) <= O.GATE_REL_L2
    # N % 8 != 0: outside the shipped predicate -> the stock path
    bind.linear_fp16(x, w[:1020])
    assert bind.route_counts()["fallback"] == 1
    monkeypatch.setenv("TEMPO_KERNELS", "0")
    bind.route_counts(reset=True)
    bind.linear_fp16(x, w)
    assert bind.route_counts() == {"tempo": 0, "fallback": 1}


def test_linear_w8a16_routes(dev, monkeypatch):
    from cuda_tempiler_b200 import bind
    a, q, s, z = O.inputs_w8_group(24, 1024, 1024, 128, seed=4)
    monkeypatch.setenv("TEMPO_KERNELS", "1")
    bind.route_counts(reset=True)
    y = bind.linear_w8a16(torch.from_numpy(a).cuda(), torch.from_numpy(q).cuda(),
                          torch.from_numpy(s).cuda(), torch.from_numpy(z).cuda(), 128)
    torch.cuda.synchronize()
    assert bind.route_counts()["tempo"] == 1
    ref = O.gemm_w_ref(a, O.dequant_group(q, s, z, 128))
    assert O.rel_l2(y.cpu().numpy(), ref) <= O.GATE_REL_L2


def test_custom_op_is_strict(dev):
    from cuda_tempiler_b200 import bind  # noqa: F401  (registers the ops)
    from cuda_tempiler_b200._lib import NotCovered
    A = torch.zeros(4, 64, dtype=torch.float16, device="cuda")
    B = torch.zeros(4095, 64, dtype=torch.float16, device="cuda")
    with pytest.raises(NotCovered):
        torch.ops.tempo.gemm_fp16(A, B)
