"""The serving binding on CPU: the custom ops are registered with fake implementations, the
TEMPO_KERNELS switch is off by default, and with it off (or for a problem the kernels do not
cover) the linear layers are the stock F.linear path, counted as fallbacks."""
import torch

from cuda_tempiler_b200 import bind


def test_ops_registered_with_fake_shapes():
    A = torch.empty(5, 64, dtype=torch.float16, device="meta")
    B = torch.empty(24, 64, dtype=torch.float16, device="meta")
    assert torch.ops.tempo.gemm_fp16(A, B).shape == (5, 24)
    W = torch.empty(32, 64, dtype=torch.int8, device="meta")
    s = torch.empty(32, dtype=torch.float16, device="meta")
    assert torch.ops.tempo.gemm_w8a16(A, W, s, None, 0).shape == (5, 32)


def test_switch_off_by_default(monkeypatch):
    monkeypatch.delenv("TEMPO_KERNELS", raising=False)
    assert not bind.enabled()
    monkeypatch.setenv("TEMPO_KERNELS", "1")
    assert bind.enabled()


def test_fallback_is_stock_linear(monkeypatch):
    monkeypatch.setenv("TEMPO_KERNELS", "1")  # on, but CPU tensors are not covered
    bind.route_counts(reset=True)
    g = torch.Generator().manual_seed(0)
    x = torch.randn(2, 3, 64, generator=g)
    w = torch.randn(16, 64, generator=g)
    assert torch.equal(bind.linear_fp16(x, w), torch.nn.functional.linear(x, w))
    q = torch.randint(-127, 128, (16, 64), generator=g, dtype=torch.int8)
    s = torch.rand(16, generator=g).half()
    y = bind.linear_w8a16(x.half(), q, s)
    ref = torch.nn.functional.linear(x.half(), (q.float() * s.float()[:, None]).half())
    assert torch.equal(y, ref)
    assert bind.route_counts() == {"tempo": 0, "fallback": 2}


def test_dequantize_group_matches_formula():
    g = torch.Generator().manual_seed(1)
    q = torch.randint(0, 256, (32, 256), generator=g, dtype=torch.uint8)
    s = (torch.rand(2, 32, generator=g) * 0.02).half()
    z = torch.randint(100, 157, (2, 32), generator=g, dtype=torch.uint8)
    w = bind.dequantize(q, s, z, 128)
    n, k = 7, 200
    want = (float(q[n, k]) - float(z[k // 128, n])) * float(s[k // 128, n])
    assert abs(float(w[n, k]) - want) <= 1e-3 * max(1.0, abs(want))


def test_covered_predicates():
    x = torch.empty(4, 64, dtype=torch.float16)
    w = torch.empty(24, 64, dtype=torch.float16)
    assert not bind.covered_fp16(x, w)  # CPU tensors
