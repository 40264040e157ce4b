"""The CPU oracle pinned against golden vectors: exact ship-probe answers and the reference's
own GPTQ generator output (tests/golden, made by make_golden.py from the reference)."""
import json
import os

import numpy as np
import torch

from oracle import gemm_oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def test_ship_probe_known_answers():
    for c in json.load(open(os.path.join(GOLD, "ship_probe_kat.json"))):
        M, N, K = c["M"], c["N"], c["K"]
        ms, ns = O.ship_probe_cells(M, N)
        assert ms.tolist() == c["m"] and ns.tolist() == c["n"]
        if M * K <= 4 * 1024 * 1024 and N * K <= 64 * 1024 * 1024:
            exp = O.ship_probe_expected(M, N, K)
            assert np.array_equal(exp, np.array(c["expected"]))


def test_fp32_oracle_on_ship_probe_cells():
    c = json.load(open(os.path.join(GOLD, "ship_probe_kat.json")))[0]
    a, b = O.ship_probe_inputs(c["M"], c["N"], c["K"])
    C = O.gemm_fp16_ref(a, b)
    got = C[np.array(c["m"]), np.array(c["n"])]
    assert O.ship_probe_maxrel(got, np.array(c["expected"])) < 1e-6


def test_gptq_repack_and_dequant_match_reference_generator():
    d = np.load(os.path.join(GOLD, "gptq_int8.npz"))
    from cuda_tempiler_b200.gptq import dequantize, repack_gptq_int8
    W, s, z = repack_gptq_int8(torch.from_numpy(d["qweight"]), torch.from_numpy(d["qzeros"]),
                               torch.from_numpy(d["scales"]), 128)
    ref = torch.from_numpy(d["W"]).float().T             # reference W is [K, N]
    got = dequantize(W, s, z, 128).half().float()
    assert torch.equal(got, ref)
    # the oracle's restatement of the formula agrees on the same repacked arrays
    o = O.dequant_group(W.numpy(), s.numpy(), z.numpy(), 128)
    assert np.array_equal(o.astype(np.float16).astype(np.float32), ref.numpy())
