"""Generate the golden fixtures in this directory by running the REFERENCE implementation
(xormal/cuda_tempiler, importable as the ``tempo`` package from a checkout given by
--reference) on fixed inputs.  Run once where the reference is available; the fixtures are
committed and the tests read only them.

Fixtures:
  rel_l2.json          reference tempo.core.op.oracle.rel_l2 on fixed vectors
  registry_match.json  reference tempo.core.emit.registry._match on predicate/keyword cases
  median_ratio.json    reference tempo.core.measure.ratio.median_ratio on fixed pairs
  wave.json            reference tempo.core.model.wave.efficiency on (ctas, quantum) cases
  recognize.json       reference TEMPO-OP parse (kernels/naive/gemm_fp16.cu) with run-time shapes
  gptq_int8.npz        reference bench/gemm_baseline.py make_gptq_int8(K=256, N=64, G=128, cpu,
                       seed=3): qweight, qzeros, scales and the dense fp16 W it reconstructs
  ship_probe_kat.json  exact fp64 values of the reference ship probe's 64 cells per shape
                       (kernels/shipped/gemm_fp16/sm_70/ship_probe.cu:41-80 patterns: multiples
                       of 1/8, so every product and sum is exact in fp64)
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    a = ap.parse_args()
    sys.path.insert(0, a.reference)
    from tempo.core.emit.registry import _match
    from tempo.core.measure.ratio import median_ratio
    from tempo.core.model.wave import efficiency
    from tempo.core.op.oracle import rel_l2
    from tempo.core.op.recognize import from_file

    rng = np.random.default_rng(0)
    cases = []
    for n in (1, 7, 64, 1000):
        x = rng.standard_normal(n).tolist()
        y = (np.array(x) + rng.standard_normal(n) * 1e-3).tolist()
        cases.append({"got": y, "ref": x, "rel_l2": rel_l2(y, x)})
    cases.append({"got": [1.0, 2.0], "ref": [0.0, 0.0], "rel_l2": None})
    json.dump(cases, open(os.path.join(HERE, "rel_l2.json"), "w"))

    preds = [({"M_max": 16}, {"M": 16}), ({"M_max": 16}, {"M": 17}), ({"M_min": 4}, {"M": 3}),
             ({"N_divides": 128}, {"N": 256}), ({"N_divides": 128}, {"N": 200}),
             ({"dtype": "fp16"}, {"dtype": "fp16"}), ({"dtype": "fp16"}, {"dtype": "int8"}),
             ({"M_max": 64, "N_divides": 8}, {"M": 1, "N": 4096}), ({"K_divides": 64}, {"M": 1})]
    json.dump([{"pred": p, "kw": k, "match": _match(p, k)} for p, k in preds],
              open(os.path.join(HERE, "registry_match.json"), "w"))

    pairs = [[[1.0, 2.0], [3.0, 3.0], [2.0, 1.0]], [[1.0, 1.0], [2.0, 1.0]], [[5.0, 0.0]]]
    json.dump([{"pairs": p, "median": median_ratio(p)} for p in pairs],
              open(os.path.join(HERE, "median_ratio.json"), "w"))
    json.dump([{"ctas": c, "quantum": q, "eff": efficiency(c, q)}
               for c, q in ((64, 80), (148, 148), (149, 148), (720, 148), (0, 148))],
              open(os.path.join(HERE, "wave.json"), "w"))

    op = from_file(os.path.join(a.reference, "kernels", "naive", "gemm_fp16.cu"),
                   {"M": 4096, "N": 15360, "K": 3840})
    json.dump({"kind": op.kind, "dtype": [op.dtype_a, op.dtype_b, op.dtype_c, op.dtype_acc],
               "layout": [op.layout_a, op.layout_b, op.layout_c], "shapes": dict(op.shapes),
               "coverage": op.coverage}, open(os.path.join(HERE, "recognize.json"), "w"))

    spec = importlib.util.spec_from_file_location(
        "ref_gemm_baseline", os.path.join(a.reference, "bench", "gemm_baseline.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    qw, qz, sc, W = mod.make_gptq_int8(256, 64, 128, "cpu", 3)
    np.savez_compressed(os.path.join(HERE, "gptq_int8.npz"), qweight=qw.numpy(),
                        qzeros=qz.numpy(), scales=sc.numpy(), W=W.numpy())

    shapes = [(1, 4096, 3840), (8, 4096, 3840), (32, 15360, 3840), (128, 4096, 3840),
              (512, 15360, 3840), (2048, 3840, 15360)]
    kat = []
    for M, N, K in shapes:
        t = np.arange(64)
        ms, ns = (t * 37) % M, (t * 53) % N
        k = np.arange(K)
        vals = []
        for m, n in zip(ms, ns):
            av = (((m * K + k) % 7) - 3) * 0.125
            bv = (((n * K + k) % 5) - 2) * 0.125
            vals.append(float(np.dot(av.astype(np.float64), bv.astype(np.float64))))
        kat.append({"M": M, "N": N, "K": K, "m": ms.tolist(), "n": ns.tolist(), "expected": vals})
    json.dump(kat, open(os.path.join(HERE, "ship_probe_kat.json"), "w"))
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
