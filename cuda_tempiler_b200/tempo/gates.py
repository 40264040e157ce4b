"""Boundary gates G1-G8 (adapted from the reference's tests/test_gates.py:60-394): they prove
the pipeline is arch-agnostic and the sm100 plugin honours the contract.  Each gate returns
(ok, message); ``main`` prints PASS/FAIL and returns non-zero on failure."""
from __future__ import annotations

import ast
import os
import sys

from .plugins import registry
from .plugins.base import OpSpec, PluginCapabilityError, PluginError, UnknownSymbol

HERE = os.path.dirname(os.path.abspath(__file__))
CORE = os.path.join(HERE, "core")
PKG = os.path.dirname(HERE)
ARCH_TOKENS = ("sm_100", "sm100", "B200", "tcgen05", "TMEM", "UMMA", "Blackwell", "nullarch")


def _core_files():
    for root, _, files in os.walk(CORE):
        for f in files:
            if f.endswith(".py"):
                yield os.path.join(root, f)


def g1_lexical():
    """G1: the pipeline (core/) names no architecture and no hardware literal."""
    bad = []
    for p in _core_files():
        text = open(p, encoding="utf-8").read()
        bad += [f"{os.path.relpath(p, HERE)}: {t}" for t in ARCH_TOKENS if t in text]
    return not bad, "; ".join(bad) or "core names no architecture"


def g2_null_refuses():
    """G2: the null plugin refuses structurally; the pipeline survives it."""
    from .core.search.prune import prune
    p = registry.load("null")
    op = OpSpec("gemm", "fp16", "fp16", "fp16", "fp32", "k", "k", "n", {"M": 8, "N": 8, "K": 8})
    try:
        list(p.skeletons.variants(op))
        return False, "variants() did not refuse"
    except AttributeError as e:
        return False, f"AttributeError instead of a structural refusal: {e}"
    except PluginError:
        pass
    cands = prune(p, op, [object()])
    return (len(cands) == 1 and not cands[0].kept), "null plugin refused; prune kept nothing"


def _toy_op():
    return OpSpec("gemm", "fp16", "fp16", "fp16", "fp32", "k", "k", "n",
                  {"M": 60, "N": 60, "K": 60}, tol_rel_l2=1e-3)


def g3_nullarch_period():
    """G3: the pipeline runs end to end on a toy architecture and reproduces T = 30 (Z)."""
    import tempfile

    from .core.emit.render import emit
    from .core.search.prune import kept, prune
    p = registry.load("nullarch")
    op = _toy_op()
    c = prune(p, op, list(p.skeletons.variants(op)))
    k = kept(c)
    if not k or k[0].bound is None:
        return False, "nothing kept"
    b = k[0].bound
    with tempfile.TemporaryDirectory() as d:
        path = emit(p, op, k[0].hyper, d)
        emitted = os.path.exists(path)
    ok = abs(b.T - 30.0) < 1e-9 and b.binding == "Z" and emitted
    return ok, f"T={b.T} bound by {b.binding}, emitted={emitted}"


def g4_closed_rates():
    """G4: a rate outside the closed table is a refusal, not a default."""
    p = registry.load("sm100")
    try:
        p.machine.latency("NO_SUCH_ATOM_CLASS")
        return False, "unknown symbol answered"
    except UnknownSymbol:
        return True, "UnknownSymbol raised"


def g5_core_imports():
    """G5: core imports no plugin but the contract, and spawns no process."""
    bad = []
    for p in _core_files():
        tree = ast.parse(open(p, encoding="utf-8").read())
        for node in ast.walk(tree):
            mods = []
            if isinstance(node, ast.Import):
                mods = [a.name for a in node.names]
            elif isinstance(node, ast.ImportFrom):
                mods = [("." * node.level) + (node.module or "")]
            for m in mods:
                if "plugins" in m and not m.endswith("plugins.base"):
                    bad.append(f"{os.path.relpath(p, HERE)} imports {m}")
                if m.split(".")[0] in ("subprocess", "multiprocessing"):
                    bad.append(f"{os.path.relpath(p, HERE)} imports {m}")
    return not bad, "; ".join(bad) or "core imports only the contract"


def _hbm_bound_op():
    return OpSpec("gemm", "fp16", "fp16", "fp16", "fp32", "k", "k", "n",
                  {"M": 16, "N": 30720, "K": 3840}, tol_rel_l2=3e-3)


def g6_perturbed_rate():
    """G6: doubling one rate (HBM bandwidth) halves exactly that channel's bound."""
    from .core.model.bound import bound
    a, b = registry.load("sm100"), registry.load("sm100_perturbed")
    op = _hbm_bound_op()
    h = next(iter(a.skeletons.variants(op)))
    ba = bound(a.skeletons.estimate_atoms(op, h), a.machine.channels())
    bb = bound(b.skeletons.estimate_atoms(op, h), b.machine.channels())
    ok = abs(bb.per_channel["HBM"] * 2 - ba.per_channel["HBM"]) < 1e-6 * ba.per_channel["HBM"]
    for ch in ba.per_channel:
        if ch != "HBM" and abs(ba.per_channel[ch] - bb.per_channel[ch]) > 1e-9:
            ok = False
    return ok, f"HBM {ba.per_channel['HBM']:.0f} -> {bb.per_channel['HBM']:.0f} cycles, others unchanged"


def g7_no_machine_paths():
    """G7: product sources carry no absolute path of a build machine."""
    bad = []
    for root, _, files in os.walk(PKG):
        if "__pycache__" in root:
            continue
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h", ".inc")):
                p = os.path.join(root, f)
                t = open(p, encoding="utf-8", errors="replace").read()
                for tok in ("/" + "root/", "/" + "home/", "/" + "tmp/"):
                    if tok in t:
                        bad.append(f"{os.path.relpath(p, PKG)}: {tok}")
    return not bad, "; ".join(bad) or "no machine paths"


def g8_two_valued_field():
    """G8: flipping consumes_registers of the operand feed must move the resource verdict."""
    a, b = registry.load("sm100"), registry.load("sm100_regstage")
    op = OpSpec("gemm", "fp16", "fp16", "fp16", "fp32", "k", "k", "n",
                {"M": 4096, "N": 15360, "K": 3840}, tol_rel_l2=3e-3)
    h = next(h for h in a.skeletons.variants(op) if h.params["bn"] == 256)

    def verdict(p):
        regs, ml, smem = p.skeletons.resources_of(op, h)
        l = p.skeletons.launch_of(op, h)
        return p.resources.verdict(regs, ml, smem, l.threads, l.min_ctas_per_sm)
    va, vb = verdict(a), verdict(b)
    return va.code != vb.code, f"TMA feed: {va.code}; register-staged feed: {vb.code}"


GATES = [("G1", g1_lexical), ("G2", g2_null_refuses), ("G3", g3_nullarch_period),
         ("G4", g4_closed_rates), ("G5", g5_core_imports), ("G6", g6_perturbed_rate),
         ("G7", g7_no_machine_paths), ("G8", g8_two_valued_field)]


def main() -> int:
    bad = 0
    for name, fn in GATES:
        try:
            ok, msg = fn()
        except Exception as e:  # a crashing gate is a failing gate
            ok, msg = False, f"{type(e).__name__}: {e}"
        print(f"{'PASS' if ok else 'FAIL'} {name} {fn.__doc__.strip().splitlines()[0]}\n     {msg}")
        bad += not ok
    print(f"GATES: {len(GATES) - bad}/{len(GATES)}")
    return 1 if bad else 0


if __name__ == "__main__":
    sys.exit(main())
