"""tempolator CLI -- stages of the pipeline for the sm_100a plugin.

  doctor                               tools and device
  plugins                              plugins and their capabilities
  selftest [--arch sm100]              plugin self-checks
  gates                                boundary gates G1..G8
  stubs --arch sm100                   honest list of what is not implemented
  recognize FILE.cu [M N K]            naive source with a TEMPO-OP block -> spec
  space --arch sm100 -M -N -K          enumerate and prune without building
  emit  --arch sm100 -M -N -K --out D  render the chosen hyperform to D/kernel_<key>.cu
  build --arch sm100 -M -N -K --out D  emit + compile (-Xptxas -v facts)
  verify --arch sm100 -M -N -K --out D build + reject spills / stack frames / missing sm_100a path
  measure --arch sm100 -M -N -K        GPU: correctness gate, then paired timing vs cuBLAS and naive
  tune [--set fp16|w8pc|w8g|all]       GPU: measured sweep of the shipped family -> JSON
  calibrate [--device N]               GPU: probe the NOT_MEASURED channels -> tempo/calib/2 record
  passport [--out FILE]                GPU: card state + gate over every production point
  ship --from TUNE.json                derive the M-ladder, write kernels/shipped/<op>/sm_100a
  ship --passport FILE                 re-freeze, writing card and gate into the manifests

Weights: --dtype-b fp16 (default) | int8 (per-channel scale) | uint8 (--scale group:128).
"""
from __future__ import annotations

import argparse
import json
import os
import sys


def _plugin(a):
    from ..plugins import registry
    return registry.load(a.arch)


def _op(a):
    from ..plugins.base import OpSpec
    scale = a.scale
    if scale is None and a.dtype_b == "int8":
        scale = "per_channel"
    if scale is None and a.dtype_b == "uint8":
        scale = "group:128"
    return OpSpec(kind="gemm", dtype_a="fp16", dtype_b=a.dtype_b, dtype_c="fp16", dtype_acc="fp32",
                  layout_a="k", layout_b=a.layout_b, layout_c="n",
                  shapes={"M": a.M, "N": a.N, "K": a.K}, scale=scale, tol_rel_l2=3e-3)


def cmd_doctor(a):
    from . import env
    env.main([])
    print("\nPLUGINS:")
    from ..plugins import registry
    for name in registry.available():
        try:
            print(f"  {name:<16} {registry.load(name).description}")
        except Exception as e:
            print(f"  {name:<16} LOAD REFUSED: {e}")
    return 0


def cmd_plugins(a):
    from ..plugins import registry
    for name in registry.available():
        p = registry.load(name)
        print(f"{name}  (arch id {p.id}, contract {p.contract})\n  {p.description}")
        try:
            print("  capabilities: " + (", ".join(sorted(p.skeletons.capabilities())) or "-"))
        except Exception as e:
            print(f"  capabilities: -- ({type(e).__name__})")
        print(f"  declared stubs: {len(p.declared_stubs())}\n")
    return 0


def cmd_selftest(a):
    from ..plugins import registry
    bad = 0
    for name in ([a.arch] if a.arch else registry.available()):
        r = registry.load(name).selftest()
        print(r.render() + "\n")
        bad += not r.green
    return 1 if bad else 0


def cmd_gates(a):
    from .. import gates
    return gates.main()


def cmd_stubs(a):
    p = _plugin(a)
    print(f"NOT IMPLEMENTED -- {p.id}")
    for s in p.declared_stubs():
        print("  * " + s)
    return 0


def cmd_recognize(a):
    from ..core.op.recognize import from_file
    from ..core.op.spec import describe, flops
    shapes = {"M": a.M, "N": a.N, "K": a.K} if a.M else {}
    op = from_file(a.source, shapes)
    print("RECOGNISED: " + describe(op))
    print(f"tolerance relL2 {op.tol_rel_l2:g}; coverage policy {op.coverage}")
    print(f"work: {flops(op):.3g} FLOP")
    return 0


def _candidates(a):
    from ..core.search.prune import prune
    p = _plugin(a)
    op = _op(a)
    return p, op, prune(p, op, list(p.skeletons.variants(op)))


def cmd_space(a):
    from ..core.search.prune import summary
    from ..core.search.space import axes_table
    p, op, cands = _candidates(a)
    print(axes_table(p) + "\n")
    for c in sorted(cands, key=lambda c: (not c.kept, getattr(c.hyper, "key", ""))):
        print("  " + c.render())
    print("\n" + summary(cands))
    return 0


def _choose(p, op, cands):
    """The shipped ladder's (measured) choice when it is among the kept candidates, else the
    kept candidate with the best model bound."""
    from ..core.search.prune import ranked
    good = ranked(cands)
    if not good:
        return None
    try:
        from ..plugins.sm100 import select_shipped
        pick = select_shipped(op)
    except Exception:
        pick = None
    if pick:
        match = [c.hyper for c in good if all(c.hyper.params.get(k) == v for k, v in pick.items())]
        if match:
            return min(match, key=lambda h: h.params.get("splits", 1))
    return good[0].hyper


def cmd_emit(a):
    from ..core.emit.render import emit
    p, op, cands = _candidates(a)
    h = _choose(p, op, cands)
    if h is None:
        print("THE PRUNER KEPT NOTHING -- nothing to emit")
        return 2
    path = emit(p, op, h, a.out)
    print(f"emitted: {path} (hyperform {h.key})")
    print(f"entry probe: {p.skeletons.entry_probe(h)}")
    a._emitted = (p, op, h, path)
    return 0


def cmd_build(a):
    from pathlib import Path
    rc = cmd_emit(a)
    if rc:
        return rc
    p, op, h, path = a._emitted
    out = Path(path).with_suffix(".o")
    br = p.toolchain.compile(Path(path), out, "obj", [], Path(a.out))
    print(f"build {'OK' if br.ok else 'FAILED'}: regs {br.regs}, spill st/ld {br.spill_st}/"
          f"{br.spill_ld}, stack frame {br.stack_frame}, smem static {br.smem_static}")
    if not br.ok:
        print(br.log[-2000:])
        return 3
    a._build = br
    return 0


def cmd_verify(a):
    rc = cmd_build(a)
    if rc:
        return rc
    br = a._build
    problems = []
    if br.stack_frame:
        problems.append(f"stack frame {br.stack_frame} B")
    if br.spill_st or br.spill_ld:
        problems.append(f"spills {br.spill_st}/{br.spill_ld} B")
    if "k_gemm_sm100" not in br.log:
        problems.append("no sm_100a entry was compiled (tcgen05 path compiled out?)")
    for msg in problems:
        print("REJECTED: " + msg)
    if not problems:
        print("VERIFIED: no spills, no stack frame, sm_100a tcgen05/TMA entry compiled")
    return 4 if problems else 0


def cmd_measure(a):
    from ..measure_stage import measure
    return measure(_plugin(a), _op(a), rounds=a.rounds)


def cmd_tune(a):
    from ... import tune
    argv = ["--set", a.set, "--rounds", str(a.rounds)]
    if a.ms:
        argv += ["--ms", a.ms]
    if a.out:
        argv += ["--out", a.out]
    return tune.main(argv)


def cmd_calibrate(a):
    from .. import calibrate_stage
    from ..plugins.sm100 import machine
    rec = calibrate_stage.run(a.device)
    path = calibrate_stage.write(rec, a.out or machine.CALIB_DIR)
    for b in rec["binds"]:
        print(f"  {b['symbol']:12s} {b['value']:.5g}  {b['note']}")
    for k, v in rec["measured"].items():
        print(f"  measured {k} = {v}")
    print(f"wrote {path}")
    return 0


def cmd_passport(a):
    from ..passport_stage import main as passport_main
    return passport_main(a.out, a.device)


def cmd_ship(a):
    from ..plugins.sm100 import ship
    rows = json.load(open(a.source)) if a.source else []
    root = a.out or os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(
        os.path.abspath(__file__)))), "kernels", "shipped")
    facts = {}
    try:
        from ... import build as libbuild
        from ..plugins.sm100.toolchain import demangle_family, parse_ptxas
        log = (libbuild.PKG / "libtempo_sm100.ptxas.log")
        if log.exists():
            for k, v in parse_ptxas(log.read_text()).items():
                name = demangle_family(k)
                if name:
                    facts[name] = v
    except Exception:
        pass
    for op, kinds in (("gemm_fp16", (0,)), ("gemm_w8a16", (1, 2))):
        prev = os.path.join(root, op, "sm_100a", "manifest.json")
        if rows:
            lad = ship.derive_ladder(rows, kinds)
            measured = [{"kind": r["kind"], "name": r.get("name"), "M": r["M"], "N": r["N"],
                         "K": r["K"], "best": r["best"], "dispatch": r["dispatch"]}
                        for r in rows if r["kind"] in kinds]
            if getattr(a, "merge", False) and os.path.exists(prev):
                m0 = json.load(open(prev))
                old = [(r["m_max"], r["bn"], r["swap"], r["group_m"], r.get("cta_group", 1))
                       for r in m0["ladder"]]
                lad, keep_from = ship.merge_ladder(lad, old, [r["M"] for r in rows
                                                              if r["kind"] in kinds])
                measured += [r for r in m0.get("rows", []) if r["M"] > keep_from]
        elif os.path.exists(prev):  # re-freeze the skeleton under the ladder already shipped
            m0 = json.load(open(prev))
            lad = [(r["m_max"], r["bn"], r["swap"], r["group_m"], r.get("cta_group", 1))
                   for r in m0["ladder"]]
            lad[-1] = (ship.INF,) + lad[-1][1:]
            measured = m0.get("rows", [])
        else:
            lad, measured = list(ship.DEFAULT_LADDER), []
        m0 = json.load(open(prev)) if os.path.exists(prev) else {}
        gate, card = m0.get("gate"), m0.get("card")
        if getattr(a, "passport", None):
            pp = json.load(open(a.passport))
            card = pp["card"]
            g = dict(pp["gate"][op])
            g["rows"] = [{k: r[k] for k in ("gemm", "M", "N", "K", "rel_l2", "spot_fp64",
                                             "uncovered") if k in r} | ({"scale": r["scale"]}
                                                                        if "scale" in r else {})
                         for r in g["rows"]]
            gate = g
        m = ship.write_ship(op, lad, root, build_facts=facts, measured=measured,
                            gate=gate, card=card)
        print(f"shipped {op}: ladder {m['ladder']}")
    if facts:
        d = os.path.join(os.path.dirname(ship.__file__), "data", "build_facts.json")
        with open(d, "w") as f:
            json.dump({"schema": "tempo/build_facts/1", "entries": facts}, f, indent=1, sort_keys=True)
    return 0


def main(argv=None):
    ap = argparse.ArgumentParser(prog="tempo", description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = ap.add_subparsers(dest="cmd", required=True)
    sub.add_parser("doctor").set_defaults(fn=cmd_doctor)
    sub.add_parser("plugins").set_defaults(fn=cmd_plugins)
    s = sub.add_parser("selftest")
    s.add_argument("--arch")
    s.set_defaults(fn=cmd_selftest)
    sub.add_parser("gates").set_defaults(fn=cmd_gates)
    s = sub.add_parser("stubs")
    s.add_argument("--arch", default="sm100")
    s.set_defaults(fn=cmd_stubs)
    s = sub.add_parser("recognize")
    s.add_argument("source")
    for k in ("M", "N", "K"):
        s.add_argument(k, nargs="?", type=int)
    s.set_defaults(fn=cmd_recognize)
    for name, fn in (("space", cmd_space), ("emit", cmd_emit), ("build", cmd_build),
                     ("verify", cmd_verify), ("measure", cmd_measure)):
        s = sub.add_parser(name)
        s.add_argument("--arch", default="sm100")
        s.add_argument("-M", type=int, required=True)
        s.add_argument("-N", type=int, required=True)
        s.add_argument("-K", type=int, required=True)
        s.add_argument("--dtype-b", default="fp16", choices=["fp16", "int8", "uint8"])
        s.add_argument("--layout-b", default="k")
        s.add_argument("--scale", default=None)
        if name in ("emit", "build", "verify"):
            s.add_argument("--out", required=True)
        if name == "measure":
            s.add_argument("--rounds", type=int, default=9)
        s.set_defaults(fn=fn)
    s = sub.add_parser("tune")
    s.add_argument("--set", default="fp16", choices=["fp16", "w8pc", "w8g", "all"])
    s.add_argument("--ms", default=None)
    s.add_argument("--rounds", type=int, default=5)
    s.add_argument("--out", default=None)
    s.set_defaults(fn=cmd_tune)
    s = sub.add_parser("calibrate")
    s.add_argument("--device", type=int, default=0)
    s.add_argument("--out", default=None, help="record directory (default: the plugin's data/calib)")
    s.set_defaults(fn=cmd_calibrate)
    s = sub.add_parser("passport")
    s.add_argument("--device", type=int, default=0)
    s.add_argument("--out", default=None)
    s.set_defaults(fn=cmd_passport)
    s = sub.add_parser("ship")
    s.add_argument("--passport", default=None,
                   help="tempo/passport/1 JSON (from `passport`): card and gate into the manifests")
    s.add_argument("--from", dest="source", default=None)
    s.add_argument("--out", default=None)
    s.add_argument("--merge", action="store_true",
                   help="re-derive only the M bands the tune rows cover; keep the shipped "
                        "ladder rows (and measured rows) above them")
    s.set_defaults(fn=cmd_ship)
    a = ap.parse_args(argv)
    return a.fn(a)


if __name__ == "__main__":
    sys.exit(main())
