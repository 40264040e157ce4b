"""The sm_100a (NVIDIA B200) plugin of the tempolator, contract ``tempo/arch/1``.

Drop-in: this directory imports its contract types relatively (``from ..base import ...``), so
copied into the reference tree as ``tempo/plugins/sm100/`` it binds to the reference's own
``tempo/plugins/base.py`` and its pipeline (``python3 -m tempo.cli emit --arch sm100 ...``)
runs it unchanged; inside this repository it binds to ``cuda_tempiler_b200.tempo.plugins.base``.
"""
from __future__ import annotations

from ..base import CONTRACT, OpSpec, PluginCapabilityError, Report
from .machine import Sm100Machine
from .memory import Sm100Memory
from .meters import Sm100Meters
from .resources import Sm100Resources, SmemBytes
from .skeletons_py import Sm100Skeletons, skel_cfg
from .sync import Sm100Sync
from .tensor import Sm100TensorUnit
from .toolchain import Sm100Toolchain


class Sm100Plugin:
    id = "sm_100a"
    contract = CONTRACT
    description = ("NVIDIA B200 (sm_100a): TMA + mbarrier pipelines, warp-specialised "
                   "tcgen05.mma into TMEM, fp16 and W8A16 (smem dequant) GEMM skeletons")

    def __init__(self):
        self.machine = Sm100Machine()
        self.memory = Sm100Memory(self.machine)
        self.tensor = Sm100TensorUnit()
        self.resources = Sm100Resources(self.machine)
        self.sync = Sm100Sync()
        self.classifier = None  # optional section: needs SASS reading, which is not done
        self.skeletons = Sm100Skeletons(self.machine, self.sync)
        self.toolchain = Sm100Toolchain()
        self.meters = Sm100Meters()

    def declared_stubs(self):
        return (
            "classifier: not provided -- classifying machine instructions requires reading the "
            "SASS of our own builds, which this project does not do; verify uses ptxas facts "
            "and ncu counters instead",
            "toolchain.disasm: refuses (same reason)",
            "meters.clock_lock: refuses -- GPU clocks are never changed, only sampled",
            "cta_group axis: only cta_group::1 is instantiated; the 2-SM pair is declared",
            "latency rates (LAT.*), TMA/epilogue/dequant channel capacities: NOT_MEASURED; the "
            "bound model is silent on them",
        )

    def selftest(self) -> Report:
        r = Report(self.id)
        r.check("contract tempo/arch/1", self.contract == CONTRACT)
        t = self.machine.symbols()
        ok = True
        for v in t.values():
            try:
                v.check()
            except Exception:
                ok = False
        r.check("every MEASURED rate carries a card with zero foreign processes", ok)
        ch = self.machine.channels()
        r.check("no SPEC rate backs a channel capacity",
                all(c.capacity.status != "SPEC" for c in ch.values()))
        r.check("UMMA capacity derived from the measured dense tensor peak",
                ch["UMMA"].capacity.measured and 0 < 1.0 / ch["UMMA"].capacity.value < 16384)
        c256 = skel_cfg(256, 0, False)
        r.check("BN=256 prefill plan: 4 stages within 227 KB, 512 TMEM columns",
                c256["stages"] == 4 and c256["smem"] <= self.machine.SMEM_PER_CTA
                and c256["tmem_cols"] == 512, str(c256))
        c16 = skel_cfg(16, 0, True)
        r.check("BN=16 decode plan: 12 stages", c16["stages"] == 12, str(c16))
        v = self.resources.verdict(100, 100, SmemBytes(c256["smem"], 512), 192, 1)
        r.check("BN=256 verdict FITS at 1 CTA/SM", v.ok and v.code == "FITS", v.explain)
        v2 = self.resources.verdict(100, 100, SmemBytes(c256["smem"], 512), 192, 2)
        r.check("two 512-column CTAs hit the TMEM wall (NO_BUDGET)", v2.code == "NO_BUDGET", v2.explain)
        v3 = self.resources.verdict(100, 100, SmemBytes(240 * 1024, 64), 192, 1)
        r.check("240 KB shared memory hits WALL_SMEM", v3.code == "WALL_SMEM")
        op = OpSpec("gemm", "fp16", "fp16", "fp16", "fp32", "k", "k", "n",
                    {"M": 4096, "N": 15360, "K": 3840}, tol_rel_l2=3e-3)
        hs = list(self.skeletons.variants(op))
        r.check("config-1 space is non-empty", len(hs) > 0, f"{len(hs)} hyperforms")
        try:
            list(self.skeletons.variants(OpSpec("gemm", "fp16", "fp16", "fp16", "fp32", "k", "n",
                                                "n", {"M": 64, "N": 64, "K": 64})))
            refused = False
        except PluginCapabilityError:
            refused = True
        r.check("layout b=n is refused structurally", refused)
        try:
            list(self.skeletons.variants(OpSpec("gemm", "fp16", "fp16", "fp16", "fp16", "k", "k",
                                                "n", {"M": 64, "N": 64, "K": 64})))
            refused = False
        except PluginCapabilityError:
            refused = True
        r.check("fp16 accumulator is refused structurally", refused)
        w8 = OpSpec("gemm", "fp16", "uint8", "fp16", "fp32", "k", "k", "n",
                    {"M": 16, "N": 5120, "K": 17408}, scale="group:128", tol_rel_l2=3e-3)
        r.check("W8A16 group-wise space is non-empty", len(list(self.skeletons.variants(w8))) > 0)
        a = self.skeletons.estimate_atoms(op, hs[0])
        r.check("atoms carry UMMA and HBM load", any("UMMA" in x.footprint for x in a)
                and any("HBM" in x.footprint for x in a))
        r.check("toolchain targets sm_100a", "arch=compute_100a,code=sm_100a" in
                " ".join(self.toolchain.arch_flags()))
        return r


def load():
    return Sm100Plugin()


def select_shipped(op):
    """The shipped dispatcher's choice for ``op`` (bn, swap, group_m, splits) when the ship
    directory of this repository is present, else None (e.g. inside another tree)."""
    import importlib.util
    import os
    name = "gemm_fp16" if op.dtype_b == "fp16" else "gemm_w8a16"
    here = os.path.dirname(os.path.abspath(__file__))
    path = os.path.join(here, "..", "..", "..", "kernels", "shipped", name, "sm_100a", "select.py")
    if not os.path.exists(path):
        return None
    spec = importlib.util.spec_from_file_location(f"tempo_ship_select_{name}", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    s = op.shapes
    pick = mod.select(name, s["M"], s["N"], s["K"], dtype_b=op.dtype_b)
    if not pick:
        return None
    return {"bn": pick["bn"], "swap": pick["swap"], "group_m": pick["group_m"]}
