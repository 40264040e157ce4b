"""Falsifier G3: a fake architecture with nothing in common with any GPU -- 13 SMs, 7-lane
warps, a 5x3x2 tensor op, two channels Z (scope sched) and Y (scope sm) -- whose hand-computed
period the arch-agnostic pipeline must reproduce end to end (recognize -> variants -> prune
-> bound -> emit).

Hand computation for op M=N=K=60 and the single hyperform "t": per iteration the skeleton
emits atoms with footprint Z = 12 units and Y = 9 units; CAP.Z = 2.5 cycles/unit (sched),
CAP.Y = 3 units/cycle (sm) with 2 resident warps -> Z: 12 * 2.5 = 30, Y: 9 * 2 / 3 = 6;
T = 30, bound by Z.
"""
from __future__ import annotations

from ..base import (CONTRACT, Atom, AtomKind, Axis, CardState, Channel, FragmentMap, Hyperform,
                    Launch, Occupancy, PluginCapabilityError, Provenance, Rate, Rendered,
                    Report, ResourceVerdict, TensorOp, TransactionKind, closed_table_get, rate)

CARD = CardState(index=0, clock_mhz=1000, foreign_procs=0, date="1970-01-01")
PROV = Provenance("hand", None, "1", "1970-01-01", "gate", "clean", CARD)


class Machine:
    def __init__(self):
        self.t = {"SMS": rate("SMS", 13, "SM", "SPEC"),
                  "CAP.Z": Rate("CAP.Z", 2.5, "cycle/unit", "MEASURED", PROV),
                  "CAP.Y": Rate("CAP.Y", 3.0, "unit/cycle", "MEASURED", PROV)}

    def arch(self):
        return "nullarch"

    def symbols(self):
        return dict(self.t)

    def channels(self):
        return {"Z": Channel("Z", "sched", self.t["CAP.Z"]), "Y": Channel("Y", "sm", self.t["CAP.Y"])}

    def latency(self, c):
        return closed_table_get(self.t, "LAT." + c)

    def sms(self):
        return self.t["SMS"]

    def schedulers_per_sm(self):
        return rate("SCHED", 1, "scheduler", "SPEC")

    def warp_slots_per_sm(self):
        return rate("SLOTS", 4, "warp", "SPEC")

    def threads_per_warp(self):
        return rate("WARP", 7, "thread", "SPEC")

    def smem_per_sm(self):
        return rate("SMEM", 1000, "B", "SPEC")

    def smem_per_cta_max(self):
        return rate("SMEM_CTA", 1000, "B", "SPEC")

    def regfile_words_per_sm(self):
        return rate("REGS", 700, "word", "SPEC")

    def clock_mhz(self):
        return rate("CLK", 1000, "MHz", "SPEC")

    def peak(self, kind):
        return closed_table_get(self.t, "PEAK." + kind)


class Resources:
    def __init__(self, sync):
        self.sync = sync

    def verdict(self, regs, max_live, smem, threads, min_ctas_per_sm=1):
        occ = Occupancy(warps_per_sm=2, ctas_per_sm=1, regs_per_thread=regs, limiter="toy")
        if smem > 1000:
            return ResourceVerdict(False, "WALL_SMEM", occ, "toy smem wall")
        if max_live > 50:
            return ResourceVerdict(False, "SPILL", occ, "toy register budget 50")
        return ResourceVerdict(True, "FITS", occ, "toy")

    def reg_budget(self, w):
        return 50

    def spill_threshold(self, m):
        return 50

    def free_spills(self):
        return 0

    def spill_cost(self, n):
        return rate("SPILL", n, "cycle", "MODEL")

    def occupancy(self, regs, smem, threads):
        return Occupancy(2, 1, regs, "toy")

    def wave_quantum(self, occ):
        return 13

    def declared_bounds_required(self):
        return False


class Sync:
    consumes_registers = False

    def transactions(self):
        return (TransactionKind("gmem->smem", "TOYLD", "TOYWAIT", "barrier",
                                rate("INFLIGHT", 2, "stage", "SPEC"), {"Z": 1.0},
                                self.consumes_registers, True, "depth"),)

    def barriers(self):
        return ()

    def rendezvous_cost(self, b, n):
        return rate("RV", 1, "cycle", "MODEL")


class Skeletons:
    def __init__(self, sync):
        self.sync = sync

    def ops(self):
        return ("gemm",)

    def axes(self):
        return (Axis("depth", frozenset({"registers"})),)

    def variants(self, op):
        if op.kind != "gemm":
            raise PluginCapabilityError("toy: gemm only")
        yield Hyperform("nullarch", {"depth": 2}, "t")

    def estimate_atoms(self, op, h):
        return [Atom(0, AtomKind.COMPUTE, "TOYMMA", {"Z": 12.0}),
                Atom(1, AtomKind.MEM_READ, "TOYLD", {"Y": 9.0})]

    def resources_of(self, op, h):
        staged = 40 if self.sync.transactions()[0].consumes_registers else 0
        return 20 + staged, 20 + staged, 500

    def launch_of(self, op, h):
        return Launch(13, 14, 500, "toy_entry")

    def render(self, op, h):
        return Rendered("// toy kernel\nvoid toy_entry() {}\n", self.launch_of(op, h), filename="toy.cu")

    def entry_probe(self, h):
        return "toy_entry"

    def capabilities(self):
        return frozenset({"toy"})


class Tensor:
    def ops(self):
        return (TensorOp("TOY.5x3x2", 5, 3, 2, ("fp16", "fp16"), "fp32",
                         FragmentMap(lambda l: [(0, 0, 0)], lambda l: [(0, 0, 0)],
                                     lambda l: [(0, 0, 0), (0, 1, 1)]),
                         rate("TOYCOST", 1, "cycle", "MODEL"), "registers"),)

    def select(self, i, a):
        return self.ops()[0]


class NullArchPlugin:
    id = "nullarch"
    contract = CONTRACT
    description = "falsifier G3/G8: toy architecture with a hand-computed period"
    sync_cls = Sync

    def __init__(self):
        self.machine = Machine()
        self.memory = None
        self.tensor = Tensor()
        self.sync = self.sync_cls()
        self.resources = Resources(self.sync)
        self.classifier = None
        self.skeletons = Skeletons(self.sync)
        self.toolchain = None
        self.meters = None

    def declared_stubs(self):
        return ("memory", "toolchain", "meters")

    def selftest(self):
        r = Report(self.id)
        r.check("toy channels declared", set(self.machine.channels()) == {"Z", "Y"})
        return r


def load():
    return NullArchPlugin()
