"""The plugin boundary: the ``tempo/arch/1`` contract.

This restates the reference's contract (reference tempo/plugins/base.py:54-660) -- the same
type names, field names and meanings, so a plugin written against either module works with
both pipelines.  The pipeline (tempo.core) never names an architecture; everything measured on
a specific machine lives in a plugin.

Rules carried over from the reference contract:

* A number carries its unit, status and provenance (``Rate``).  ``MEASURED`` requires a card
  state with zero foreign processes; ``SPEC`` (a datasheet figure) may never enter a time bound.
* A plugin that cannot do something refuses *structurally* (``PluginCapabilityError`` /
  ``NotSupported``), never with AttributeError.
* Unknown contract majors are rejected at load time.
* Enum values are ASCII (they travel into manifest.json).

Version: ``tempo/arch/1``.  Thread-block clusters are not expressible as a barrier scope in v1
(``BarrierKind.scope`` is closed to warp|cta); the sm100 plugin declares its 2-SM pairing as an
opaque skeleton axis instead.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from enum import Enum
from pathlib import Path
from typing import (Any, Callable, ContextManager, Iterable, Iterator, Literal, Mapping,
                    Optional, Protocol, Sequence, runtime_checkable)

CONTRACT = "tempo/arch/1"
CONTRACT_MAJOR = "tempo/arch"

ArchId = str  # e.g. "sm_100a"; the pipeline never compares it with a literal


# ----------------------------------------------------------------------------- errors
class PluginError(Exception):
    """Root of every boundary error; the pipeline catches these, not AttributeError."""


class PluginCapabilityError(PluginError):
    """The plugin cannot do what was asked: a structural refusal, not a crash."""


class UnknownSymbol(PluginError):
    """A rate outside the closed ``Machine.symbols()`` table was requested."""


class ContractError(PluginError):
    """The plugin broke the contract (unknown major, MEASURED without a card, ...)."""


class NotSupported(PluginError):
    """An optional capability is not implemented: a legal answer, not a defect."""


# ----------------------------------------------------------------------------- provenance
STATUS = ("MEASURED", "SPEC", "MODEL", "UPPER_BOUND", "NOT_MEASURED")


@dataclass(frozen=True)
class CardState:
    """State of the card when a number was measured; a MEASURED rate needs one."""
    index: int
    clock_mhz: int
    foreign_procs: int
    date: str


@dataclass(frozen=True)
class Provenance:
    tool: str
    counter: Optional[str]
    version: str
    date: str
    who: str
    observability: Literal["clean", "code_edit", "derived"]
    card: Optional[CardState] = None


@dataclass(frozen=True)
class Rate:
    """A number with its unit, status and provenance."""
    symbol: str
    value: float
    units: str
    status: Literal["MEASURED", "SPEC", "MODEL", "UPPER_BOUND", "NOT_MEASURED"]
    prov: Optional[Provenance] = None
    note: str = ""

    def __post_init__(self):
        if self.status not in STATUS:
            raise ContractError(f"status {self.status!r} not in {STATUS}")

    @property
    def measured(self) -> bool:
        return self.status == "MEASURED"

    def check(self) -> None:
        """Loader-enforced rules: MEASURED needs a card with zero foreign processes."""
        if self.status == "MEASURED":
            if self.prov is None or self.prov.card is None:
                raise ContractError(f"{self.symbol}: MEASURED without a card state")
            if self.prov.card.foreign_procs != 0:
                raise ContractError(f"{self.symbol}: MEASURED with {self.prov.card.foreign_procs} "
                                    "foreign processes on the card")


def spec_forbidden_in_time_bound(r: Rate) -> None:
    """A datasheet (SPEC) figure may not enter a time bound: MEASURED or UPPER_BOUND only."""
    if r.status == "SPEC":
        raise ContractError(f"{r.symbol}: SPEC rate used in a time bound")


# ----------------------------------------------------------------------------- atoms (the IR)
class AtomKind(str, Enum):
    COMPUTE = "COMPUTE"
    MEM_READ = "MEM_READ"
    MEM_WRITE = "MEM_WRITE"
    XFER_ISSUE = "XFER_ISSUE"  # split transaction: issue ...
    XFER_WAIT = "XFER_WAIT"    # ... and wait
    BARRIER = "BARRIER"
    BRANCH = "BRANCH"
    SPILL = "SPILL"
    OTHER = "OTHER"


@dataclass(frozen=True)
class Dep:
    src_uid: int
    type: Literal["RAW", "WAR", "WAW", "CTRL", "XFER"]
    distance: int = 0
    min_gap: float = 0.0


@dataclass(frozen=True)
class Atom:
    """A unit of load: a footprint of occupied cycles per channel.  ``op_id`` is opaque."""
    uid: int
    kind: AtomKind
    op_id: str
    footprint: Mapping[str, float]
    latency: float = 0.0
    token: Optional[str] = None
    deps: tuple = ()
    region: str = "body"


# ----------------------------------------------------------------------------- 1. machine
@dataclass(frozen=True)
class Channel:
    """Something occupied over an interval.  scope "sched": capacity is cycles per command;
    scope "sm": capacity is units per cycle for the whole SM."""
    name: str
    scope: Literal["sched", "sm"]
    capacity: Rate


@runtime_checkable
class Machine(Protocol):
    def arch(self) -> ArchId: ...
    def symbols(self) -> Mapping[str, Rate]: ...
    def channels(self) -> Mapping[str, Channel]: ...
    def latency(self, atom_class: str) -> Rate: ...
    def sms(self) -> Rate: ...
    def schedulers_per_sm(self) -> Rate: ...
    def warp_slots_per_sm(self) -> Rate: ...
    def threads_per_warp(self) -> Rate: ...
    def smem_per_sm(self) -> Rate: ...
    def smem_per_cta_max(self) -> Rate: ...
    def regfile_words_per_sm(self) -> Rate: ...
    def clock_mhz(self) -> Rate: ...
    def peak(self, kind: str) -> Rate: ...


# ----------------------------------------------------------------------------- 2. memory
@dataclass(frozen=True)
class WavefrontCost:
    degree: float
    floor: float
    wavefronts: float


@dataclass(frozen=True)
class MemLevel:
    name: str
    bytes_: Rate
    bandwidth: Rate
    latency: Rate


@dataclass(frozen=True)
class Layout:
    """Shared-memory array layout: the input of the bank-conflict law."""
    name: str
    row_words: int
    rows: int
    elem_bytes: int
    swizzle: Optional[str] = None


@runtime_checkable
class Memory(Protocol):
    def levels(self) -> tuple: ...
    def wavefronts(self, lane_words: Sequence, width_bytes: int) -> WavefrontCost: ...
    def alignment_rule(self, width_bytes: int) -> int: ...
    def pad_family(self, layout: Layout) -> Iterable[int]: ...
    def swizzle_family(self, layout: Layout) -> Iterable[str]: ...
    def residency_policy(self) -> str: ...


# ----------------------------------------------------------------------------- 3. tensor unit
@dataclass(frozen=True)
class FragmentMap:
    """lane -> [(row, col, register slot)] for A, B and C of one tensor instruction."""
    a: Callable[[int], Sequence]
    b: Callable[[int], Sequence]
    c: Callable[[int], Sequence]


@dataclass(frozen=True)
class TensorOp:
    id: str
    m: int
    n: int
    k: int
    in_dtypes: tuple
    acc_dtype: str
    frag: FragmentMap
    cost: Rate
    operand_source: Literal["registers", "smem_direct"]
    loader: Optional[str] = None
    exact_while: Optional[str] = None


@runtime_checkable
class TensorUnit(Protocol):
    def ops(self) -> tuple: ...
    def select(self, in_dtypes: tuple, acc_dtype: str) -> TensorOp: ...


def acc_regs_per_thread(warp_tile: tuple, op: TensorOp) -> int:
    """Accumulator registers per thread, derived from the fragment map (never a constant)."""
    m, n = warp_tile
    per_op = len(op.frag.c(0))
    return per_op * (m // op.m) * (n // op.n)


def operand_loads_per_mma(warp_tile: tuple, op: TensorOp) -> float:
    """Fragment loads per tensor instruction: (MB + NB) / (MB * NB) in units of the op."""
    mb = warp_tile[0] // op.m
    nb = warp_tile[1] // op.n
    if mb <= 0 or nb <= 0:
        raise ContractError(f"warp tile {warp_tile!r} smaller than {op.id}")
    return (mb + nb) / float(mb * nb)


# ----------------------------------------------------------------------------- 4. resources
RESOURCE_CODES = ("FITS", "SPILL", "WALL_REG", "WALL_SMEM", "NO_BUDGET")


@dataclass(frozen=True)
class Occupancy:
    warps_per_sm: int
    ctas_per_sm: int
    regs_per_thread: int
    limiter: str


@dataclass(frozen=True)
class ResourceVerdict:
    ok: bool
    code: Literal["FITS", "SPILL", "WALL_REG", "WALL_SMEM", "NO_BUDGET"]
    occ: Occupancy
    explain: str  # for the report only; the pipeline never branches on the text

    def __post_init__(self):
        if self.code not in RESOURCE_CODES:
            raise ContractError(f"verdict code {self.code!r} not in {RESOURCE_CODES}")


@runtime_checkable
class Resources(Protocol):
    def reg_budget(self, warps_per_sm: int) -> int: ...
    def spill_threshold(self, max_live: int) -> int: ...
    def free_spills(self) -> int: ...
    def spill_cost(self, n: int) -> Rate: ...
    def occupancy(self, regs: int, smem_bytes: int, threads: int) -> Occupancy: ...
    def verdict(self, regs: int, max_live: int, smem_bytes: int, threads: int,
                min_ctas_per_sm: int = 1) -> ResourceVerdict: ...
    def wave_quantum(self, occ: Occupancy) -> int: ...
    def declared_bounds_required(self) -> bool: ...


# ----------------------------------------------------------------------------- 5. sync
@dataclass(frozen=True)
class TransactionKind:
    """How data is fed.  ``consumes_registers`` is the two-valued field the G8 falsifier flips."""
    id: str
    issue_op: str
    wait_op: Optional[str]
    granularity: Literal["instruction", "group", "barrier"]
    in_flight_max: Rate
    occupies: Mapping[str, float]
    consumes_registers: bool
    consumes_smem_staging: bool
    depth_axis: Optional[str] = None


@dataclass(frozen=True)
class BarrierKind:
    id: str
    scope: Literal["warp", "cta"]
    phased: bool
    counted: bool
    cost: Rate


@runtime_checkable
class Sync(Protocol):
    def transactions(self) -> tuple: ...
    def barriers(self) -> tuple: ...
    def rendezvous_cost(self, barrier_id: str, participants: int) -> Rate: ...


# ----------------------------------------------------------------------------- 6. classifier
@dataclass(frozen=True)
class AtomClass:
    channel: str
    cycles: float
    width_bytes: int
    latency_class: str
    predicated: bool


@runtime_checkable
class Classifier(Protocol):
    def classify(self, instr_text: str) -> AtomClass: ...
    def decode(self, binary: Path, kernel_regex: str) -> Any: ...
    def control_fields(self, word: int) -> Any: ...


# ----------------------------------------------------------------------------- 7. skeletons
@dataclass(frozen=True)
class Hyperform:
    plugin: ArchId
    params: Mapping[str, Any]  # opaque to the pipeline
    key: str                   # stable hash -> kernel and ship-directory name


@dataclass(frozen=True)
class Axis:
    name: str
    affects: frozenset


@dataclass(frozen=True)
class Launch:
    grid_ctas: int
    threads: int
    smem_bytes: int
    entry: str
    min_ctas_per_sm: int = 1  # residency declared to the compiler (sets its register budget)


@dataclass(frozen=True)
class Rendered:
    source: str
    launch: Launch
    includes: tuple = ()
    notes: str = ""
    filename: str = "kernel.cuh"  # a file with explicit instantiations must be a .cu


@runtime_checkable
class Skeletons(Protocol):
    def ops(self) -> tuple: ...
    def axes(self) -> tuple: ...
    def variants(self, op: "OpSpec") -> Iterator[Hyperform]: ...
    def estimate_atoms(self, op: "OpSpec", h: Hyperform) -> list: ...
    def resources_of(self, op: "OpSpec", h: Hyperform) -> tuple: ...
    def launch_of(self, op: "OpSpec", h: Hyperform) -> Launch: ...
    def render(self, op: "OpSpec", h: Hyperform) -> Rendered: ...
    def entry_probe(self, h: Hyperform) -> str: ...
    def capabilities(self) -> frozenset: ...


# ----------------------------------------------------------------------------- 8. toolchain
@dataclass(frozen=True)
class BuildResult:
    ok: bool
    binary: Optional[Path]
    regs: int
    spill_st: int
    spill_ld: int
    stack_frame: int
    smem_static: int
    smem_dynamic: int
    ldl_stl_in_loops: Optional[int]
    log: str


@dataclass(frozen=True)
class EnvReq:
    name: str
    path: Optional[str]
    what: str


@runtime_checkable
class Toolchain(Protocol):
    def arch_flags(self) -> list: ...
    def compile(self, source: Path, out: Path, mode: str, extra: list,
                build_dir: Path) -> BuildResult: ...
    def disasm(self, binary: Path) -> str: ...
    def requirements(self) -> list: ...


@runtime_checkable
class Meters(Protocol):
    def counters(self, kind: str) -> list: ...
    def profile(self, binary: Path, kernel: str, counters: list) -> Mapping[str, float]: ...
    def clock_lock(self, card: int, mhz: int) -> ContextManager: ...


# ----------------------------------------------------------------------------- pipeline side
@dataclass(frozen=True)
class OpSpec:
    """The *declared* operation (parsed from a TEMPO-OP block, never from arbitrary C++)."""
    kind: str
    dtype_a: str
    dtype_b: str
    dtype_c: str
    dtype_acc: str
    layout_a: str
    layout_b: str
    layout_c: str
    shapes: Mapping[str, int]
    scale: Optional[str] = None
    tol_rel_l2: float = 0.0
    coverage: str = "atomic_stamp"


@dataclass
class Report:
    """A plugin's self-check report."""
    name: str
    ok: int = 0
    total: int = 0
    lines: list = field(default_factory=list)

    def check(self, label: str, cond: bool, note: str = "") -> bool:
        self.total += 1
        if cond:
            self.ok += 1
        self.lines.append(("ok   " if cond else "FAIL ", label, note))
        return bool(cond)

    @property
    def green(self) -> bool:
        return self.total > 0 and self.ok == self.total

    def render(self) -> str:
        out = [f"PLUGIN SELF-CHECK {self.name}"]
        for st, label, note in self.lines:
            out.append(f"  {st} {label}" + (f"  -- {note}" if note else ""))
        out.append(f"  TOTAL: {self.ok}/{self.total}")
        return "\n".join(out)


@runtime_checkable
class Plugin(Protocol):
    id: ArchId
    contract: str
    description: str
    machine: Machine
    memory: Memory
    tensor: TensorUnit
    resources: Resources
    sync: Sync
    classifier: Optional[Classifier]
    skeletons: Skeletons
    toolchain: Toolchain
    meters: Meters

    def declared_stubs(self) -> tuple: ...
    def selftest(self) -> Report: ...


# ----------------------------------------------------------------------------- plugin helpers
def rate(symbol, value, units, status, note="", prov=None) -> Rate:
    return Rate(symbol=symbol, value=float(value), units=units, status=status, note=note, prov=prov)


def not_measured(symbol, units, note="") -> Rate:
    """A rate that does not exist yet; printed as such."""
    return Rate(symbol=symbol, value=float("nan"), units=units, status="NOT_MEASURED", note=note)


def closed_table_get(table: Mapping[str, Rate], symbol: str) -> Rate:
    """Closed rate table: a missing symbol is a refusal, never a default."""
    try:
        return table[symbol]
    except KeyError:
        raise UnknownSymbol(f"rate {symbol!r} is not declared (closed table of "
                            f"{len(table)} symbols)") from None
