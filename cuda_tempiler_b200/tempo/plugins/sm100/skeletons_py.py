"""Section 7 -- skeletons and search axes of the sm_100a plugin.

One hand-written skeleton family, ``gemm_sm100`` (skeletons/gemm_sm100/kernel.cuh): a
persistent, warp-specialised TMA -> mbarrier -> tcgen05.mma -> TMEM -> epilogue GEMM with
an optional shared-memory dequant stage for 8-bit weights.  Axes:

  bn         MMA N tile (UMMA N): swap-AB {16, 32, 64, 128}; prefill {64, 128, 256}
  swap_ab    1 = weights on the 128-row MMA side, activations on the narrow N side (decode);
             2 = the same with 8-bit weights dequantised in shared memory instead of TMEM
  splits     k-split count; partials in a caller workspace, last-arriving CTA reduces
  group_m    raster group height (128-row tiles) for L2 reuse of operand tiles
  weight     0 fp16, 1 int8 per-channel (scale in the epilogue), 2 uint8 group-wise
             ((q - z) * s applied in the dequant stage, since s varies along K)
  stages     derived: the deepest ring that fits 227 KB next to the epilogue staging
  cta_group  1, or 2: fp16 256 x bn tiles (bn 128..256 step 32) on a 2-CTA cluster
             (tcgen05.mma.cta_group::2), the width picked by a wave-count model, where
             splits 2 turns a ragged last wave into a stream-K region (one contiguous k-block
             run per cluster, partials reduced by the last cluster to finish a tile)
  tmem_bufs  2 (double-buffered fp32 accumulator)

The operation contract follows the reference (C = A * B^T, layouts a=k b=k c=n, fp32
accumulate; reference tempo/plugins/sm70/lower.py:106-127 refuses b=n and an fp16 accumulator
the same way, structurally).
"""
from __future__ import annotations

import json
import math
import os

from ..base import (Atom, AtomKind, Axis, Hyperform, Launch, PluginCapabilityError, Rendered)
from .resources import SmemBytes

HERE = os.path.dirname(os.path.abspath(__file__))
SKEL_DIR = os.path.join(HERE, "skeletons", "gemm_sm100")
FAMILY = "gemm_sm100"
BM, BK = 128, 64
MAX_DYN_SMEM = 232448
SWAP_BN = (16, 32, 64, 128)
SWAP_SDQ_BN = (32, 64, 128)  # swap 2 (shared-memory dequant) instantiations
PREFILL_BN = (64, 128, 256)
PAIR_BN = (256, 224, 192, 160, 128)
GEMV_MAX_M = 16  # the streaming GEMV (bn 0) covers M <= 16 (k_gemv_sm100 MM 1, 2, 4, 8, 16)  # 2-CTA tile widths (k_gemm_sm100_pair<BN>)
GEMV_THREADS = 128  # k_gemv_sm100: one CTA of 128 threads per `rows` weight rows (kGemvThreads)
GEMV_MIN_CTAS_PER_SM = 12  # launch.cuh kGemvMinCtasPerSm


GEMV_MMA_MIN_CTAS_PER_SM = 8  # launch.cuh kGemvMmaMinCtasPerSm
GEMV_MMA_MAX_SPLIT = 8  # kGemvMmaMaxSplit: k-slices of a 16-row group on one cluster


def gemv_mma_min_m(wq: int) -> int:
    """From this M the dispatcher's GEMV uses the warp tensor-core variant (launch.cuh
    gemv_mma_min_m): 5 for fp16 weights, 3 for 8-bit weights."""
    return 5 if wq == 0 else 3


def gemv_mma_splits(N: int, K: int, wq: int, sms: int = 148) -> int:
    """Cluster k-split of the tensor-core GEMV, as launch.cuh gemv_mma_splits()."""
    groups = -(-N // 16)
    want = GEMV_MMA_MIN_CTAS_PER_SM * (sms if sms > 0 else 148)
    nch = K // (8 if wq == 0 else 16)
    s = 1
    while s < GEMV_MMA_MAX_SPLIT and groups * s < want and nch // (2 * s) >= 16:
        s *= 2
    return s


def gemv_rows(N: int, M: int, sms: int = 148) -> int:
    """Weight rows per GEMV CTA, as launch.cuh gemv_rows(): the widest of 4, 2, 1 (2 at most
    for M > 4) that leaves at least GEMV_MIN_CTAS_PER_SM CTAs per SM."""
    want = GEMV_MIN_CTAS_PER_SM * (sms if sms > 0 else 148)
    r = 2 if M > 4 else 4
    while r > 1:
        if N // r >= want:
            return r
        r //= 2
    return 1
SPLITS = (1, 2, 3, 4, 6, 8)


def _ru(x, a):
    return (x + a - 1) // a * a


def pair_cfg(bn: int) -> dict:
    """Python mirror of ``PairCfg<BN>`` (2-CTA 256 x BN tiles, per CTA)."""
    stage = BM * BK * 2 + _ru((bn // 2) * BK * 2, 1024)
    epi, bar = 4 * 2 * 2048, 512
    stages = min((MAX_DYN_SMEM - 1024 - epi - bar) // stage, 8)
    acc_stride = 128 if bn <= 128 else 256  # TMEM columns per accumulator buffer
    return dict(stage_bytes=stage, stages=stages, smem=1024 + stages * stage + epi + bar,
                threads=192, tmem_cols=2 * acc_stride)


def skel_cfg(bn: int, wq: int, swap: int) -> dict:
    """Python mirror of ``SkelCfg<BN, WQ, SWAP, SMEMDQ>`` in kernel.cuh (shared-memory plan);
    swap 2 = swapped with the 8-bit weights dequantised in shared memory (SMEMDQ);
    bn == 0 is the decode GEMV (no dynamic shared memory, no TMEM, GEMV_THREADS threads)."""
    if bn == 0:
        return dict(stage_bytes=0, stages=0, smem=0, threads=GEMV_THREADS, tmem_cols=0)
    ta = bool(wq) and swap == 1  # 8-bit weights dequantised into TMEM as the A operand
    wrows = (BM if swap else bn) if wq else 0
    ks = 128 if ta else BK  # k elements per stage
    p_bytes, q_bytes, raw = (0 if ta else BM * BK * 2), bn * ks * 2, wrows * ks
    q_off = _ru(p_bytes, 1024)
    raw_off = q_off + _ru(q_bytes, 1024)
    sz = wrows * 3 * (ks // BK) if wq == 2 else 0
    stage = raw_off + _ru(raw + sz, 1024)
    epi = 0 if swap else 4 * 2 * 2048
    bar = 1024
    smem_stages = (MAX_DYN_SMEM - 1024 - epi - bar) // stage
    stages = (min(smem_stages, 24) & ~1) if ta else min(smem_stages, 12)
    nacc = 4 if bn <= 32 else (2 if bn <= 64 else 1)  # accumulators per tile
    cols = 2 * bn * nacc
    tmem = 512 if ta else (32 if cols <= 32 else 1 << (cols - 1).bit_length())
    return dict(stage_bytes=stage, stages=stages, smem=1024 + stages * stage + epi + bar,
                threads=32 * (6 + (8 if ta else 4 if wq else 0)), tmem_cols=tmem)


def weight_kind(op) -> int:
    if op.dtype_b == "fp16":
        return 0
    if op.dtype_b == "int8":
        return 1
    if op.dtype_b == "uint8":
        return 2
    raise PluginCapabilityError(f"weight dtype {op.dtype_b!r} is not offered")


def group_size(op) -> int:
    s = op.scale or ""
    if s.startswith("group:"):
        return int(s.split(":", 1)[1])
    return 128


def check_op(op) -> int:
    """Structural refusals (never AttributeError): returns the weight kind."""
    if op.kind != "gemm":
        raise PluginCapabilityError(f"operation {op.kind!r}: only 'gemm' has a skeleton")
    if (op.layout_a, op.layout_b, op.layout_c) != ("k", "k", "n"):
        raise PluginCapabilityError(
            f"layout a={op.layout_a} b={op.layout_b} c={op.layout_c}: the skeleton computes "
            "C = A * B^T with both operands K-major (a=k b=k c=n)")
    if op.dtype_acc != "fp32":
        raise PluginCapabilityError(f"accumulator {op.dtype_acc!r}: fp32 accumulation only")
    if op.dtype_a != "fp16" or op.dtype_c != "fp16":
        raise PluginCapabilityError(f"A/C {op.dtype_a}/{op.dtype_c}: fp16 only")
    wq = weight_kind(op)
    M, N, K = op.shapes["M"], op.shapes["N"], op.shapes["K"]
    if N % 8 or K % (16 if wq else 8):
        raise PluginCapabilityError(f"N={N}, K={K}: TMA needs 16-byte row strides "
                                    f"(N % 8, K % {16 if wq else 8})")
    if wq == 1 and op.scale not in (None, "per_channel"):
        raise PluginCapabilityError(f"int8 weights take a per-channel scale, not {op.scale!r}")
    if wq == 2:
        g = group_size(op)
        if g % 64 or K % g:
            raise PluginCapabilityError(f"group size {g}: must be a multiple of 64 dividing K={K}")
    return wq


def key_of(p: dict) -> str:
    if p["bn"] == 0 and p.get("gemv") == "mma":
        return f"gemv_mma_sm100_wq{p['weight']}_mg{p['mg']}_sp{p['splits']}"
    if p["bn"] == 0:
        return f"gemv_sm100_wq{p['weight']}_m{p['mm']}_r{p['rows']}"
    return (f"{FAMILY}_bn{p['bn']}_sw{p['swap']}_sp{p['splits']}_gm{p['group_m']}"
            f"_wq{p['weight']}_cg{p['cta_group']}")


def entry_name(p: dict) -> str:
    if p.get("cta_group", 1) == 2:
        return f"tempo_sm100::k_gemm_sm100_pair<{p['bn']}>"
    if p["bn"] == 0 and p.get("gemv") == "mma":
        return f"tempo_sm100::k_gemv_mma_sm100<{p['weight']}, {p['mg']}>"
    if p["bn"] == 0:
        return f"tempo_sm100::k_gemv_sm100<{p['weight']}, {p.get('mm', 4)}, {p.get('rows', 4)}>"
    if p["swap"] == 2:
        return f"tempo_sm100::k_gemm_sm100<{p['bn']}, {p['weight']}, true, true>"
    return f"tempo_sm100::k_gemm_sm100<{p['bn']}, {p['weight']}, {'true' if p['swap'] else 'false'}>"


def problem_geometry(op, p):
    """Units per SM-sized work item; a 2-CTA tile counts as two 128-row units."""
    M, N, K = op.shapes["M"], op.shapes["N"], op.shapes["K"]
    rows_p, rows_q = (N, M) if p["swap"] else (M, N)
    tiles = math.ceil(rows_p / BM) * math.ceil(rows_q / p["bn"])
    num_kb = math.ceil(K / BK)
    if p.get("cta_group", 1) == 2:
        tiles = 2 * math.ceil(M / 256) * math.ceil(N / p["bn"])
        if p["splits"] > 1:  # stream-K: the k-blocks spread evenly over the SMs
            return dict(tiles=tiles, num_kb=num_kb, splits=1, units=tiles,
                        kb_per_unit=num_kb, balanced=True)
    splits = max(1, min(p["splits"], num_kb))
    return dict(tiles=tiles, num_kb=num_kb, splits=splits, units=tiles * splits,
                kb_per_unit=math.ceil(num_kb / splits))


class Sm100Skeletons:
    def __init__(self, machine, sync=None, build_facts=None):
        self.m = machine
        self.sync = sync
        self._facts = build_facts if build_facts is not None else _load_facts()

    def _staging_regs(self, p) -> int:
        """Registers a feed path costs when it passes through registers (the G8 field): the
        whole in-flight ring divided over the CTA's threads.  TMA bypasses registers (0)."""
        if self.sync is None:
            return 0
        tk = next((t for t in self.sync.transactions() if t.id == "gmem->smem"), None)
        if tk is None or not tk.consumes_registers:
            return 0
        c = skel_cfg(p["bn"], p["weight"], int(p["swap"]))
        return (c["stages"] * c["stage_bytes"]) // (4 * c["threads"])

    def ops(self):
        return ("gemm",)

    def axes(self):
        return (
            Axis("bn", frozenset({"tmem", "smem", "umma_shape", "waves"})),
            Axis("swap_ab", frozenset({"umma_shape", "waves", "epilogue"})),
            Axis("splits", frozenset({"waves", "workspace", "hbm"})),
            Axis("group_m", frozenset({"l2"})),
            Axis("weight", frozenset({"hbm", "smem", "dequant"})),
            Axis("stages", frozenset({"smem", "latency_hiding"})),
            Axis("cta_group", frozenset({"smem", "umma_shape"})),
            Axis("tmem_bufs", frozenset({"tmem", "epilogue_overlap"})),
        )

    def variants(self, op):
        wq = check_op(op)
        M, N, K = op.shapes["M"], op.shapes["N"], op.shapes["K"]
        num_kb = math.ceil(K / BK)
        forms, forms_out = [], []
        if M <= GEMV_MAX_M:
            mm = 1 if M == 1 else 2 if M == 2 else 4 if M <= 4 else 8 if M <= 8 else 16
            p = dict(family=FAMILY, bn=0, swap=0, splits=1, group_m=0, weight=wq, stages=0,
                     cta_group=1, tmem_bufs=0, mm=mm,
                     rows=gemv_rows(N, M, int(self.m.sms().value)))
            if wq == 2:
                p["group_size"] = group_size(op)
            forms_out.append(Hyperform(plugin=self.m.arch(), params=p, key=key_of(p)))
            # the warp tensor-core GEMV: 16 weight rows per CTA, k-slices on a cluster
            p = dict(family=FAMILY, bn=0, swap=0, group_m=2, weight=wq, stages=0,
                     cta_group=1, tmem_bufs=0, gemv="mma", mg=1 if M <= 8 else 2,
                     splits=gemv_mma_splits(N, K, wq, int(self.m.sms().value)))
            if wq == 2:
                p["group_size"] = group_size(op)
            forms_out.append(Hyperform(plugin=self.m.arch(), params=p, key=key_of(p)))
        if M <= 256:
            forms += [(bn, 1) for bn in SWAP_BN]
            if wq:  # swapped 8-bit weights dequantised in shared memory instead of TMEM
                forms += [(bn, 2) for bn in SWAP_SDQ_BN]
        forms += [(bn, 0) for bn in PREFILL_BN]
        if wq == 0 and M > 128:  # 2-CTA cluster tiles (cta_group::2); splits 2 = stream-K
            for bn in PAIR_BN:
                for splits in (1, 2):
                    c = pair_cfg(bn)
                    p = dict(family=FAMILY, bn=bn, swap=0, splits=splits, group_m=16, weight=0,
                             stages=c["stages"], cta_group=2, tmem_bufs=2)
                    forms_out.append(Hyperform(plugin=self.m.arch(), params=p, key=key_of(p)))
        for bn, swap in forms:
            for splits in SPLITS:
                if splits > 1 and splits > num_kb // 2:
                    continue
                for gm in ((8,) if swap else (8, 16)):
                    c = skel_cfg(bn, wq, int(swap))
                    p = dict(family=FAMILY, bn=bn, swap=swap, splits=splits, group_m=gm,
                             weight=wq, stages=c["stages"], cta_group=1, tmem_bufs=2)
                    if wq == 2:
                        p["group_size"] = group_size(op)
                    forms_out.append(Hyperform(plugin=self.m.arch(), params=p, key=key_of(p)))
        # Most promising first (a pipeline that emits the first kept variant gets the measured
        # ladder's pick): ladder (bn, swap) match, then the plugin's own cycle estimate.
        pick = ladder_pick(op, wq)
        forms_out.sort(key=lambda h: (0 if pick and (h.params["bn"], h.params["swap"],
                                                     h.params.get("cta_group", 1)) == pick else 1,
                                      self._estimate_cycles(op, h), h.params["splits"], h.key))
        yield from forms_out

    def _estimate_cycles(self, op, h) -> float:
        ch = self.m.channels()
        load: dict = {}
        for a in self.estimate_atoms(op, h):
            for k, v in a.footprint.items():
                load[k] = load.get(k, 0.0) + v
        best = 0.0
        for k, v in load.items():
            c = ch.get(k)
            if c is None or c.capacity.status in ("NOT_MEASURED", "SPEC"):
                continue
            best = max(best, v * c.capacity.value)
        return best

    def estimate_atoms(self, op, h):
        """Whole-launch load of the busiest SM on each channel (scope "sched" channels turn
        it into cycles): UMMA FLOPs, shared-memory operand reads, TMA feed bytes, this SM's
        share of the compulsory HBM traffic, epilogue bytes and dequantised elements."""
        p = h.params
        M, N, K = op.shapes["M"], op.shapes["N"], op.shapes["K"]
        sms = int(self.m.sms().value)
        if p["bn"] == 0:  # streaming GEMV: HBM stream shared by all SMs
            w_bytes = 1 if p["weight"] else 2
            hbm = (2.0 * M * K + w_bytes * N * K + 2.0 * M * N) / sms
            if p.get("gemv") == "mma":  # warp MMAs of 16 x 8 x 16 (8 or 16 activation rows)
                mmas = -(-N // 16) * (K / 16.0) * p["mg"] / sms
                return [Atom(0, AtomKind.MEM_READ, "LDG.128.STREAM", {"HBM": hbm}),
                        Atom(1, AtomKind.COMPUTE, "HMMA.16816.F32", {"FMA": mmas * 2048.0})]
            return [Atom(0, AtomKind.MEM_READ, "LDG.128.STREAM", {"HBM": hbm}),
                    Atom(1, AtomKind.COMPUTE, "HFMA2", {"FMA": 2.0 * M * N * K / sms})]
        g = problem_geometry(op, p)
        if g.get("balanced"):
            kb = g["units"] * g["kb_per_unit"] / sms
            waves = g["units"] / sms
        else:
            waves = math.ceil(g["units"] / sms)
            kb = waves * g["kb_per_unit"]
        bn, wq = p["bn"], p["weight"]
        flops = kb * 2.0 * BM * bn * BK
        b_rows = bn // 2 if p.get("cta_group", 1) == 2 else bn  # B rows this SM holds
        ta = bool(wq) and p["swap"] == 1  # A operand (weights) from TMEM, not shared memory
        smem_rd = kb * ((0 if ta else BM) + b_rows) * BK * 2.0
        w_rows = BM if p["swap"] else bn
        act_rows = bn if p["swap"] else BM
        if p.get("cta_group", 1) == 2:
            w_rows = b_rows
        tma = kb * (act_rows * BK * 2.0 + w_rows * BK * (1.0 if wq else 2.0))
        w_bytes = 1 if wq else 2
        hbm_total = 2.0 * M * K + w_bytes * N * K + 2.0 * M * N
        if p["splits"] > 1:
            hbm_total += 2.0 * g["tiles"] * p["splits"] * BM * bn * 4.0
        hbm = hbm_total / min(sms, g["units"])
        epi = waves * BM * bn * (4.0 if p["splits"] > 1 else 2.0)
        atoms = [
            Atom(0, AtomKind.XFER_ISSUE, "TMA.LOAD.2D", {"TMA_L2": tma}, token="stage"),
            Atom(1, AtomKind.XFER_WAIT, "MBAR.WAIT", {}, token="stage"),
            Atom(2, AtomKind.MEM_READ, "SMEM.UMMA_OPERANDS", {"SMEM_RD": smem_rd}),
            Atom(3, AtomKind.COMPUTE, f"UMMA.F16.M128N{bn}K16", {"UMMA": flops}),
            Atom(4, AtomKind.MEM_READ, "HBM.STREAM", {"HBM": hbm}),
            Atom(5, AtomKind.MEM_WRITE, "EPI.TMEM_TO_GLOBAL", {"EPI": epi}, region="epilogue"),
        ]
        if wq:
            # CAP.DEQ is measured for 4 dequant warps; the TMEM-A tiles run 8
            atoms.append(Atom(6, AtomKind.COMPUTE, "DEQUANT.U8_TO_F16",
                              {"DEQ": kb * w_rows * BK * (0.5 if ta else 1.0)}, region="dequant"))
        return atoms

    def resources_of(self, op, h):
        p = h.params
        c = pair_cfg(p["bn"]) if p.get("cta_group", 1) == 2 else \
            skel_cfg(p["bn"], p["weight"], int(p["swap"]))
        regs = self._facts.get(entry_name(p), {}).get("regs", 128 if p["bn"] else 64)
        if p["bn"]:
            regs += self._staging_regs(p)
        return regs, regs, SmemBytes(c["smem"], c["tmem_cols"])

    def launch_of(self, op, h):
        p = h.params
        c = pair_cfg(p["bn"]) if p.get("cta_group", 1) == 2 else \
            skel_cfg(p["bn"], p["weight"], int(p["swap"]))
        if p["bn"] == 0 and p.get("gemv") == "mma":
            return Launch(grid_ctas=-(-op.shapes["N"] // 16) * p["splits"], threads=GEMV_THREADS,
                          smem_bytes=0, entry=entry_name(p), min_ctas_per_sm=1)
        if p["bn"] == 0:
            return Launch(grid_ctas=-(-op.shapes["N"] // p["rows"]), threads=GEMV_THREADS,
                          smem_bytes=0,
                          entry=entry_name(p), min_ctas_per_sm=1)
        g = problem_geometry(op, p)
        return Launch(grid_ctas=min(g["units"], int(self.m.sms().value)), threads=c["threads"],
                      smem_bytes=c["smem"], entry=entry_name(p), min_ctas_per_sm=1)

    def render(self, op, h):
        """A self-contained translation unit: the skeleton text (PTX wrappers + kernel
        template), an explicit instantiation through an extern "C" entry probe, and the
        hyperform's launch facts as comments."""
        p = h.params
        src = skeleton_source()
        probe = f"tempo_entry_probe_{h.key}"
        inst = (f"\n// ---- hyperform {h.key}\n"
                f"// op: M={op.shapes['M']} N={op.shapes['N']} K={op.shapes['K']} "
                f"{op.dtype_a}*{op.dtype_b}->{op.dtype_c} acc {op.dtype_acc}\n"
                f"// params: {json.dumps(p, sort_keys=True)}\n"
                f"extern \"C\" const void* {probe}() {{\n"
                f"  return reinterpret_cast<const void*>(&{entry_name(p)});\n}}\n")
        return Rendered(source=src + inst, launch=self.launch_of(op, h),
                        includes=("cuda.h", "cuda_fp16.h"), notes=f"entry probe {probe}",
                        filename=f"kernel_{h.key}.cu")

    def entry_probe(self, h):
        return f"tempo_entry_probe_{h.key} -> {entry_name(h.params)}"

    def capabilities(self):
        return frozenset({"gemm_fp16", "gemm_w8a16_per_channel", "gemm_w8a16_group",
                          "swap_ab", "split_k", "tcgen05", "tma", "persistent"})


DEFAULT_LADDER = [(4, 0, 0), (16, 16, 1), (32, 32, 1), (64, 64, 1), (256, 128, 1), (1 << 31, 256, 0)]


def ladder_pick(op, wq: int):
    """(bn, swap) of the shipped M-ladder for this problem: the ship directory's select.py
    when this repository's ship tree is present, else the built-in default ladder."""
    M = op.shapes["M"]
    name = "gemm_fp16" if wq == 0 else "gemm_w8a16"
    path = os.path.join(HERE, "..", "..", "..", "kernels", "shipped", name, "sm_100a", "select.py")
    rows = DEFAULT_LADDER
    if os.path.exists(path):
        import importlib.util
        spec = importlib.util.spec_from_file_location(f"tempo_ship_ladder_{name}", path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        rows = [(r[0], r[1], r[2], r[4] if len(r) > 4 else 1) for r in mod.LADDER]
    for row in rows:
        if M <= row[0]:
            cg = row[3] if len(row) > 3 else 1
            return (row[1], row[2], cg if wq == 0 else 1)
    return None


def _strip_local_includes(text: str) -> str:
    out = []
    for line in text.split("\n"):
        s = line.strip()
        if s.startswith("#include \"") or s == "#pragma once":
            continue
        out.append(line)
    return "\n".join(out)


def skeleton_source(with_launch: bool = False) -> str:
    """Concatenated skeleton text: PTX wrappers, kernel template (and optionally the naive
    kernels and the host launch layer), local includes removed so it stands alone."""
    parts = ["sm100_ptx.cuh", "kernel.cuh"] + (["naive.cuh", "launch.cuh"] if with_launch else [])
    txt = ["#pragma once"] if with_launch else []
    for name in parts:
        with open(os.path.join(SKEL_DIR, name), encoding="utf-8") as f:
            txt.append(f"// ===== {name}\n" + _strip_local_includes(f.read()))
    return "\n".join(txt) + "\n"


def _load_facts() -> dict:
    path = os.path.join(HERE, "data", "build_facts.json")
    if os.path.exists(path):
        with open(path, encoding="utf-8") as f:
            return json.load(f).get("entries", {})
    return {}
