"""Section 5 -- synchronisation and transactions on sm_100a.

Data movement is asynchronous and bypasses registers: TMA tile loads complete as transaction
bytes on an mbarrier; tcgen05.mma reads shared memory through descriptors and reports through
tcgen05.commit onto an mbarrier.  Only the epilogue's TMEM -> register load consumes registers.
The 2-SM pairing (cta_group::2) is a skeleton axis, not a barrier scope: contract v1 closes
``BarrierKind.scope`` to warp|cta.
"""
from __future__ import annotations

from ..base import BarrierKind, PluginCapabilityError, TransactionKind, not_measured, rate


class Sm100Sync:
    def transactions(self):
        return (
            TransactionKind(id="gmem->smem", issue_op="cp.async.bulk.tensor.2d",
                            wait_op="mbarrier.try_wait.parity", granularity="barrier",
                            in_flight_max=rate("TMA.STAGES_MAX", 12, "stage", "SPEC"),
                            occupies={"TMA_L2": 1.0}, consumes_registers=False,
                            consumes_smem_staging=True, depth_axis="stages"),
            TransactionKind(id="smem->tmem(mma)", issue_op="tcgen05.mma.cta_group::1.kind::f16",
                            wait_op="tcgen05.commit+mbarrier", granularity="barrier",
                            in_flight_max=rate("UMMA.TMEM_BUFS", 2, "accumulator", "SPEC"),
                            occupies={"UMMA": 1.0, "SMEM_RD": 1.0}, consumes_registers=False,
                            consumes_smem_staging=False, depth_axis="tmem_bufs"),
            TransactionKind(id="tmem->reg", issue_op="tcgen05.ld.sync.aligned.32x32b",
                            wait_op="tcgen05.wait::ld", granularity="instruction",
                            in_flight_max=rate("TMEM.LD_INFLIGHT", 1, "load", "SPEC"),
                            occupies={"EPI": 1.0}, consumes_registers=True,
                            consumes_smem_staging=False, depth_axis=None),
            TransactionKind(id="smem->gmem", issue_op="cp.async.bulk.tensor.2d.global.shared::cta",
                            wait_op="cp.async.bulk.wait_group.read", granularity="group",
                            in_flight_max=rate("TMA.STORE_GROUPS", 2, "group", "SPEC"),
                            occupies={"EPI": 1.0}, consumes_registers=False,
                            consumes_smem_staging=True, depth_axis=None),
        )

    def barriers(self):
        return (
            BarrierKind("mbarrier", "cta", phased=True, counted=True,
                        cost=not_measured("COST.MBARRIER", "cycle")),
            BarrierKind("bar.sync", "cta", phased=False, counted=True,
                        cost=not_measured("COST.BAR_SYNC", "cycle")),
            BarrierKind("syncwarp", "warp", phased=False, counted=False,
                        cost=not_measured("COST.SYNCWARP", "cycle")),
        )

    def rendezvous_cost(self, barrier_id: str, participants: int):
        if barrier_id not in {b.id for b in self.barriers()}:
            raise PluginCapabilityError(f"barrier {barrier_id!r} is not declared")
        return not_measured(f"COST.{barrier_id.upper()}.{participants}", "cycle")
