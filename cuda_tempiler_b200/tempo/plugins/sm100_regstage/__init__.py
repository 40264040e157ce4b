"""Falsifier G8: the sm100 plugin with exactly one two-valued field flipped -- the
gmem->smem transaction ``consumes_registers`` = True (a register-staged feed instead of TMA).
The resource verdict must move."""
from __future__ import annotations

import dataclasses

from ..sm100 import Sm100Plugin
from ..sm100.sync import Sm100Sync


class RegStageSync(Sm100Sync):
    def transactions(self):
        out = []
        for t in super().transactions():
            if t.id == "gmem->smem":
                t = dataclasses.replace(t, consumes_registers=True)
            out.append(t)
        return tuple(out)


class RegStagePlugin(Sm100Plugin):
    id = "sm_100a_regstage"
    description = "falsifier G8: sm100 with a register-staged operand feed"

    def __init__(self):
        super().__init__()
        self.sync = RegStageSync()
        self.skeletons.sync = self.sync


def load():
    return RegStagePlugin()
