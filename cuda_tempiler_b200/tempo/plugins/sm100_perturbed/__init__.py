"""Falsifier G6: the sm100 plugin with exactly one rate changed -- CAP.HBM halved (twice the
bandwidth).  Only the HBM channel's bound may move, and it must halve."""
from __future__ import annotations

import dataclasses

from ..sm100 import Sm100Plugin


class PerturbedPlugin(Sm100Plugin):
    id = "sm_100a_perturbed"
    description = "falsifier G6: sm100 with CAP.HBM halved"

    def __init__(self):
        super().__init__()
        m = self.machine
        hbm = m._table["CAP.HBM"]
        m._table["CAP.HBM"] = dataclasses.replace(hbm, value=hbm.value / 2.0)
        m._channels["HBM"] = dataclasses.replace(m._channels["HBM"], capacity=m._table["CAP.HBM"])


def load():
    return PerturbedPlugin()
