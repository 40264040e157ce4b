"""CPU tests of the calibration loop: the tempo/calib/2 record rules (restated from the
reference's tempo/core/calib/schema.py and load.py) and the sm_100a machine table loading
measured channel rates from the plugin's data/calib records."""
import copy
import json
import math

import pytest

from cuda_tempiler_b200.tempo.core.calib import load as L
from cuda_tempiler_b200.tempo.core.calib.schema import CalibError, validate


def record(**kw):
    r = {
        "schema": "tempo/calib/2", "id": "t", "kind": "rate", "plugin": "sm_100a",
        "quantity": "q", "units": "u", "taken_with": {"tool": "probe", "counter": "clock64",
                                                       "version": "1"},
        "shape": {}, "card": {"index": 0, "clock_mhz": 1900, "foreign_procs": 0},
        "observability": "clean", "provenance": {"date": "2026-12-02", "who": "test"},
        "binds": [{"symbol": "CAP.TMA_L2", "value": 0.02, "note": "50 B/cycle"},
                  {"symbol": "LAT.HBM", "value": 900.0}],
    }
    r.update(kw)
    return r


def test_schema_rules():
    validate(record())
    for f in ("id", "kind", "plugin", "card", "provenance", "taken_with"):
        r = record()
        del r[f]
        with pytest.raises(CalibError):
            validate(r)
    with pytest.raises(CalibError):
        validate(record(schema="tempo/calib/1"))           # version 1 has no plugin field
    with pytest.raises(CalibError):
        validate(record(kind="guess"))
    with pytest.raises(CalibError):
        validate(record(observability="vibes"))
    with pytest.raises(CalibError):                         # foreign processes: invalid
        validate(record(card={"index": 0, "foreign_procs": 1}))
    with pytest.raises(CalibError):                         # unknown count: invalid too
        validate(record(card={"index": 0}))
    with pytest.raises(CalibError):
        validate(record(binds=[{"symbol": "CAP.DEQ", "value": float("nan")}]))


def test_apply_direction_and_closed_table(tmp_path, monkeypatch):
    from cuda_tempiler_b200.tempo.plugins.sm100 import machine
    monkeypatch.setattr(machine, "CALIB_DIR", str(tmp_path))   # the uncalibrated table
    base = machine.Sm100Machine().symbols()
    assert base["CAP.TMA_L2"].status == "NOT_MEASURED"
    out = L.apply(base, [record()], "sm_100a")
    assert out["CAP.TMA_L2"].status == "MEASURED" and out["CAP.TMA_L2"].value == 0.02
    assert out["CAP.TMA_L2"].units == base["CAP.TMA_L2"].units
    out["CAP.TMA_L2"].check()                               # card with zero foreign processes
    assert out["LAT.HBM"].value == 900.0
    # architectural constants are never re-measured
    out2 = L.apply(base, [record(binds=[{"symbol": "SMS", "value": 100}])], "sm_100a")
    assert out2["SMS"].value == 148
    with pytest.raises(KeyError):                           # a refusal, not an extension
        L.apply(base, [record(binds=[{"symbol": "CAP.WARP_DRIVE", "value": 1.0}])], "sm_100a")
    with pytest.raises(CalibError):                         # another plugin's record
        L.apply(base, [record(plugin="sm_70")], "sm_100a")


def test_machine_loads_records(tmp_path, monkeypatch):
    from cuda_tempiler_b200.tempo.plugins.sm100 import machine
    (tmp_path / "a.json").write_text(json.dumps(record()))
    (tmp_path / "b.json").write_text(json.dumps(record(id="other", plugin="sm_70")))
    monkeypatch.setattr(machine, "CALIB_DIR", str(tmp_path))
    m = machine.Sm100Machine()
    assert m.calibration == ["t"]                           # the sm_70 record is not ours
    assert m.symbols()["CAP.TMA_L2"].measured
    assert m.channels()["TMA_L2"].capacity.value == 0.02
    assert math.isnan(m.symbols()["CAP.EPI"].value)        # still NOT_MEASURED
    # a bad record is an error, not a silence
    (tmp_path / "c.json").write_text(json.dumps(record(id="bad", card={"foreign_procs": 2})))
    with pytest.raises(CalibError):
        machine.Sm100Machine()


def test_shipped_calibration_record_is_valid():
    """The committed record (made by `tempo calibrate` on a B200) validates and loads."""
    import glob
    import os
    from cuda_tempiler_b200.tempo.plugins.sm100 import machine
    files = glob.glob(os.path.join(machine.CALIB_DIR, "*.json"))
    if not files:
        pytest.skip("no calibration record committed")
    for f in files:
        validate(json.load(open(f)))
    m = machine.Sm100Machine()
    for sym in ("CAP.TMA_L2", "CAP.DEQ", "CAP.EPI", "LAT.TMA_L2", "LAT.HBM"):
        assert m.symbols()[sym].measured, sym
