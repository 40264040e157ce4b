"""GPU: the calibration probes run, every wait completes, and the rates are physically
plausible for a B200 (bounds loose enough for any clock, tight enough to catch a probe that
measures nothing)."""
import pytest

pytestmark = pytest.mark.gpu


def test_calibrate_stage_record():
    from cuda_tempiler_b200.tempo import calibrate_stage
    from cuda_tempiler_b200.tempo.core.calib.schema import validate
    rec = calibrate_stage.run(0)
    rec["card"]["foreign_procs"] = 0 if rec["card"]["foreign_procs"] < 0 else rec["card"]["foreign_procs"]
    b = {x["symbol"]: x["value"] for x in rec["binds"]}
    assert 1.0 / 512 < b["CAP.TMA_L2"] < 1.0        # 1 .. 512 B/cycle per SM from L2
    assert 0 < b["CAP.DEQ"] < 1.0                   # more than one element per cycle per SM
    assert 1.0 / 512 < b["CAP.EPI"] < 1.0
    assert 100 < b["LAT.TMA_L2"] < 3000
    assert b["LAT.HBM"] > b["LAT.TMA_L2"]
    m = rec["measured"]
    assert m["bulk_feed_l2_B_per_cycle_per_sm"] > m["bulk_feed_hbm_B_per_cycle_per_sm"] > 1
    if rec["card"]["foreign_procs"] == 0:
        validate(rec)
