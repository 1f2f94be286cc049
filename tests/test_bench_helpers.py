"""bench.py's bookkeeping, on CPU: a DRAM-traffic constant is reported only while the
kernel source it was captured from is unchanged, and a sampled CPU step is
extrapolated to the whole batch with its fixed part counted once."""
import hashlib
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_traffic_constants_match_their_sources():
    for (cfg, units), t in bench.MEASURED_TRAFFIC.items():
        value, why = bench.measured_traffic(cfg, units)
        digest = hashlib.sha256(open(os.path.join(ROOT, t["source"]), "rb").read()).hexdigest()
        assert digest == t["sha256"], f"{t['source']} changed since its capture: retake it"
        assert value == t["bytes"] and "capture" in why


def test_changed_source_reports_null(monkeypatch):
    key = next(iter(bench.MEASURED_TRAFFIC))
    stale = dict(bench.MEASURED_TRAFFIC[key], sha256="0" * 64)
    monkeypatch.setitem(bench.MEASURED_TRAFFIC, key, stale)
    value, why = bench.measured_traffic(*key)
    assert value is None and "changed" in why
    assert bench.measured_traffic("c1", 1) == (None, "no capture of this workload")


def test_extrapolation():
    # 10 s measured on 256 of 65536 rows, 2 s of it the absmax pass over every row
    full = bench.extrapolate(65536, 256, 10.0, 2.0)
    assert abs(full - (2.0 + 8.0 * 256)) < 1e-9
    assert bench.extrapolate(100, 100, 3.0, 0.0) == 3.0
