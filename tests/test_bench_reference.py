"""bench.py's reference arm (`--impl reference`): the CPU restatement of the reference
path timed on the host cores, one JSON line with the contract's keys.  Runs on CPU."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


# runs bench.py in-process, then reports whether the product library was ever mapped
_RUN = ("import runpy, sys; sys.argv = ['bench.py'] + sys.argv[1:]; "
        "runpy.run_path('bench.py', run_name='__main__'); "
        "print('MAPPED', 'librg_npu' in open('/proc/self/maps').read())")


@pytest.mark.parametrize("extra", [["--config", "c1"], ["--config", "c1", "--precision", "fp16"],
                                   ["--config", "c1", "--precision", "f32"],
                                   ["--config", "c3a", "--batch", "256"],
                                   ["--config", "c3a", "--batch", "256", "--weight-quant", "per_channel"]])
def test_reference_arm_line(oracle_lib, extra):
    r = subprocess.run([sys.executable, "-c", _RUN, "--impl", "reference", "--steps", "1", "--warmup", "1"] + extra,
                       capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    # the reference arm builds its model and input with oracle/ alone
    assert "MAPPED False" in r.stdout
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0 and d["higher_is_better"] is True
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["config"]["per_gpu_batch"] >= d["sample_per_step"] >= 1
