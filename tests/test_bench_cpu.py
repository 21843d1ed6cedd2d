"""CPU: the reference arm of bench.py (the reference's own v0 on the host cores, no GPU) prints the one
JSON line of the benchmark contract with the keys the driver reads."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_the_contract_line():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "3",
                        "--warmup", "3"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    if "unavailable" in d:
        pytest.skip(d["unavailable"])
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["steps"] == 3 and d["warmup"] == 3 and d["higher_is_better"] is True and d["unit"] == "TFLOPS"
    assert d["value"] > 0 and d["cpu_baseline"]["value"] == d["value"]
    assert d["cpu_baseline"]["kind"] in ("reference", "port") and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["config"]["m"] == d["config"]["n"] == d["config"]["k"] == 4096


def test_bench_rejects_too_few_warmups():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--warmup", "2"],
                       capture_output=True, text=True, timeout=120, cwd=ROOT)
    assert r.returncode != 0 and "warmup" in r.stderr


def test_output_check_catches_a_planted_mistake():
    """bench.check_rows (the bench's own check of its timed output against golden rows) passes the
    golden rows themselves and fails a planted error in each tier."""
    import numpy as np
    sys.path.insert(0, ROOT)
    import bench
    rows, gold = bench.golden("cfg1_4096_seed1")
    assert bench.check_rows(gold.copy(), gold, "f32", "f16")["ok"]
    bad = gold.copy()
    bad[3, 17] = np.float16(float(gold[3, 17]) * 1.01 + 0.5)
    assert not bench.check_rows(bad, gold, "f32", "f16")["ok"]
    nan = gold.copy()
    nan[0, 0] = np.float16("nan")
    assert not bench.check_rows(nan, gold, "f32", "f16")["ok"]
    rows2, gold2 = bench.golden("cfg2_4096_seed2")
    assert bench.check_rows(gold2.copy(), gold2, "f16", "f16")["ok"]
    assert not bench.check_rows(gold2 * np.float16(1.01), gold2, "f16", "f16")["ok"]
    rows3, gold3 = bench.golden("cfg3_sgemm_4096_seed3")
    assert bench.check_rows(gold3.copy(), gold3, "f32", "f32")["ok"]
    assert not bench.check_rows(gold3 * np.float32(1.0001), gold3, "f32", "f32")["ok"]
    rows4, gold4 = bench.golden("cfg4a_16384_seed4")
    assert bench.check_rows(gold4.copy(), gold4, "f32", "f16")["ok"]
    assert not bench.check_rows(gold4[:, ::-1].copy(), gold4, "f32", "f16")["ok"]
