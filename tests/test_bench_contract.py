"""bench.py's JSON line contract, checked on the reference arm (host cores only).

The reference arm times the reference's grouped CPU forward (restated in
oracle/cpu_reference.py) on whole batches and prints one JSON line with the
same metric, unit and direction as the CUDA arm, plus its own cpu_baseline and
a zero-copy e2e object.  A small layer and batch keep this a few seconds; the
CUDA arm's line is exercised by the GPU runs.
"""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _reference_line(*args):
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    out = subprocess.run(
        [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", *args],
        cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, out.stdout
    return json.loads(lines[0])


@pytest.mark.parametrize("model", ["gptoss", "lfm2", "dense"])
def test_reference_arm_prints_one_contract_line(model):
    d = _reference_line("--model", model, "--tokens", "64", "--experts", "8", "--steps", "1",
                        "--warmup", "1")
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config", "e2e",
                "cpu_baseline"):
        assert key in d, key
    assert d["impl"] == "reference"
    assert d["unit"] == "tokens/s" and d["higher_is_better"] is True
    assert d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] == 1
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert "workload" in d["config"] and "model" not in d["config"]
    assert d["e2e"]["value"] == d["value"] and d["e2e"]["unit"] == d["unit"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] in ("port", "reference")
    assert cb["cores"] >= 1 and cb["sample"].startswith("full batch")


def test_every_row_parity_helper():
    # bench.rows_parity judges the GPU forward's rows against the CPU
    # forward's on the path's bar; a non-finite row fails it
    sys.path.insert(0, ROOT)
    import bench
    want = np.linspace(-3.0, 3.0, 40, dtype=np.float32).reshape(4, 10)
    ok = bench.rows_parity(want + 1e-3, want)
    assert ok["pass"] and ok["rows"] == 4 and abs(ok["max_abs"] - 1e-3) < 1e-6
    bad = bench.rows_parity(want + 0.05, want)
    assert not bad["pass"] and bad["max_abs"] > bench.MAX_ABS
    nan = want.copy()
    nan[2, 3] = np.nan
    r = bench.rows_parity(nan, want)
    assert not r["pass"] and r["max_abs"] == float("inf")
