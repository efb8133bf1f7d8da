"""bench.py's reference arm on the host cores: the one JSON line the benchmark
contract asks for (metric, value, unit, step counts, cpu_baseline, e2e), the
config-3 extra, and silence on every rank but rank 0.  No GPU is needed: the
reference arm times the reference's CPU path only."""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(env_extra):
    env = dict(os.environ)
    env.update(env_extra)
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "1"],
                       cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    return [ln for ln in r.stdout.splitlines() if ln.startswith("{")]


def test_reference_arm_line():
    lines = _run({"RANK": "0", "WORLD_SIZE": "1"})
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == "W4A8 GEMV HBM GB/s (decode projection sweep, M=1)"
    assert d["unit"] == "GB/s" and d["value"] > 0
    assert d["n_gpus"] == 1 and d["steps"] == 1
    assert d["warmup"] == 3  # raised to the contract's minimum of 3 warm-up steps, and reported so
    assert d["higher_is_better"] is True and d["scaling"] == "weak" and d["vs_baseline"] is None
    assert d["ms_per_step"] > 0 and d["config"]["workload"] == "decode_sweep_c2"
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["unit"] == "GB/s" and cb["kind"] == "port" and cb["cores"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    c3 = d["extra"]["c3_lmhead_argmax"]
    assert c3["us_per_token"] > 0 and c3["tok_s"] > 0


def test_reference_arm_other_ranks_silent():
    assert _run({"RANK": "1", "WORLD_SIZE": "2"}) == []
