"""The JSON line of `bench.py --impl reference` (the CPU arm, which needs no
GPU): one line, the keys the bench contract names, and the same metric and
workload as our own arm's line."""
import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def test_reference_arm_line():
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                        "--steps", "1", "--warmup", "3"], cwd=ROOT, env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip().startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    for k in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
              "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
              "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference" and d["n_gpus"] == 1 and d["steps"] == 1
    assert d["warmup"] >= 3 and d["value"] > 0 and d["higher_is_better"] is True
    assert d["metric"] == "micro-ops/sec (requests/s) of the 16K mixed-op request stream"
    assert d["config"]["workload"] == ("mixed_24op: 16384 requests, 24 ops, f32, sizes "
                                       "log-uniform [256, 32768], flush every 512")
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
