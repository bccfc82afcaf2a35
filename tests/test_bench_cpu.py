"""bench.py's reference arm on the host: `--impl reference` times the
reference's CPU path (the oracle restatement of the forward on the host
threads) and prints one JSON line with the contract's keys: the same metric
and unit as the GPU arm, `impl: reference`, the CPU sample it timed in
`cpu_baseline`, and an `e2e` object with no host<->device bytes.  One page,
one step: about fifteen seconds on the host."""
import json
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                        "--steps", "1", "--warmup", "0"],
                       capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.strip()]
    assert len(lines) == 1, lines
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["unit"] == "pages/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 1 and d["warmup"] == 0 and d["n_gpus"] == 1
    assert d["metric"].startswith("pages/s")
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["unit"] == "pages/s"
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert d["config"]["workload"]
