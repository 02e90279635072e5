"""The reference arm of bench.py on CPU: one JSON line with the fields the
benchmark contract names (the arm times the torch-CPU restatement of the
reference's per-head decode on the host cores; no GPU involved)."""
import json
import os
import subprocess
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_contract_line():
    res = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference",
                          "--steps", "1", "--warmup", "1"], capture_output=True, text=True,
                         timeout=600, cwd=REPO)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [x for x in res.stdout.splitlines() if x.startswith("{")]
    assert len(lines) == 1, res.stdout[-2000:]
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "dtype", "config"):
        assert key in d, key
    assert d["unit"] == "tokens/s" and d["higher_is_better"] is True and d["value"] > 0
    assert d["config"]["workload"] == "qwen3-8b-attn-ctx131072-b16"
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] == "port" and cb["cores"] >= 1
    assert cb["unit"] == "tokens/s" and cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
