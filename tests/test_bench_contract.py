"""The benchmark's JSON contract, on the CPU: `bench.py --impl reference`
(the reference's CPU expert loop, the arm the driver runs beside ours) prints
one JSON line with the keys and types the driver reads.  No GPU."""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]

REQUIRED = {
    "metric": str, "value": float, "unit": str, "n_gpus": int, "steps": int, "warmup": int,
    "ms_per_step": float, "higher_is_better": bool, "scaling": str, "dtype": str, "data": str,
    "config": dict, "impl": str, "cpu_baseline": dict, "e2e": dict,
}


def test_reference_arm_prints_one_contract_line():
    proc = subprocess.run(
        [sys.executable, "bench.py", "--impl", "reference", "--steps", "3", "--warmup", "3"],
        cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [l for l in proc.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, proc.stdout
    d = json.loads(lines[0])
    for key, typ in REQUIRED.items():
        assert key in d, key
        assert isinstance(d[key], typ), (key, type(d[key]))
    assert "vs_baseline" in d
    assert d["impl"] == "reference"
    assert d["metric"] == "moe_layer_tokens_per_s" and d["unit"] == "tokens/s"
    assert d["n_gpus"] == 1 and d["steps"] == 3 and d["warmup"] == 3
    assert d["higher_is_better"] is True and d["value"] > 0
    assert d["config"]["tokens"] == 72214 and "workload" in d["config"]
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert "sample" in cb
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
