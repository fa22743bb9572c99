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


# Runs the reference arm in-process, then reports whether this repository's
# library or package was ever loaded into that process.
_RUN_REFERENCE_ARM = """
import runpy, sys
sys.argv = ["bench.py", "--impl", "reference", "--steps", "3", "--warmup", "3"]
runpy.run_path("bench.py", run_name="__main__")
maps = open("/proc/self/maps").read()
print("LOADED_LIB", "libcti_b200" in maps, "PACKAGE", "cti_b200" in sys.modules)
"""


def test_reference_arm_prints_one_contract_line():
    proc = subprocess.run([sys.executable, "-c", _RUN_REFERENCE_ARM], cwd=ROOT,
                          capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stderr[-2000:]
    # The reference arm runs only the reference's CPU code path.
    assert "LOADED_LIB False PACKAGE False" in proc.stdout, proc.stdout
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
    # The same config object as our arm's line: the whole batch, no sample.
    sys.path.insert(0, str(ROOT))
    import bench

    synth = bench.load_synth()
    assert d["config"] == bench.workload_config(synth.CFG2, 72214)
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert "sample" in cb
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_stage_bandwidths_algorithmic_bytes():
    """The cfg2 line's `stages_hbm`: algorithmic bytes of router, dispatch
    and combine at T = 72,214, D = 256, E = 16 (38.7 / 113.3 / 112.1 MB; the
    dispatch figure includes the scan's pass over the block histograms), over
    the stage times."""
    sys.path.insert(0, str(ROOT))
    import bench

    stages = {"router": 0.030, "dispatch": 0.030, "combine": 0.025, "ffn_fused": 0.18}
    out = bench.stage_bandwidths(stages, 72214, 256, 16, 6552.6)
    assert set(out) == {"router", "dispatch", "combine"}
    assert round(out["router"]["bytes"] / 1e6, 1) == 38.7
    assert round(out["dispatch"]["bytes"] / 1e6, 1) == 113.3
    assert round(out["combine"]["bytes"] / 1e6, 1) == 112.1
    c = out["combine"]
    assert abs(c["gbs"] - c["bytes"] / 25e-6 / 1e9) < 1e-6
    assert abs(c["frac_of_hbm"] - c["gbs"] / 6552.6) < 1e-12
    assert bench.stage_bandwidths({"router": 0.03}, 1000, 128, 8, 6552.6).keys() == {"router"}
