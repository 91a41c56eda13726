"""bench.py's reference arm runs on the host cores alone: its JSON line keeps the
contract (the requested steps and warm-up, the reference-arm fields)."""
import json
import subprocess
import sys

from tests.conftest import ROOT


def test_reference_arm_json_line():
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "5", "--warmup", "3"],
                       capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    line = [ln for ln in r.stdout.splitlines() if ln.startswith("{")][-1]
    d = json.loads(line)
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["steps"] == 5 and d["warmup"] == 3
    assert d["value"] > 0 and d["cpu_baseline"]["value"] == d["value"] and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    # the same config dict as the GPU arm's headline line (bench.headline_config), so the
    # two arms describe one workload; the pool sample is reported beside it
    assert set(d["config"]) == {"workload", "hidden", "inter", "experts", "top_k", "layers", "weights",
                                "hidden_states", "l2", "parallelism"}
    assert d["config"]["layers"] == 48 and "layers_per_step" in d
