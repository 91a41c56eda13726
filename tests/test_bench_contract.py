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


def test_headline_parallelism_labels():
    # N > 1 runs the expert-parallel decode of one token stream (strong scaling) unless
    # --replicas; both arms print the same labels from the same function
    r = subprocess.run([sys.executable, "-c",
                        "import sys; sys.path.insert(0, '.'); import bench; "
                        "print(bench.headline_parallelism(1, False), bench.headline_parallelism(8, False), "
                        "bench.headline_parallelism(8, True), bench.headline_config(48, 8)['parallelism'])"],
                       capture_output=True, text=True, timeout=120, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    out = r.stderr + r.stdout   # bench.py points fd 1 at stderr on import
    assert "('single GPU', 'weak') ('ep8', 'strong') ('replicas', 'weak') ep8" in out


def test_ep_split_from_stamps():
    # the per-layer split of the expert-parallel decode, from synthetic phase stamps:
    # layer l starts at 20,000 l ns; stamps 12 / 13 / 7 (values pushed, received, sums sent)
    # at +8,750 / +11,750 / +13,750 ns on the slowest CTA (bench.py imports in a child:
    # it points file descriptor 1 at stderr)
    r = subprocess.run([sys.executable, "-c", """
import sys, json
sys.path.insert(0, '.')
import numpy as np
import bench
L, G = 5, 4
st = np.zeros((L, G, 32), np.uint64)
for l in range(L):
    base = 20000 * l
    for c in range(G):
        st[l, c, 0] = base + 100 * c
        st[l, c, 12] = base + 8000 + 250 * c
        st[l, c, 13] = base + 11000 + 250 * c
        st[l, c, 7] = base + 13000 + 250 * c
print(json.dumps(bench.ep_split(st)))
"""], capture_output=True, text=True, timeout=120, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    import json as _json
    d = _json.loads([ln for ln in (r.stderr + r.stdout).splitlines() if ln.startswith("{")][-1])
    assert d == {"layer_us": 20.0, "partial_us": 8.75, "exchange_us": 3.0, "combine_us": 2.0}


def test_batched_kernel_choices_match_the_library_modes():
    # --batched-kernels maps onto the expert-matmul modes the library defines
    # (tg_internal.h BATCHED_*; tgx_set_batched_kernels / tgx_ep_set_kernels accept 0..3)
    import re
    r = subprocess.run([sys.executable, "-c",
                        "import sys, json; sys.path.insert(0, '.'); import bench; print(json.dumps(bench.KERNELS))"],
                       capture_output=True, text=True, timeout=120, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    kernels = json.loads([ln for ln in (r.stderr + r.stdout).splitlines() if ln.startswith("{")][-1])
    src = (ROOT / "tinygiant_b200" / "csrc" / "tg_internal.h").read_text()
    modes = dict(re.findall(r"BATCHED_(\w+) = (\d)", src))
    assert {k: int(v) for k, v in modes.items()} == {"AUTO": 0, "DP4A": 1, "MMA": 2, "MMA_FAST": 3}
    assert kernels == {"auto": 0, "dp4a": 1, "mma": 2, "mma-fast": 3}
    for f in ("tg_capi.cu", "tg_ep.cu"):
        assert "kernels >= 0 && kernels <= 3" in (ROOT / "tinygiant_b200" / "csrc" / f).read_text(), f
