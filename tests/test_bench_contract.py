"""bench.py's reference arm on the CPU: the JSON line the benchmark driver
reads (one line, the GPU arm's metric, unit and config, `impl: reference`, a
`cpu_baseline` describing the run and an `e2e` object with no host copies),
on a 32-token sample so that it finishes in well under a minute. The GPU arm
prints the same keys; it needs a B200 and is exercised by the GPU runs.
"""
import json
import subprocess
import sys

from conftest import ROOT

sys.path.insert(0, str(ROOT))


def test_reference_arm_json_line():
    import bench
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                        "--steps", "1", "--warmup", "1", "--cpu-tokens", "32"],
                       capture_output=True, text=True, timeout=600, cwd=str(ROOT))
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == bench.METRIC and d["unit"] == bench.UNIT
    assert d["value"] > 0 and d["ms_per_step"] > 0 and d["higher_is_better"] is True
    assert d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] == 1
    for key in ("scaling", "vs_baseline", "dtype", "data"):
        assert key in d, key
    assert d["config"]["workload"] == "moe_layer_fwd"
    assert d["config"]["tokens_per_gpu"] == 16384 and d["config"]["experts"] == 256
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["unit"] == bench.UNIT
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and "32 tokens" in cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == bench.UNIT
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
