"""bench.py's reference arm runs on the CPU and prints the contract's JSON line."""
import json
import subprocess
import sys

from conftest import REPO


def test_reference_arm_json_line():
    r = subprocess.run([sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--config", "c2",
                        "--steps", "1", "--warmup", "3"], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["value"] > 0 and line["unit"] == "tokens/s"
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]


def test_launch_count_model():
    sys.path.insert(0, str(REPO))
    import bench

    k, slabs = bench.launches_per_step(bench.CONFIGS["c4"], 1, 0)
    assert slabs == 4 and k == 2 + 1 + 3 * 4
    k8, slabs8 = bench.launches_per_step(bench.CONFIGS["c4"], 8, 0)
    assert slabs8 == 2
