"""bench.py's reference arm runs on the CPU and prints the contract's JSON line."""
import json
import os
import subprocess
import sys

from conftest import REPO


def test_reference_arm_json_line():
    # torchrun exports OMP_NUM_THREADS=1 to every rank; the arm must still
    # give the reference's BLAS every host core.
    env = dict(os.environ, OMP_NUM_THREADS="1")
    r = subprocess.run([sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--config", "c2",
                        "--steps", "1", "--warmup", "3"], capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["value"] > 0 and line["unit"] == "tokens/s"
    expected_kind = "reference" if (REPO / "baseline" / "_ref" / "NimbleML").is_dir() else "port"
    assert line["cpu_baseline"]["kind"] == expected_kind
    assert line["cpu_baseline"]["cores"] == len(os.sched_getaffinity(0))
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]


def test_launch_count_model():
    sys.path.insert(0, str(REPO))
    import bench

    k, slabs = bench.launches_per_step(bench.CONFIGS["c4"], 1, 0)
    assert slabs == 4 and k == 2 + 1 + 3 * 4
    # A shard of a split vocabulary follows the 2 GiB budget alone: one slab
    # at 4 and 8 ranks (N x V/P x 2 bytes <= 2 GiB), two at 2 ranks.
    assert bench.launches_per_step(bench.CONFIGS["c4"], 8, 0)[1] == 1
    assert bench.launches_per_step(bench.CONFIGS["c4"], 4, 0)[1] == 1
    assert bench.launches_per_step(bench.CONFIGS["c4"], 2, 0)[1] == 2
    # fp32: two TF32 rounding passes per step (once per forward + backward pair).
    k2, slabs2 = bench.launches_per_step(bench.CONFIGS["c2"], 1, 0)
    assert k2 == 2 + 1 + 3 * slabs2 + 2
