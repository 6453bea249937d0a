"""bench.py's reference arm prints one JSON line with the contract's keys,
on the small cfg0 scene (without a GPU the arm times the CPU restatement on
the host cores; on a GPU box it times the reference's own CUDA kernels)."""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_prints_contract_line():
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--config", "cfg0",
                          "--steps", "1", "--warmup", "1", "--cpu-budget", "1"],
                         capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    for key in ("impl", "metric", "value", "unit", "higher_is_better", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    sys.path.insert(0, str(ROOT))
    import bench

    assert line["impl"] == "reference" and line["metric"] == bench.METRIC and line["unit"] == "iters/s"
    assert line["value"] > 0 and line["higher_is_better"] is True
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": "iters/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_without_output():
    import os

    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--config", "cfg0",
                          "--gpus", "2", "--steps", "1", "--warmup", "1", "--cpu-budget", "1"],
                         capture_output=True, text=True, timeout=300, cwd=ROOT, env=env)
    assert out.returncode == 0, out.stderr[-2000:]
    assert out.stdout.strip() == ""
