"""bench.py's reference arm (``--impl reference``) on the host: the reference's
dense-mask CPU path (oracle port) on bounded row samples, one JSON line with the
contract's keys and the arm's marker, the native arm's workload string, the
warm-up it was given, and nothing of hilberta_b200 loaded; no GPU needed."""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent

RUNNER = """
import runpy, sys
sys.argv = ["bench.py", "--impl", "reference", "--steps", "2", "--warmup", "3", "--config", "1024_t4k1",
            "--cpu-seconds", "0.5"]
runpy.run_path("bench.py", run_name="__main__")
print("NATIVE_MODULES", sorted(m for m in sys.modules if m.startswith("hilberta_b200")))
"""


def test_reference_arm_prints_contract_line():
    res = subprocess.run([sys.executable, "-c", RUNNER], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = res.stdout.strip().splitlines()
    assert lines[-1] == "NATIVE_MODULES []"
    line = json.loads(lines[-2])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["unit"] == "TFLOP/s" and line["value"] > 0
    assert line["steps"] == 2 and line["warmup"] == 3
    sys.path.insert(0, str(ROOT))
    import bench

    assert line["config"]["workload"] == bench.workload_name("1024_t4k1", 24, 4608)
    # the whole config object is the one the native arm prints for the same arguments
    active = line["config"]["active_blocks_per_phase"]
    assert line["config"] == bench.shared_config("1024_t4k1", 24, 4608, 1, "bhnd", active)
    assert line["ms_per_step"] < 5000  # measured wall time of one bounded sample, not an extrapolation
    assert line["extrapolated"]["ms_per_call"] > 0
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
