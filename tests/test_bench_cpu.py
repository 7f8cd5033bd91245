"""bench.py's host-side contract without a GPU: the algorithmic byte count
the roofline and GB/s figures use, and the reference arm (the CPU path of the
reference, restated in oracle/cpu_path.py), which prints the JSON line the
benchmark driver reads."""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_algorithmic_bytes():
    # K*N/2 packed + (K/128)*N*2 scales + M*K*2 activations + M*N*2 outputs
    assert bench.alg_bytes(1, 4096, 4096) == 8_667_136
    assert bench.alg_bytes(1, 4096, 1024) == 2_172_928
    assert bench.alg_bytes(1, 4096, 14336) == 30_314_496
    assert bench.alg_bytes(1, 14336, 4096) == 30_314_496


def test_reference_arm_json_line():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                          "--steps", "2", "--warmup", "3"], capture_output=True, text=True, timeout=600,
                         cwd=ROOT, check=True).stdout
    lines = [l for l in out.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["metric"] == bench.METRIC and d["unit"] == "GB/s"
    assert d["higher_is_better"] is True and d["steps"] == 2 and d["warmup"] == 3
    assert d["value"] > 0 and d["cpu_baseline"]["value"] == d["value"]
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["config"]["workload"] == bench.WORKLOAD
