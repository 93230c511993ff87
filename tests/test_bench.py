"""bench.py on the CPU: the algorithmic byte models its roofline lines use,
and the JSON contract of the reference arm (`--impl reference`, the
reference's CPU implementation restated in the oracle) on the small
operating point. No GPU needed."""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(REPO))

import bench  # noqa: E402


def test_msda_byte_model_matches_the_stated_totals():
    # Decoder B4 Q300 M8 D32 L4 K4 S22223 bf16: 40.86 MB forward, 126.61 MB
    # backward (corner rows, params, outputs, gradients, one zero-fill).
    fwd, bwd = bench.algorithmic_bytes(4, 22223, 300, 8, 32, 4, 4, 2)
    assert (fwd, bwd) == (40857600, 126613504)
    # Encoder (Q = S): 3.03 GB forward, 6.05 GB backward.
    fwd, bwd = bench.algorithmic_bytes(4, 22223, 22223, 8, 32, 4, 4, 2)
    assert round(fwd / 1e6, 1) == 3026.6 and round(bwd / 1e6, 1) == 6053.2


def test_gather_byte_models():
    fwd, bwd, units = bench.gather_algorithmic_bytes("grid_sample", bench.GATHER_WORKLOADS["grid_sample"])
    assert units == 8 * 128 * 128 and fwd + bwd == 504889344
    fwd, bwd, units = bench.gather_algorithmic_bytes("roi_align", bench.GATHER_WORKLOADS["roi_align"])
    assert units == 1024 and fwd + bwd == 1871486976


def test_reference_arm_json_contract():
    out = subprocess.run([sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--config", "small",
                          "--steps", "1", "--warmup", "3"], capture_output=True, text=True, timeout=600,
                         cwd=REPO)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "queries/s" and d["higher_is_better"] is True
    assert d["metric"] == bench.METRIC and d["value"] > 0 and d["n_gpus"] == 1
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "queries/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
    assert d["config"]["workload"].startswith("small") and d["config"]["global_batch"] == 1
