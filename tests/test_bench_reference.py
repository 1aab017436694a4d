"""bench.py's reference arm runs without a GPU and prints the driver's JSON line for the chosen
configuration, at that configuration's precision (C3: float64; C5: float32). The arm runs the
bench's own workload; here it is shrunk to 12^3 cells so the check takes seconds."""

import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.parametrize("config,dtype,scaling", [("c5", "f32", "weak"), ("c3", "f64", "weak")])
def test_reference_arm_line(config, dtype, scaling):
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                          "--config", config, "--steps", "1", "--warmup", "0", "--cells", "12"],
                         capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["config"]["name"] == config
    assert line["dtype"] == dtype and line["scaling"] == scaling
    assert line["unit"] == "atom-steps/s" and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]
    assert line["steps"] == 1 and line["warmup"] == 0
    assert line["config"]["total_atoms"] == 4 * 12 ** 3
