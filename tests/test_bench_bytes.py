"""bench.py's roofline byte model, on CPU: the algorithmic bytes of the density phase, the force
pass and the whole step for the C3 workload's measured counts (2,048,000 owned atoms, 365,405
ghosts, 437,756,210 listed pairs, 176,772,660 kept edges counted both ways), as a B200 run of the
bench reported them, and the rule that names the density phase in the line's roofline."""

import importlib.util
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def bench_module():
    spec = importlib.util.spec_from_file_location("ljx_bench", ROOT / "bench.py")
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def test_c3_algorithmic_bytes():
    bench = bench_module()
    nlocal, nall = 2_048_000, 2_048_000 + 365_405
    density, force, step = bench.algorithmic_bytes(437_756_210, nlocal, nall, 176_772_660,
                                                   "float64", newton=False)
    assert force == 918_314_840
    assert step == 4_214_286_780
    assert density == 4 * 437_756_210 + 12 * nlocal + 32 * nall + 4 * 176_772_660 + 8 * nlocal
    # The density phase carries the list read: the larger bytes, so the line's roofline phase.
    assert density > 2.5 * force
    # Float32 halves the staged positions and the F' and rho words; newton on adds the ghost
    # rows' rho and force round trips to the step.
    d32, f32, s32 = bench.algorithmic_bytes(437_756_210, nlocal, nall, 176_772_660, "float32",
                                            newton=False)
    assert f32 < force and s32 < step and d32 < density
    _, _, s_on = bench.algorithmic_bytes(437_756_210, nlocal, nall, 176_772_660, "float64",
                                         newton=True)
    assert s_on - step == (nall - nlocal) * (2 * 8 + 48)
