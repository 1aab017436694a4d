"""ljx_force_only: the steps where LAMMPS asks for neither energy nor virial (all but thermo
steps; the reference runs its force-only program there, cpp/pair_jax_kokkos.cpp:1055-1057).

The EAM force pass then sums no energy and no virial. Its forces must equal those of the full
pass to rounding (the same per-pair terms; without the sums the compiler may fuse a multiply and
an add where the full pass keeps both, so the last bit can differ), in every force mode and both
precisions, through the engine and through the pair style with eflag = vflag = 0; the step's
result reports energy and virial as zero and the edge count as usual. A full step after a
force-only one reports its totals again.
"""

import numpy as np
import pytest
import torch

from cases import F32_TOTAL_REL, F64_TOTAL_REL, eam_case
from test_gpu_force_to_host import engine_step
from test_gpu_parity import MODE_SETUP, run_pair

pytestmark = pytest.mark.gpu


def engine_forces(pair, system, ev):
    eng, plan = pair.engine, pair.plan
    atoms, nl = system.atoms(), system.list.struct()
    system.f.zero_()
    eng.pack_atoms(atoms)
    eng.density(atoms, nl, system.newton_pair)
    if plan.reverse_density:
        rows, width, elem = eng.feature_rows(0)
        system.comm.reverse(rows, width, elem)
    eng.embed(atoms)
    if plan.forward_fp:
        rows, width, elem = eng.feature_rows(1)
        system.comm.forward(rows, width, elem)
    if ev:
        eng.force(atoms, nl, system.newton_pair, 1.0)
    else:
        eng.force_only(atoms, nl, system.newton_pair, 1.0)
    res = eng.read_result()
    if system.newton_pair:
        system.comm.reverse_forces(system.f)
    return system.f.cpu().numpy().copy(), res


@pytest.mark.parametrize("precision", ["float64", "float32"])
@pytest.mark.parametrize("mode", list(MODE_SETUP))
def test_force_only_equals_full_forces(tmp_path, mode, precision):
    case = eam_case(elements=("Cu", "Zr"), cells=(5, 5, 5), seed=29, nr=2000, nrho=2000)
    pair, system, _ = run_pair(tmp_path, case, mode, precision)
    f_full, full = engine_forces(pair, system, ev=True)
    f_only, only = engine_forces(pair, system, ev=False)
    scale = float(np.max(np.abs(f_full)))
    tol = 1e-13 if precision == "float64" else 1e-5
    assert float(np.max(np.abs(f_only - f_full))) <= tol * scale
    assert only.energy == 0.0 and list(only.virial) == [0.0] * 6
    assert only.edge_count == full.edge_count and only.overflow == 0
    assert full.energy != 0.0
    # The totals come back with the next full step (half lists scatter rho with atomics, so the
    # step repeats to the precision's tolerance, not bit for bit).
    _, again = engine_forces(pair, system, ev=True)
    rel = F64_TOTAL_REL if precision == "float64" else F32_TOTAL_REL
    assert again.energy == pytest.approx(full.energy, rel=rel)


def test_pair_style_runs_force_only_without_ev_flags(tmp_path):
    case = eam_case(cells=(5, 5, 5), seed=13, nr=2000, nrho=2000)
    pair, system, full = run_pair(tmp_path, case, "rows-full", "float64")
    f_full = system.f[: case.nlocal].cpu().numpy().copy()
    system.f.zero_()
    res = pair.compute(system, eflag=False, vflag=False)
    torch.cuda.synchronize()
    f_only = system.f[: case.nlocal].cpu().numpy()
    assert float(np.max(np.abs(f_only - f_full))) <= 1e-13 * float(np.max(np.abs(f_full)))
    assert res.energy == 0.0 and res.edge_count == full.edge_count
    # The next step that asks for the energy reports it again.
    system.f.zero_()
    res = pair.compute(system, eflag=True, vflag=False)
    assert res.energy == pytest.approx(full.energy, rel=1e-12)


def test_streamed_and_force_only_steps_interleave(tmp_path):
    """A force-only step between streamed full steps leaves the streamed rows and totals
    intact."""
    case = eam_case(cells=(4, 4, 4), seed=3, nr=800, nrho=800)
    pair, system, _ = run_pair(tmp_path, case, "rows-full", "float64")
    f_host = torch.empty((case.nlocal, 3), dtype=torch.float64).pin_memory()
    first = engine_step(pair, system, f_host, 4)
    engine_forces(pair, system, ev=False)
    second = engine_step(pair, system, f_host, 4)
    assert second.energy == first.energy
    np.testing.assert_array_equal(f_host.numpy(), system.f[: case.nlocal].cpu().numpy())
