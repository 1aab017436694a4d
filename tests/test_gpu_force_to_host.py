"""ljx_force_to_host: the force pass in row pieces with each piece's owned force rows copied to
pinned host memory as soon as it finishes (the device-to-host copy of LAMMPS's forces overlapped
with the pass).

- The host rows equal the device rows of the same call bit for bit. With every pair evaluated
  from both rows (LJX_OWNED_HALF=0) they also equal the rows of a one-launch ljx_force bit for
  bit (every row's force is one warp's sum either way); with owned pairs held once (the
  default) the neighbor shares arrive by atomics in another order, so to rounding. The step
  totals (energy, virial) are block sums in another grouping, so they agree to the float64
  totals tolerance (1e-12).
- Every piece count from 1 to 16, float64 and float32, EAM full list newton off and LJ
  edge-force bundles; the pieces split rows unevenly and some are empty.
- Modes whose rows scatter into other rows (newton on, half lists) are refused before launch.
- A list whose row r is not atom r: the result read after the step fails.
"""

import numpy as np
import pytest
import torch

from cases import F32_TOTAL_REL, F64_FORCE_REL, F64_TOTAL_REL, device_system, eam_case, host_list
from conftest import load_package
from test_gpu_parity import lj_case, oracle_step, run_pair

pytestmark = pytest.mark.gpu


def engine_step(pair, system, f_host=None, pieces=4):
    """One pair-style step on the pair's engine; the force pass streamed when f_host is given."""
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
    if f_host is None:
        eng.force(atoms, nl, system.newton_pair, 1.0)
    else:
        eng.force_to_host(atoms, nl, system.newton_pair, f_host, 1.0, pieces)
    return eng.read_result()


def pinned_rows(n):
    return torch.full((n, 3), float("nan"), dtype=torch.float64).pin_memory()


@pytest.mark.parametrize("owned_half", ["0", "1"])
@pytest.mark.parametrize("precision", ["float64", "float32"])
def test_eam_rows_stream_to_host(tmp_path, oracle, monkeypatch, precision, owned_half):
    monkeypatch.setenv("LJX_OWNED_HALF", owned_half)
    case = eam_case(elements=("Cu", "Zr"), cells=(5, 5, 5), seed=23, nr=2000, nrho=2000)
    pair, system, res = run_pair(tmp_path, case, "rows-full", precision)
    one = engine_step(pair, system)
    f_one = system.f[: case.nlocal].cpu().numpy().copy()
    ref = oracle_step(oracle, case, system, "rows-full", precision)
    fmax = float(np.max(np.abs(ref.forces)))
    assert float(np.max(np.abs(f_one - ref.forces))) <= (
        F64_FORCE_REL if precision == "float64" else 1e-5) * fmax
    for pieces in (1, 2, 3, 7, 16):
        f_host = pinned_rows(case.nlocal)
        got = engine_step(pair, system, f_host, pieces)
        np.testing.assert_array_equal(f_host.numpy(), system.f[: case.nlocal].cpu().numpy())
        if owned_half == "0":
            np.testing.assert_array_equal(f_host.numpy(), f_one)
        else:
            tol = 1e-13 if precision == "float64" else 1e-6
            assert float(np.max(np.abs(f_host.numpy() - f_one))) <= tol * fmax
        assert got.edge_count == one.edge_count and got.overflow == 0
        # Float densities summed by atomics in another order move the float totals more.
        trel = F64_TOTAL_REL if precision == "float64" or owned_half == "0" else F32_TOTAL_REL
        assert got.energy == pytest.approx(one.energy, rel=trel)
        vs = float(np.max(np.abs(one.virial)))
        assert float(np.max(np.abs(np.array(got.virial) - np.array(one.virial)))) <= trel * vs


def test_lj_edge_rows_stream_to_host(tmp_path):
    ljx = load_package()
    x_all, owner, nlocal, cutoff, skin = lj_case(cells=(8, 8, 8))
    nall = len(x_all)
    path = tmp_path / "lj.json"
    ljx.write_bundle(path, potential=ljx.lj_potential(1.0, 1.0), max_atoms=nall + 32,
                     max_edges=(nall + 32) * 96, cutoff=cutoff, unit_style="lj",
                     precision="float64", force_output="edge-force", newton="off")
    x = torch.as_tensor(x_all, device="cuda")
    system = ljx.System(x=x, type=torch.ones(nall, dtype=torch.int32, device="cuda"),
                        f=torch.zeros_like(x), nlocal=nlocal, nghost=nall - nlocal,
                        newton_pair=False, unit_style="lj", ntypes=1)
    system.list = ljx.synth.neighbor_list(x_all, nlocal, cutoff + skin, half=False)
    system.comm = ljx.SelfComm(torch.as_tensor(owner, device="cuda"), nlocal)
    pair = ljx.PairJax()
    pair.coeff(system, "*", "*", str(path))
    pair.init_style(system)
    pair.compute(system)
    one = engine_step(pair, system)
    f_one = system.f[:nlocal].cpu().numpy().copy()
    for pieces in (1, 5, 16):
        f_host = pinned_rows(nlocal)
        got = engine_step(pair, system, f_host, pieces)
        np.testing.assert_array_equal(f_host.numpy(), f_one)
        assert got.edge_count == one.edge_count
        assert got.energy == pytest.approx(one.energy, rel=F64_TOTAL_REL)


def test_scattering_modes_are_refused(tmp_path):
    ljx = load_package()
    case = eam_case(cells=(4, 4, 4), seed=5, nr=800, nrho=800)
    for mode in ("ghost", "half-unique"):
        pair, system, _ = run_pair(tmp_path, case, mode, "float64")
        with pytest.raises(ljx.LjxError, match="each list row holds its atom's whole force"):
            engine_step(pair, system, pinned_rows(case.nlocal))
        # Nothing was launched: the next plain step still works.
        engine_step(pair, system)


def test_rows_out_of_atom_order_fail_at_the_result(tmp_path):
    ljx = load_package()
    case = eam_case(cells=(4, 4, 4), seed=9, nr=800, nrho=800)
    pair, system, _ = run_pair(tmp_path, case, "rows-full", "float64")
    lst = system.list
    il, nn, nb, stride, maxn = host_list(lst)
    assert np.array_equal(il[: lst.inum], np.arange(lst.inum))
    swapped = lst.ilist.clone()
    swapped[[0, 1]] = swapped[[1, 0]]
    lst.ilist = swapped
    lst.ago = 0
    with pytest.raises(ljx.LjxError, match="not their own atom"):
        engine_step(pair, system, pinned_rows(case.nlocal))
    # The flag is per step: with the rows back in order the streamed step is accepted again.
    lst.ilist = torch.as_tensor(il, device="cuda")
    engine_step(pair, system, pinned_rows(case.nlocal))
