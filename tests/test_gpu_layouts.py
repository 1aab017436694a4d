"""GPU parity for the remaining contract layouts the loader accepts (cpp/lammps_jax_model.cpp:
212-315): neighbor-matrix EAM bundles (CopyNeighborMatrixFunctor, cpp/pair_jax_kokkos.cpp:121-155;
capacity check :1069-1075), max_owned (:1040-1046) and EAM edge-force bundles
(make_setfl_edge_force, python/lammps_jax/eam.py:383-398, added by AddEdgeForcesFunctor,
cpp/pair_jax_kokkos.cpp:195-225).

The physics of each layout is the same step as the sparse-edge atom-force bundles, so each case
is checked against the oracle mode with that force distribution. Tolerances: float64 forces within
1e-10 of max |F|, energy and virial within 1e-12 relative.
"""

import numpy as np
import pytest
import torch

from cases import device_system, eam_case
from conftest import load_package
from test_gpu_parity import assert_parity, oracle_step

pytestmark = pytest.mark.gpu


def run_bundle(tmp_path, case, *, newton_pair, half, name, **bundle_kw):
    ljx = load_package()
    path = tmp_path / f"{name}.json"
    nall = len(case.x_all)
    kw = dict(potential=ljx.eam_potential(case.text), max_atoms=nall + 64, cutoff=case.cutoff,
              unit_style="metal", precision="float64", n_species=case.ntypes)
    kw.update(bundle_kw)
    ljx.write_bundle(path, **kw)
    system = device_system(case, newton=newton_pair, half=half)
    pair = ljx.PairJax(device=0)
    pair.settings()
    pair.coeff(system, "*", "*", str(path))
    plan = pair.init_style(system)
    assert bool(plan["half_list"]) == half
    return ljx, pair, system


def compute(pair, system):
    res = pair.compute(system, eflag=True, vflag=True)
    if system.newton_pair:
        system.comm.reverse_forces(system.f)
    torch.cuda.synchronize()
    return res


@pytest.mark.parametrize("newton,mode", [(False, "rows-full"), (True, "ghost")])
def test_neighbor_matrix_eam(tmp_path, oracle, newton, mode):
    case = eam_case(elements=("Cu", "Zr"), cells=(5, 5, 5), seed=51, nr=2000, nrho=2000)
    ljx, pair, system = run_bundle(tmp_path, case, newton_pair=newton, half=False, name=f"m{mode}",
                                   max_neighbors=320, newton="on" if newton else "off",
                                   comm=not newton)
    assert pair.bundle.contract["input_layout"] == ljx.abi.LAYOUT_NEIGHBOR_MATRIX
    res = compute(pair, system)
    ref = oracle_step(oracle, case, system, mode, "float64")
    assert_parity(res, system, ref, "float64", case)
    widest = int(system.list.numneigh[: case.nlocal].max().item())
    assert res.widest_row == widest


def test_neighbor_matrix_capacity_message(tmp_path):
    case = eam_case(cells=(4, 4, 4), seed=53, nr=500, nrho=500)
    ljx, pair, system = run_bundle(tmp_path, case, newton_pair=False, half=False, name="mcap",
                                   max_neighbors=100, newton="off", comm=True)
    widest = int(system.list.numneigh[: case.nlocal].max().item())
    assert widest > 100
    with pytest.raises(ljx.LammpsError) as err:
        compute(pair, system)
    assert str(err.value) == (f"LAMMPS-JAX neighbor capacity exceeded: global max {widest} "
                              "neighbors per atom, capacity 100")


def test_max_owned_rows(tmp_path, oracle):
    case = eam_case(cells=(4, 4, 4), seed=55, nr=500, nrho=500)
    ljx, pair, system = run_bundle(tmp_path, case, newton_pair=False, half=False, name="owned",
                                   max_neighbors=320, newton="off", comm=True,
                                   max_owned=case.nlocal + 8)
    res = compute(pair, system)
    assert_parity(res, system, oracle_step(oracle, case, system, "rows-full", "float64"),
                  "float64", case)
    ljx, pair, system = run_bundle(tmp_path, case, newton_pair=False, half=False, name="owned_small",
                                   max_neighbors=320, newton="off", comm=True,
                                   max_owned=case.nlocal - 8)
    with pytest.raises(ljx.LammpsError) as err:
        compute(pair, system)
    assert "owned-row capacity exceeded" in str(err.value)


# Newton off: a plain bundle (the loader refuses communicating edge-force bundles without newton,
# cpp/lammps_jax_model.cpp); newton on: the communicating half-edge export.
@pytest.mark.parametrize("newton,half,mode", [(False, False, "rows-full"),
                                              (True, True, "half-unique")])
def test_eam_edge_force_bundles(tmp_path, oracle, newton, half, mode):
    case = eam_case(elements=("Cu", "Zr"), cells=(5, 5, 5), seed=57, nr=2000, nrho=2000)
    nall = len(case.x_all)
    ljx, pair, system = run_bundle(tmp_path, case, newton_pair=newton, half=half, name=f"e{mode}",
                                   max_edges=(nall + 64) * 128, force_output="edge-force",
                                   newton="on" if newton else "off", comm=newton, half_edges=half)
    assert pair.bundle.contract["force_layout"] == ljx.abi.FORCE_EDGE
    res = compute(pair, system)
    ref = oracle_step(oracle, case, system, mode, "float64")
    assert_parity(res, system, ref, "float64", case)
    if not newton:
        # AddEdgeForcesFunctor with newton off adds to senders only: ghost rows stay untouched.
        assert not np.any(system.f[case.nlocal:].cpu().numpy())
