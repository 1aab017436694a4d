"""GPU parity of energy-only evaluation (LAMMPS eflag_only for MC moves; the reference's
execute_energy path, cpp/pair_jax_kokkos.cpp:997-1001, 1051-1053) and the reference's refusals of
per-atom energy and virial (:995-996).

An energy-only step reports the same total energy as a full step on the same positions (within
1e-12 relative in float64) and leaves forces and the virial untouched.
"""

import numpy as np
import pytest
import torch

from cases import F64_TOTAL_REL, eam_case, host_list
from conftest import load_package
from test_gpu_parity import LJ_MODES, MODE_SETUP, lj_case, oracle_step, run_pair

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode", ["rows-full", "ghost", "half-unique"])
def test_eam_energy_only(tmp_path, oracle, mode):
    case = eam_case(elements=("Cu", "Zr"), cells=(5, 5, 5), seed=61, nr=2000, nrho=2000)
    pair, system, res_full = run_pair(tmp_path, case, mode, "float64")
    ref = oracle_step(oracle, case, system, mode, "float64")
    system.f.zero_()
    system.list.ago = 1  # the cached candidate lists of the full step are reused
    before = list(pair.virial)
    # LAMMPS's MC energy call: eflag set, eflag_only set, no virial; the tallies follow ev_init.
    res = pair.compute(system, eflag=True, vflag=False, eflag_only=True)
    torch.cuda.synchronize()
    assert res.energy == pytest.approx(ref.energy, rel=F64_TOTAL_REL)
    assert pair.eng_vdwl == pytest.approx(ref.energy, rel=F64_TOTAL_REL)
    assert not torch.any(system.f != 0).item()
    assert list(pair.virial) == before  # vflag off: the virial tally is left alone
    assert res.edge_count == ref.count


@pytest.mark.parametrize("mode", list(LJ_MODES))
def test_lj_energy_only(tmp_path, oracle, mode):
    ljx = load_package()
    force_output, newton, half = LJ_MODES[mode]
    x_all, owner, nlocal, cutoff, skin = lj_case()
    nall = len(x_all)
    path = tmp_path / "lj.json"
    ljx.write_bundle(path, potential=ljx.lj_potential(1.0, 1.0), max_atoms=nall + 32,
                     max_edges=(nall + 32) * 96, cutoff=cutoff, unit_style="lj",
                     precision="float64", force_output=force_output,
                     newton="on" if newton else "off")
    x = torch.as_tensor(x_all, device="cuda")
    system = ljx.System(x=x, type=torch.ones(nall, dtype=torch.int32, device="cuda"),
                        f=torch.zeros_like(x), nlocal=nlocal, nghost=nall - nlocal,
                        newton_pair=newton, unit_style="lj", ntypes=1)
    system.list = ljx.synth.neighbor_list(x_all, nlocal, cutoff + skin, half=half)
    system.comm = ljx.SelfComm(torch.as_tensor(owner, device="cuda"), nlocal)
    pair = ljx.PairJax(device=0)
    pair.settings()
    pair.coeff(system, "*", "*", str(path))
    pair.init_style(system)
    res = pair.compute(system, eflag_only=True)
    torch.cuda.synchronize()
    ref = oracle.lj_step(x_all, nlocal, owner, host_list(system.list), epsilon=1.0, sigma=1.0,
                         cutoff=cutoff, force_output=force_output, newton_pair=newton,
                         precision="float64")
    assert res.energy == pytest.approx(ref.energy, rel=F64_TOTAL_REL)
    assert not torch.any(system.f != 0).item()
    assert res.edge_count == ref.count


@pytest.mark.parametrize("flag,message", [
    ("eflag_atom", "pair jax/kk does not support per-atom energy output"),
    ("vflag_atom", "pair jax/kk does not support per-atom virial output"),
])
def test_per_atom_outputs_refused(tmp_path, flag, message):
    ljx = load_package()
    case = eam_case(cells=(3, 3, 3), seed=63, nr=500, nrho=500)
    pair, system, _ = run_pair(tmp_path, case, "rows-full", "float64")
    with pytest.raises(ljx.LammpsError) as err:
        pair.compute(system, **{flag: True})
    assert str(err.value) == message
