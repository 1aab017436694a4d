"""Per-atom energy and virial (eflag_atom / vflag_atom) through the pair style, on the GPU.

The reference refuses both flags (cpp/pair_jax_kokkos.cpp:995-996); with LAMMPS's per-atom
arrays registered (ljx_pair_set_atom_tallies) the pair style fills them as LAMMPS's ev_tally
splits a pair term: the embedding energy F(rho_i) to atom i, half of each pair's energy and half
of its virial -rij (x) F to each atom (a full-list row takes its own half). Checked against a
per-atom restatement built from the CPU oracle's own edge arrays (its packed edges, densities,
F' and per-edge forces, with the pair spline evaluated by the oracle's spline routine), row by
row over owned and ghost rows, and through the size-independent sums: the per-atom energies and
virials add up to the step's totals. Without registered arrays the refusal stands
(tests/test_gpu_energy_only.py).
"""

import numpy as np
import pytest
import torch

from cases import F64_FORCE_REL, F64_TOTAL_REL, device_system, eam_case, host_list, write_eam_bundle
from conftest import load_package
from test_gpu_parity import LJ_MODES, MODE_SETUP, lj_case

pytestmark = pytest.mark.gpu

ORACLE_MODE = {"ghost": 0, "rows-full": 1, "half-unique": 2}


def eam_tally_reference(oracle, case, lst, mode):
    """(eatom, vatom, energy, virial) over all rows from the oracle's edges and model output."""
    tables = oracle.parse_setfl_text(case.text)
    x, types, nlocal = case.x_all, case.types_all, case.nlocal
    nall = len(x)
    ilist, numneigh, neighbors, stride, maxneigh = lst
    senders, receivers, mask, count, _ = oracle.pack_edges(
        x, ilist, numneigh, neighbors, 1, stride, nlocal, maxneigh, nall,
        int(numneigh[:nlocal].sum()) + 1, tables["cutoff"], nlocal=nlocal)
    species = (types - 1).astype(np.int32)
    out = oracle.eam_model(tables, x, species, nlocal, nall - nlocal, senders, receivers, mask,
                           mode, owner=case.owner)
    s, r = senders[:count], receivers[:count]
    d = x[r] - x[s]
    rr = np.sqrt((d * d).sum(1))
    keep = rr * rr < tables["cutoff"] ** 2
    s, r, d, rr = s[keep], r[keep], d[keep], rr[keep]
    fe = out.edge_force[:count][keep]
    # Pair energy phi = (r phi)(r) / r per edge, by the oracle's spline routine.
    phi = np.empty(len(s))
    rows = tables["pair_index"][species[s], species[r]]
    for row in np.unique(rows):
        sel = rows == row
        phi[sel] = oracle.spline_eval(tables["pair"][row], rr[sel], tables["dr"]) / rr[sel]
    half = mode == "half-unique"
    eatom = np.zeros(nall)
    for el in range(len(tables["elements"])):
        sel = np.nonzero(species[:nlocal] == el)[0]
        eatom[sel] += oracle.spline_eval(tables["embedding"][el], out.rho[sel], tables["drho"],
                                         extrapolate=True)
    np.add.at(eatom, s, 0.5 * phi)
    if half:
        np.add.at(eatom, r, 0.5 * phi)
    c = np.stack([d[:, 0] * fe[:, 0], d[:, 1] * fe[:, 1], d[:, 2] * fe[:, 2],
                  d[:, 0] * fe[:, 1], d[:, 0] * fe[:, 2], d[:, 1] * fe[:, 2]], axis=1)
    vatom = np.zeros((nall, 6))
    np.add.at(vatom, s, -0.5 * c)
    if mode != "rows-full":
        np.add.at(vatom, r, -0.5 * c)
    return eatom, vatom, out.energy, out.virial


@pytest.mark.parametrize("mode", list(MODE_SETUP))
def test_eam_per_atom_energy_and_virial(tmp_path, oracle, mode):
    ljx = load_package()
    newton, half = MODE_SETUP[mode]
    case = eam_case(elements=("Cu", "Zr"), cells=(4, 4, 4), seed=11, nr=2000, nrho=2000)
    path = write_eam_bundle(tmp_path, case, mode=mode, precision="float64")
    system = device_system(case, newton=newton, half=half)
    pair = ljx.PairJax(device=0)
    pair.coeff(system, "*", "*", str(path))
    pair.init_style(system)
    nall = len(case.x_all)
    eatom = torch.full((nall,), 7.0, dtype=torch.float64, device="cuda")  # ev_setup zeroes
    vatom = torch.full((nall, 6), 7.0, dtype=torch.float64, device="cuda")
    pair.set_atom_tallies(eatom, vatom)
    res = pair.compute(system, eflag=True, vflag=True, eflag_atom=True, vflag_atom=True)
    torch.cuda.synchronize()
    e_ref, v_ref, energy_ref, virial_ref = eam_tally_reference(oracle, case,
                                                               host_list(system.list), mode)
    got_e, got_v = eatom.cpu().numpy(), vatom.cpu().numpy()
    rows = nall if newton else case.nlocal   # ev_setup's rows; ghost rows stay 7 with newton off
    if not newton:
        assert np.all(got_e[case.nlocal:] == 7.0) and np.all(got_v[case.nlocal:] == 7.0)
    escale = float(np.max(np.abs(e_ref)))
    vscale = float(np.max(np.abs(v_ref)))
    assert float(np.max(np.abs(got_e[:rows] - e_ref[:rows]))) <= F64_FORCE_REL * escale
    assert float(np.max(np.abs(got_v[:rows] - v_ref[:rows]))) <= F64_FORCE_REL * vscale
    # The per-atom tallies add up to the step's totals.
    assert got_e[:rows].sum() == pytest.approx(res.energy, rel=F64_TOTAL_REL)
    vtot = float(np.max(np.abs(np.array(res.virial))))
    assert np.max(np.abs(got_v[:rows].sum(0) - np.array(res.virial))) <= 1e-11 * vtot
    assert res.energy == pytest.approx(energy_ref, rel=F64_TOTAL_REL)


@pytest.mark.parametrize("mode", list(LJ_MODES))
def test_lj_per_atom_energy_and_virial(tmp_path, oracle, mode):
    """LJ: per-atom energy against the edge sum of the 12-6 energy (0.5 per directed edge of a
    full list; half of each pair to each atom of a half list), and both sums against the totals,
    with a pair_coeff scale."""
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
    pair = ljx.PairJax()
    scale = 0.75
    pair.coeff(system, "*", "*", str(path), str(scale))
    pair.init_style(system)
    eatom = torch.zeros(nall, dtype=torch.float64, device="cuda")
    vatom = torch.zeros(nall, 6, dtype=torch.float64, device="cuda")
    pair.set_atom_tallies(eatom, vatom)
    res = pair.compute(system, eflag=True, vflag=True, eflag_atom=True, vflag_atom=True)
    torch.cuda.synchronize()
    ilist, numneigh, neighbors, stride, maxneigh = host_list(system.list)
    s, r, m, count, _ = oracle.pack_edges(x_all, ilist, numneigh, neighbors, 1, stride, nlocal,
                                          maxneigh, nall, int(numneigh[:nlocal].sum()) + 1,
                                          cutoff, nlocal=nlocal)
    s, r = s[:count], r[:count]
    d = x_all[r] - x_all[s]
    r2 = (d * d).sum(1)
    keep = (r2 > 1e-12) & (r2 < cutoff * cutoff)
    s, r, r2 = s[keep], r[keep], r2[keep]
    a6 = (1.0 / r2) ** 3
    u = 4.0 * (a6 * a6 - a6)
    # Whole pair energy per edge of a half list, half per directed edge of a full list.
    ew = 1.0 if half else 0.5
    e_ref = np.zeros(nall)
    if half:
        np.add.at(e_ref, s, 0.5 * ew * u)
        np.add.at(e_ref, r, 0.5 * ew * u)
    else:
        np.add.at(e_ref, s, ew * u)
    e_ref *= scale
    rows = nall if newton else nlocal
    got_e, got_v = eatom.cpu().numpy(), vatom.cpu().numpy()
    assert float(np.max(np.abs(got_e - e_ref))) <= F64_FORCE_REL * float(np.max(np.abs(e_ref)))
    assert got_e[:rows].sum() == pytest.approx(res.energy, rel=F64_TOTAL_REL)
    vtot = float(np.max(np.abs(np.array(res.virial))))
    assert np.max(np.abs(got_v[:rows].sum(0) - np.array(res.virial))) <= 1e-11 * vtot


def test_per_atom_flags_refused_without_arrays(tmp_path):
    """The reference's refusal stays in place until LAMMPS's arrays are registered, and comes
    back when they are withdrawn."""
    ljx = load_package()
    case = eam_case(cells=(3, 3, 3), nr=800, nrho=800)
    path = write_eam_bundle(tmp_path, case, mode="rows-full", precision="float64")
    system = device_system(case, newton=False, half=False)
    pair = ljx.PairJax(device=0)
    pair.coeff(system, "*", "*", str(path))
    pair.init_style(system)
    with pytest.raises(ljx.LammpsError, match="does not support per-atom energy output"):
        pair.compute(system, eflag_atom=True)
    eatom = torch.zeros(len(case.x_all), dtype=torch.float64, device="cuda")
    pair.set_atom_tallies(eatom, None)
    pair.compute(system, eflag=True, eflag_atom=True)
    with pytest.raises(ljx.LammpsError, match="does not support per-atom virial output"):
        pair.compute(system, vflag_atom=True)
    pair.set_atom_tallies(None, None)
    with pytest.raises(ljx.LammpsError, match="does not support per-atom energy output"):
        pair.compute(system, eflag_atom=True)
