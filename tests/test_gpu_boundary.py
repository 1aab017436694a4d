"""Pairs on and next to the two cutoffs, on the GPU through the C ABI, against the oracle.

The reference keeps a listed pair when r^2 <= rc^2 in double, each product and sum rounded on
its own (cpp/pair_jax_kokkos.cpp:84-91); LAMMPS lists a pair when r^2 < (rc + skin)^2. ljx
decides both in float first and falls back to that double test only inside a rounding band
around the cutoff, so the cases that matter are pairs whose double r^2 equals the cutoff or
lies a few ulps from it.

The crystal is simple cubic with spacing 3.25 A (an exact binary fraction), 7 x 7 x 7 cells,
model cutoff 6.5 A (two spacings) and skin 3.25 A (list cutoff 9.75 A, three spacings). Each
column of atoms along y is displaced as a whole in x and z by a seeded offset of up to 0.1 A (a
multiple of 2^-20), so the forces do not cancel by symmetry while two atoms of one column differ
in y alone. Each atom's y carries a further seeded offset of -2..2 units of 2^-47 (exact at every
coordinate of the ghost shell). Within a column:
- pairs two spacings apart with equal offsets have r^2 = 42.25 exactly, on the model cutoff;
- pairs three spacings apart with equal offsets have r^2 = 95.0625 exactly, on the list cutoff;
- the others land 13 to 52 ulps (model cutoff) or 10 to 39 ulps (list cutoff) inside or
  outside it.
"""

import numpy as np
import pytest
import torch

from cases import (F32_FORCE_REL, F32_TOTAL_REL, F64_FORCE_REL, F64_TOTAL_REL, Case,
                   canonical_edges, copy_device, device_system, host_list, write_eam_bundle)
from conftest import load_package
from test_gpu_parity import LJ_MODES, MODE_SETUP, assert_parity, oracle_step

SPACING = 3.25
CELLS = 7
UNIT = 2.0 ** -47
COLUMN_SHIFT = 104857  # 0.1 A in units of 2^-20


def boundary_case(seed=5):
    ljx = load_package()
    synth = ljx.synth
    rng = np.random.default_rng(seed)
    g = np.arange(CELLS) * SPACING
    z, y, x = np.meshgrid(g, g, g, indexing="ij")  # x fastest, as LAMMPS's spatial sort
    pos = np.stack([x.ravel(), y.ravel(), z.ravel()], axis=1)
    iz, iy, ix = np.meshgrid(*(np.arange(CELLS),) * 3, indexing="ij")
    column = (iz * CELLS + ix).ravel()
    shift = rng.integers(-COLUMN_SHIFT, COLUMN_SHIFT + 1, size=(CELLS * CELLS, 2)) * 2.0 ** -20
    pos[:, 0] += shift[column, 0]
    pos[:, 2] += shift[column, 1]
    pos[:, 1] += rng.integers(-2, 3, size=len(pos)) * UNIT
    box = np.full(3, CELLS * SPACING)
    cutoff, skin = 6.5, SPACING
    x_all, owner = synth.periodic_ghosts(pos, box, cutoff + skin)
    types = np.ones(len(pos), np.int32)
    types_all = np.concatenate([types, types[owner]]).astype(np.int32)
    text = synth.synthetic_setfl(("Cu",), nr=2000, nrho=2000)
    return Case(text, x_all, types_all, len(pos), owner, box, cutoff, skin, 1)


def squared_distances(case):
    """Double r^2 (separately rounded, as the reference's test) of every owned-ghost pair."""
    xi = case.x_all[: case.nlocal, None, :]
    d = xi - case.x_all[None, :, :]
    return (d[..., 0] * d[..., 0] + d[..., 1] * d[..., 1]) + d[..., 2] * d[..., 2]


def test_case_has_pairs_on_and_next_to_both_cutoffs():
    case = boundary_case()
    r2 = squared_distances(case)
    for cut in (case.cutoff, case.cutoff + case.skin):
        c2 = cut * cut
        assert np.count_nonzero(r2 == c2) > 0
        near = np.abs(r2 - c2)
        assert np.count_nonzero((r2 < c2) & (near < 1e-12)) > 0
        assert np.count_nonzero((r2 > c2) & (near < 1e-12)) > 0


@pytest.mark.gpu
def test_boundary_neighbor_list(oracle):
    case = boundary_case()
    for half in (False, True):
        system = device_system(case, newton=half, half=half)
        il, nn, nb, stride, maxn = host_list(system.list)
        o_il, o_nn, o_nb, o_stride, o_max = oracle.build_list(case.x_all, case.nlocal,
                                                              case.cutoff + case.skin, half=half)
        np.testing.assert_array_equal(nn[: case.nlocal], o_nn[: case.nlocal])
        for i in range(case.nlocal):
            mine = np.sort(nb[i + np.arange(nn[i]) * stride])
            theirs = np.sort(o_nb[i + np.arange(o_nn[i]) * o_stride])
            np.testing.assert_array_equal(mine, theirs)


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["rows-full", "ghost", "half-unique"])
def test_boundary_pack_edges_bit_exact(tmp_path, oracle, mode):
    ljx = load_package()
    case = boundary_case()
    newton, half = MODE_SETUP[mode]
    path = write_eam_bundle(tmp_path, case, mode=mode, precision="float64")
    system = device_system(case, newton=newton, half=half)
    engine = ljx.Engine(ljx.Bundle.load(path))
    atoms, nl = system.atoms(), system.list.struct()
    engine.pack_atoms(atoms)
    engine.pack_edges(atoms, nl, newton)
    s_ptr, r_ptr, m_ptr, cap = engine.edges()
    torch.cuda.synchronize()
    senders = copy_device(s_ptr, cap, np.int32)
    receivers = copy_device(r_ptr, cap, np.int32)
    mask = copy_device(m_ptr, cap, np.uint8).astype(bool)
    il, nn, nb, stride, maxn = host_list(system.list)
    o_s, o_r, o_m, count, overflow = oracle.pack_edges(
        case.x_all, il, nn, nb, 1, stride, case.nlocal, maxn, engine.contract["max_atoms"], cap,
        case.cutoff, nlocal=case.nlocal)
    assert overflow == 0
    assert int(mask.sum()) == count
    a = canonical_edges(senders[:count], receivers[:count])
    b = canonical_edges(o_s[:count], o_r[:count])
    np.testing.assert_array_equal(a[0], b[0])
    np.testing.assert_array_equal(a[1], b[1])
    # The kept set reaches the pairs exactly on the model cutoff and nothing past it.
    d = case.x_all[a[0]] - case.x_all[a[1]]
    kept_r2 = (d[:, 0] * d[:, 0] + d[:, 1] * d[:, 1]) + d[:, 2] * d[:, 2]
    c2 = case.cutoff * case.cutoff
    assert np.count_nonzero(kept_r2 == c2) > 0
    assert np.all(kept_r2 <= c2)


@pytest.mark.gpu
@pytest.mark.parametrize("precision", ["float64", "float32"])
@pytest.mark.parametrize("cache", [True, False])
@pytest.mark.parametrize("mode", ["rows-full", "ghost", "half-unique"])
def test_boundary_eam_step(tmp_path, oracle, mode, cache, precision):
    """One step in either precision; the kept count is the double test's in both."""
    ljx = load_package()
    case = boundary_case()
    newton, half = MODE_SETUP[mode]
    path = write_eam_bundle(tmp_path, case, mode=mode, precision=precision)
    system = device_system(case, newton=newton, half=half)
    system.list.ago = 0 if cache else -1
    pair = ljx.PairJax(device=0)
    pair.settings()
    pair.coeff(system, "*", "*", str(path))
    pair.init_style(system)
    res = pair.compute(system, eflag=True, vflag=True)
    if newton:
        system.comm.reverse_forces(system.f)
    torch.cuda.synchronize()
    ref = oracle_step(oracle, case, system, mode, precision)
    assert_parity(res, system, ref, precision, case)


@pytest.mark.gpu
@pytest.mark.parametrize("precision", ["float64", "float32"])
@pytest.mark.parametrize("mode", list(LJ_MODES))
def test_boundary_lj_step(tmp_path, oracle, mode, precision):
    """LJ does not vanish at the cutoff, so a pair on rc that the model evaluated (r^2 <= rc^2
    instead of r^2 < rc^2) would show in the forces and the energy; the kept count checks the
    pack's r^2 <= rc^2. sigma = 2.9 puts the spacing near the potential's minimum."""
    ljx = load_package()
    force_output, newton, half = LJ_MODES[mode]
    case = boundary_case()
    nall, nlocal = len(case.x_all), case.nlocal
    sigma = 2.9
    path = tmp_path / "lj.json"
    ljx.write_bundle(path, potential=ljx.lj_potential(1.0, sigma), max_atoms=nall + 32,
                     max_edges=(nall + 32) * 96, cutoff=case.cutoff, unit_style="lj",
                     precision=precision, force_output=force_output,
                     newton="on" if newton else "off")
    x = torch.as_tensor(case.x_all, device="cuda")
    system = ljx.System(x=x, type=torch.ones(nall, dtype=torch.int32, device="cuda"),
                        f=torch.zeros_like(x), nlocal=nlocal, nghost=nall - nlocal,
                        newton_pair=newton, unit_style="lj", ntypes=1)
    system.list = ljx.synth.neighbor_list(case.x_all, nlocal, case.cutoff + case.skin, half=half)
    system.comm = ljx.SelfComm(torch.as_tensor(case.owner, device="cuda"), nlocal)
    pair = ljx.PairJax()
    pair.coeff(system, "*", "*", str(path))
    pair.init_style(system)
    res = pair.compute(system)
    if newton:
        system.comm.reverse_forces(system.f)
    torch.cuda.synchronize()
    ref = oracle.lj_step(case.x_all, nlocal, case.owner, host_list(system.list), epsilon=1.0,
                         sigma=sigma, cutoff=case.cutoff, force_output=force_output,
                         newton_pair=newton, precision=precision)
    forces = system.f[:nlocal].cpu().numpy()
    fmax = float(np.max(np.abs(ref.forces)))
    frel = F64_FORCE_REL if precision == "float64" else F32_FORCE_REL
    trel = F64_TOTAL_REL if precision == "float64" else F32_TOTAL_REL
    assert float(np.max(np.abs(forces - ref.forces))) <= frel * fmax
    assert res.energy == pytest.approx(ref.energy, rel=trel)
    vscale = float(np.max(np.abs(ref.virial)))
    assert float(np.max(np.abs(np.array(res.virial) - ref.virial))) <= trel * vscale
    assert res.edge_count == ref.count
