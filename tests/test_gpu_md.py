"""NVE trajectories through the pair style on the device (lammps-jax_b200/md.py) against the same
trajectories with the CPU oracle's forces.

- C1: LJ 12-6, fcc 8x8x4 cells (1024 atoms) at reduced density 0.8442 with +-0.05 sigma jitter,
  rc 2.5, skin 0.3, edge-force bundle, full list, newton off, float64; seeded Gaussian
  velocities at T* = 0.7; one force evaluation, then 100 NVE steps at dt = 0.005 with
  `neigh_modify every 1 delay 0 check yes` (a rebuild, with new borders, whenever an atom has
  moved more than half the skin).
- C3-shaped EAM: Cu fcc 6x6x6 cells with 0.08 A jitter, full list, newton off, float64, metal
  units, dt = 1 fs, a list rebuild every 10 steps (check no), velocities at 600 K, borders kept
  while no atom has moved half the skin (the bench's device-only rebuild).

The oracle side restates LAMMPS's Verlet + fix nve (fix_nve.cpp) in numpy with the oracle's
forces and its own neighbor lists, re-bordering at every rebuild. Position and energy tolerances
allow for the growth of rounding differences along 100 steps of a chaotic trajectory.
"""

import numpy as np
import pytest
import torch

from conftest import load_package

pytestmark = pytest.mark.gpu


def oracle_nve(oracle, forces_fn, x_owned, v, box, cut, skin, dt, mass, ftm2v, steps, every,
               check):
    """Velocity Verlet with the oracle's forces: returns per-step pair energies, the final
    positions and velocities, and the number of list builds."""
    ljx = load_package()
    nlocal = len(x_owned)
    dtfm = 0.5 * dt * ftm2v / mass[:, None]
    state = {}

    def borders(x):
        x = np.mod(x, box)
        x[x >= box] -= box[np.nonzero(x >= box)[1]]
        x_all, owner = ljx.synth.periodic_ghosts(x, box, cut)
        shift = np.round((x_all[nlocal:] - x[owner]) / box) * box
        state.update(x_all=x_all, owner=owner, shift=shift, xhold=x.copy(),
                     lst=oracle.build_list(x_all, nlocal, cut))
        state["builds"] = state.get("builds", 0) + 1

    borders(np.array(x_owned, np.float64))
    f, e = forces_fn(state["x_all"], state["owner"], state["lst"])
    energies = [e]
    v = np.array(v, np.float64)
    ago = 0
    for _ in range(steps):
        x = state["x_all"][:nlocal]
        v += dtfm * f
        x = x + dt * v
        ago += 1
        rebuild = False
        if ago % every == 0:
            rebuild = (not check) or \
                float(np.max(np.sum((x - state["xhold"]) ** 2, axis=1))) > 0.25 * skin * skin
        if rebuild:
            borders(x)
            ago = 0
        else:
            state["x_all"] = np.concatenate([x, x[state["owner"]] + state["shift"]])
        f, e = forces_fn(state["x_all"], state["owner"], state["lst"])
        v += dtfm * f
        energies.append(e)
    return np.array(energies), state["x_all"][:nlocal].copy(), v, state["builds"]


def test_c1_lj_nve_trajectory(tmp_path, oracle):
    ljx = load_package()
    from lammps_jax_b200 import md
    density, cells, cutoff, skin, dt = 0.8442, (8, 8, 4), 2.5, 0.3, 0.005
    a = (4.0 / density) ** (1.0 / 3.0)
    lattice = ljx.synth.fcc(cells, a, jitter=0.0, seed=3)
    rng = np.random.default_rng(3)
    x0 = np.mod(lattice.x + rng.uniform(-0.05, 0.05, lattice.x.shape), lattice.box)
    n = len(x0)
    assert n == 1024
    v0 = md.maxwell_velocities(np.ones(n), 0.7, "lj", seed=12345)
    path = tmp_path / "lj.json"
    ljx.write_bundle(path, potential=ljx.lj_potential(1.0, 1.0), max_atoms=4 * n,
                     max_edges=4 * n * 96, cutoff=cutoff, unit_style="lj", precision="float64",
                     force_output="edge-force", newton="off")
    pair = ljx.PairJax()
    run = md.NVE(pair, x0, np.ones(n, np.int32), lattice.box, [1.0], cutoff=cutoff, skin=skin,
                 dt=dt, units="lj", newton_pair=False, half_list=False, v=v0, every=1,
                 check=True, borders="always")
    pair.coeff(run.system, "*", "*", str(path))
    assert not pair.init_style(run.system)["half_list"]
    energies = [run.setup().energy]
    t0 = run.thermo(run.pair.last)
    assert t0.temp == pytest.approx(0.7, rel=1e-12)
    for _ in range(100):
        energies.append(run.step(eflag=True).energy)
    torch.cuda.synchronize()
    t1 = run.thermo(run.pair.last)
    x_gpu = run.system.x[:n].cpu().numpy()
    v_gpu = run.v.cpu().numpy()

    def lj_forces(x_all, owner, lst):
        r = oracle.lj_step(x_all, n, owner, lst, epsilon=1.0, sigma=1.0, cutoff=cutoff,
                           force_output="edge-force", newton_pair=False)
        return r.forces, r.energy

    e_ref, x_ref, v_ref, builds = oracle_nve(oracle, lj_forces, x0, v0, lattice.box,
                                             cutoff + skin, skin, dt, np.ones(n), 1.0, 100, 1,
                                             True)
    assert run.builds == builds > 3           # the same rebuild steps on both sides
    # Unwrapped positions: both sides wrap at the same rebuilds.
    assert float(np.max(np.abs(x_gpu - x_ref))) < 1e-9
    assert float(np.max(np.abs(v_gpu - v_ref))) < 1e-8
    np.testing.assert_allclose(energies, e_ref, rtol=1e-10)
    # NVE: the total energy stays put (truncated, unshifted LJ: pairs crossing rc jolt it).
    assert abs(t1.etotal - t0.etotal) < 2e-3 * abs(t0.etotal)


def test_c3_shaped_eam_nve_device_rebuilds(tmp_path, oracle):
    ljx = load_package()
    from lammps_jax_b200 import md
    cutoff, skin, dt = 6.5, 2.0, 0.001
    text = ljx.synth.synthetic_setfl(("Cu",), nr=2000, nrho=2000)
    atoms = ljx.synth.fcc((6, 6, 6), 3.615, jitter=0.08, seed=5)
    n = len(atoms.x)
    mass = np.array([63.546])
    v0 = md.maxwell_velocities(np.full(n, mass[0]), 600.0, "metal", seed=6)
    path = tmp_path / "cu.json"
    ljx.write_bundle(path, potential=ljx.eam_potential(text), max_atoms=6 * n,
                     max_edges=6 * n * 128, cutoff=cutoff, unit_style="metal",
                     precision="float64", force_output="atom-force", newton="off", comm=True)
    pair = ljx.PairJax()
    run = md.NVE(pair, atoms.x, atoms.types, atoms.box, mass, cutoff=cutoff, skin=skin, dt=dt,
                 units="metal", newton_pair=False, half_list=False, v=v0, every=10, check=False,
                 borders="when-needed")
    pair.coeff(run.system, "*", "*", str(path))
    pair.init_style(run.system)
    energies = [run.setup().energy]
    for _ in range(40):
        energies.append(run.step(eflag=True).energy)
    torch.cuda.synchronize()
    assert run.builds == 5 and run.border_builds == 1   # 4 device-only rebuilds
    tables = oracle.parse_setfl_text(text)

    def eam_forces(x_all, owner, lst):
        types_all = np.ones(len(x_all), np.int32)
        r = oracle.eam_step(tables, x_all, types_all, n, owner, lst, mode="rows-full")
        return r.forces, r.energy

    e_ref, x_ref, v_ref, builds = oracle_nve(oracle, eam_forces, atoms.x, v0, atoms.box,
                                             cutoff + skin, skin, dt, mass[atoms.types - 1],
                                             md.UNITS["metal"]["ftm2v"], 40, 10, False)
    assert builds == 5
    x_gpu = np.mod(run.system.x[:n].cpu().numpy(), atoms.box)
    x_ref = np.mod(x_ref, atoms.box)
    d = x_gpu - x_ref
    d -= atoms.box * np.round(d / atoms.box)
    assert float(np.max(np.abs(d))) < 1e-9
    np.testing.assert_allclose(energies, e_ref, rtol=1e-11)
