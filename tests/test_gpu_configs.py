"""GPU parity at the benchmark configurations' own sizes.

C1 (LJ fcc 8x8x4, 1024 atoms) already runs at full size in test_gpu_parity.test_lj_matches_oracle.
Here:
- C2: synthetic binary Cu-Zr EAM, 8192 atoms of seeded random packing at 0.058 atoms/A^3 with a
  2.0 A hard core, 64/36 species, half list with newton on (the half-unique communicating export),
  128 edges per atom, float64.
- C3: Cu fcc 80^3 cells = 2,048,000 atoms with 0.08 A Gaussian jitter, full list, newton off,
  float64, rebuild state as the bench runs it (candidate cache built this step).
Both are checked against the CPU oracle on the same inputs and list. C3 also checks a
size-independent property: the forces of a periodic system sum to zero.

Tolerances: float64 forces within 1e-10 of the max-abs force, energy and virial 1e-12 relative.
"""

import numpy as np
import pytest
import torch

from cases import F64_FORCE_REL, F64_TOTAL_REL, Case, host_list, write_eam_bundle
from conftest import load_package
from test_gpu_parity import assert_parity, oracle_step

pytestmark = pytest.mark.gpu


def run_case(tmp_path, case, mode, newton, half):
    ljx = load_package()
    path = write_eam_bundle(tmp_path, case, mode=mode, precision="float64")
    x = torch.as_tensor(case.x_all, device="cuda")
    system = ljx.System(x=x, type=torch.as_tensor(case.types_all, device="cuda"),
                        f=torch.zeros_like(x), nlocal=case.nlocal,
                        nghost=len(case.x_all) - case.nlocal, newton_pair=newton,
                        unit_style="metal", ntypes=case.ntypes)
    system.list = ljx.synth.neighbor_list(case.x_all, case.nlocal, case.cutoff + case.skin,
                                          half=half)
    system.comm = ljx.SelfComm(torch.as_tensor(case.owner, device="cuda"), case.nlocal)
    pair = ljx.PairJax(device=0)
    pair.settings()
    pair.coeff(system, "*", "*", str(path))
    assert bool(pair.init_style(system)["half_list"]) == half
    res = pair.compute(system, eflag=True, vflag=True)
    if newton:
        system.comm.reverse_forces(system.f)
    torch.cuda.synchronize()
    return system, res


def test_c2_binary_amorphous(tmp_path, oracle):
    ljx = load_package()
    synth = ljx.synth
    atoms = synth.random_packing(8192, 0.058, 2.0, seed=2)
    types = synth.substitutional(len(atoms.x), (0.64, 0.36), seed=3)
    cutoff, skin = 6.5, 2.0
    x_all, owner = synth.periodic_ghosts(atoms.x, atoms.box, cutoff + skin)
    types_all = np.concatenate([types, types[owner]]).astype(np.int32)
    case = Case(synth.synthetic_setfl(("Cu", "Zr")), x_all, types_all, len(atoms.x), owner,
                atoms.box, cutoff, skin, 2)
    system, res = run_case(tmp_path, case, "half-unique", newton=True, half=True)
    ref = oracle_step(oracle, case, system, "half-unique", "float64")
    assert_parity(res, system, ref, "float64", case)


def test_c3_full_size(tmp_path, oracle):
    ljx = load_package()
    synth = ljx.synth
    atoms = synth.fcc((80, 80, 80), 3.615, jitter=0.08, seed=2024)
    cutoff, skin = 6.5, 2.0
    x_all, owner = synth.periodic_ghosts(atoms.x, atoms.box, cutoff + skin)
    case = Case(synth.synthetic_setfl(("Cu",)), x_all, np.ones(len(x_all), np.int32),
                len(atoms.x), owner, atoms.box, cutoff, skin, 1)
    assert case.nlocal == 2_048_000
    system, res = run_case(tmp_path, case, "rows-full", newton=False, half=False)
    forces = system.f[: case.nlocal]
    fmax = float(forces.abs().max().item())
    # Momentum: pair forces cancel, so the sum is rounding only (2 M terms of size <= fmax).
    total = forces.sum(dim=0).abs().max().item()
    assert total <= 1e-10 * fmax * case.nlocal ** 0.5
    ref = oracle_step(oracle, case, system, "rows-full", "float64")
    ferr = float(np.max(np.abs(forces.cpu().numpy() - ref.forces)))
    assert ferr <= F64_FORCE_REL * float(np.max(np.abs(ref.forces)))
    assert res.energy == pytest.approx(ref.energy, rel=F64_TOTAL_REL)
    assert res.edge_count == ref.count
