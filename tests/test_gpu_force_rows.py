"""ljx_force_rows: the EAM force pass in two parts, so that the F'(rho) exchange can run under it.

ljx_density marks the list rows that keep a ghost neighbor (the candidate-cache build marks rows
with a ghost candidate). ROWS_LOCAL runs the force pass over the other rows (they read no ghost
F'), ROWS_GHOST over the marked ones; in that order they must
leave the forces, energy, virial and kept count of one ljx_force call, to rounding (the sums run
in another order), in every force mode and both precisions, over the candidate cache and over
the list pass. The crystal (8 x 8 x 8 fcc cells, periodic images as ghosts) has rows of both
kinds: atoms more than rc from every face keep no ghost. The ghost part alone, out of order, and
LJ bundles are refused. The overlap itself, with the exchange on a side stream over NCCL, is
checked on two GPUs by tests/multirank_parity.py.
"""

import numpy as np
import pytest
import torch

from cases import F32_TOTAL_REL, F64_TOTAL_REL, eam_case
from conftest import load_package
from test_gpu_parity import MODE_SETUP, lj_case, run_pair

pytestmark = pytest.mark.gpu


def engine_step(pair, system, ago, split):
    """One step through the engine; the force pass whole or in its two parts."""
    ljx = load_package()
    eng, plan = pair.engine, pair.plan
    atoms, nl = system.atoms(), system.list.struct()
    nl.ago = ago
    system.f.zero_()
    eng.pack_atoms(atoms)
    eng.density(atoms, nl, system.newton_pair)
    if plan.reverse_density:
        rows, width, elem = eng.feature_rows(0)
        system.comm.reverse(rows, width, elem)
    eng.embed(atoms)
    local = None
    if plan.forward_fp:
        rows, width, elem = eng.feature_rows(1)
        system.comm.forward(rows, width, elem)
    if split:
        eng.force_rows(atoms, nl, system.newton_pair, ljx.abi.ROWS_LOCAL, 1.0)
        torch.cuda.synchronize()
        local = system.f.cpu().numpy().copy()
        eng.force_rows(atoms, nl, system.newton_pair, ljx.abi.ROWS_GHOST, 1.0)
    else:
        eng.force(atoms, nl, system.newton_pair, 1.0)
    res = eng.read_result()
    if system.newton_pair:
        system.comm.reverse_forces(system.f)
    return system.f.cpu().numpy().copy(), res, local


@pytest.mark.parametrize("cache", [True, False])
@pytest.mark.parametrize("precision", ["float64", "float32"])
@pytest.mark.parametrize("mode", list(MODE_SETUP))
def test_two_parts_equal_one_pass(tmp_path, mode, precision, cache):
    case = eam_case(elements=("Cu", "Zr"), cells=(8, 8, 8), seed=31, nr=2000, nrho=2000)
    pair, system, _ = run_pair(tmp_path, case, mode, precision)
    # With the cache: the whole pass on the list's first step (the cache and its row marks are
    # built), the two parts on the next step over that cache. Without: the list pass both times.
    f_one, one, _ = engine_step(pair, system, 0 if cache else -1, split=False)
    f_two, two, local = engine_step(pair, system, 1 if cache else -1, split=True)
    scale = float(np.max(np.abs(f_one)))
    tol = 1e-12 if precision == "float64" else 1e-5
    assert float(np.max(np.abs(f_two - f_one))) <= tol * scale
    rel = F64_TOTAL_REL if precision == "float64" else F32_TOTAL_REL
    assert two.energy == pytest.approx(one.energy, rel=rel)
    vscale = float(np.max(np.abs(one.virial)))
    assert float(np.max(np.abs(np.array(two.virial) - np.array(one.virial)))) <= rel * vscale
    assert two.edge_count == one.edge_count and two.overflow == 0
    # Both parts hold rows: the local part alone moved some forces, but not all of them.
    owned = local[: case.nlocal]
    assert np.any(owned != 0.0)
    assert float(np.max(np.abs(owned - f_two[: case.nlocal]))) > 1e-3 * scale


def test_ghost_part_needs_local_part(tmp_path):
    ljx = load_package()
    case = eam_case(cells=(5, 5, 5), seed=13, nr=500, nrho=500)
    pair, system, _ = run_pair(tmp_path, case, "rows-full", "float64")
    eng = pair.engine
    atoms, nl = system.atoms(), system.list.struct()
    eng.pack_atoms(atoms)
    eng.density(atoms, nl, False)
    eng.embed(atoms)
    with pytest.raises(ljx.abi.LjxError, match="must follow"):
        eng.force_rows(atoms, nl, False, ljx.abi.ROWS_GHOST, 1.0)
    with pytest.raises(ljx.abi.LjxError, match="row part"):
        eng.force_rows(atoms, nl, False, 7, 1.0)
    # A local part, then a new density pass: the ghost part must again wait for a local part.
    eng.force_rows(atoms, nl, False, ljx.abi.ROWS_LOCAL, 1.0)
    eng.density(atoms, nl, False)
    with pytest.raises(ljx.abi.LjxError, match="must follow"):
        eng.force_rows(atoms, nl, False, ljx.abi.ROWS_GHOST, 1.0)
    eng.read_result()


def test_lj_bundle_is_refused(tmp_path):
    ljx = load_package()
    x_all, owner, nlocal, cutoff, skin = lj_case()
    nall = len(x_all)
    path = tmp_path / "lj.json"
    ljx.write_bundle(path, potential=ljx.lj_potential(1.0, 1.0), max_atoms=nall + 32,
                     max_edges=(nall + 32) * 96, cutoff=cutoff, unit_style="lj",
                     precision="float64", force_output="atom-force", newton="on")
    x = torch.as_tensor(x_all, device="cuda")
    system = ljx.System(x=x, type=torch.ones(nall, dtype=torch.int32, device="cuda"),
                        f=torch.zeros_like(x), nlocal=nlocal, nghost=nall - nlocal,
                        newton_pair=True, unit_style="lj", ntypes=1)
    system.list = ljx.synth.neighbor_list(x_all, nlocal, cutoff + skin, half=False)
    pair = ljx.PairJax()
    pair.coeff(system, "*", "*", str(path))
    pair.init_style(system)
    atoms, nl = system.atoms(), system.list.struct()
    with pytest.raises(ljx.abi.LjxError, match="EAM bundles only"):
        pair.engine.force_rows(atoms, nl, True, ljx.abi.ROWS_LOCAL, 1.0)
