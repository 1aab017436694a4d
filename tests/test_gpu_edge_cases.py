"""Edge cases of the force path on the GPU, through the pair style's C ABI, against the oracle.

The reference's own tests pin the same behaviour: padded edges contribute exactly zero and padded
force rows stay 0.0 (tests/test_eam.py:570-601, tests/test_eam_pallas.py:35); the pack drops every
pair past the cutoff (cpp/pair_jax_kokkos.cpp:84-91); capacity is checked against the kept count
(:1063-1075). Cases:
- an empty rank (no owned or ghost atoms);
- atoms whose listed neighbors all lie between rc and rc + skin (every listed pair masked);
- ragged rows: a dense cluster beside isolated atoms, so rows keep from 0 to ~80 pairs;
- the edge capacity exactly at the kept count (fits; rows spill and re-walk the list) and one
  below it (the reference's capacity message);
- ghost force rows left exactly 0.0 with newton off.
"""

import numpy as np
import pytest
import torch

from cases import F64_TOTAL_REL, Case, write_eam_bundle
from conftest import load_package
from test_gpu_parity import MODE_SETUP, assert_parity, oracle_step

pytestmark = pytest.mark.gpu


def pair_for(tmp_path, case, mode, **bundle_kw):
    ljx = load_package()
    newton, half = MODE_SETUP[mode]
    path = write_eam_bundle(tmp_path, case, mode=mode, precision="float64", **bundle_kw)
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
    pair.init_style(system)
    return pair, system


def compute(pair, system):
    res = pair.compute(system, eflag=True, vflag=True)
    if system.newton_pair:
        system.comm.reverse_forces(system.f)
    torch.cuda.synchronize()
    return res


def periodic_case(x, box, types=None, elements=("Cu",)):
    ljx = load_package()
    synth = ljx.synth
    cutoff, skin = 6.5, 2.0
    x = np.asarray(x, np.float64)
    t = np.ones(len(x), np.int32) if types is None else np.asarray(types, np.int32)
    x_all, owner = synth.periodic_ghosts(x, box, cutoff + skin)
    types_all = np.concatenate([t, t[owner]]).astype(np.int32)
    return Case(synth.synthetic_setfl(elements, nr=2000, nrho=2000), x_all, types_all, len(x),
                owner, np.asarray(box, np.float64), cutoff, skin, len(elements))


def test_empty_rank(tmp_path):
    """No owned or ghost atoms: zero energy, virial and kept pairs, no error."""
    ljx = load_package()
    text = ljx.synth.synthetic_setfl(("Cu",), nr=500, nrho=500)
    path = tmp_path / "empty.json"
    ljx.write_bundle(path, potential=ljx.eam_potential(text), max_atoms=64, max_edges=64 * 128,
                     cutoff=6.5, unit_style="metal", precision="float64",
                     force_output="atom-force", newton="off", comm=True)
    # One-row buffers so every pointer is a real allocation; the counts say there are no atoms.
    x = torch.zeros(1, 3, dtype=torch.float64, device="cuda")
    system = ljx.System(x=x, type=torch.ones(1, dtype=torch.int32, device="cuda"),
                        f=torch.zeros_like(x), nlocal=0, nghost=0, newton_pair=False,
                        unit_style="metal", ntypes=1)
    system.list = ljx.NeighborList(ilist=torch.zeros(1, dtype=torch.int32, device="cuda"),
                                   numneigh=torch.zeros(1, dtype=torch.int32, device="cuda"),
                                   neighbors=torch.zeros(32, dtype=torch.int32, device="cuda"),
                                   slot_stride=32, maxneighs=1, inum=0)
    system.comm = ljx.SelfComm(torch.zeros(1, dtype=torch.int32, device="cuda")[:0], 0)
    pair = ljx.PairJax(device=0)
    pair.coeff(system, "*", "*", str(path))
    pair.init_style(system)
    for ago in (0, 1):
        system.list.ago = ago
        res = compute(pair, system)
        assert res.energy == 0.0 and list(res.virial) == [0.0] * 6
        assert res.edge_count == 0 and res.overflow == 0
    assert float(system.f.abs().max().item()) == 0.0


@pytest.mark.parametrize("mode", ["rows-full", "ghost", "half-unique"])
def test_every_listed_pair_masked(tmp_path, oracle, mode):
    """A simple-cubic lattice at 7.0 A: each atom lists its 6 neighbors (within rc + skin =
    8.5 A) but keeps none (rc = 6.5 A). Energy is N F(0); forces and virial are exactly 0."""
    n = 8
    g = np.arange(n) * 7.0
    x = np.stack(np.meshgrid(g, g, g, indexing="ij"), -1).reshape(-1, 3) + 0.5
    case = periodic_case(x, np.full(3, n * 7.0))
    pair, system = pair_for(tmp_path, case, mode)
    # Each pair is listed (once per direction on a full list, once on a half list) and masked.
    assert int(system.list.numneigh[: case.nlocal].sum().item()) >= 3 * case.nlocal
    res = compute(pair, system)
    ref = oracle_step(oracle, case, system, mode, "float64")
    assert res.edge_count == ref.count == 0
    assert float(system.f.abs().max().item()) == 0.0
    assert list(res.virial) == [0.0] * 6
    assert res.energy == pytest.approx(ref.energy, rel=F64_TOTAL_REL)
    tables = oracle.parse_setfl_text(case.text)
    assert res.energy == pytest.approx(case.nlocal * tables["embedding"][0, 0, 0],
                                       rel=F64_TOTAL_REL)


@pytest.mark.parametrize("mode", ["rows-full", "ghost", "half-unique"])
def test_ragged_rows(tmp_path, oracle, mode):
    """A jittered fcc cluster (4x4x4 cells, binary) in a 60 A box beside isolated atoms more
    than rc + skin from everything: rows keep from 0 to ~80 pairs, cached steps included."""
    ljx = load_package()
    cluster = ljx.synth.fcc((4, 4, 4), 3.615, jitter=0.08, seed=61, wrap=False,
                            sort_binsize=None).x + 15.0
    far = np.array([[50.0, 50.0, 50.0], [50.0, 5.0, 40.0], [5.0, 50.0, 45.0], [40.0, 40.0, 5.0]])
    x = np.concatenate([cluster, far])
    types = ljx.synth.substitutional(len(x), (0.64, 0.36), seed=62)
    case = periodic_case(x, np.full(3, 60.0), types, elements=("Cu", "Zr"))
    pair, system = pair_for(tmp_path, case, mode)
    res = compute(pair, system)
    ref = oracle_step(oracle, case, system, mode, "float64")
    assert_parity(res, system, ref, "float64", case)
    f = system.f[: case.nlocal].cpu().numpy()
    assert np.all(f[-4:] == 0.0)   # the isolated atoms feel nothing
    for ago in (1, 2):             # the candidate cache over the same ragged rows
        system.f.zero_()
        system.list.ago = ago
        res = compute(pair, system)
        assert_parity(res, system, ref, "float64", case)


def test_edge_capacity_at_the_kept_count(tmp_path, oracle):
    """max_edges equal to the kept count fits (rows past the per-row capacity re-walk the list);
    one less raises the reference's capacity message."""
    ljx = load_package()
    atoms = ljx.synth.fcc((5, 5, 5), 3.615, jitter=0.08, seed=67)
    case = periodic_case(atoms.x, atoms.box)
    probe, system = pair_for(tmp_path, case, "rows-full", scale_name="probe")
    kept = compute(probe, system).edge_count
    nall = len(case.x_all)
    pair, system = pair_for(tmp_path, case, "rows-full", max_atoms=nall, max_edges=kept,
                            scale_name="exact")
    res = compute(pair, system)
    ref = oracle_step(oracle, case, system, "rows-full", "float64")
    assert res.edge_count == ref.count == kept
    assert_parity(res, system, ref, "float64", case)
    assert np.all(system.f[case.nlocal:].cpu().numpy() == 0.0)  # ghost rows, newton off
    pair, system = pair_for(tmp_path, case, "rows-full", max_atoms=nall, max_edges=kept - 1,
                            scale_name="short")
    with pytest.raises(ljx.LammpsError) as err:
        compute(pair, system)
    assert str(err.value).startswith("LAMMPS-JAX edge capacity exceeded: global max "
                                     f"{kept} edges, capacity {kept - 1}")
