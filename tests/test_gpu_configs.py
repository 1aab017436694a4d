"""GPU parity at the benchmark configurations' own sizes.

C1 (LJ fcc 8x8x4, 1024 atoms) already runs at full size in test_gpu_parity.test_lj_matches_oracle.
Here:
- C2: synthetic binary Cu-Zr EAM, 8192 atoms of seeded random packing at 0.058 atoms/A^3 with a
  2.0 A hard core, 64/36 species, half list with newton on (the half-unique communicating export),
  128 edges per atom, float64.
- C3: Cu fcc 80^3 cells = 2,048,000 atoms with 0.08 A Gaussian jitter, full list, newton off,
  in float64 and in float32 (the two precisions C3 names), rebuild state as the bench runs it
  (candidate cache built this step); forces, energy, virial and the kept count.
- C5: the edge-pack stress test, a binary Cu-Zr liquid at 1.2x fcc density with a 2.0 A core,
  2,048,000 atoms (a 32,000-atom periodic tile repeated 4x4x4), full list with a 2.0 A skin so
  that about half the listed pairs are masked out, 160 edges per atom, float32, a fresh list.
Both are checked against the CPU oracle on the same inputs and list. C3 also checks a
size-independent property: the forces of a periodic system sum to zero. C5 packs the reference's
edge ABI (ljx_pack_edges) as well: bit-exact after the canonical sort on one tile, and at full
size the kept count, the padding, and order-free checksums of the (receiver, sender) pairs.

Tolerances: float64 forces within 1e-10 of the max-abs force, energy and virial 1e-12 relative;
float32 forces within 1e-5 of the max-abs force, energy and virial 1e-5 relative.
"""

import numpy as np
import pytest
import torch

from cases import F32_FORCE_REL, F64_FORCE_REL, Case, canonical_edges, copy_device, write_eam_bundle
from conftest import load_package
from test_gpu_parity import assert_parity, oracle_step

pytestmark = pytest.mark.gpu


def run_case(tmp_path, case, mode, newton, half, precision="float64", edges_per_atom=128,
             pair_out=None):
    ljx = load_package()
    path = write_eam_bundle(tmp_path, case, mode=mode, precision=precision,
                            edges_per_atom=edges_per_atom)
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
    if pair_out is not None:
        pair_out.append(pair)
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


@pytest.mark.parametrize("precision", ["float64", "float32"])
def test_c3_full_size(tmp_path, oracle, precision):
    """C3 at its own size in both precisions it names: forces, energy, virial and the kept count
    against the oracle, and the momentum sum of the periodic crystal."""
    ljx = load_package()
    synth = ljx.synth
    atoms = synth.fcc((80, 80, 80), 3.615, jitter=0.08, seed=2024)
    cutoff, skin = 6.5, 2.0
    x_all, owner = synth.periodic_ghosts(atoms.x, atoms.box, cutoff + skin)
    case = Case(synth.synthetic_setfl(("Cu",)), x_all, np.ones(len(x_all), np.int32),
                len(atoms.x), owner, atoms.box, cutoff, skin, 1)
    assert case.nlocal == 2_048_000
    system, res = run_case(tmp_path, case, "rows-full", newton=False, half=False,
                           precision=precision)
    forces = system.f[: case.nlocal]
    fmax = float(forces.abs().max().item())
    # Momentum: pair forces cancel, so the sum is rounding only (2 M terms of size <= fmax).
    frel = F64_FORCE_REL if precision == "float64" else F32_FORCE_REL
    total = forces.sum(dim=0).abs().max().item()
    assert total <= frel * fmax * case.nlocal ** 0.5
    ref = oracle_step(oracle, case, system, "rows-full", precision)
    assert_parity(res, system, ref, precision, case)


C5_DENSITY = 1.2 * 4 / 3.615 ** 3  # 1.2x the synthetic Cu fcc density, atoms/A^3
C5_TILE = 32_000


def c5_case(tiles):
    ljx = load_package()
    synth = ljx.synth
    types = synth.substitutional(C5_TILE, (0.64, 0.36), seed=2025)
    atoms = synth.liquid_packing(C5_TILE, C5_DENSITY, 2.0, seed=2024, tiles=tiles, types=types)
    cutoff, skin = 6.5, 2.0
    x_all, owner = synth.periodic_ghosts(atoms.x, atoms.box, cutoff + skin)
    types_all = np.concatenate([atoms.types, atoms.types[owner]]).astype(np.int32)
    return Case(synth.synthetic_setfl(("Cu", "Zr")), x_all, types_all, len(atoms.x), owner,
                atoms.box, cutoff, skin, 2)


def pack_reference_abi(pair, system):
    """ljx_pack_edges into the engine's reference-ABI arrays: (senders, receivers) of the kept
    edges, the count, and whether every slot past the count holds the padding."""
    engine = pair.engine
    atoms, nl = system.atoms(), system.list.struct()
    engine.pack_atoms(atoms)
    engine.pack_edges(atoms, nl, system.newton_pair)
    s_ptr, r_ptr, m_ptr, cap = engine.edges()
    res = engine.read_result()
    count = res.edge_count
    assert res.overflow == 0
    senders = copy_device(s_ptr, count, np.int32)
    receivers = copy_device(r_ptr, count, np.int32)
    mask = copy_device(m_ptr, cap, np.uint8)
    pad = engine.contract["max_atoms"]
    tail_s = copy_device(s_ptr + 4 * count, cap - count, np.int32)
    tail_r = copy_device(r_ptr + 4 * count, cap - count, np.int32)
    padded = (bool(np.all(mask[:count] == 1)) and not np.any(mask[count:])
              and bool(np.all(tail_s == pad)) and bool(np.all(tail_r == pad)))
    return senders, receivers, count, padded


def pair_checksums(senders, receivers):
    """Order-free checksums of a set of (receiver, sender) pairs: the wrapped sum and the xor of
    a 64-bit mix (splitmix64's finalizer) of each pair's key."""
    k = (receivers.astype(np.uint64) << np.uint64(32)) | senders.astype(np.uint64)
    k ^= k >> np.uint64(30)
    k *= np.uint64(0xBF58476D1CE4E5B9)
    k ^= k >> np.uint64(27)
    k *= np.uint64(0x94D049BB133111EB)
    k ^= k >> np.uint64(31)
    return int(np.sum(k, dtype=np.uint64)), int(np.bitwise_xor.reduce(k))


@pytest.mark.parametrize("tiles", [1, 4])
def test_c5_liquid_edge_pack_stress(tmp_path, oracle, tiles):
    case = c5_case(tiles)
    assert case.nlocal == C5_TILE * tiles ** 3
    pairs = []
    system, res = run_case(tmp_path, case, "rows-full", newton=False, half=False,
                           precision="float32", edges_per_atom=160, pair_out=pairs)
    ref = oracle_step(oracle, case, system, "rows-full", "float32")
    assert_parity(res, system, ref, "float32", case)
    # About half of the listed pairs (rc 6.5 A of a 8.5 A list) are masked out.
    listed = int(system.list.numneigh[: case.nlocal].sum().item())
    assert 0.35 < res.edge_count / listed < 0.55
    senders, receivers, count, padded = pack_reference_abi(pairs[0], system)
    assert count == ref.count and padded
    if tiles == 1:
        a = canonical_edges(senders, receivers)
        b = canonical_edges(ref.senders[:count], ref.receivers[:count])
        np.testing.assert_array_equal(a[0], b[0])
        np.testing.assert_array_equal(a[1], b[1])
    else:
        assert pair_checksums(senders, receivers) == pair_checksums(ref.senders[:count],
                                                                    ref.receivers[:count])
