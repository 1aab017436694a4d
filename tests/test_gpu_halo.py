"""libljx's NCCL halo (include/ljx_halo.h) on one GPU.

A one-rank communicator exercises every part of the library's exchange: the swap table of a
z-slab that is its own neighbour along z, the gather and scatter-add kernels, and (with
LJX_HALO_SELF_BY_NCCL) grouped ncclSend/ncclRecv to the rank itself; ljx_read_result_all runs
its on-stream NCCL all-reduce. Checked against the host restatement of the swap semantics
(halo.apply_swaps) bit for bit, and through a whole EAM step against the CPU oracle in the two
exchange patterns of the benchmark (C3: forward F'; C4: reverse rho, forward F', reverse forces).
The multi-rank case is tests/test_gpu_multirank.py.
"""

import ctypes

import numpy as np
import pytest
import torch

from cases import F64_FORCE_REL, F64_TOTAL_REL
from conftest import load_package

pytestmark = pytest.mark.gpu

CUT = 8.5
A_CUZR = 0.64 * 3.615 + 0.36 * 4.525


def one_rank_halo(ljx, swaps, flags):
    from lammps_jax_b200.halo import NcclHalo
    lib = ljx.load()
    buf = (ctypes.c_ubyte * ljx.abi.HALO_ID_BYTES)()
    assert lib.ljx_halo_unique_id(buf) == ljx.abi.OK, lib.ljx_halo_create_error()
    return NcclHalo(swaps, 0, 1, torch.cuda.current_device(), unique_id=bytes(buf), flags=flags)


def slab(ljx, cells=(4, 4, 4), fractions=(0.64, 0.36)):
    return ljx.synth.slab_decomposition(cells, A_CUZR, 0.08, 5, 0, 1, CUT, fractions=fractions)


@pytest.mark.parametrize("flags", [0, 1])
@pytest.mark.parametrize("width,dtype", [(1, np.float64), (3, np.float64), (1, np.float32)])
def test_halo_rows_match_swap_semantics(flags, width, dtype):
    ljx = load_package()
    from lammps_jax_b200.halo import apply_swaps, slab_swaps
    s = slab(ljx)
    swaps = slab_swaps(s, 0, 1)
    halo = one_rank_halo(ljx, swaps, flags)
    try:
        rng = np.random.default_rng(3)
        elem = np.dtype(dtype).itemsize
        # Integer-valued rows: sums are exact in any order, so the comparison is bitwise.
        rows = rng.integers(0, 1000, size=(len(s.x), width)).astype(dtype)
        rows[s.nlocal:] = -1
        dev = torch.as_tensor(rows, device="cuda")
        halo.forward(dev.data_ptr(), width, elem)
        expect = apply_swaps([rows.copy()], [swaps], forward=True)[0]
        torch.cuda.synchronize()
        np.testing.assert_array_equal(dev.cpu().numpy(), expect)
        partial = rng.integers(0, 100, size=(len(s.x), width)).astype(dtype)
        dev = torch.as_tensor(partial, device="cuda")
        halo.reverse(dev.data_ptr(), width, elem)
        expect = apply_swaps([partial.copy()], [swaps], forward=False)[0]
        torch.cuda.synchronize()
        np.testing.assert_array_equal(dev.cpu().numpy(), expect)
    finally:
        halo.close()


def eam_slab_step(tmp_path, ljx, oracle, s, mode, flags, max_edges_per_atom=128):
    """One EAM step of slab `s` through the engine and the NCCL halo, and the oracle's."""
    from lammps_jax_b200.halo import slab_swaps
    from test_decomposition import combined_owner
    newton, half = (False, False) if mode == "rows-full" else (True, True)
    text = ljx.synth.synthetic_setfl(("Cu", "Zr"), nr=2000, nrho=2000)
    nall = len(s.x)
    path = tmp_path / f"{mode}.json"
    ljx.write_bundle(path, potential=ljx.eam_potential(text), max_atoms=nall + 64,
                     max_edges=(nall + 64) * max_edges_per_atom, cutoff=6.5, unit_style="metal",
                     precision="float64", force_output="atom-force",
                     newton="on" if newton else "off", comm=True, half_edges=half, n_species=2)
    x = torch.as_tensor(s.x, device="cuda")
    system = ljx.System(x=x, type=torch.as_tensor(s.types, device="cuda"), f=torch.zeros_like(x),
                        nlocal=s.nlocal, nghost=nall - s.nlocal, newton_pair=newton,
                        unit_style="metal", ntypes=2)
    system.list = ljx.synth.neighbor_list(s.x, s.nlocal, CUT, half=half)
    pair = ljx.PairJax()
    pair.coeff(system, "*", "*", str(path))
    pair.init_style(system)
    plan, eng = pair.plan, pair.engine
    halo = one_rank_halo(ljx, slab_swaps(s, 0, 1), flags)
    try:
        atoms, nl = system.atoms(), system.list.struct()
        fp_rows, width, elem = eng.feature_rows(1)
        rho_rows = eng.feature_rows(0)[0]
        eng.pack_atoms(atoms)
        eng.density(atoms, nl, newton)
        if plan.reverse_density:
            halo.reverse(rho_rows, width, elem)
        eng.embed(atoms)
        if plan.forward_fp:
            halo.forward(fp_rows, width, elem)
        eng.force(atoms, nl, newton, 1.0)
        if plan.reverse_force:
            halo.reverse_forces(system.f)
        res = halo.result_all(eng)
        torch.cuda.synchronize()
        forces = system.f[:s.nlocal].cpu().numpy()
    finally:
        halo.close()
    owners, _ = combined_owner([s])
    lst = (system.list.ilist.cpu().numpy(), system.list.numneigh.cpu().numpy(),
           system.list.neighbors.cpu().numpy(), system.list.slot_stride, system.list.maxneighs)
    ref = oracle.eam_step(oracle.parse_setfl_text(text), s.x, s.types, s.nlocal,
                          owners[0].astype(np.int32), lst, mode=mode, precision="float64")
    return res, forces, ref


@pytest.mark.parametrize("flags", [0, 1])
@pytest.mark.parametrize("mode", ["rows-full", "half-unique"])
def test_halo_eam_step_matches_oracle(tmp_path, oracle, mode, flags):
    ljx = load_package()
    s = slab(ljx)
    res, forces, ref = eam_slab_step(tmp_path, ljx, oracle, s, mode, flags)
    fmax = float(np.max(np.abs(ref.forces)))
    assert float(np.max(np.abs(forces - ref.forces))) <= F64_FORCE_REL * fmax
    assert res.energy == pytest.approx(ref.energy, rel=F64_TOTAL_REL)
    assert res.local_energy == res.energy
    vscale = float(np.max(np.abs(ref.virial)))
    assert float(np.max(np.abs(np.array(res.virial) - ref.virial))) <= F64_TOTAL_REL * vscale
    assert res.edge_count == ref.count and res.edge_max == ref.count
    assert res.overflow == 0


def test_halo_result_reports_capacity_overflow(tmp_path, oracle):
    """An edge capacity below the kept count sets the collective overflow flag (the pair style's
    "edge capacity exceeded" check), with the global max count; the step stays correct."""
    ljx = load_package()
    s = slab(ljx)
    res, forces, ref = eam_slab_step(tmp_path, ljx, oracle, s, "rows-full", 0,
                                     max_edges_per_atom=5)
    assert res.overflow == 1
    assert res.edge_max == ref.count
    fmax = float(np.max(np.abs(ref.forces)))
    assert float(np.max(np.abs(forces - ref.forces))) <= F64_FORCE_REL * fmax


def test_halo_rejects_rows_wider_than_its_table():
    ljx = load_package()
    from lammps_jax_b200.halo import slab_swaps
    s = slab(ljx)
    halo = one_rank_halo(ljx, slab_swaps(s, 0, 1), 0)
    try:
        rows = torch.zeros(len(s.x), 4, dtype=torch.float64, device="cuda")
        with pytest.raises(ljx.abi.LjxError, match="exceed"):
            halo.forward(rows.data_ptr(), 4, 8)
    finally:
        halo.close()
