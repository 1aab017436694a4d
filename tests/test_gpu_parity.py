"""GPU parity: libljx through its C ABI against the CPU oracle on identical seeded inputs.

Tolerances (stated by the engine's contract): float64 per-atom forces within 1e-10 of the
max-abs force, total energy and virial within 1e-12 relative; float32 forces within 1e-5 of the
max-abs force; packed edge lists bit-exact after a canonical (receiver, sender) sort.
"""

import numpy as np
import pytest
import torch

from cases import (F32_FORCE_REL, F32_TOTAL_REL, F64_FORCE_REL, F64_TOTAL_REL, canonical_edges,
                   copy_device, device_system, eam_case, host_list, write_eam_bundle)
from conftest import load_package

pytestmark = pytest.mark.gpu

MODE_SETUP = {  # mode -> (newton_pair, half list)
    "ghost": (True, False),
    "rows-full": (False, False),
    "half-unique": (True, True),
}


def run_pair(tmp_path, case, mode, precision, scale=1.0, **bundle_kw):
    ljx = load_package()
    newton, half = MODE_SETUP[mode]
    path = write_eam_bundle(tmp_path, case, mode=mode, precision=precision, **bundle_kw)
    system = device_system(case, newton=newton, half=half)
    pair = ljx.PairJax(device=0)
    pair.settings()
    args = ["*", "*", str(path)] + ([str(scale)] if scale != 1.0 else [])
    pair.coeff(system, *args)
    assert bool(pair.init_style(system)["half_list"]) == half
    res = pair.compute(system, eflag=True, vflag=True)
    if newton:
        system.comm.reverse_forces(system.f)  # LAMMPS's own reverse comm of ghost forces
    torch.cuda.synchronize()
    return pair, system, res


def oracle_step(oracle, case, system, mode, precision, scale=1.0):
    tables = oracle.parse_setfl_text(case.text)
    return oracle.eam_step(tables, case.x_all, case.types_all, case.nlocal, case.owner,
                           host_list(system.list), mode=mode, precision=precision, scale=scale)


def assert_parity(res, system, ref, precision, case):
    forces = system.f[: case.nlocal].cpu().numpy()
    fmax = float(np.max(np.abs(ref.forces)))
    frel = F64_FORCE_REL if precision == "float64" else F32_FORCE_REL
    trel = F64_TOTAL_REL if precision == "float64" else F32_TOTAL_REL
    ferr = float(np.max(np.abs(forces - ref.forces)))
    assert ferr <= frel * fmax, f"force err {ferr:.3e} vs max |F| {fmax:.3e}"
    assert res.energy == pytest.approx(ref.energy, rel=trel)
    vscale = float(np.max(np.abs(ref.virial)))
    verr = float(np.max(np.abs(np.array(res.virial) - ref.virial)))
    assert verr <= trel * vscale, f"virial err {verr:.3e} of {vscale:.3e}"
    assert res.edge_count == ref.count
    assert res.overflow == 0


def test_neighbor_list_matches_oracle(oracle):
    case = eam_case(cells=(5, 5, 5), seed=11, nr=500, nrho=500)
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


def test_device_binning_matches_host():
    """ljx_neigh_bin's counting sort equals the host binning: same bin starts, and atoms in
    index order within each bin."""
    ljx = load_package()
    case = eam_case(cells=(5, 5, 5), seed=19, nr=500, nrho=500)
    cut = case.cutoff + case.skin
    builder = ljx.synth.DeviceListBuilder(case.x_all, case.nlocal, cut)
    builder.launch(torch.as_tensor(case.x_all, device="cuda"))
    torch.cuda.synchronize()
    lo, binsize, nb, start, order = ljx.synth.bin_atoms(case.x_all, cut)
    np.testing.assert_array_equal(builder.bin_start.cpu().numpy(), start)
    np.testing.assert_array_equal(builder.bin_atoms.cpu().numpy(), order)


@pytest.mark.parametrize("mode", ["rows-full", "ghost", "half-unique"])
def test_pack_edges_bit_exact(tmp_path, oracle, mode):
    ljx = load_package()
    case = eam_case(elements=("Cu", "Zr"), cells=(5, 5, 5), seed=13, nr=500, nrho=500)
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
    max_atoms = engine.contract["max_atoms"]
    o_s, o_r, o_m, count, overflow = oracle.pack_edges(
        case.x_all, il, nn, nb, 1, stride, case.nlocal, maxn, max_atoms, cap, case.cutoff,
        nlocal=case.nlocal)
    assert overflow == 0
    assert int(mask.sum()) == count
    assert np.all(mask[:count]) and not np.any(mask[count:])
    a = canonical_edges(senders[:count], receivers[:count])
    b = canonical_edges(o_s[:count], o_r[:count])
    np.testing.assert_array_equal(a[0], b[0])
    np.testing.assert_array_equal(a[1], b[1])
    assert np.all(senders[count:] == max_atoms) and np.all(receivers[count:] == max_atoms)
    # A second pack with fewer atoms restores the padding past the new count.
    res = engine.read_result()
    assert res.edge_count == count


@pytest.mark.parametrize("precision", ["float64", "float32"])
@pytest.mark.parametrize("mode", ["rows-full", "ghost", "half-unique"])
@pytest.mark.parametrize("elements", [("Cu",), ("Cu", "Zr")])
def test_eam_matches_oracle(tmp_path, oracle, mode, precision, elements):
    case = eam_case(elements=elements, cells=(5, 5, 5), seed=17, nr=5000, nrho=5000)
    pair, system, res = run_pair(tmp_path, case, mode, precision)
    ref = oracle_step(oracle, case, system, mode, precision)
    assert_parity(res, system, ref, precision, case)
    # Per-atom density of owned rows (the comm-site feature).
    rho = pair.engine.feature_tensor(0, case.nlocal).cpu().numpy().astype(np.float64)
    rtol = 1e-12 if precision == "float64" else 1e-5
    np.testing.assert_allclose(rho, ref.rho[: case.nlocal].astype(np.float64), rtol=rtol)


def funcfl_text(nrho=2000, nr=2000, cutoff=6.5):
    """A single-element funcfl table (LAMMPS pair_style eam format): F(rho), the effective charge
    Z(r) (r*phi = 27.2 * 0.529 * Z^2) and rho(r), smooth and zero at the cutoff."""
    ljx = load_package()
    synth = ljx.synth
    dr = cutoff / (nr - 1)
    r = np.arange(nr) * dr
    rho_e = synth.fcc_shell_density("Cu", cutoff)
    drho = 3.0 * rho_e / (nrho - 1)
    rho = np.arange(nrho) * drho
    embed = -3.54 * np.sqrt(rho / rho_e) + 0.15 * (rho - rho_e) ** 2
    z = 1.1 * np.exp(-1.2 * (r - 2.2)) * synth.taper(r, cutoff)
    lines = ["funcfl table for the parity tests", "29 63.546 3.615 fcc",
             f"{nrho} {drho!r} {nr} {dr!r} {cutoff!r}"]
    values = np.concatenate([embed, z, synth.density_fn("Cu", r, cutoff)])
    lines += [" ".join(f"{v:.17g}" for v in values[k:k + 5]) for k in range(0, len(values), 5)]
    return "\n".join(lines) + "\n"


@pytest.mark.parametrize("mode", ["rows-full", "ghost", "half-unique"])
def test_funcfl_bundle_matches_oracle(tmp_path, oracle, mode):
    """A funcfl bundle (pair_style eam tables, eam.py:233-262) through the same engine: forces,
    energy and virial against the oracle with the oracle's own funcfl reader."""
    ljx = load_package()
    text = funcfl_text()
    case = eam_case(cells=(5, 5, 5), seed=71, nr=100, nrho=100)  # geometry; tables replaced
    newton, half = MODE_SETUP[mode]
    kwargs = dict(potential=ljx.bundle.funcfl_potential(text, "Cu"),
                  max_atoms=len(case.x_all) + 64, max_edges=(len(case.x_all) + 64) * 128,
                  cutoff=case.cutoff, unit_style="metal", precision="float64", n_species=1,
                  force_output="atom-force")
    if mode == "ghost":
        kwargs.update(newton="on")
    elif mode == "rows-full":
        kwargs.update(newton="off", comm=True)
    else:
        kwargs.update(newton="on", comm=True, half_edges=True)
    path = tmp_path / f"funcfl_{mode}.json"
    ljx.write_bundle(path, **kwargs)
    system = device_system(case, newton=newton, half=half)
    pair = ljx.PairJax(device=0)
    pair.coeff(system, "*", "*", str(path))
    pair.init_style(system)
    res = pair.compute(system, eflag=True, vflag=True)
    if newton:
        system.comm.reverse_forces(system.f)
    torch.cuda.synchronize()
    (tmp_path / "Cu.eam").write_text(text)
    tables = oracle.load_funcfl(tmp_path / "Cu.eam")
    ref = oracle.eam_step(tables, case.x_all, case.types_all, case.nlocal, case.owner,
                          host_list(system.list), mode=mode, precision="float64")
    assert_parity(res, system, ref, "float64", case)


def test_eam_scale_and_extrapolation(tmp_path, oracle):
    # Compressed lattice: densities run past rhomax, so F(rho) extrapolates linearly.
    case = eam_case(cells=(5, 5, 5), a=2.9, jitter=0.05, seed=19, nr=2000, nrho=2000)
    pair, system, res = run_pair(tmp_path, case, "rows-full", "float64", scale=0.5)
    ref = oracle_step(oracle, case, system, "rows-full", "float64", scale=0.5)
    tables = oracle.parse_setfl_text(case.text)
    assert (ref.rho[: case.nlocal] > (tables["nrho"] - 1) * tables["drho"]).sum() >= 10
    assert_parity(res, system, ref, "float64", case)


def test_spilled_rows_match(tmp_path, oracle):
    """Rows wider than the compacted row capacity re-walk the list; results are unchanged."""
    case = eam_case(cells=(5, 5, 5), seed=23, nr=1000, nrho=1000)
    nall = len(case.x_all)
    # Enough total capacity for every kept pair, but fewer slots per row than most rows keep.
    pair, system, res = run_pair(tmp_path, case, "rows-full", "float64",
                                 max_atoms=nall + 64, max_edges=(nall + 64) * 40)
    ref = oracle_step(oracle, case, system, "rows-full", "float64")
    assert ref.count <= (nall + 64) * 40
    assert_parity(res, system, ref, "float64", case)


def test_edge_capacity_overflow_message(tmp_path):
    ljx = load_package()
    case = eam_case(cells=(5, 5, 5), seed=29, nr=500, nrho=500)
    with pytest.raises(ljx.LammpsError, match="edge capacity exceeded"):
        run_pair(tmp_path, case, "rows-full", "float64", max_edges=1000)


def test_atom_capacity_message(tmp_path):
    ljx = load_package()
    case = eam_case(cells=(5, 5, 5), seed=31, nr=500, nrho=500)
    with pytest.raises(ljx.LammpsError, match="atom capacity exceeded"):
        run_pair(tmp_path, case, "rows-full", "float64", max_atoms=100)


LJ_MODES = {  # name -> (force_output, newton_pair, half list)
    "edge-newton-off": ("edge-force", False, False),
    "edge-newton-on": ("edge-force", True, True),
    "atom-newton-on": ("atom-force", True, False),
}


def lj_case(seed=3, cells=(8, 8, 4), density=0.8442, jitter=0.05, skin=0.3, cutoff=2.5):
    ljx = load_package()
    a = (4.0 / density) ** (1.0 / 3.0)
    atoms = ljx.synth.fcc(cells, a, jitter=0.0, seed=seed)
    rng = np.random.default_rng(seed)
    x = np.mod(atoms.x + rng.uniform(-jitter, jitter, atoms.x.shape), atoms.box)
    x_all, owner = ljx.synth.periodic_ghosts(x, atoms.box, cutoff + skin)
    return x_all, owner, len(x), cutoff, skin


@pytest.mark.parametrize("precision", ["float64", "float32"])
@pytest.mark.parametrize("mode", list(LJ_MODES))
def test_lj_matches_oracle(tmp_path, oracle, mode, precision):
    ljx = load_package()
    force_output, newton, half = LJ_MODES[mode]
    x_all, owner, nlocal, cutoff, skin = lj_case()
    nall = len(x_all)
    path = tmp_path / "lj.json"
    ljx.write_bundle(path, potential=ljx.lj_potential(1.0, 1.0), max_atoms=nall + 32,
                     max_edges=(nall + 32) * 96, cutoff=cutoff, unit_style="lj",
                     precision=precision, force_output=force_output,
                     newton="on" if newton else "off")
    x = torch.as_tensor(x_all, device="cuda")
    system = ljx.System(x=x, type=torch.ones(nall, dtype=torch.int32, device="cuda"),
                        f=torch.zeros_like(x), nlocal=nlocal, nghost=nall - nlocal,
                        newton_pair=newton, unit_style="lj", ntypes=1)
    system.list = ljx.synth.neighbor_list(x_all, nlocal, cutoff + skin, half=half)
    system.comm = ljx.SelfComm(torch.as_tensor(owner, device="cuda"), nlocal)
    pair = ljx.PairJax()
    pair.coeff(system, "*", "*", str(path))
    assert bool(pair.init_style(system)["half_list"]) == half
    res = pair.compute(system)
    if newton:
        system.comm.reverse_forces(system.f)
    torch.cuda.synchronize()
    ref = oracle.lj_step(x_all, nlocal, owner, host_list(system.list), epsilon=1.0, sigma=1.0,
                         cutoff=cutoff, force_output=force_output, newton_pair=newton,
                         precision=precision)
    forces = system.f[:nlocal].cpu().numpy()
    fmax = float(np.max(np.abs(ref.forces)))
    frel = F64_FORCE_REL if precision == "float64" else F32_FORCE_REL
    trel = F64_TOTAL_REL if precision == "float64" else F32_TOTAL_REL
    assert float(np.max(np.abs(forces - ref.forces))) <= frel * fmax
    assert res.energy == pytest.approx(ref.energy, rel=trel)
    vscale = float(np.max(np.abs(ref.virial)))
    assert float(np.max(np.abs(np.array(res.virial) - ref.virial))) <= trel * vscale
    assert res.edge_count == ref.count


def test_comm_rows_roundtrip():
    """Forward pack/unpack copies rows; reverse pack/unpack adds them (a15)."""
    ljx = load_package()
    lib = ljx.load()
    import ctypes
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rng = np.random.default_rng(5)
    for dtype, elem in ((torch.float64, 8), (torch.float32, 4)):
        width = 3
        n_rows, n_send = 200, 37
        rows = torch.as_tensor(rng.random((n_rows, width)), dtype=dtype, device="cuda")
        send = torch.as_tensor(rng.choice(120, n_send, replace=False).astype(np.int32),
                               device="cuda")
        words = width * elem // 4
        slots = (width * elem + 7) // 8
        buf = torch.zeros(n_send * slots, dtype=torch.float64, device="cuda")
        assert lib.ljx_comm_pack_forward(stream, ctypes.c_void_p(rows.data_ptr()), words,
                                         ctypes.c_void_p(send.data_ptr()), n_send,
                                         ctypes.c_void_p(buf.data_ptr()), slots) == 0
        first = 150
        out = rows.clone()
        assert lib.ljx_comm_unpack_forward(stream, ctypes.c_void_p(out.data_ptr()), words, first,
                                           n_send, ctypes.c_void_p(buf.data_ptr()), slots) == 0
        torch.cuda.synchronize()
        ref = rows.cpu().numpy()
        got = out.cpu().numpy()
        np.testing.assert_array_equal(got[first:first + n_send], ref[send.cpu().numpy()])
        np.testing.assert_array_equal(got[:first], ref[:first])
        # Reverse: rows[first..first+n) packed, then added into the sendlist rows.
        n_rev = 40
        rbuf = torch.zeros(n_rev * slots, dtype=torch.float64, device="cuda")
        assert lib.ljx_comm_pack_reverse(stream, ctypes.c_void_p(rows.data_ptr()), words, 100,
                                         n_rev, ctypes.c_void_p(rbuf.data_ptr()), slots) == 0
        dest = torch.zeros_like(rows)
        rsend = torch.as_tensor(rng.choice(100, n_rev, replace=False).astype(np.int32),
                                device="cuda")
        assert lib.ljx_comm_unpack_reverse(stream, ctypes.c_void_p(dest.data_ptr()), width, elem,
                                           ctypes.c_void_p(rsend.data_ptr()), n_rev,
                                           ctypes.c_void_p(rbuf.data_ptr()), slots) == 0
        torch.cuda.synchronize()
        expect = np.zeros_like(ref)
        expect[rsend.cpu().numpy()] += ref[100:100 + n_rev]
        np.testing.assert_array_equal(dest.cpu().numpy(), expect)
