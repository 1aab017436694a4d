"""The GPU path against the reference's own outputs, with no oracle in between.

The fixtures in tests/golden/ were produced by the reference itself (tests/golden/make_golden.py:
python/lammps_jax/eam.py and examples/export_model.py under a numpy stand-in for jax.numpy, and
the reference test suite's independent numpy port of PairEAM::compute). Here each fixture's edge
list becomes a LAMMPS neighbor list (rows = senders, one slot per edge) on a rank that owns every
atom and has no ghosts, and the pair style computes it through the C ABI. Tolerances are the
reference tests' own: float64 energy rel 1e-12 and forces atol 1e-10 (tests/test_eam.py:334-335,
:428-429); float32 atol 2e-5 * (1 + max|F|) (tests/test_eam_pallas.py:28-35).
"""

import numpy as np
import pytest
import torch

from conftest import GOLDEN, golden, load_package

pytestmark = pytest.mark.gpu


def f32_force_tol(ref):
    return 2e-5 * (1.0 + float(np.max(np.abs(ref))))


def list_from_edges(n, senders, receivers):
    """A LAMMPS-style list (Kokkos LayoutLeft) holding receiver j in row i for each edge."""
    ljx = load_package()
    stride = max(32, (n + 31) // 32 * 32)
    counts = np.bincount(senders, minlength=n).astype(np.int32)
    maxn = max(1, int(counts.max()))
    nb = np.zeros(stride * maxn, np.int32)
    fill = np.zeros(n, np.int64)
    for s, r in zip(senders.tolist(), receivers.tolist()):
        nb[s + fill[s] * stride] = r
        fill[s] += 1
    dev = lambda a: torch.as_tensor(np.ascontiguousarray(a), device="cuda")  # noqa: E731
    return ljx.NeighborList(ilist=dev(np.arange(n, dtype=np.int32)), numneigh=dev(counts),
                            neighbors=dev(nb), slot_stride=stride, maxneighs=maxn, inum=n)


def run_cluster(tmp_path, text, cutoff, pos, species, senders, receivers, *, mode, precision,
                potential=None, unit_style="metal", ntypes=2):
    ljx = load_package()
    n = len(pos)
    kw = dict(potential=potential or ljx.eam_potential(text), max_atoms=n + 32,
              max_edges=(n + 32) * 64, cutoff=cutoff, unit_style=unit_style,
              precision=precision, force_output="atom-force", n_species=ntypes)
    if mode == "rows-full":
        kw.update(newton="off", comm=True)
        newton = False
    else:  # half-unique: half list, newton on
        kw.update(newton="on", comm=True, half_edges=True)
        newton = True
    path = tmp_path / f"golden_{mode}_{precision}.json"
    ljx.write_bundle(path, **kw)
    x = torch.as_tensor(np.ascontiguousarray(pos, np.float64), device="cuda")
    system = ljx.System(x=x, type=torch.as_tensor((np.asarray(species) + 1).astype(np.int32),
                                                  device="cuda"),
                        f=torch.zeros_like(x), nlocal=n, nghost=0, newton_pair=newton,
                        unit_style=unit_style, ntypes=ntypes)
    system.list = list_from_edges(n, np.asarray(senders), np.asarray(receivers))
    system.list.half = mode != "rows-full"
    system.comm = ljx.SelfComm(torch.zeros(1, dtype=torch.int32, device="cuda")[:0], n)
    pair = ljx.PairJax(device=0)
    pair.coeff(system, "*", "*", str(path))
    pair.init_style(system)
    res = pair.compute(system, eflag=True, vflag=True)
    torch.cuda.synchronize()
    return res, system.f.cpu().numpy()


def tiny_setfl(oracle):
    text = (GOLDEN / "tiny.eam.alloy").read_text()
    return text, oracle.parse_setfl_text(text)["cutoff"]


def test_tiny_setfl_f64_matches_reference(tmp_path, oracle):
    g = golden("golden_tiny_setfl.npz")
    text, cutoff = tiny_setfl(oracle)
    res, f = run_cluster(tmp_path, text, cutoff, g["positions"], g["species"], g["senders"],
                         g["receivers"], mode="rows-full", precision="float64")
    assert res.energy == pytest.approx(float(g["native_energy"]), rel=1e-12)
    assert res.energy == pytest.approx(float(np.sum(g["energy_f64"])), rel=1e-12)
    np.testing.assert_allclose(f, g["native_forces"], rtol=0, atol=1e-10)


def test_tiny_setfl_f32_matches_reference(tmp_path, oracle):
    g = golden("golden_tiny_setfl.npz")
    text, cutoff = tiny_setfl(oracle)
    res, f = run_cluster(tmp_path, text, cutoff, g["positions"], g["species"], g["senders"],
                         g["receivers"], mode="rows-full", precision="float32")
    ref = np.zeros((len(g["positions"]), 3))
    np.add.at(ref, g["senders"], g["edge_force_f32"].astype(np.float64))
    assert res.energy == pytest.approx(float(np.sum(g["energy_f32"])), rel=1e-5)
    np.testing.assert_allclose(f, ref, rtol=0, atol=f32_force_tol(ref))


@pytest.mark.parametrize("tag,precision", [("f64", "float64"), ("f32", "float32")])
def test_half_edges_match_reference(tmp_path, oracle, tag, precision):
    """The half-unique export on a half list: energy and the edge forces summed per atom
    (sender +F, receiver -F) of the reference's half-edge model."""
    g = golden("golden_tiny_setfl.npz")
    text, cutoff = tiny_setfl(oracle)
    hs, hr = g["half_senders"], g["half_receivers"]
    res, f = run_cluster(tmp_path, text, cutoff, g["half_positions"], g["half_species"], hs, hr,
                         mode="half-unique", precision=precision)
    fe = g[f"half_edge_force_{tag}"].astype(np.float64)
    ref = np.zeros((len(g["half_positions"]), 3))
    np.add.at(ref, hs, fe)
    np.add.at(ref, hr, -fe)
    rel = 1e-12 if tag == "f64" else 1e-5
    assert res.energy == pytest.approx(float(np.sum(g[f"half_energy_{tag}"])), rel=rel)
    atol = 1e-10 if tag == "f64" else f32_force_tol(ref)
    np.testing.assert_allclose(f, ref, rtol=0, atol=atol)


@pytest.mark.parametrize("tag,precision", [("f64", "float64"), ("f32", "float32")])
def test_lj_matches_reference(tmp_path, tag, precision):
    """examples/export_model.py's LJ (eps = sigma = 1) as an edge-force bundle on a full list with
    newton off (energy 1/2 per directed edge): per-step energy against the reference's per-atom
    energies, forces against central differences of the reference energy."""
    ljx = load_package()
    g = golden("golden_lj.npz")
    pos, s, r = g["positions"], g["senders"], g["receivers"]
    n = len(pos)
    path = tmp_path / f"lj_{tag}.json"
    ljx.write_bundle(path, potential=ljx.lj_potential(1.0, 1.0), max_atoms=n + 32,
                     max_edges=(n + 32) * 64, cutoff=float(g["cutoff"]), unit_style="lj",
                     precision=precision, force_output="edge-force", newton="off")
    x = torch.as_tensor(np.ascontiguousarray(pos, np.float64), device="cuda")
    system = ljx.System(x=x, type=torch.ones(n, dtype=torch.int32, device="cuda"),
                        f=torch.zeros_like(x), nlocal=n, nghost=0, newton_pair=False,
                        unit_style="lj", ntypes=1)
    system.list = list_from_edges(n, np.asarray(s), np.asarray(r))
    system.comm = ljx.SelfComm(torch.zeros(1, dtype=torch.int32, device="cuda")[:0], n)
    pair = ljx.PairJax(device=0)
    pair.coeff(system, "*", "*", str(path))
    pair.init_style(system)
    res = pair.compute(system, eflag=True, vflag=True)
    torch.cuda.synchronize()
    ref = float(np.sum(g[f"energy_{tag}_s0.5"]))
    assert res.energy == pytest.approx(ref, rel=1e-12 if tag == "f64" else 2e-6)
    fd = g["fd_forces_s0.5"]
    f = system.f.cpu().numpy()
    tol = 1e-5 * np.max(np.abs(fd)) if tag == "f64" else f32_force_tol(fd)
    np.testing.assert_allclose(f, fd, rtol=0, atol=tol)
