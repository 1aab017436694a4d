"""Pins the CPU oracle against vectors produced by the lammps-jax reference itself.

The fixtures (tests/golden/make_golden.py) come from the reference's own eam.py / export_model.py
run under a numpy stand-in for jax.numpy, and from the reference test suite's independent numpy
port of PairEAM::compute. Tolerances are the reference tests' own: tests/test_eam.py:334-335
(rel/atol 1e-12 in float64), :428-429 (forces atol 1e-10), test_eam_pallas.py:28-35 (float32
atol 2e-5 * (1 + max|F|)).
"""

import numpy as np
import pytest

from conftest import CUZR_TABLE, GOLDEN, golden


def f32_force_tol(ref):
    return 2e-5 * (1.0 + float(np.max(np.abs(ref))))


def sum_sender_forces(edge_force, senders, n):
    out = np.zeros((n, 3))
    np.add.at(out, senders, edge_force.astype(np.float64))
    return out


def test_spline_coefficients_match_reference(oracle):
    g = golden("golden_spline.npz")
    coeffs = oracle.spline_coefficients(g["values"])
    np.testing.assert_array_equal(coeffs, g["coeffs"])
    np.testing.assert_allclose(coeffs, g["native_coeffs"], rtol=0, atol=1e-14)


@pytest.mark.parametrize("tag,dtype", [("f64", np.float64), ("f32", np.float32)])
@pytest.mark.parametrize("ext", [0, 1])
@pytest.mark.parametrize("der", [0, 1])
def test_spline_lookup_matches_reference(oracle, tag, dtype, ext, der):
    g = golden("golden_spline.npz")
    out = oracle.spline_eval(g["coeffs"], g["x"], dtype(g["delta"]), extrapolate=ext,
                             derivative=der, dtype=dtype)
    ref = g[f"{tag}_ext{ext}_der{der}"]
    rtol = 1e-15 if dtype == np.float64 else 2e-7
    np.testing.assert_allclose(out, ref, rtol=rtol, atol=rtol * np.max(np.abs(ref)))


def test_setfl_parse_matches_reference(oracle):
    g = golden("golden_tiny_setfl.npz")
    tables = oracle.load_setfl(GOLDEN / "tiny.eam.alloy")
    assert tables["elements"] == ["A", "B"]
    assert tables["masses"] == [10.0, 20.0]
    for key in ("embedding", "density", "pair", "pair_index"):
        np.testing.assert_array_equal(tables[key], g[key])


def _model(oracle, tables, pos, spc, s, r, mode, dtype):
    n = pos.shape[0]
    return oracle.eam_model(tables, pos, spc, n, 0, s, r, np.ones(len(s), np.uint8), mode,
                            dtype=dtype)


def test_setfl_f64_matches_reference_and_native_port(oracle):
    g = golden("golden_tiny_setfl.npz")
    tables = oracle.load_setfl(GOLDEN / "tiny.eam.alloy")
    pos, spc, s, r = g["positions"], g["species"], g["senders"], g["receivers"]
    ghost = _model(oracle, tables, pos, spc, s, r, "ghost", np.float64)
    rows = _model(oracle, tables, pos, spc, s, r, "rows-full", np.float64)
    # Per-atom energies of make_setfl_energy (rel 1e-12, test_eam.py:334).
    np.testing.assert_allclose(ghost.atom_energy, g["energy_f64"], rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(rows.atom_energy, g["energy_f64"], rtol=1e-12, atol=1e-12)
    assert ghost.energy == pytest.approx(float(np.sum(g["energy_f64"])), rel=1e-12)
    # Per-edge forces of make_setfl_edge_force.
    fmax = float(np.max(np.abs(g["edge_force_f64"])))
    np.testing.assert_allclose(rows.edge_force, g["edge_force_f64"], rtol=0, atol=1e-12 * fmax)
    # The independent PairEAM::compute port (test_eam.py:397-429): energy rel 1e-12, forces 1e-10.
    assert ghost.energy == pytest.approx(float(g["native_energy"]), rel=1e-12)
    np.testing.assert_allclose(ghost.model_force, g["native_forces"], rtol=0, atol=1e-10)
    np.testing.assert_allclose(rows.model_force, g["native_forces"], rtol=0, atol=1e-10)
    np.testing.assert_allclose(ghost.rho, g["native_density"], rtol=1e-12, atol=1e-12)
    # The fixture drives >= 10 atoms past rhomax (test_eam.py:412-413).
    rhomax = (tables["nrho"] - 1) * tables["drho"]
    assert int((ghost.rho > rhomax).sum()) >= 10
    # -dE/dx of the reference energy by central differences.
    fd = g["fd_forces"]
    np.testing.assert_allclose(ghost.model_force, fd, rtol=0, atol=1e-6 * np.max(np.abs(fd)))
    # Per-edge virial equals f.r over the model forces when every endpoint is a real row.
    assert np.allclose(ghost.virial, oracle.virial_fdotr(pos, ghost.model_force), rtol=1e-12,
                       atol=1e-12)


def test_setfl_f32_matches_reference(oracle):
    g = golden("golden_tiny_setfl.npz")
    tables = oracle.load_setfl(GOLDEN / "tiny.eam.alloy")
    pos, spc, s, r = g["positions"], g["species"], g["senders"], g["receivers"]
    rows = _model(oracle, tables, pos, spc, s, r, "rows-full", np.float32)
    np.testing.assert_allclose(rows.atom_energy, g["energy_f32"], rtol=1e-5, atol=1e-5)
    ref = g["edge_force_f32"]
    np.testing.assert_allclose(rows.edge_force, ref, rtol=0, atol=f32_force_tol(ref))
    np.testing.assert_allclose(rows.model_force, g["native_forces"], rtol=0,
                               atol=f32_force_tol(g["native_forces"]))


@pytest.mark.parametrize("tag,dtype", [("f64", np.float64), ("f32", np.float32)])
def test_half_pairing_matches_reference(oracle, tag, dtype):
    g = golden("golden_tiny_setfl.npz")
    tables = oracle.load_setfl(GOLDEN / "tiny.eam.alloy")
    pos, spc = g["half_positions"], g["half_species"]
    hs, hr = g["half_senders"], g["half_receivers"]
    half = _model(oracle, tables, pos, spc, hs, hr, "half-unique", dtype)
    full = _model(oracle, tables, pos, spc, g["full_senders"], g["full_receivers"], "rows-full",
                  dtype)
    rel = 1e-12 if dtype == np.float64 else 1e-5
    # Totals agree with the reference's half and full builders and with each other
    # (test_half_edges_match_full_pairing, test_eam.py:467-508).
    assert half.energy == pytest.approx(float(np.sum(g[f"half_energy_{tag}"])), rel=rel)
    assert full.energy == pytest.approx(float(np.sum(g[f"half_full_energy_{tag}"])), rel=rel)
    ref = g[f"half_edge_force_{tag}"]
    atol = 1e-12 * np.max(np.abs(ref)) if dtype == np.float64 else f32_force_tol(ref)
    np.testing.assert_allclose(half.edge_force, ref, rtol=0, atol=atol)
    np.testing.assert_allclose(half.model_force, full.model_force, rtol=0,
                               atol=atol * 10 if dtype == np.float64 else atol)


@pytest.mark.skipif(not CUZR_TABLE.exists(), reason="CuZr table lives in the reference checkout")
@pytest.mark.parametrize("tag,dtype", [("f64", np.float64), ("f32", np.float32)])
def test_cuzr_cluster_matches_reference(oracle, tag, dtype):
    g = golden("golden_cuzr_cluster.npz")
    tables = oracle.load_setfl(CUZR_TABLE)
    np.testing.assert_array_equal(tables["density"][:, 1000], g["density_row1000"])
    np.testing.assert_array_equal(tables["pair"][:, 1000], g["pair_row1000"])
    np.testing.assert_array_equal(tables["embedding"][:, 500], g["embedding_row500"])
    pos = g["positions"].astype(np.float64)
    out = _model(oracle, tables, pos, g["species"], g["senders"], g["receivers"], "rows-full",
                 dtype)
    ref_e, ref_f = g[f"energy_{tag}"], g[f"edge_force_{tag}"]
    if dtype == np.float64:
        np.testing.assert_allclose(out.atom_energy, ref_e, rtol=1e-12, atol=1e-12)
        np.testing.assert_allclose(out.edge_force, ref_f, rtol=0,
                                   atol=1e-12 * np.max(np.abs(ref_f)))
        assert out.energy == pytest.approx(float(g["native_energy"]), rel=1e-12)
        np.testing.assert_allclose(out.model_force, g["native_forces"], rtol=0, atol=1e-10)
    else:
        np.testing.assert_allclose(out.atom_energy, ref_e, rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(out.edge_force, ref_f, rtol=0, atol=f32_force_tol(ref_f))


@pytest.mark.parametrize("tag,dtype", [("f64", np.float64), ("f32", np.float32)])
@pytest.mark.parametrize("scale", [0.5, 1.0])
def test_lj_matches_reference(oracle, tag, dtype, scale):
    g = golden("golden_lj.npz")
    pos = g["positions"]
    s, r = g["senders"], g["receivers"]
    atom_energy, edge_force, model_force, energy, _ = oracle.lj_model(
        1.0, 1.0, float(g["cutoff"]), scale, pos, pos.shape[0], 0, s, r,
        np.ones(len(s), np.uint8), 0.5, dtype=dtype)
    ref = g[f"energy_{tag}_s{scale}"]
    rel = 1e-12 if dtype == np.float64 else 2e-6
    np.testing.assert_allclose(atom_energy, ref, rtol=rel, atol=rel * np.max(np.abs(ref)))
    if dtype == np.float64 and scale == 0.5:
        fd = g["fd_forces_s0.5"]
        np.testing.assert_allclose(model_force, fd, rtol=0, atol=1e-5 * np.max(np.abs(fd)))
        # Full list: summing per-edge dU/drij at the senders gives the same atom forces.
        summed = sum_sender_forces(edge_force, s, pos.shape[0])
        np.testing.assert_allclose(summed, model_force, rtol=0, atol=1e-9 * np.max(np.abs(fd)))
