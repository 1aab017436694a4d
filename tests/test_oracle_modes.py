"""CPU checks of the oracle's pair-style flow on periodic boxes (no GPU).

The three EAM distribution modes the engine implements — plain bundle on a full list with
newton on (ghost), full list with newton off and an F'(rho) forward exchange (rows-full), and
the half-unique half list with newton on (reverse rho, forward F') — must give the same owned
forces, energy and virial once LAMMPS's reverse comm has folded ghost forces into their owners.
An all-pairs minimum-image evaluation with the same splines is the independent referee.
"""

import numpy as np
import pytest

from cases import F64_FORCE_REL, F64_TOTAL_REL, eam_case

MODES = ["ghost", "rows-full", "half-unique"]


def run_mode(oracle, case, mode, precision="float64"):
    tables = oracle.parse_setfl_text(case.text)
    half = mode == "half-unique"
    lst = oracle.build_list(case.x_all, case.nlocal, case.cutoff + case.skin, half=half)
    return oracle.eam_step(tables, case.x_all, case.types_all, case.nlocal, case.owner, lst,
                           mode=mode, precision=precision)


def minimum_image_reference(oracle, case):
    """All-pairs EAM with minimum image (box > 2 cutoffs): energy, forces, virial."""
    t = oracle.parse_setfl_text(case.text)
    x = case.x_all[: case.nlocal]
    spc = case.types_all[: case.nlocal] - 1
    n = len(x)
    d = x[None, :, :] - x[:, None, :]          # d[i, j] = x_j - x_i
    d -= case.box * np.round(d / case.box)
    r = np.sqrt((d * d).sum(-1))
    np.fill_diagonal(r, np.inf)
    within = r < t["cutoff"]
    ii, jj = np.nonzero(within)
    rr = r[ii, jj]
    rho = np.zeros(n)
    for s in range(len(t["elements"])):
        sel = spc[jj] == s
        np.add.at(rho, ii[sel], oracle.spline_eval(t["density"][s], rr[sel], t["dr"]))
    energy = 0.0
    fp = np.zeros(n)
    for s in range(len(t["elements"])):
        sel = spc == s
        energy += oracle.spline_eval(t["embedding"][s], rho[sel], t["drho"], extrapolate=True).sum()
        fp[sel] = oracle.spline_eval(t["embedding"][s], rho[sel], t["drho"], extrapolate=True,
                                     derivative=True)
    psip = np.zeros_like(rr)
    phi = np.zeros_like(rr)
    for a in range(len(t["elements"])):
        for b in range(len(t["elements"])):
            sel = (spc[ii] == a) & (spc[jj] == b)
            if not sel.any():
                continue
            pr = t["pair_index"][a, b]
            z2 = oracle.spline_eval(t["pair"][pr], rr[sel], t["dr"])
            z2p = oracle.spline_eval(t["pair"][pr], rr[sel], t["dr"], derivative=True)
            ph = z2 / rr[sel]
            php = (z2p - ph) / rr[sel]
            rhojp = oracle.spline_eval(t["density"][b], rr[sel], t["dr"], derivative=True)
            rhoip = oracle.spline_eval(t["density"][a], rr[sel], t["dr"], derivative=True)
            psip[sel] = fp[ii[sel]] * rhojp + fp[jj[sel]] * rhoip + php
            phi[sel] = ph
    energy += 0.5 * phi.sum()
    fe = (psip / rr)[:, None] * d[ii, jj]
    forces = np.zeros((n, 3))
    np.add.at(forces, ii, fe)
    vir = -0.5 * np.einsum("e,ea,eb->ab", psip / rr, d[ii, jj], d[ii, jj])
    virial = np.array([vir[0, 0], vir[1, 1], vir[2, 2], vir[0, 1], vir[0, 2], vir[1, 2]])
    return energy, forces, virial


@pytest.mark.parametrize("elements", [("Cu",), ("Cu", "Zr")])
def test_modes_agree_with_minimum_image(oracle, elements):
    case = eam_case(elements=elements, cells=(4, 4, 4), seed=3, nr=800, nrho=800)
    e_ref, f_ref, v_ref = minimum_image_reference(oracle, case)
    fmax = np.max(np.abs(f_ref))
    for mode in MODES:
        out = run_mode(oracle, case, mode)
        assert np.max(np.abs(out.forces - f_ref)) <= F64_FORCE_REL * fmax, mode
        assert out.energy == pytest.approx(e_ref, rel=F64_TOTAL_REL), mode
        vscale = np.max(np.abs(v_ref))
        assert np.max(np.abs(out.virial - v_ref)) <= 1e-11 * vscale, (mode, out.virial, v_ref)


def test_pack_counts_and_padding(oracle):
    case = eam_case(cells=(4, 4, 4), seed=5, nr=800, nrho=800)
    out = run_mode(oracle, case, "rows-full")
    assert out.overflow == 0
    assert out.count == int(out.mask.sum())
    assert np.all(out.senders[out.count:] == len(case.x_all))
    assert np.all(out.receivers[out.count:] == len(case.x_all))
