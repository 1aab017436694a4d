"""Owned pairs held once (the default for EAM full lists with newton off).

The density pass keeps, per row i, the owned neighbors j > i and every ghost; each owned pair's
density share and force reach the neighbor's row by atomics (Newton's third law), and its energy
and virial count for both directions. The kept pairs, forces, energy, virial and edge count are
those of evaluating every pair from both rows (LJX_OWNED_HALF=0), to rounding: the engine's
float64 contract (forces 1e-10 of max |F|, totals 1e-12) with a margin, checked here at 1e-13.
Covered: float64 and float32, one and two species, over the candidate cache and over the list
(neighbor->ago < 0), and the fallback to full rows when some owned atom has no list row.
"""

import numpy as np
import pytest
import torch

from cases import F64_TOTAL_REL, eam_case, host_list
from test_gpu_parity import oracle_step, run_pair

pytestmark = pytest.mark.gpu


def step(tmp_path, case, precision, ago, owned_half, monkeypatch, inum=None):
    monkeypatch.setenv("LJX_OWNED_HALF", owned_half)
    pair, system, _ = run_pair(tmp_path, case, "rows-full", precision)
    if inum is not None:
        system.list.inum = inum
    system.list.ago = ago
    system.f.zero_()
    res = pair.compute(system, eflag=True, vflag=True)
    torch.cuda.synchronize()
    return system, res


@pytest.mark.parametrize("ago", [0, -1])
@pytest.mark.parametrize("elements", [("Cu",), ("Cu", "Zr")])
@pytest.mark.parametrize("precision", ["float64", "float32"])
def test_owned_pairs_once_equal_both_rows(tmp_path, oracle, monkeypatch, precision, elements,
                                          ago):
    case = eam_case(elements=elements, cells=(5, 5, 5), seed=41, nr=2000, nrho=2000)
    sys_b, both = step(tmp_path, case, precision, ago, "0", monkeypatch)
    f_both = sys_b.f[: case.nlocal].cpu().numpy().copy()
    sys_o, once = step(tmp_path, case, precision, ago, "1", monkeypatch)
    f_once = sys_o.f[: case.nlocal].cpu().numpy().copy()
    fmax = float(np.max(np.abs(f_both)))
    tol = 1e-13 if precision == "float64" else 1e-5
    assert float(np.max(np.abs(f_once - f_both))) <= tol * fmax
    trel = 1e-13 if precision == "float64" else 1e-5
    assert once.energy == pytest.approx(both.energy, rel=trel)
    vs = float(np.max(np.abs(both.virial)))
    assert float(np.max(np.abs(np.array(once.virial) - np.array(both.virial)))) <= trel * vs
    assert once.edge_count == both.edge_count and once.widest_row == both.widest_row
    assert once.overflow == 0
    if precision == "float64":
        ref = oracle_step(oracle, case, sys_o, "rows-full", precision)
        assert float(np.max(np.abs(f_once - ref.forces))) <= 1e-10 * float(np.max(np.abs(ref.forces)))
        assert once.energy == pytest.approx(ref.energy, rel=F64_TOTAL_REL)
        assert once.edge_count == ref.count


def test_rows_missing_from_the_list_keep_full_rows(tmp_path, monkeypatch):
    """A list that leaves some owned atoms without a row cannot hold owned pairs once (the
    lower atom's row may be missing): the engine keeps full rows, so both settings agree bit
    for bit."""
    case = eam_case(cells=(4, 4, 4), seed=17, nr=800, nrho=800)
    inum = case.nlocal - 7
    sys_b, both = step(tmp_path, case, "float64", 0, "0", monkeypatch, inum=inum)
    f_both = sys_b.f.cpu().numpy().copy()
    sys_o, once = step(tmp_path, case, "float64", 0, "1", monkeypatch, inum=inum)
    np.testing.assert_array_equal(sys_o.f.cpu().numpy(), f_both)
    assert once.energy == both.energy and once.edge_count == both.edge_count
    il, nn, _, _, _ = host_list(sys_o.list)
    assert int(nn[il[inum:case.nlocal]].sum()) > 0  # the dropped rows had neighbors
