"""GPU parity of the row-group candidate cache across steps (ljx_list.ago).

The engine caches, per group of 8 list rows, the union of their neighbors within rc plus a
margin of 8 % of rc when LAMMPS reports a fresh list (ago == 0), and reuses it while ago > 0.
It rebuilds on the device once some atom has moved more than half the margin. Each case moves
the atoms between steps on the same LAMMPS list and checks the step against the oracle at the
new positions. Tolerances are the engine's contract (float64 forces 1e-10 of max |F|, energy
and virial 1e-12 relative).
"""

import numpy as np
import pytest
import torch

from cases import eam_case, host_list
from conftest import load_package
from test_gpu_parity import MODE_SETUP, assert_parity, oracle_step, run_pair

pytestmark = pytest.mark.gpu

MARGIN = 0.08  # kGroupMargin in csrc/engine.cu: fraction of rc


def owners_of_all(case):
    return np.concatenate([np.arange(case.nlocal), case.owner])


def moved_case(case, shift):
    """The case with every owned atom shifted by shift[i] and its ghost images with it."""
    x_all = case.x_all + shift[owners_of_all(case)]
    return type(case)(**{**case.__dict__, "x_all": x_all})


def step_again(pair, system, case, ago):
    system.x.copy_(torch.as_tensor(case.x_all, device="cuda"))
    system.f.zero_()
    system.list.ago = ago
    res = pair.compute(system, eflag=True, vflag=True)
    if system.newton_pair:
        system.comm.reverse_forces(system.f)
    torch.cuda.synchronize()
    return res


@pytest.mark.parametrize("mode", ["rows-full", "ghost", "half-unique"])
def test_cached_steps_follow_small_moves(tmp_path, oracle, mode):
    case = eam_case(elements=("Cu", "Zr"), cells=(5, 5, 5), seed=31, nr=2000, nrho=2000)
    pair, system, res = run_pair(tmp_path, case, mode, "float64")
    assert_parity(res, system, oracle_step(oracle, case, system, mode, "float64"), "float64", case)
    rng = np.random.default_rng(5)
    limit = 0.5 * MARGIN * case.cutoff
    for ago in (1, 2, 3):
        # Random moves below half the margin: the cached unions stay valid.
        d = rng.normal(size=(case.nlocal, 3))
        d *= (0.9 * limit * rng.random((case.nlocal, 1))) / np.linalg.norm(d, axis=1, keepdims=True)
        case = moved_case(case, d)
        res = step_again(pair, system, case, ago)
        ref = oracle_step(oracle, case, system, mode, "float64")
        assert_parity(res, system, ref, "float64", case)


@pytest.mark.parametrize("mode", ["rows-full", "half-unique"])
def test_large_move_rebuilds_on_device(tmp_path, oracle, mode):
    """One atom jumps past half the margin toward a listed partner that lay outside rc + margin
    when the cache was built. Only a rebuild can find the pair, so the step matches the oracle
    only if the device rebuilt the unions."""
    case = eam_case(cells=(5, 5, 5), seed=37, nr=2000, nrho=2000)
    pair, system, res = run_pair(tmp_path, case, mode, "float64")
    il, nn, nb, stride, maxn = host_list(system.list)
    rc = case.cutoff
    a = 0
    listed = nb[a + np.arange(nn[a]) * stride]
    dist = np.linalg.norm(case.x_all[listed] - case.x_all[a], axis=1)
    far = listed[(dist > rc * (1 + MARGIN) + 0.05) & (dist < rc * (1 + MARGIN) + 0.4)]
    assert len(far) > 0
    b = int(far[0])
    v = case.x_all[b] - case.x_all[a]
    r = float(np.linalg.norm(v))
    shift = np.zeros((case.nlocal, 3))
    shift[a] = v / r * (r - (rc - 0.2))  # now 0.2 A inside the cutoff
    assert np.linalg.norm(shift[a]) > 0.5 * MARGIN * rc
    case = moved_case(case, shift)
    res = step_again(pair, system, case, ago=1)
    ref = oracle_step(oracle, case, system, mode, "float64")
    assert_parity(res, system, ref, "float64", case)


@pytest.mark.parametrize("mode", ["rows-full", "ghost", "half-unique"])
def test_cache_off_walks_the_list(tmp_path, oracle, mode):
    """ago < 0: every step filters the whole list (no cache)."""
    ljx = load_package()
    case = eam_case(elements=("Cu", "Zr"), cells=(5, 5, 5), seed=41, nr=2000, nrho=2000)
    newton, half = MODE_SETUP[mode]
    from cases import device_system, write_eam_bundle
    path = write_eam_bundle(tmp_path, case, mode=mode, precision="float64")
    system = device_system(case, newton=newton, half=half)
    system.list.ago = -1
    pair = ljx.PairJax(device=0)
    pair.settings()
    pair.coeff(system, "*", "*", str(path))
    pair.init_style(system)
    res = pair.compute(system, eflag=True, vflag=True)
    if newton:
        system.comm.reverse_forces(system.f)
    torch.cuda.synchronize()
    assert_parity(res, system, oracle_step(oracle, case, system, mode, "float64"), "float64", case)


def test_cache_policy_over_list_ages(tmp_path, oracle):
    """The engine caches candidates for a fresh list only if the previous list lived at least 4
    steps; otherwise that list's steps take the list pass. A sequence with long lists, a list of
    one step and the switch back covers cached, rebuilt and list-pass steps; every step matches
    the oracle."""
    case = eam_case(elements=("Cu", "Zr"), cells=(5, 5, 5), seed=43, nr=2000, nrho=2000)
    pair, system, res = run_pair(tmp_path, case, "rows-full", "float64")
    rng = np.random.default_rng(9)
    limit = 0.5 * MARGIN * case.cutoff
    for ago in (1, 2, 3, 4, 0, 1, 2, 3, 4, 0, 0, 1, 2, 3, 4, 0, 1):
        d = rng.normal(size=(case.nlocal, 3))
        d *= (0.2 * limit * rng.random((case.nlocal, 1))) / np.linalg.norm(d, axis=1, keepdims=True)
        case = moved_case(case, d)
        res = step_again(pair, system, case, ago)
        ref = oracle_step(oracle, case, system, "rows-full", "float64")
        assert_parity(res, system, ref, "float64", case)


def test_spilled_groups_walk_their_lists(tmp_path, oracle):
    """A compacted row capacity of 40 gives every group a union capacity of 160 and a row
    candidate capacity of 80, which C3-density rows (about 108 candidates) exceed: every group is
    past capacity, and the cached steps walk the rows' lists instead."""
    case = eam_case(cells=(5, 5, 5), seed=47, nr=2000, nrho=2000)
    nall = len(case.x_all)
    pair, system, res = run_pair(tmp_path, case, "rows-full", "float64",
                                 max_atoms=nall + 64, max_edges=(nall + 64) * 40)
    assert_parity(res, system, oracle_step(oracle, case, system, "rows-full", "float64"),
                  "float64", case)
    rng = np.random.default_rng(3)
    limit = 0.5 * MARGIN * case.cutoff
    for ago in (1, 2):
        d = rng.normal(size=(case.nlocal, 3))
        d *= (0.5 * limit * rng.random((case.nlocal, 1))) / np.linalg.norm(d, axis=1, keepdims=True)
        case = moved_case(case, d)
        res = step_again(pair, system, case, ago)
        assert_parity(res, system, oracle_step(oracle, case, system, "rows-full", "float64"),
                      "float64", case)


def test_cache_build_is_deterministic(tmp_path, monkeypatch):
    """The cache build numbers each union in first-seen order of one warp's walk over the
    group's lists, so a repeated run gives bitwise the same forces and energy on the build step
    and on the cached steps after it. (Full list, newton off, every pair evaluated from both of
    its rows (LJX_OWNED_HALF=0): every sum has a fixed order. Holding owned pairs once and the
    newton-on modes scatter to neighbors with atomics.)"""
    monkeypatch.setenv("LJX_OWNED_HALF", "0")
    mode = "rows-full"
    case = eam_case(elements=("Cu", "Zr"), cells=(5, 5, 5), seed=53, nr=2000, nrho=2000)
    rng = np.random.default_rng(8)
    limit = 0.5 * MARGIN * case.cutoff
    moves = []
    for _ in range(3):
        d = rng.normal(size=(case.nlocal, 3))
        d *= (0.5 * limit * rng.random((case.nlocal, 1))) / np.linalg.norm(d, axis=1, keepdims=True)
        moves.append(d)

    def run():
        pair, system, res = run_pair(tmp_path, case, mode, "float64")
        out = [(system.f[: case.nlocal].cpu().numpy().copy(), res.energy, tuple(res.virial))]
        c = case
        for ago, d in enumerate(moves, start=1):
            c = moved_case(c, d)
            r = step_again(pair, system, c, ago)
            out.append((system.f[: case.nlocal].cpu().numpy().copy(), r.energy, tuple(r.virial)))
        return out

    first, second = run(), run()
    for (fa, ea, va), (fb, eb, vb) in zip(first, second):
        np.testing.assert_array_equal(fa, fb)
        assert ea == eb and va == vb
