"""The allocation-free LJ entry point against the engine path (GPU).

ljx_lj_force_noalloc exists for callers that cannot call cudaMalloc (another framework holds
the device memory, e.g. JAX/XLA preallocation, or the caller must stay inside a memory pool it
does not own). It runs the engine's LJ kernels with scratch in a fixed device array inside the
library, so this test checks it against ljx_force on the same lj/cut bundle, in each force
distribution an lj/cut bundle can ask for, twice in a row (the array keeps the previous call's
contents), that further calls leave the device's free memory unchanged, and that oversize
systems are refused. This file sorts last so a run that stops at the first failure has run
every other test first.
"""

import ctypes

import numpy as np
import pytest
import torch

from conftest import load_package

pytestmark = pytest.mark.gpu

# name -> (force_output, newton_pair, half list): the three distributions ljx_lj_force_noalloc
# selects (edge forces on a full list, edge forces on a half list with newton on, atom forces).
MODES = {
    "edge-newton-off": ("edge-force", False, False),
    "edge-newton-on": ("edge-force", True, True),
    "atom-newton-on": ("atom-force", True, False),
}


def lj_system(ljx, cells=(8, 8, 4), density=0.8442, jitter=0.05, seed=3, cutoff=2.5, skin=0.3):
    a = (4.0 / density) ** (1.0 / 3.0)
    atoms = ljx.synth.fcc(cells, a, jitter=0.0, seed=seed)
    rng = np.random.default_rng(seed)
    x = np.mod(atoms.x + rng.uniform(-jitter, jitter, atoms.x.shape), atoms.box)
    x_all, owner = ljx.synth.periodic_ghosts(x, atoms.box, cutoff + skin)
    return x_all, owner, len(x), cutoff, skin


@pytest.mark.parametrize("precision", ["float64", "float32"])
@pytest.mark.parametrize("mode", list(MODES))
def test_noalloc_lj_matches_engine(tmp_path, mode, precision):
    ljx = load_package()
    lib = ljx.load()
    force_output, newton, half = MODES[mode]
    x_all, owner, nlocal, cutoff, skin = lj_system(ljx)
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
    pair = ljx.PairJax()
    pair.coeff(system, "*", "*", str(path))
    assert bool(pair.init_style(system)["half_list"]) == half
    ref = pair.compute(system)
    torch.cuda.synchronize()
    # Every row, ghosts included: newton-on modes leave ghost partials for the reverse comm.
    f_ref = system.f.clone()

    prec = ljx.abi.FLOAT64 if precision == "float64" else ljx.abi.FLOAT32
    layout = ljx.abi.FORCE_EDGE if force_output == "edge-force" else ljx.abi.FORCE_ATOM
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    result = torch.zeros(9, dtype=torch.float64, device="cuda")
    atoms, nl = system.atoms(), system.list.struct()

    def call():
        return lib.ljx_lj_force_noalloc(stream, ctypes.byref(atoms), ctypes.byref(nl), 1.0, 1.0,
                                        cutoff, prec, layout, int(newton), 1.0,
                                        ctypes.c_void_p(result.data_ptr()))

    fmax = float(f_ref.abs().max())
    frel = 1e-10 if precision == "float64" else 1e-5
    trel = 1e-12 if precision == "float64" else 1e-5
    vscale = max(abs(v) for v in ref.virial)
    for k in range(2):
        system.f.zero_()
        status = call()
        assert status == ljx.abi.OK, (k, status)
        torch.cuda.synchronize()
        assert float((system.f - f_ref).abs().max()) <= frel * fmax, k
        r = result.cpu().numpy()
        assert r[0] == pytest.approx(ref.energy, rel=trel), k
        assert np.max(np.abs(r[1:7] - np.array(ref.virial))) <= trel * vscale, k
        assert int(r[7]) == ref.edge_count and int(r[8]) == ref.widest_row, k

    # Nothing is allocated per call: after the calls above (every kernel already loaded), more
    # calls leave the device's free memory where it was.
    free_before = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        assert call() == ljx.abi.OK
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before


def test_noalloc_refuses_oversize_systems():
    ljx = load_package()
    lib = ljx.load()
    f = torch.zeros(1, 3, dtype=torch.float64, device="cuda")
    atoms = ljx.abi.Atoms(0, 0, f.data_ptr(), 40000, 1000)
    nl = ljx.abi.NeighList(0, 0, 0, 1, 40000, 40000, 0, 1)
    result = torch.zeros(9, dtype=torch.float64, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    status = lib.ljx_lj_force_noalloc(stream, ctypes.byref(atoms), ctypes.byref(nl), 1.0, 1.0,
                                      2.5, ljx.abi.FLOAT64, ljx.abi.FORCE_EDGE, 0, 1.0,
                                      ctypes.c_void_p(result.data_ptr()))
    assert status == ljx.abi.ERR_CAPACITY
