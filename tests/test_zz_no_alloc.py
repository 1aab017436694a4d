"""The allocation-free LJ entry point against the engine path (GPU).

ljx_lj_force_noalloc exists for callers that cannot call cudaMalloc (another framework holds
the device memory, e.g. JAX/XLA preallocation, or the caller must stay inside a memory pool it
does not own). It runs the engine's LJ kernels with scratch in a fixed device array inside the
library, so this test checks it against ljx_force on the same lj/cut bundle, twice in a row
(the array keeps the previous call's contents), and checks that oversize systems are refused.
This file sorts last so a run that stops at the first failure has run every other test first.
"""

import ctypes

import numpy as np
import pytest
import torch

from conftest import load_package

pytestmark = pytest.mark.gpu


def lj_system(ljx, cells=(8, 8, 4), density=0.8442, jitter=0.05, seed=3, cutoff=2.5, skin=0.3):
    a = (4.0 / density) ** (1.0 / 3.0)
    atoms = ljx.synth.fcc(cells, a, jitter=0.0, seed=seed)
    rng = np.random.default_rng(seed)
    x = np.mod(atoms.x + rng.uniform(-jitter, jitter, atoms.x.shape), atoms.box)
    x_all, owner = ljx.synth.periodic_ghosts(x, atoms.box, cutoff + skin)
    return x_all, owner, len(x), cutoff, skin


@pytest.mark.parametrize("precision", ["float64", "float32"])
def test_noalloc_lj_matches_engine(tmp_path, precision):
    ljx = load_package()
    lib = ljx.load()
    x_all, owner, nlocal, cutoff, skin = lj_system(ljx)
    nall = len(x_all)
    path = tmp_path / "lj.json"
    ljx.write_bundle(path, potential=ljx.lj_potential(1.0, 1.0), max_atoms=nall + 32,
                     max_edges=(nall + 32) * 96, cutoff=cutoff, unit_style="lj",
                     precision=precision, force_output="edge-force", newton="off")
    x = torch.as_tensor(x_all, device="cuda")
    system = ljx.System(x=x, type=torch.ones(nall, dtype=torch.int32, device="cuda"),
                        f=torch.zeros_like(x), nlocal=nlocal, nghost=nall - nlocal,
                        newton_pair=False, unit_style="lj", ntypes=1)
    system.list = ljx.synth.neighbor_list(x_all, nlocal, cutoff + skin, half=False)
    pair = ljx.PairJax()
    pair.coeff(system, "*", "*", str(path))
    pair.init_style(system)
    ref = pair.compute(system)
    torch.cuda.synchronize()
    f_ref = system.f.clone()

    prec = ljx.abi.FLOAT64 if precision == "float64" else ljx.abi.FLOAT32
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    result = torch.zeros(9, dtype=torch.float64, device="cuda")
    for call in range(2):
        system.f.zero_()
        atoms, nl = system.atoms(), system.list.struct()
        status = lib.ljx_lj_force_noalloc(stream, ctypes.byref(atoms), ctypes.byref(nl), 1.0, 1.0,
                                          cutoff, prec, ljx.abi.FORCE_EDGE, 0, 1.0,
                                          ctypes.c_void_p(result.data_ptr()))
        assert status == ljx.abi.OK, (call, status)
        torch.cuda.synchronize()
        fmax = float(f_ref.abs().max())
        frel = 1e-10 if precision == "float64" else 1e-5
        assert float((system.f - f_ref).abs().max()) <= frel * fmax, call
        r = result.cpu().numpy()
        trel = 1e-12 if precision == "float64" else 1e-5
        assert r[0] == pytest.approx(ref.energy, rel=trel), call
        vscale = max(abs(v) for v in ref.virial)
        assert np.max(np.abs(r[1:7] - np.array(ref.virial))) <= 10 * trel * vscale, call
        assert int(r[7]) == ref.edge_count and int(r[8]) == ref.widest_row, call


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
