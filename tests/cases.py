"""Shared builders for the parity tests: one seeded system, its bundle, and both evaluations.

A case is a periodic box owned by one rank: owned atoms first, then the ghost images LAMMPS
would create within the list cutoff (model cutoff + skin). The GPU path runs through libljx's C
ABI (PairJax -> ljx_* entry points); the CPU oracle (oracle/oracle.py) runs the reference's
per-step flow on the same coordinates and the same neighbor list.
"""

from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path

import numpy as np

from conftest import load_package

F64_FORCE_REL = 1e-10   # per-atom forces vs max-abs force (float64)
F64_TOTAL_REL = 1e-12   # total energy and virial (float64)
F32_FORCE_REL = 1e-5    # per-atom forces vs max-abs force (float32)
F32_TOTAL_REL = 1e-5    # total energy and virial (float32)


@dataclass
class Case:
    text: str
    x_all: np.ndarray
    types_all: np.ndarray
    nlocal: int
    owner: np.ndarray
    box: np.ndarray
    cutoff: float
    skin: float
    ntypes: int


def eam_case(elements=("Cu",), cells=(4, 4, 4), a=3.615, jitter=0.08, seed=1, skin=2.0,
             nr=5000, nrho=5000, fractions=None) -> Case:
    ljx = load_package()
    synth = ljx.synth
    text = synth.synthetic_setfl(elements, nr=nr, nrho=nrho)
    cutoff = 6.5
    n = 4 * cells[0] * cells[1] * cells[2]
    types = None
    if len(elements) > 1:
        types = synth.substitutional(n, fractions or (0.64, 0.36), seed=seed + 100)
    atoms = synth.fcc(cells, a, jitter=jitter, seed=seed, types=types)
    x_all, owner = synth.periodic_ghosts(atoms.x, atoms.box, cutoff + skin)
    types_all = np.concatenate([atoms.types, atoms.types[owner]]).astype(np.int32)
    return Case(text, x_all, types_all, len(atoms.x), owner, atoms.box, cutoff, skin,
                len(elements))


def write_eam_bundle(tmp_path: Path, case: Case, *, mode: str, precision: str,
                     edges_per_atom: int = 128, max_atoms=None, max_edges=None, scale_name="b"):
    ljx = load_package()
    nall = len(case.x_all)
    max_atoms = max_atoms or nall + 64
    kwargs = dict(potential=ljx.eam_potential(case.text), max_atoms=max_atoms,
                  cutoff=case.cutoff, unit_style="metal", precision=precision,
                  n_species=case.ntypes)
    if max_edges is None:
        max_edges = max_atoms * edges_per_atom
    if mode == "ghost":        # plain setfl export: full list, newton on, no exchange
        kwargs.update(force_output="atom-force", newton="on", max_edges=max_edges)
    elif mode == "rows-full":  # full list, newton off, F'(rho) forward exchange
        kwargs.update(force_output="atom-force", newton="off", max_edges=max_edges, comm=True)
    elif mode == "half-unique":  # half list, newton on, rho reverse + F' forward exchanges
        kwargs.update(force_output="atom-force", newton="on", max_edges=max_edges, comm=True,
                      half_edges=True)
    else:
        raise ValueError(mode)
    path = tmp_path / f"{scale_name}_{mode}_{precision}.json"
    ljx.write_bundle(path, **kwargs)
    return path


def device_system(case: Case, newton: bool, half: bool):
    import torch
    ljx = load_package()
    x = torch.as_tensor(case.x_all, device="cuda")
    t = torch.as_tensor(case.types_all, device="cuda")
    f = torch.zeros_like(x)
    nl = ljx.synth.neighbor_list(case.x_all, case.nlocal, case.cutoff + case.skin, half=half)
    comm = ljx.SelfComm(torch.as_tensor(case.owner, device="cuda"), case.nlocal)
    return ljx.System(x=x, type=t, f=f, nlocal=case.nlocal, nghost=len(case.x_all) - case.nlocal,
                      newton_pair=newton, unit_style="metal", ntypes=case.ntypes, list=nl,
                      comm=comm)


def host_list(nl):
    """(ilist, numneigh, neighbors, stride, maxneigh) numpy copy of a device NeighborList."""
    return (nl.ilist.cpu().numpy(), nl.numneigh.cpu().numpy(), nl.neighbors.cpu().numpy(),
            nl.slot_stride, nl.maxneighs)


def copy_device(ptr: int, count: int, dtype) -> np.ndarray:
    import torch
    ljx = load_package()
    nbytes = count * np.dtype(dtype).itemsize
    buf = torch.empty(max(nbytes, 1), dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    ljx.engine._cuda_memcpy_dtod(buf.data_ptr(), ptr, nbytes)
    return buf.cpu().numpy()[:nbytes].view(dtype).copy()


def rel_err(a, b, scale):
    return float(np.max(np.abs(np.asarray(a) - np.asarray(b)))) / max(float(scale), 1e-300)


def canonical_edges(senders, receivers):
    order = np.lexsort((senders, receivers))
    return senders[order], receivers[order]
