"""CPU ORACLE — TEST INFRASTRUCTURE ONLY.

Python side of the CPU restatement of the lammps-jax reference's EAM/LJ force path. Only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg import this module,
and only as the checker (or as the labelled CPU stand-in for the reference's own CPU path). The
product package never imports it.

The arithmetic lives in ``eam_oracle.c`` (built into ``liboracle.so`` by ``oracle/Makefile``);
this module parses setfl files (a restatement of python/lammps_jax/eam.py:174-262), wraps the C
routines with numpy arrays, and strings them into the pair style's per-step flow
(cpp/pair_jax_kokkos.cpp:989-1102) for one rank whose ghosts are periodic images.
Parity is pinned against vectors produced by the reference itself: see tests/golden/.
"""

from __future__ import annotations

import ctypes
import gzip
import os
import subprocess
from dataclasses import dataclass
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

FUNCFL_Z2R_SCALE = 27.2 * 0.529  # Hartree*Bohr -> eV*Angstrom (eam.py:230)

_lib = None


def build() -> Path:
    """Compile liboracle.so with the committed Makefile (gcc; no GPU needed)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        _lib = ctypes.CDLL(str(LIB_PATH))
    return _lib


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None else None


# ---------------------------------------------------------------------------------------------
# Tables (eam.py:115-262)
# ---------------------------------------------------------------------------------------------

def spline_coefficients(values) -> np.ndarray:
    """(n, 4) cubic coefficients of a uniform table: eam.py:115-135, via the C restatement."""
    f = np.ascontiguousarray(values, dtype=np.float64)
    out = np.empty((f.size, 4), np.float64)
    lib().orc_spline_coefficients(_p(f), ctypes.c_int(f.size), _p(out))
    return out


def read_table_lines(path) -> list[str]:
    opener = gzip.open if str(path).endswith(".gz") else open
    with opener(path, "rt") as handle:
        return handle.read().splitlines()


def parse_setfl_text(text: str, name: str = "<setfl>") -> dict:
    """DYNAMO setfl (eam/alloy) tables: a restatement of eam.py:174-227.

    Three comment lines; then element count and names, then nrho drho nr dr cutoff, then per
    element a header line (number, mass, lattice constant, lattice), F(rho) and rho(r); then the
    lower triangle of r*phi tables in file order.
    """
    lines = text.splitlines()
    tokens = " ".join(lines[3:]).split()
    n_el = int(tokens[0])
    elements = tokens[1:1 + n_el]
    pos = 1 + n_el
    nrho, drho, nr, dr, cutoff = tokens[pos:pos + 5]
    nrho, nr = int(nrho), int(nr)
    drho, dr, cutoff = float(drho), float(dr), float(cutoff)
    pos += 5
    masses, embedding, density = [], [], []
    for _ in range(n_el):
        masses.append(float(tokens[pos + 1]))
        pos += 4
        embedding.append(spline_coefficients(np.array(tokens[pos:pos + nrho], np.float64)))
        pos += nrho
        density.append(spline_coefficients(np.array(tokens[pos:pos + nr], np.float64)))
        pos += nr
    pair = []
    pair_index = np.zeros((n_el, n_el), np.int32)
    for i in range(n_el):
        for j in range(i + 1):
            pair_index[i, j] = pair_index[j, i] = len(pair)
            pair.append(spline_coefficients(np.array(tokens[pos:pos + nr], np.float64)))
            pos += nr
    if pos != len(tokens):
        raise ValueError(f"{name}: {len(tokens) - pos} unparsed trailing values")
    return dict(elements=elements, masses=masses, nrho=nrho, drho=drho, nr=nr, dr=dr,
                cutoff=cutoff, embedding=np.stack(embedding), density=np.stack(density),
                pair=np.stack(pair), pair_index=pair_index)


def load_setfl(path) -> dict:
    return parse_setfl_text("\n".join(read_table_lines(path)), str(path))


def load_funcfl(path) -> dict:
    """Single-element funcfl: eam.py:233-262 (Z(r) becomes r*phi = 27.2*0.529*Z^2)."""
    lines = read_table_lines(path)
    mass = float(lines[1].split()[1])
    tokens = " ".join(lines[2:]).split()
    nrho, nr = int(tokens[0]), int(tokens[2])
    drho, dr, cutoff = float(tokens[1]), float(tokens[3]), float(tokens[4])
    values = np.array(tokens[5:], np.float64)
    if values.size != nrho + 2 * nr:
        raise ValueError(f"{path}: expected {nrho + 2 * nr} table values, got {values.size}")
    z = values[nrho:nrho + nr]
    return dict(elements=[str(path).rsplit("/", 1)[-1].split(".")[0]], masses=[mass],
                nrho=nrho, drho=drho, nr=nr, dr=dr, cutoff=cutoff,
                embedding=spline_coefficients(values[:nrho])[None],
                density=spline_coefficients(values[nrho + nr:])[None],
                pair=spline_coefficients(FUNCFL_Z2R_SCALE * z * z)[None],
                pair_index=np.zeros((1, 1), np.int32))


def spline_eval(coeffs, x, delta, extrapolate=False, derivative=False, dtype=np.float64):
    """eam.py:138-164 on one table, at contract precision `dtype`."""
    c = np.ascontiguousarray(coeffs, dtype)
    xs = np.ascontiguousarray(np.atleast_1d(x), dtype)
    out = np.empty_like(xs)
    fn = lib().orc_spline_eval_f64 if dtype == np.float64 else lib().orc_spline_eval_f32
    real = ctypes.c_double if dtype == np.float64 else ctypes.c_float
    fn(_p(c), ctypes.c_int(c.shape[0]), _p(xs), ctypes.c_int(xs.size), real(delta),
       ctypes.c_int(int(extrapolate)), ctypes.c_int(int(derivative)), _p(out))
    return out


# ---------------------------------------------------------------------------------------------
# Pair-style flow (cpp/pair_jax_kokkos.cpp)
# ---------------------------------------------------------------------------------------------

NEIGHMASK = 0x1FFFFFFF


def build_list(x, nlocal, cutoff, half=False, maxneigh=None):
    """Owned-row neighbor list in LAMMPS/Kokkos LayoutLeft (neighbors[i + jj*stride]).

    Returns (ilist, numneigh, neighbors_flat, stride, maxneigh). Pairs strictly inside `cutoff`
    (list cutoff = model cutoff + skin); `half` keeps each pair once (owned j > i, or a ghost j
    ordered after i in (z, y, x)).
    """
    x = np.ascontiguousarray(x, np.float64)
    nall = x.shape[0]
    if maxneigh is None:
        maxneigh = 64
        while True:
            out = build_list(x, nlocal, cutoff, half, maxneigh)
            if out[1].max(initial=0) < maxneigh:
                return out
            maxneigh *= 2
    stride = max(nlocal, 1)
    neighbors = np.full(stride * maxneigh, 0, np.int32)
    numneigh = np.zeros(max(nall, 1), np.int32)
    widest = lib().orc_build_list(_p(x), ctypes.c_int(nall), ctypes.c_int(nlocal),
                                  ctypes.c_double(cutoff), ctypes.c_int(int(half)),
                                  _p(neighbors), ctypes.c_long(stride), ctypes.c_int(maxneigh),
                                  _p(numneigh))
    if widest > maxneigh:
        numneigh[:nlocal] = np.minimum(numneigh[:nlocal], maxneigh)
    ilist = np.arange(nlocal, dtype=np.int32)
    return ilist, numneigh, neighbors, stride, maxneigh


def pack_edges(x, ilist, numneigh, neighbors, atom_stride, slot_stride, num_rows, maxneighs,
               max_atoms, max_edges, cutoff, half_edges=False, unique_boundary=False,
               duplicate_reverse_edges=False, nlocal=0):
    """cpp/pair_jax_kokkos.cpp:77-117 + :811-873. Returns (senders, receivers, mask, count,
    overflow) in row/slot order with the padding contract past `count`."""
    x = np.ascontiguousarray(x, np.float64)
    senders = np.empty(max_edges, np.int32)
    receivers = np.empty(max_edges, np.int32)
    mask = np.empty(max_edges, np.uint8)
    overflow = ctypes.c_int(0)
    count = lib().orc_pack_edges(
        _p(x), _p(np.ascontiguousarray(ilist, np.int32)),
        _p(np.ascontiguousarray(numneigh, np.int32)), _p(np.ascontiguousarray(neighbors, np.int32)),
        ctypes.c_long(atom_stride), ctypes.c_long(slot_stride), ctypes.c_int(num_rows),
        ctypes.c_int(maxneighs), ctypes.c_int(max_atoms), ctypes.c_int(max_edges),
        ctypes.c_double(cutoff * cutoff), ctypes.c_int(int(half_edges)),
        ctypes.c_int(int(unique_boundary)), ctypes.c_int(int(duplicate_reverse_edges)),
        ctypes.c_int(nlocal), _p(senders), _p(receivers), _p(mask), ctypes.byref(overflow))
    return senders, receivers, mask.astype(bool), int(count), int(overflow.value)


@dataclass
class ModelOutput:
    rho: np.ndarray
    fp: np.ndarray
    atom_energy: np.ndarray
    model_force: np.ndarray
    edge_force: np.ndarray
    energy: float
    virial: np.ndarray


EAM_MODES = {"ghost": 0, "rows-full": 1, "half-unique": 2}


def eam_model(tables, positions, species, nlocal, nghost, senders, receivers, mask, mode,
              owner=None, dtype=np.float64):
    """One model evaluation on packed edges (see orc_eam_model in eam_oracle_impl.h)."""
    n_rows = positions.shape[0]
    n_edges = senders.shape[0]
    real = ctypes.c_double if dtype == np.float64 else ctypes.c_float
    fn = lib().orc_eam_model_f64 if dtype == np.float64 else lib().orc_eam_model_f32
    emb = np.ascontiguousarray(tables["embedding"], dtype)
    den = np.ascontiguousarray(tables["density"], dtype)
    par = np.ascontiguousarray(tables["pair"], dtype)
    pos = np.ascontiguousarray(positions, dtype)
    spc = np.ascontiguousarray(species, np.int32)
    own = np.ascontiguousarray(owner if owner is not None else np.zeros(1), np.int32)
    out = ModelOutput(np.empty(n_rows, dtype), np.empty(n_rows, dtype), np.empty(n_rows, dtype),
                      np.empty((n_rows, 3), dtype), np.empty((n_edges, 3), dtype), 0.0,
                      np.empty(6))
    energy = ctypes.c_double(0)
    cutoff_sq = np.asarray(tables["cutoff"] * tables["cutoff"], dtype)
    fn(ctypes.c_int(len(tables["elements"])), ctypes.c_int(tables["nrho"]),
       ctypes.c_int(tables["nr"]), real(tables["drho"]), real(tables["dr"]), real(cutoff_sq),
       _p(emb), _p(den), _p(par), _p(pos), _p(spc), ctypes.c_int(n_rows), ctypes.c_int(nlocal),
       ctypes.c_int(nghost), _p(np.ascontiguousarray(senders, np.int32)),
       _p(np.ascontiguousarray(receivers, np.int32)), _p(np.ascontiguousarray(mask, np.uint8)),
       ctypes.c_int(n_edges), ctypes.c_int(EAM_MODES[mode]), _p(own), _p(out.rho), _p(out.fp),
       _p(out.atom_energy), _p(out.model_force), _p(out.edge_force), ctypes.byref(energy),
       _p(out.virial))
    out.energy = float(energy.value)
    return out


def lj_model(epsilon, sigma, cutoff, edge_energy_scale, positions, nlocal, nghost, senders,
             receivers, mask, virial_weight, dtype=np.float64):
    """examples/export_model.py:16-74 on packed edges (see orc_lj_model)."""
    n_rows = positions.shape[0]
    n_edges = senders.shape[0]
    real = ctypes.c_double if dtype == np.float64 else ctypes.c_float
    fn = lib().orc_lj_model_f64 if dtype == np.float64 else lib().orc_lj_model_f32
    pos = np.ascontiguousarray(positions, dtype)
    atom_energy = np.empty(n_rows, dtype)
    edge_force = np.empty((n_edges, 3), dtype)
    model_force = np.empty((n_rows, 3), dtype)
    virial = np.empty(6)
    energy = ctypes.c_double(0)
    # Python-double constants cast to the contract dtype, as jnp.asarray(...) does (:24-26).
    fn(real(np.asarray(4.0 * epsilon, dtype)), real(np.asarray(sigma * sigma, dtype)),
       real(np.asarray(cutoff * cutoff, dtype)), real(np.asarray(edge_energy_scale, dtype)),
       _p(pos), ctypes.c_int(n_rows), ctypes.c_int(nlocal), ctypes.c_int(nghost),
       _p(np.ascontiguousarray(senders, np.int32)), _p(np.ascontiguousarray(receivers, np.int32)),
       _p(np.ascontiguousarray(mask, np.uint8)), ctypes.c_int(n_edges),
       ctypes.c_double(virial_weight), _p(atom_energy), _p(edge_force), _p(model_force),
       ctypes.byref(energy), _p(virial))
    return atom_energy, edge_force, model_force, float(energy.value), virial


def virial_fdotr(x, f):
    """cpp/pair_jax_kokkos.cpp:228-245 over all rows given."""
    x = np.ascontiguousarray(x, np.float64)
    f = np.ascontiguousarray(f, np.float64)
    v = np.empty(6)
    lib().orc_virial_fdotr(_p(x), _p(f), ctypes.c_int(x.shape[0]), _p(v))
    return v


def set_threads(n: int) -> None:
    lib().orc_set_num_threads(ctypes.c_int(n))


def num_threads() -> int:
    return int(lib().orc_num_threads())


@dataclass
class StepResult:
    forces: np.ndarray      # owned-row LAMMPS forces after the step (and reverse comm)
    f_all: np.ndarray       # LAMMPS f over all rows before the LAMMPS reverse comm
    energy: float           # scale * E as added to eng_vdwl
    virial: np.ndarray      # pair virial (fdotr for newton on; per-edge for newton off)
    rho: np.ndarray
    fp: np.ndarray
    count: int
    overflow: int
    senders: np.ndarray
    receivers: np.ndarray
    mask: np.ndarray


def eam_step(tables, x, types, nlocal, owner, list_, *, mode, precision="float64",
             max_atoms=None, max_edges=None, scale=1.0):
    """One pair-style compute (cpp/pair_jax_kokkos.cpp:989-1102) for an EAM bundle on one rank.

    mode: 'ghost' (plain bundle, full list, newton on), 'rows-full' (full list, newton off,
    forward comm of rho) or 'half-unique' (half-unique comm bundle, newton on). `list_` is the
    tuple build_list returns. Ghost rows are periodic images (owner[g]); after the pair style adds
    its forces, newton-on modes apply LAMMPS's reverse comm of ghost forces to owners.
    """
    dtype = np.float64 if precision == "float64" else np.float32
    nall = x.shape[0]
    nghost = nall - nlocal
    max_atoms = max_atoms or nall
    ilist, numneigh, neighbors, stride, maxneigh = list_
    if max_edges is None:
        max_edges = int(numneigh[:nlocal].sum()) + 1
    # The pair style hands half-unique bundles LAMMPS's native half list, which already holds
    # one direction per pair, so neither packer rule applies (pair_jax_kokkos.cpp:425-431,854-865).
    senders, receivers, mask, count, overflow = pack_edges(
        x, ilist, numneigh, neighbors, 1, stride, nlocal, maxneigh, max_atoms, max_edges,
        tables["cutoff"], nlocal=nlocal)
    positions = np.zeros((max_atoms, 3), dtype)
    species = np.zeros(max_atoms, np.int32)
    positions[:nall] = x.astype(dtype)
    species[:nall] = types - 1
    out = eam_model(tables, positions, species, nlocal, nghost, senders, receivers, mask, mode,
                    owner=owner, dtype=dtype)
    f = np.zeros((nall, 3))
    newton_on = mode != "rows-full"
    rows = nall if newton_on else nlocal
    f[:rows] += scale * out.model_force[:rows].astype(np.float64)
    if newton_on:
        virial = virial_fdotr(x, f)
    else:
        virial = scale * out.virial
    f_all = f.copy()
    if newton_on:
        np.add.at(f, np.asarray(owner[:nghost]), f[nlocal:nall])
    return StepResult(f[:nlocal].copy(), f_all, scale * out.energy, virial, out.rho, out.fp,
                      count, overflow, senders, receivers, mask)


def lj_step(x, nlocal, owner, list_, *, epsilon, sigma, cutoff, force_output="edge-force",
            newton_pair=False, precision="float64", max_atoms=None, max_edges=None, scale=1.0,
            pair_sum=False):
    """One pair-style compute for an LJ bundle (examples/export_model.py + pair_jax_kokkos.cpp).

    Edge-force bundles add dU/drij to the sender and, with newton on, subtract it from the
    receiver (AddEdgeForcesFunctor, :195-225); atom-force bundles add the autodiff forces of the
    0.5-per-edge energy over all rows (AddForcesFunctor, newton on). The per-edge energy scale
    follows export_lj (:107). Newton-on runs take the f.r virial over all rows, then fold ghost
    forces into owners; newton-off runs report the per-edge virial.
    """
    dtype = np.float64 if precision == "float64" else np.float32
    nall = x.shape[0]
    nghost = nall - nlocal
    max_atoms = max_atoms or nall
    ilist, numneigh, neighbors, stride, maxneigh = list_
    edge = force_output == "edge-force"
    duplicate = bool(newton_pair and pair_sum and not edge)
    if max_edges is None:
        max_edges = 2 * int(numneigh[:nlocal].sum()) + 1
    senders, receivers, mask, count, overflow = pack_edges(
        x, ilist, numneigh, neighbors, 1, stride, nlocal, maxneigh, max_atoms, max_edges, cutoff,
        duplicate_reverse_edges=duplicate, nlocal=nlocal)
    positions = np.zeros((max_atoms, 3), dtype)
    positions[:nall] = x.astype(dtype)
    escale = 1.0 if (edge and newton_pair) else 0.5
    atom_energy, edge_force, model_force, energy, virial_edge = lj_model(
        epsilon, sigma, cutoff, escale, positions, nlocal, nghost, senders, receivers, mask,
        1.0 if newton_pair else 0.5, dtype=dtype)
    f = np.zeros((nall, 3))
    if edge:
        c = min(count, max_edges)
        fe = scale * edge_force[:c].astype(np.float64)
        np.add.at(f, senders[:c], fe)
        if newton_pair:
            np.add.at(f, receivers[:c], -fe)
    else:
        rows = nall if newton_pair else nlocal
        f[:rows] += scale * model_force[:rows].astype(np.float64)
    virial = virial_fdotr(x, f) if newton_pair else scale * virial_edge
    f_all = f.copy()
    if newton_pair:
        np.add.at(f, np.asarray(owner[:nghost]), f[nlocal:nall])
    return StepResult(f[:nlocal].copy(), f_all, scale * energy, virial, None, None, count,
                      overflow, senders, receivers, mask)
