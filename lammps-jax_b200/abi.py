"""ctypes binding of libljx.so (include/ljx.h, ljx_neigh.h, ljx_pair.h, ljx_md.h, ljx_halo.h).

The library is the product: there is no Python or CPU fallback. Loading fails loudly when the
shared object is missing or lacks a declared symbol.
"""

from __future__ import annotations

import ctypes
from ctypes import (POINTER, Structure, c_char, c_char_p, c_double, c_int, c_longlong, c_size_t,
                    c_uint8, c_void_p)
from pathlib import Path

from .build import LIB

MAX_COMM_WIDTHS = 16

OK, ERR_INVALID, ERR_CUDA, ERR_CAPACITY, ERR_BUNDLE, ERR_UNSUPPORTED = range(6)
LAYOUT_SPARSE_EDGE, LAYOUT_NEIGHBOR_MATRIX = 0, 1
FORCE_ATOM, FORCE_EDGE = 0, 1
NEWTON_ANY, NEWTON_ON, NEWTON_OFF = 0, 1, 2
FLOAT32, FLOAT64 = 0, 1
PAIRING_FULL, PAIRING_HALF, PAIRING_HALF_UNIQUE = 0, 1, 2
POTENTIAL_NONE, POTENTIAL_EAM, POTENTIAL_LJ = 0, 1, 2


class Contract(Structure):
    _fields_ = [
        ("input_layout", c_int), ("max_atoms", c_int), ("max_edges", c_int),
        ("max_neighbors", c_int), ("cutoff", c_double), ("unit_style", c_char * 16),
        ("precision", c_int), ("force_layout", c_int), ("newton", c_int), ("n_hops", c_int),
        ("half_edges", c_int), ("edge_pairing", c_int), ("n_comm_widths", c_int),
        ("comm_widths", c_int * MAX_COMM_WIDTHS), ("n_comm_sites", c_int),
        ("comm_sites", c_int * 3), ("uses_box", c_int), ("pair_sum", c_int),
        ("n_species", c_int), ("max_owned", c_int), ("format", c_char * 48),
        ("platform", c_char * 16), ("has_force_program", c_int), ("has_energy_program", c_int),
        ("has_energy_and_forces_program", c_int), ("potential", c_int), ("n_elements", c_int),
        ("lj_epsilon", c_double), ("lj_sigma", c_double), ("lj_edge_energy_scale", c_double),
    ]


class Atoms(Structure):
    _fields_ = [("x", c_void_p), ("type", c_void_p), ("f", c_void_p), ("nlocal", c_int),
                ("nghost", c_int)]


class NeighList(Structure):
    _fields_ = [("ilist", c_void_p), ("numneigh", c_void_p), ("neighbors", c_void_p),
                ("atom_stride", c_longlong), ("slot_stride", c_longlong), ("inum", c_int),
                ("gnum", c_int), ("maxneighs", c_int), ("ago", c_int)]


class Result(Structure):
    _fields_ = [("energy", c_double), ("virial", c_double * 6), ("edge_count", c_longlong),
                ("overflow", c_int), ("widest_row", c_int)]


COMM_FN = ctypes.CFUNCTYPE(c_int, c_void_p, c_void_p, c_int, c_int, c_void_p)
REDUCE_FN = ctypes.CFUNCTYPE(c_int, c_void_p, POINTER(c_int), c_int)


class PairHost(Structure):
    _fields_ = [("ctx", c_void_p), ("forward_comm", COMM_FN), ("reverse_comm", COMM_FN),
                ("allreduce_max", REDUCE_FN)]


HALO_ID_BYTES = 128
HALO_SELF_BY_NCCL = 1


class Swap(Structure):
    _fields_ = [("stage", c_int), ("send_rank", c_int), ("recv_rank", c_int),
                ("sendlist", c_void_p), ("sendnum", c_int), ("firstrecv", c_int),
                ("recvnum", c_int)]


class ResultAll(Structure):
    _fields_ = [("energy", c_double), ("virial", c_double * 6), ("edge_count", c_longlong),
                ("edge_max", c_longlong), ("overflow", c_int), ("widest_row", c_int),
                ("local_energy", c_double)]


EFLAG_GLOBAL, VFLAG_GLOBAL, EFLAG_ATOM, VFLAG_ATOM, EFLAG_ONLY = 1, 2, 4, 8, 16


class Plan(Structure):
    _fields_ = [("half_list", c_int), ("reverse_density", c_int), ("forward_fp", c_int),
                ("reverse_force", c_int), ("comm_width", c_int), ("comm_elem_bytes", c_int)]


# Every symbol the headers declare: (name, restype, argtypes).
ROWS_LOCAL = 1  # ljx_force_rows parts (include/ljx.h)
ROWS_GHOST = 2

SIGNATURES = [
    ("ljx_bundle_load", c_int, [c_char_p, POINTER(c_void_p)]),
    ("ljx_bundle_load_string", c_int, [c_char_p, c_size_t, POINTER(c_void_p)]),
    ("ljx_bundle_error", c_char_p, []),
    ("ljx_bundle_contract", c_int, [c_void_p, POINTER(Contract)]),
    ("ljx_bundle_eam_tables", c_int, [c_void_p, POINTER(c_int), POINTER(c_int), POINTER(c_int),
                                      POINTER(c_double), POINTER(c_double), POINTER(c_double),
                                      c_void_p, c_void_p, c_void_p]),
    ("ljx_bundle_free", None, [c_void_p]),
    ("ljx_engine_create", c_int, [c_void_p, c_int, POINTER(c_void_p)]),
    ("ljx_engine_destroy", None, [c_void_p]),
    ("ljx_engine_error", c_char_p, [c_void_p]),
    ("ljx_engine_plan", c_int, [c_void_p, c_int, POINTER(Plan)]),
    ("ljx_pack_atoms", c_int, [c_void_p, c_void_p, POINTER(Atoms)]),
    ("ljx_pack_edges", c_int, [c_void_p, c_void_p, POINTER(Atoms), POINTER(NeighList), c_int]),
    ("ljx_edges", c_int, [c_void_p, POINTER(c_void_p), POINTER(c_void_p), POINTER(c_void_p),
                          POINTER(c_int)]),
    ("ljx_density", c_int, [c_void_p, c_void_p, POINTER(Atoms), POINTER(NeighList), c_int]),
    ("ljx_embed", c_int, [c_void_p, c_void_p, POINTER(Atoms)]),
    ("ljx_force", c_int, [c_void_p, c_void_p, POINTER(Atoms), POINTER(NeighList), c_int,
                          c_double]),
    ("ljx_force_rows", c_int, [c_void_p, c_void_p, POINTER(Atoms), POINTER(NeighList), c_int,
                               c_double, c_int]),
    ("ljx_force_only", c_int, [c_void_p, c_void_p, POINTER(Atoms), POINTER(NeighList), c_int,
                               c_double]),
    ("ljx_force_to_host", c_int, [c_void_p, c_void_p, POINTER(Atoms), POINTER(NeighList), c_int,
                                  c_double, c_void_p, c_int]),
    ("ljx_energy", c_int, [c_void_p, c_void_p, POINTER(Atoms), POINTER(NeighList), c_int,
                           c_double]),
    ("ljx_read_result", c_int, [c_void_p, c_void_p, POINTER(Result)]),
    ("ljx_feature_rows", c_int, [c_void_p, c_int, POINTER(c_void_p), POINTER(c_int),
                                 POINTER(c_int)]),
    ("ljx_comm_pack_forward", c_int, [c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p,
                                      c_int]),
    ("ljx_comm_unpack_forward", c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p,
                                        c_int]),
    ("ljx_comm_pack_reverse", c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_int]),
    ("ljx_comm_unpack_reverse", c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_int,
                                        c_void_p, c_int]),
    ("ljx_comm_zero_rows", c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int]),
    ("ljx_halo_forward_self", c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_int, c_int]),
    ("ljx_halo_reverse_self", c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_int, c_int]),
    ("ljx_lj_force_noalloc", c_int, [c_void_p, POINTER(Atoms), POINTER(NeighList), c_double,
                                     c_double, c_double, c_int, c_int, c_int, c_double,
                                     c_void_p]),
    ("ljx_set_atom_tallies", c_int, [c_void_p, c_void_p, c_void_p, c_double]),
    ("ljx_engine_launches", c_longlong, [c_void_p]),
    ("ljx_pair_create", c_int, [c_int, POINTER(c_void_p)]),
    ("ljx_pair_destroy", None, [c_void_p]),
    ("ljx_pair_error", c_char_p, [c_void_p]),
    ("ljx_pair_settings", c_int, [c_void_p, c_int, POINTER(c_char_p)]),
    ("ljx_pair_coeff", c_int, [c_void_p, c_int, POINTER(c_char_p), c_char_p, c_int]),
    ("ljx_pair_init_style", c_int, [c_void_p, c_int, c_int, POINTER(c_double), POINTER(c_double),
                                    c_int, POINTER(c_char_p), POINTER(Plan)]),
    ("ljx_pair_init_one", c_double, [c_void_p]),
    ("ljx_pair_compute", c_int, [c_void_p, c_void_p, POINTER(Atoms), POINTER(NeighList), c_int,
                                 c_int, POINTER(PairHost), POINTER(Result)]),
    ("ljx_pair_tally", c_int, [c_void_p, POINTER(c_double), POINTER(c_double)]),
    ("ljx_pair_set_atom_tallies", c_int, [c_void_p, c_void_p, c_void_p]),
    ("ljx_pair_bundle", c_void_p, [c_void_p]),
    ("ljx_pair_engine", c_void_p, [c_void_p]),
    ("ljx_version", c_char_p, []),
    ("ljx_neigh_bin", c_int, [c_void_p, c_void_p, c_int, c_void_p, c_double, c_void_p,
                              c_void_p, c_void_p, c_void_p, c_void_p]),
    ("ljx_neigh_build", c_int, [c_void_p, c_void_p, c_int, c_int, c_double, c_int, c_void_p,
                                c_double, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                c_longlong, c_int, c_void_p, c_void_p]),
    ("ljx_nve_initial", c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int,
                                c_double, POINTER(c_double), c_int]),
    ("ljx_nve_final", c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, POINTER(c_double),
                              c_int]),
    ("ljx_ghost_positions", c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p]),
    ("ljx_max_displacement", c_int, [c_void_p, c_void_p, c_void_p, c_int, c_void_p]),
    ("ljx_halo_unique_id", c_int, [c_void_p]),
    ("ljx_halo_create", c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, POINTER(c_void_p)]),
    ("ljx_halo_destroy", None, [c_void_p]),
    ("ljx_halo_error", c_char_p, [c_void_p]),
    ("ljx_halo_create_error", c_char_p, []),
    ("ljx_halo_set_swaps", c_int, [c_void_p, POINTER(Swap), c_int, c_int]),
    ("ljx_halo_forward", c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int]),
    ("ljx_halo_reverse", c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int]),
    ("ljx_read_result_all", c_int, [c_void_p, c_void_p, c_void_p, POINTER(ResultAll)]),
    ("ljx_halo_allreduce_sum", c_int, [c_void_p, c_void_p, c_void_p, c_int]),
    ("ljx_halo_launches", c_longlong, [c_void_p]),
]

_lib: ctypes.CDLL | None = None


class LjxError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


def load(path: Path | None = None) -> ctypes.CDLL:
    """Load libljx.so and bind every declared entry point; raises if anything is missing."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    so = Path(path) if path is not None else LIB
    if not so.exists():
        raise RuntimeError(f"{so} is missing: build it with __graft_entry__.build() "
                           "(nvcc, sm_100a); the ljx force path has no CPU fallback")
    lib = ctypes.CDLL(str(so))
    for name, restype, argtypes in SIGNATURES:
        fn = getattr(lib, name)  # AttributeError names the missing symbol
        fn.restype = restype
        fn.argtypes = argtypes
    if path is None:
        _lib = lib
    return lib
