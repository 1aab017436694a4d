"""ljx — B200-native EAM/LJ force engine behind lammps-jax's `pair_style jax/kk` surface.

The product is libljx.so (csrc/, C ABI in include/ljx.h): hand-written sm_100a kernels for
the per-step edge pack, EAM density, embedding and the fused force/energy/virial pass, LJ as the
one-pass case, and the halo pack/unpack of the comm sites. This package is the host side:
build recipe, ctypes binding, bundle writer/reader, a mirror of the reference pair style
(PairJaxKokkos) and the synthetic-workload harness (synth, halo, md).
"""

from . import abi, build, md, synth  # noqa: F401
from .abi import LjxError, load  # noqa: F401
from .build import build_library  # noqa: F401
from .bundle import (Bundle, add_potential, bundle_dict, eam_potential,  # noqa: F401
                     funcfl_potential, lj_potential, write_bundle)
from .engine import Engine, LammpsError, NeighborList, PairJax, SelfComm, System  # noqa: F401

__all__ = ["abi", "build", "md", "synth", "LjxError", "load", "build_library", "Bundle",
           "add_potential", "bundle_dict", "eam_potential", "funcfl_potential", "lj_potential",
           "write_bundle", "Engine", "LammpsError",
           "NeighborList", "PairJax", "SelfComm", "System"]
