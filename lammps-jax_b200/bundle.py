"""Bundle files: write the reference's JSON schema plus the potential block, read via the C loader.

write_bundle produces what python/lammps_jax/export.py:523-566 writes (same format tags, same
sorted keys, same contract keys) with a `potential` object carrying the physics in readable
form; the serialized-program slots stay empty because this engine computes EAM and LJ natively.
Reading always goes through the library's loader (ljx_bundle_load), so Python sees exactly the
validation the LAMMPS pair style sees.
"""

from __future__ import annotations

import base64
import ctypes
import json
from pathlib import Path

import numpy as np

from . import abi

BUNDLE_FORMAT = "lammps-jax-json"
DISTRIBUTED_BUNDLE_FORMAT = "lammps-jax-json-distributed"
HALF_EDGE_BUNDLE_FORMAT = "lammps-jax-json-half-edge"


def eam_potential(setfl_text: str) -> dict:
    return {"potential_kind": "eam/alloy",
            "setfl_b64": base64.b64encode(setfl_text.encode("ascii")).decode("ascii")}


def funcfl_potential(funcfl_text: str, element: str = "funcfl") -> dict:
    return {"potential_kind": "eam", "funcfl_element": element,
            "funcfl_b64": base64.b64encode(funcfl_text.encode("ascii")).decode("ascii")}


def lj_potential(epsilon: float, sigma: float, edge_energy_scale: float | None = None) -> dict:
    out = {"potential_kind": "lj/cut", "lj_epsilon": float(epsilon), "lj_sigma": float(sigma)}
    if edge_energy_scale is not None:
        out["lj_edge_energy_scale"] = float(edge_energy_scale)
    return out


def bundle_dict(*, potential: dict, max_atoms: int, cutoff: float, unit_style: str,
                precision: str = "float32", force_output: str = "atom-force", newton: str = "on",
                max_edges: int | None = None, max_neighbors: int | None = None, n_hops: int = 1,
                comm: bool = False, half_edges: bool = False, comm_widths=None, comm_sites=None,
                uses_box: bool = False, pair_sum: bool = False, n_species: int | None = None,
                max_owned: int | None = None, platform: str = "cuda") -> dict:
    """The bundle JSON object (keys as export.py writes them)."""
    if (max_edges is None) == (max_neighbors is None):
        raise ValueError("give exactly one of max_edges (sparse edges) or max_neighbors "
                         "(neighbor matrix)")
    unique = comm and half_edges
    widths = list(comm_widths if comm_widths is not None else ([1] if comm else []))
    sites = list(comm_sites if comm_sites is not None else ([len(widths)] * 3 if comm else [0, 0, 0]))
    contract = {
        "input_layout": "neighbor-matrix" if max_neighbors is not None else "sparse-edge",
        "max_atoms": int(max_atoms),
        "cutoff": float(cutoff),
        "unit_style": unit_style,
        "precision": precision,
        "force_output": force_output,
        "newton": newton,
        "n_hops": int(n_hops),
        "edge_pairing": "half-unique" if unique else "half" if half_edges else "full",
        "comm_widths": widths,
        "comm_sites": sites,
        "custom_call_targets": [],
        "uses_box": bool(uses_box),
        "pair_sum": bool(pair_sum),
    }
    if max_neighbors is not None:
        contract["max_neighbors"] = int(max_neighbors)
    else:
        contract["max_edges"] = int(max_edges)
    if n_species is not None:
        contract["n_species"] = int(n_species)
    if max_owned is not None:
        contract["max_owned"] = int(max_owned)
    distributed = n_hops > 1 or comm
    return {
        "format": HALF_EDGE_BUNDLE_FORMAT if half_edges
        else DISTRIBUTED_BUNDLE_FORMAT if distributed else BUNDLE_FORMAT,
        "programs": {"force_mlir_b64": "", "energy_mlir_b64": "",
                     "energy_and_forces_mlir_b64": ""},
        "export_info": {"exporter": "ljx", "platform": platform},
        "compile_options_b64": "",
        "contract": contract,
        "potential": dict(potential),
    }


def write_bundle(path, **kwargs) -> dict:
    data = bundle_dict(**kwargs)
    Path(path).write_text(json.dumps(data, indent=2, sort_keys=True) + "\n", encoding="utf-8")
    return data


def add_potential(path, potential: dict) -> dict:
    """Insert the potential block into a bundle another exporter wrote (the reference's
    export_model, python/lammps_jax/export.py:523-566, keeps its programs, contract and
    export_info); the file is rewritten the way that exporter writes it (sorted keys, indent 2,
    trailing newline). lammps-jax_b200/export_potential.patch makes the exporter itself take a
    `potential=` argument instead."""
    data = json.loads(Path(path).read_text(encoding="utf-8"))
    data["potential"] = dict(potential)
    Path(path).write_text(json.dumps(data, indent=2, sort_keys=True) + "\n", encoding="utf-8")
    return data


def _decode(value) -> str:
    return value.decode() if isinstance(value, bytes) else value


class Bundle:
    """A bundle parsed and validated by the library's loader (ljx_bundle_load)."""

    def __init__(self, handle: int, owned: bool = True):
        self._handle = ctypes.c_void_p(handle)
        self._lib = abi.load()
        self._owned = owned

    @classmethod
    def load(cls, path) -> "Bundle":
        lib = abi.load()
        out = ctypes.c_void_p()
        status = lib.ljx_bundle_load(str(path).encode(), ctypes.byref(out))
        if status != abi.OK:
            raise abi.LjxError(status, _decode(lib.ljx_bundle_error()))
        return cls(out.value)

    @classmethod
    def from_string(cls, text: str) -> "Bundle":
        lib = abi.load()
        raw = text.encode()
        out = ctypes.c_void_p()
        status = lib.ljx_bundle_load_string(raw, len(raw), ctypes.byref(out))
        if status != abi.OK:
            raise abi.LjxError(status, _decode(lib.ljx_bundle_error()))
        return cls(out.value)

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._handle

    def contract_struct(self) -> abi.Contract:
        c = abi.Contract()
        status = self._lib.ljx_bundle_contract(self._handle, ctypes.byref(c))
        if status != abi.OK:
            raise abi.LjxError(status, "ljx_bundle_contract failed")
        return c

    @property
    def contract(self) -> dict:
        c = self.contract_struct()
        out = {}
        for name, _ in c._fields_:
            value = getattr(c, name)
            if isinstance(value, bytes):
                value = value.decode()
            elif hasattr(value, "__len__"):
                value = list(value)
            out[name] = value
        out["comm_widths"] = out["comm_widths"][: out["n_comm_widths"]]
        out["comm_sites"] = out["comm_sites"][: out["n_comm_sites"]]
        return out

    def eam_tables(self) -> dict:
        n_el, nrho, nr = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        drho, dr, cut = ctypes.c_double(), ctypes.c_double(), ctypes.c_double()
        status = self._lib.ljx_bundle_eam_tables(self._handle, ctypes.byref(n_el),
                                                 ctypes.byref(nrho), ctypes.byref(nr),
                                                 ctypes.byref(drho), ctypes.byref(dr),
                                                 ctypes.byref(cut), None, None, None)
        if status != abi.OK:
            raise abi.LjxError(status, "bundle has no EAM tables")
        emb = np.empty((n_el.value, nrho.value, 4))
        den = np.empty((n_el.value, nr.value, 4))
        par = np.empty((n_el.value * (n_el.value + 1) // 2, nr.value, 4))
        self._lib.ljx_bundle_eam_tables(self._handle, None, None, None, None, None, None,
                                        emb.ctypes.data_as(ctypes.c_void_p),
                                        den.ctypes.data_as(ctypes.c_void_p),
                                        par.ctypes.data_as(ctypes.c_void_p))
        return {"nrho": nrho.value, "drho": drho.value, "nr": nr.value, "dr": dr.value,
                "cutoff": cut.value, "embedding": emb, "density": den, "pair": par,
                "elements": [str(k) for k in range(n_el.value)]}

    def __del__(self):
        try:
            if self._handle and self._owned:
                self._lib.ljx_bundle_free(self._handle)
                self._handle = ctypes.c_void_p()
        except Exception:
            pass
