"""Host side of the drop-in for the harness and the tests: handles on the engine and on the pair
style.

`PairJax` drives libljx's pair style (include/ljx_pair.h, csrc/pair.cpp), the C++ restatement of
cpp/pair_jax_kokkos.cpp — settings (:573-580), coeff (:582-663), init_style (:665-785), init_one
(:787-792) and compute (:989-1102) — with the same arguments, checks and error messages. Every
array operation runs in libljx on a CUDA stream; torch supplies device memory and streams only.

`System` stands in for the LAMMPS state the pair style reads (x, type, f, nlocal, nghost, the
neighbor list) and `SelfComm` for LAMMPS's comm on one rank whose ghosts are periodic images.
"""

from __future__ import annotations

import builtins
import ctypes
from dataclasses import dataclass, field

import torch

from . import abi
from .bundle import Bundle


def _ptr(t: torch.Tensor | None):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream(stream=None) -> ctypes.c_void_p:
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


class LammpsError(RuntimeError):
    """error->all / error->one of the pair style: the run aborts with this message."""


@dataclass
class NeighborList:
    """A NeighListKokkos view on the device (Kokkos LayoutLeft: neighbors[i + jj*stride])."""
    ilist: torch.Tensor
    numneigh: torch.Tensor
    neighbors: torch.Tensor
    slot_stride: int
    maxneighs: int
    inum: int
    atom_stride: int = 1
    gnum: int = 0
    half: bool = False
    # neighbor->ago: steps since the list was built (0 on a build step); negative turns the
    # engine's per-group candidate cache off.
    ago: int = 0

    def struct(self) -> abi.NeighList:
        return abi.NeighList(self.ilist.data_ptr(), self.numneigh.data_ptr(),
                             self.neighbors.data_ptr(), self.atom_stride, self.slot_stride,
                             self.inum, self.gnum, self.maxneighs, self.ago)


@dataclass
class System:
    """LAMMPS per-rank state on the device: owned rows first, then ghosts."""
    x: torch.Tensor            # float64 [nall, 3]
    type: torch.Tensor         # int32 [nall], 1-based
    f: torch.Tensor            # float64 [nall, 3]
    nlocal: int
    nghost: int
    newton_pair: bool = True
    unit_style: str = "metal"
    ntypes: int = 1
    list: NeighborList | None = None
    comm: object = None
    fixes: builtins.list = field(default_factory=builtins.list)
    molecular: bool = False
    special_lj: tuple = (1.0, 1.0, 1.0, 1.0)     # force->special_lj[0..3]
    special_coul: tuple = (1.0, 1.0, 1.0, 1.0)   # force->special_coul[0..3]

    @property
    def nall(self) -> int:
        return self.nlocal + self.nghost

    def atoms(self) -> abi.Atoms:
        return abi.Atoms(self.x.data_ptr(), self.type.data_ptr(), self.f.data_ptr(), self.nlocal,
                         self.nghost)


class SelfComm:
    """LAMMPS comm for one rank with periodic images: ghost row nlocal+g mirrors owner[g]."""

    def __init__(self, owner: torch.Tensor, nlocal: int):
        self.owner = owner.to(torch.int32).contiguous()
        self.nlocal = nlocal
        self.nghost = int(owner.numel())
        self.lib = abi.load()

    def forward(self, rows: int, width: int, elem_bytes: int, stream=None):
        st = self.lib.ljx_halo_forward_self(_stream(stream), ctypes.c_void_p(rows), width,
                                            elem_bytes, _ptr(self.owner), self.nlocal, self.nghost)
        if st != abi.OK:
            raise LammpsError("forward comm failed")

    def reverse(self, rows: int, width: int, elem_bytes: int, stream=None):
        st = self.lib.ljx_halo_reverse_self(_stream(stream), ctypes.c_void_p(rows), width,
                                            elem_bytes, _ptr(self.owner), self.nlocal, self.nghost)
        if st != abi.OK:
            raise LammpsError("reverse comm failed")

    def reverse_forces(self, f: torch.Tensor, stream=None):
        """LAMMPS's own reverse comm of ghost force rows (newton on)."""
        self.reverse(f.data_ptr(), 3, 8, stream)

    def allreduce_max(self, values):
        return list(values)


class Engine:
    """One ljx_engine: device buffers sized from the bundle contract."""

    def __init__(self, bundle: Bundle, device: int = 0, handle: int | None = None):
        """A new engine for `bundle`, or (handle given) a view of an engine someone else owns,
        such as the one behind a PairJax."""
        self.lib = abi.load()
        self.bundle = bundle
        self._owned = handle is None
        if handle is None:
            out = ctypes.c_void_p()
            status = self.lib.ljx_engine_create(bundle.handle, device, ctypes.byref(out))
            if status != abi.OK:
                raise abi.LjxError(status, self.lib.ljx_bundle_error().decode())
            self._h = out
        else:
            self._h = ctypes.c_void_p(handle)
        self.contract = bundle.contract
        self.f64 = self.contract["precision"] == abi.FLOAT64

    def _check(self, status: int):
        if status != abi.OK:
            raise abi.LjxError(status, self.lib.ljx_engine_error(self._h).decode())

    def plan(self, newton_pair: bool) -> abi.Plan:
        plan = abi.Plan()
        self._check(self.lib.ljx_engine_plan(self._h, int(newton_pair), ctypes.byref(plan)))
        return plan

    def pack_atoms(self, atoms: abi.Atoms, stream=None):
        self._check(self.lib.ljx_pack_atoms(self._h, _stream(stream), ctypes.byref(atoms)))

    def pack_edges(self, atoms: abi.Atoms, nl: abi.NeighList, newton_pair: bool, stream=None):
        self._check(self.lib.ljx_pack_edges(self._h, _stream(stream), ctypes.byref(atoms),
                                            ctypes.byref(nl), int(newton_pair)))

    def edges(self):
        s, r, m = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
        cap = ctypes.c_int()
        self._check(self.lib.ljx_edges(self._h, ctypes.byref(s), ctypes.byref(r),
                                       ctypes.byref(m), ctypes.byref(cap)))
        return s.value, r.value, m.value, cap.value

    def density(self, atoms, nl, newton_pair, stream=None):
        self._check(self.lib.ljx_density(self._h, _stream(stream), ctypes.byref(atoms),
                                         ctypes.byref(nl), int(newton_pair)))

    def embed(self, atoms, stream=None):
        self._check(self.lib.ljx_embed(self._h, _stream(stream), ctypes.byref(atoms)))

    def force(self, atoms, nl, newton_pair, scale=1.0, stream=None):
        self._check(self.lib.ljx_force(self._h, _stream(stream), ctypes.byref(atoms),
                                       ctypes.byref(nl), int(newton_pair), float(scale)))

    def force_rows(self, atoms, nl, newton_pair, part, scale=1.0, stream=None):
        """One part of the force pass (ljx_force_rows): abi.ROWS_LOCAL, the rows without a
        ghost neighbor (they may run while the F' exchange is in flight), then abi.ROWS_GHOST,
        the others; together they are force()."""
        self._check(self.lib.ljx_force_rows(self._h, _stream(stream), ctypes.byref(atoms),
                                            ctypes.byref(nl), int(newton_pair), float(scale),
                                            int(part)))

    def force_only(self, atoms, nl, newton_pair, scale=1.0, stream=None):
        """The forces without the energy and virial sums (steps where LAMMPS asks for
        neither); the next read_result reports energy and virial as zero."""
        self._check(self.lib.ljx_force_only(self._h, _stream(stream), ctypes.byref(atoms),
                                            ctypes.byref(nl), int(newton_pair), float(scale)))

    def force_to_host(self, atoms, nl, newton_pair, f_host, scale=1.0, pieces=4, stream=None):
        """ljx_force with the owned force rows copied into `f_host` (a pinned CPU float64
        tensor of nlocal x 3) piece by piece while the pass runs; complete once the stream has
        drained (read_result)."""
        if f_host.device.type != "cpu" or f_host.dtype != torch.float64 or not f_host.is_contiguous():
            raise ValueError("f_host must be a contiguous float64 CPU tensor")
        if f_host.numel() < 3 * atoms.nlocal:
            raise ValueError("f_host holds fewer than nlocal rows")
        self._check(self.lib.ljx_force_to_host(self._h, _stream(stream), ctypes.byref(atoms),
                                               ctypes.byref(nl), int(newton_pair), float(scale),
                                               ctypes.c_void_p(f_host.data_ptr()), int(pieces)))

    def energy(self, atoms, nl, newton_pair, scale=1.0, stream=None):
        self._check(self.lib.ljx_energy(self._h, _stream(stream), ctypes.byref(atoms),
                                        ctypes.byref(nl), int(newton_pair), float(scale)))

    def read_result(self, stream=None) -> abi.Result:
        res = abi.Result()
        self._check(self.lib.ljx_read_result(self._h, _stream(stream), ctypes.byref(res)))
        return res

    def feature_rows(self, which: int):
        rows = ctypes.c_void_p()
        width, elem = ctypes.c_int(), ctypes.c_int()
        self._check(self.lib.ljx_feature_rows(self._h, which, ctypes.byref(rows),
                                              ctypes.byref(width), ctypes.byref(elem)))
        return rows.value, width.value, elem.value

    def feature_tensor(self, which: int, rows: int) -> torch.Tensor:
        """Copy of the first `rows` feature values (test helper; synchronizes)."""
        ptr, width, elem = self.feature_rows(which)
        dtype = torch.float64 if elem == 8 else torch.float32
        out = torch.empty(rows * width, dtype=dtype, device="cuda")
        torch.cuda.synchronize()
        _cuda_memcpy_dtod(out.data_ptr(), ptr, rows * width * elem)
        return out

    @property
    def launches(self) -> int:
        return int(self.lib.ljx_engine_launches(self._h))

    def close(self):
        if getattr(self, "_h", None) and getattr(self, "_owned", True):
            self.lib.ljx_engine_destroy(self._h)
        self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


_cudart = None


def _cuda_memcpy_dtod(dst: int, src: int, nbytes: int):
    global _cudart
    if _cudart is None:
        import glob
        cands = sorted(glob.glob("/usr/local/cuda/lib64/libcudart.so*"))
        for c in cands:
            try:
                _cudart = ctypes.CDLL(c)
                break
            except OSError:
                continue
        if _cudart is None:
            raise RuntimeError("libcudart not found")
    status = _cudart.cudaMemcpy(ctypes.c_void_p(dst), ctypes.c_void_p(src), ctypes.c_size_t(nbytes),
                                3)
    if status != 0:
        raise RuntimeError(f"cudaMemcpy failed ({status})")


class PairJax:
    """pair_style jax/kk: a handle on libljx's pair style (include/ljx_pair.h), the C++ restatement
    of PairJaxKokkos. The methods take the LAMMPS state from a `System`; checks, their order and
    messages are the library's (the reference's). `system.comm` serves the exchanges."""

    def __init__(self, device: int = 0):
        self.lib = abi.load()
        self.device = device
        out = ctypes.c_void_p()
        if self.lib.ljx_pair_create(device, ctypes.byref(out)) != abi.OK:
            raise LammpsError("Failed to create pair jax/kk")
        self._h = out
        self.bundle: Bundle | None = None
        self.engine: Engine | None = None
        self.plan: abi.Plan | None = None
        self.last = None

    def _check(self, status: int):
        if status != abi.OK:
            raise LammpsError(self.lib.ljx_pair_error(self._h).decode())

    @staticmethod
    def _argv(args):
        raw = [str(a).encode() for a in args]
        return len(raw), (ctypes.c_char_p * max(1, len(raw)))(*raw)

    def settings(self, *args):
        n, argv = self._argv(args)
        self._check(self.lib.ljx_pair_settings(self._h, n, argv))

    def coeff(self, system: System, *args):
        self.engine = None
        n, argv = self._argv(args)
        status = self.lib.ljx_pair_coeff(self._h, n, argv, system.unit_style.encode(),
                                         system.ntypes)
        handle = self.lib.ljx_pair_bundle(self._h)
        self.bundle = Bundle(handle, owned=False) if handle else None
        eng = self.lib.ljx_pair_engine(self._h)
        if eng:
            self.engine = Engine(self.bundle, self.device, handle=eng)
        self._check(status)

    @property
    def model_loaded(self) -> bool:
        return self.engine is not None

    def init_style(self, system: System):
        fixes = [str(f).encode() for f in system.fixes]
        arr = (ctypes.c_char_p * max(1, len(fixes)))(*fixes)
        lj = (ctypes.c_double * 4)(*system.special_lj)
        coul = (ctypes.c_double * 4)(*system.special_coul)
        plan = abi.Plan()
        self._check(self.lib.ljx_pair_init_style(self._h, int(system.newton_pair),
                                                 int(system.molecular), lj, coul, len(fixes), arr,
                                                 ctypes.byref(plan)))
        self.plan = plan
        return {"half_list": bool(plan.half_list)}

    def init_one(self) -> float:
        return float(self.lib.ljx_pair_init_one(self._h))

    def set_atom_tallies(self, eatom: torch.Tensor | None, vatom: torch.Tensor | None):
        """Register LAMMPS's per-atom arrays (eatom [nmax] and vatom [nmax, 6] float64 device
        tensors, or None) for computes with eflag_atom / vflag_atom."""
        self._tallies = (eatom, vatom)  # kept alive while registered
        self._check(self.lib.ljx_pair_set_atom_tallies(self._h, _ptr(eatom), _ptr(vatom)))

    def compute(self, system: System, eflag: bool = True, vflag: bool = True, stream=None, *,
                eflag_atom: bool = False, vflag_atom: bool = False, eflag_only: bool = False):
        """One force evaluation; forces are added into system.f (ghost rows too, newton on).
        eflag_only is LAMMPS's energy-only request (MC moves): the energy alone."""
        if system.list is None:
            raise LammpsError("LAMMPS-JAX requires a Kokkos device neighbor list")
        flags = ((abi.EFLAG_GLOBAL if eflag else 0) | (abi.VFLAG_GLOBAL if vflag else 0) |
                 (abi.EFLAG_ATOM if eflag_atom else 0) | (abi.VFLAG_ATOM if vflag_atom else 0) |
                 (abi.EFLAG_ONLY if eflag_only else 0))
        comm = system.comm
        failures = []

        def forward(_ctx, rows, width, elem, strm):
            try:
                comm.forward(rows, width, elem, stream)
                return 0
            except Exception as err:  # reported through the pair style's status
                failures.append(err)
                return 1

        def reverse(_ctx, rows, width, elem, strm):
            try:
                comm.reverse(rows, width, elem, stream)
                return 0
            except Exception as err:
                failures.append(err)
                return 1

        def reduce(_ctx, values, n):
            try:
                if hasattr(comm, "allreduce_max"):
                    out = comm.allreduce_max([values[k] for k in range(n)])
                    for k in range(n):
                        values[k] = int(out[k])
                return 0
            except Exception as err:
                failures.append(err)
                return 1

        host = abi.PairHost(None, abi.COMM_FN(forward), abi.COMM_FN(reverse),
                            abi.REDUCE_FN(reduce))
        res = abi.Result()
        atoms = system.atoms()
        nl = system.list.struct()
        status = self.lib.ljx_pair_compute(self._h, _stream(stream), ctypes.byref(atoms),
                                           ctypes.byref(nl), int(system.newton_pair), flags,
                                           ctypes.byref(host), ctypes.byref(res))
        if status != abi.OK and failures:
            raise LammpsError(f"{self.lib.ljx_pair_error(self._h).decode()} ({failures[0]})")
        self._check(status)
        self.last = res
        return res

    def _tally(self):
        e = ctypes.c_double()
        v = (ctypes.c_double * 6)()
        self.lib.ljx_pair_tally(self._h, ctypes.byref(e), v)
        return e.value, list(v)

    @property
    def eng_vdwl(self) -> float:
        return self._tally()[0]

    @property
    def virial(self) -> list:
        return self._tally()[1]

    def close(self):
        if getattr(self, "_h", None):
            self.engine = None
            self.lib.ljx_pair_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
