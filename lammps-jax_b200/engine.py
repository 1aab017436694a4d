"""Host side of the drop-in: the engine handle and a mirror of PairJaxKokkos.

`PairJax` follows cpp/pair_jax_kokkos.cpp — settings (:573-580), coeff (:582-663), init_style
(:665-785), init_one (:787-792) and compute (:989-1102) — with the same arguments, the same
checks and the same error messages, but every array operation goes to libljx through its C ABI
on a CUDA stream. torch supplies device memory and streams only.

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

    def __init__(self, bundle: Bundle, device: int = 0):
        self.lib = abi.load()
        self.bundle = bundle
        out = ctypes.c_void_p()
        status = self.lib.ljx_engine_create(bundle.handle, device, ctypes.byref(out))
        if status != abi.OK:
            raise abi.LjxError(status, self.lib.ljx_bundle_error().decode())
        self._h = out
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
        if getattr(self, "_h", None):
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
    """pair_style jax/kk on the ljx engine (mirror of PairJaxKokkos)."""

    PLATFORM = "cuda"

    def __init__(self, device: int = 0):
        self.device = device
        self.scale = 1.0
        self.bundle: Bundle | None = None
        self.engine: Engine | None = None
        self.model_loaded = False
        self.plan: abi.Plan | None = None
        self.eng_vdwl = 0.0
        self.virial = [0.0] * 6
        self.last = None

    def settings(self, *args):
        # pair_style jax/kk [plugin-path]: the path is accepted and ignored (no PJRT plugin).
        if len(args) > 1:
            raise LammpsError("Illegal pair_style jax/kk command")

    def coeff(self, system: System, *args):
        if len(args) < 3 or len(args) > 4:
            raise LammpsError("Illegal pair_coeff jax/kk command")
        if len(args) == 4:
            self.scale = float(args[3])
        try:
            self.bundle = Bundle.load(args[2])
        except abi.LjxError as err:
            raise LammpsError(f"Failed to load LAMMPS-JAX model: {err}") from err
        c = self.bundle.contract
        if c["unit_style"] != system.unit_style:
            raise LammpsError("LAMMPS-JAX model unit style does not match current units")
        if c["n_species"] > 0 and system.ntypes > c["n_species"]:
            raise LammpsError(
                f"LAMMPS-JAX model distinguishes {c['n_species']} species but the system defines "
                f"{system.ntypes} atom types; types beyond the model's range would silently map "
                "to its last species")
        if c["platform"] != self.PLATFORM:
            raise LammpsError(
                f"LAMMPS-JAX model was exported for {c['platform']} but this build runs "
                f"{self.PLATFORM}; re-export it with platform=\"{self.PLATFORM}\"")
        try:
            self.engine = Engine(self.bundle, self.device)
        except abi.LjxError as err:
            raise LammpsError(f"Failed to initialize LAMMPS-JAX runtime: {err}") from err
        self.model_loaded = True

    def init_style(self, system: System):
        if not self.model_loaded:
            raise LammpsError("LAMMPS-JAX model has not been loaded")
        for fix in system.fixes:
            if not system.newton_pair and any(k in fix for k in ("npt", "nph", "press",
                                                                 "box/relax", "msst")):
                raise LammpsError(f"Fix {fix} requires pair virial; run pair jax/kk with newton "
                                  "pair on")
        try:
            self.plan = self.engine.plan(system.newton_pair)
        except abi.LjxError as err:
            raise LammpsError(str(err)) from err
        return {"half_list": bool(self.plan.half_list)}

    def init_one(self) -> float:
        return float(self.bundle.contract["cutoff"])

    def compute(self, system: System, eflag: bool = True, vflag: bool = True, stream=None, *,
                eflag_atom: bool = False, vflag_atom: bool = False, eflag_only: bool = False):
        """One force evaluation; forces are added into system.f (ghost rows too, newton on).

        eflag_only is LAMMPS's energy-only request (MC moves): the energy alone, no forces or
        virial (cpp/pair_jax_kokkos.cpp:997-1001). The bundle's potential block always provides
        the energy, so the reference's energy-program check cannot fail here."""
        if not self.model_loaded or self.engine is None:
            raise LammpsError("LAMMPS-JAX runtime is not initialized")
        if eflag_atom:
            raise LammpsError("pair jax/kk does not support per-atom energy output")
        if vflag_atom:
            raise LammpsError("pair jax/kk does not support per-atom virial output")
        if system.list is None:
            raise LammpsError("LAMMPS-JAX requires a Kokkos device neighbor list")
        eng, plan = self.engine, self.plan
        atoms = system.atoms()
        nl = system.list.struct()
        newton = system.newton_pair
        try:
            eng.pack_atoms(atoms, stream)
        except abi.LjxError as err:
            if err.status == abi.ERR_CAPACITY:
                raise LammpsError(str(err)) from err
            raise LammpsError(f"LAMMPS-JAX compute failed: {err}") from err
        try:
            eng.density(atoms, nl, newton, stream)
            if plan.reverse_density:
                rows, width, elem = eng.feature_rows(0)
                system.comm.reverse(rows, width, elem, stream)
            eng.embed(atoms, stream)
            if eflag_only:
                eng.energy(atoms, nl, newton, self.scale, stream)
            else:
                if plan.forward_fp:
                    rows, width, elem = eng.feature_rows(1)
                    system.comm.forward(rows, width, elem, stream)
                eng.force(atoms, nl, newton, self.scale, stream)
            res = eng.read_result(stream)
        except abi.LjxError as err:
            raise LammpsError(f"LAMMPS-JAX compute failed: {err}") from err
        c = self.bundle.contract
        if res.overflow:
            if c["input_layout"] == abi.LAYOUT_NEIGHBOR_MATRIX:
                raise LammpsError(
                    f"LAMMPS-JAX neighbor capacity exceeded: global max {res.widest_row} neighbors "
                    f"per atom, capacity {c['max_neighbors']}")
            raise LammpsError(f"LAMMPS-JAX edge capacity exceeded: global max {res.edge_count} "
                              f"edges, capacity {c['max_edges']}")
        if eflag or eflag_only:
            self.eng_vdwl += res.energy
        if vflag and not eflag_only:
            for k in range(6):
                self.virial[k] += res.virial[k]
        self.last = res
        return res
