"""NVE molecular dynamics around the pair style, on the device.

The standalone harness's stand-in for LAMMPS's run loop on one rank that owns a periodic box
(Verlet::run with `fix nve`):
  1. FixNVE::initial_integrate (ljx_nve_initial);
  2. Neighbor::decide: ago += 1; every `every` steps, rebuild when any owned atom has moved more
     than half the skin since the last build ("check yes"), or unconditionally ("check no");
  3. on a rebuild: Domain::pbc + Comm::borders (wrap the owned atoms into the box and make the
     ghost shell again, on the host) and the device neighbor build; otherwise Comm::forward_comm
     of positions to the ghost images (ljx_ghost_positions);
  4. force clear, pair->compute with neighbor->ago, the reverse comm of ghost forces (newton on);
  5. FixNVE::final_integrate (ljx_nve_final).
`borders="when-needed"` keeps the ghost set between rebuilds for as long as no owned atom has
moved more than half the skin since it was made; the rebuild is then the device list build alone.
That gives the same forces as LAMMPS's re-bordering (every pair within the list cutoff of the
old shell is still present, as in LAMMPS between two rebuilds) and keeps large systems off the
host. Units follow LAMMPS's `update->set_units` constants for `lj` and `metal`.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from . import abi, synth
from .engine import LammpsError, SelfComm, System

# force->boltz, force->mvv2e, force->ftm2v (LAMMPS update.cpp, units lj / metal).
UNITS = {
    "lj": {"boltz": 1.0, "mvv2e": 1.0, "ftm2v": 1.0},
    "metal": {"boltz": 8.617343e-5, "mvv2e": 1.0364269e-4, "ftm2v": 1.0 / 1.0364269e-4},
}


def maxwell_velocities(masses, temperature, units, seed):
    """Seeded Gaussian velocities with zero total momentum, scaled to `temperature` over 3N - 3
    degrees of freedom (LAMMPS `velocity all create T seed dist gaussian mom yes`; LAMMPS's own
    random stream differs, the distribution is the same)."""
    u = UNITS[units]
    m = np.asarray(masses, np.float64)[:, None]
    rng = np.random.default_rng(seed)
    v = rng.normal(size=(len(m), 3)) / np.sqrt(m)
    v -= (m * v).sum(0) / m.sum()
    dof = 3 * len(m) - 3
    t_now = float((m * v * v).sum()) * u["mvv2e"] / (dof * u["boltz"])
    return v * np.sqrt(temperature / t_now)


@dataclass
class Thermo:
    step: int
    pe: float
    ke: float
    temp: float

    @property
    def etotal(self) -> float:
        return self.pe + self.ke


class NVE:
    """Velocity-Verlet NVE of `system` under `pair` (a coeff'ed, init_style'd PairJax).

    `x_owned` [nlocal, 3], `types` [nlocal] (1-based) and `box` describe the owned atoms; the
    ghost shell reaches `cutoff + skin`. `mass` is per type. `v` (owned velocities) defaults to
    zero."""

    def __init__(self, pair, x_owned, types, box, mass, *, cutoff, skin, dt, units,
                 newton_pair, half_list, v=None, every=1, check=True, borders="always",
                 maxneigh=None, device="cuda"):
        if borders not in ("always", "when-needed"):
            raise ValueError(borders)
        self.lib = abi.load()
        self.pair, self.box = pair, np.asarray(box, np.float64)
        self.cut, self.skin, self.dt, self.units = cutoff + skin, skin, dt, units
        self.newton, self.half, self.every, self.check = newton_pair, half_list, every, check
        self.borders, self.maxneigh, self.device = borders, maxneigh, device
        self.types_owned = np.asarray(types, np.int32)
        self.nlocal = len(self.types_owned)
        self.mass = np.asarray(mass, np.float64)
        self.ntypes = len(self.mass)
        u = UNITS[units]
        self.dtfm = (ctypes.c_double * self.ntypes)(*(0.5 * dt * u["ftm2v"] / self.mass))
        v0 = np.zeros((self.nlocal, 3)) if v is None else np.asarray(v, np.float64)
        self.v = torch.as_tensor(v0.copy(), device=device)
        self.mass_atom = torch.as_tensor(self.mass[self.types_owned - 1], device=device)
        self.disp = torch.zeros(1, dtype=torch.float64, device=device)
        self.step_count = 0
        self.builds = 0
        self.border_builds = 0
        self._make_borders(np.asarray(x_owned, np.float64))
        self.ago = 0

    # -- LAMMPS's pbc + borders + neighbor build -------------------------------------------
    def _make_borders(self, x_owned):
        x_owned = np.mod(x_owned, self.box)
        x_owned[x_owned >= self.box] -= self.box[np.nonzero(x_owned >= self.box)[1]]
        x_all, owner = synth.periodic_ghosts(x_owned, self.box, self.cut)
        nall = len(x_all)
        types_all = np.concatenate([self.types_owned, self.types_owned[owner]]).astype(np.int32)
        shift = x_all[self.nlocal:] - x_owned[owner]
        shift = np.round(shift / self.box) * self.box  # exact 0 or +-L per dimension
        x = torch.as_tensor(x_all, device=self.device)
        self.system = System(x=x, type=torch.as_tensor(types_all, device=self.device),
                             f=torch.zeros_like(x), nlocal=self.nlocal, nghost=nall - self.nlocal,
                             newton_pair=self.newton, unit_style=self.units, ntypes=self.ntypes)
        self.owner = torch.as_tensor(owner, device=self.device)
        self.shift = torch.as_tensor(shift, device=self.device)
        self.system.comm = SelfComm(self.owner, self.nlocal)
        self.lists = synth.DeviceListBuilder(x_all, self.nlocal, self.cut, half=self.half,
                                             maxneigh=self.maxneigh, margin=self.skin,
                                             device=self.device)
        self.system.list = self.lists.build(x)
        self.xhold = x[: self.nlocal].clone()      # positions at the last list build
        self.xborder = self.xhold.clone()          # positions when the ghost set was made
        self.builds += 1
        self.border_builds += 1

    def _stream(self):
        return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def _max_disp2(self, ref) -> float:
        st = self.lib.ljx_max_displacement(self._stream(), ctypes.c_void_p(self.system.x.data_ptr()),
                                           ctypes.c_void_p(ref.data_ptr()), self.nlocal,
                                           ctypes.c_void_p(self.disp.data_ptr()))
        if st != abi.OK:
            raise LammpsError(f"ljx_max_displacement failed ({st})")
        return float(self.disp.item())

    def _ghosts(self):
        st = self.lib.ljx_ghost_positions(self._stream(), ctypes.c_void_p(self.system.x.data_ptr()),
                                          self.nlocal, self.system.nghost,
                                          ctypes.c_void_p(self.owner.data_ptr()),
                                          ctypes.c_void_p(self.shift.data_ptr()))
        if st != abi.OK:
            raise LammpsError(f"ljx_ghost_positions failed ({st})")

    def _reneighbor(self):
        half_skin2 = 0.25 * self.skin * self.skin
        if self.borders == "when-needed" and self._max_disp2(self.xborder) <= half_skin2:
            self._ghosts()
            self.lists.launch(self.system.x)
            if int(self.lists.widest.item()) > self.lists.maxneigh:
                self.maxneigh = int(self.lists.widest.item()) + 16
                self._make_borders(self.system.x[: self.nlocal].cpu().numpy())
            else:
                self.xhold.copy_(self.system.x[: self.nlocal])
                self.builds += 1
        else:
            self._make_borders(self.system.x[: self.nlocal].cpu().numpy())

    def _decide(self) -> bool:
        """Neighbor::decide with delay 0."""
        self.ago += 1
        if self.ago % self.every:
            return False
        if not self.check:
            return True
        return self._max_disp2(self.xhold) > 0.25 * self.skin * self.skin

    # -- the step ----------------------------------------------------------------------------
    def force(self, eflag=True, vflag=True):
        """Force clear + pair->compute (+ reverse comm of ghost forces with newton on)."""
        s = self.system
        s.f.zero_()
        s.list.ago = self.ago
        res = self.pair.compute(s, eflag=eflag, vflag=vflag)
        if self.newton:
            s.comm.reverse_forces(s.f)
        return res

    def setup(self):
        """Verlet::setup: the forces of the starting positions (LAMMPS `run 0`)."""
        self.ago = 0
        return self.force()

    def step(self, eflag=False, vflag=False):
        s = self.system
        st = self.lib.ljx_nve_initial(self._stream(), ctypes.c_void_p(s.x.data_ptr()),
                                      ctypes.c_void_p(self.v.data_ptr()),
                                      ctypes.c_void_p(s.f.data_ptr()),
                                      ctypes.c_void_p(s.type.data_ptr()), self.nlocal, self.dt,
                                      self.dtfm, self.ntypes)
        if st != abi.OK:
            raise LammpsError(f"ljx_nve_initial failed ({st})")
        if self._decide():
            self._reneighbor()
            self.ago = 0
        else:
            self._ghosts()
        res = self.force(eflag, vflag)
        s = self.system
        st = self.lib.ljx_nve_final(self._stream(), ctypes.c_void_p(self.v.data_ptr()),
                                    ctypes.c_void_p(s.f.data_ptr()),
                                    ctypes.c_void_p(s.type.data_ptr()), self.nlocal, self.dtfm,
                                    self.ntypes)
        if st != abi.OK:
            raise LammpsError(f"ljx_nve_final failed ({st})")
        self.step_count += 1
        return res

    def thermo(self, res) -> Thermo:
        """pe (the pair energy of `res`), ke and temp of the current velocities."""
        u = UNITS[self.units]
        mv2 = float((self.mass_atom[:, None] * self.v * self.v).sum().item())
        ke = 0.5 * u["mvv2e"] * mv2
        temp = mv2 * u["mvv2e"] / ((3 * self.nlocal - 3) * u["boltz"])
        return Thermo(self.step_count, float(res.energy), ke, temp)
