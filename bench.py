"""Benchmark: EAM force + energy + virial throughput (atom-steps/s) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ljx|reference] [--precision P]

A step is one pair-style compute of the hot path on resident inputs: stage positions (a1),
fused list filter/compaction + EAM density (a2+a6), embedding (a8), forward exchange of F'(rho)
to the ghost images (a15), fused force/energy/virial (a9-a13), and the energy/virial readback.
Workload at N=1: the 2,048,000-atom Cu fcc configuration (80^3 cells, a = 3.615 A, Gaussian
jitter 0.08 A, synthetic EAM, rc 6.5 A, skin 2.0 A), float64, full list with newton off.
The neighbor list is built once and held fixed (positions are static across timed steps); the
list alone (about 1.9 GB) is larger than the 126 MB L2, so no separate flush is needed.

--impl reference times the CPU restatement of the reference's path (oracle/, OpenMP on all host
threads) on the same 2,048,000-atom workload, the same warm-up and timed steps, and prints the
same line with "impl": "reference".

Multi-GPU runs (torchrun, one rank per GPU) use spatial decomposition along z: every rank owns a
2,048,000-atom slab of a larger crystal (weak scaling) and exchanges F'(rho) of its boundary
atoms with its two z-neighbors each step through libljx's NCCL halo (ljx_halo); the step totals
and the collective capacity check are one on-stream NCCL all-reduce.

The c3 line also carries a "c4" object: the 16,384,000-atom C4 crystal (the same atoms at every
GPU count) split over the run's GPUs (strong scaling), with its total energy, virial and a
sample of forces by global atom id, so runs at different GPU counts compare atom by atom.

--config c4 is the strong-scaling case (16,384,000-atom binary crystal split over the GPUs, half
list, newton on: reverse rho, forward F'(rho) and reverse force exchanges). --config c5 is the
edge-pack stress test on one GPU (2,048,000-atom dense binary liquid, float32, fresh list every
step, about half the listed pairs outside rc).
"""

from __future__ import annotations

import argparse
import importlib.util
import json
import os
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
METRIC = "EAM atom-steps/s (force+energy+virial)"
UNIT = "atom-steps/s"
CUTOFF, SKIN, A_CU, JITTER = 6.5, 2.0, 3.615, 0.08

# Bench workloads ([3] and [4]). c3: weak scaling, 80^3 cells per GPU,
# single-species Cu, full list, newton off. c4: strong scaling, 160^3 cells in all split into
# z-slabs, binary Cu-Zr 64/36, half list with newton on (the half-unique communicating export).
# c5: the edge-pack stress test, a dense binary liquid in float32 with a fresh list every step.
CONFIGS = {
    "c3": {"cells": 80, "strong": False, "elements": ("Cu",), "fractions": None, "newton": False,
           "half": False, "scaling": "weak", "lattice": A_CU, "edges_per_atom": 128,
           "title": "C3: Cu fcc {c}^3 cells per GPU, synthetic EAM rc 6.5 A skin 2.0 A, full list, "
                    "newton off, forward F'(rho) exchange"},
    # C4 names no lattice constant; Vegard's law between the synthetic Cu (3.615 A) and Zr
    # (4.525 A) lattices at 64/36 keeps the random alloy near zero pressure.
    # Edge capacity 64 per atom for the half list (~43 kept per row) also keeps max_edges inside
    # the contract's int range at 16.4 M atoms.
    "c4": {"cells": 160, "strong": True, "elements": ("Cu", "Zr"), "fractions": (0.64, 0.36),
           "newton": True, "half": True, "scaling": "strong", "lattice": 0.64 * 3.615 + 0.36 * 4.525,
           "edges_per_atom": 64,
           "title": "C4: binary Cu-Zr (64/36) fcc {c}^3 cells in all (a = 3.943 A), split over the GPUs, "
                    "synthetic EAM rc 6.5 A skin 2.0 A, half list, newton on, reverse rho + "
                    "forward F'(rho) + reverse force exchanges"},
    # 1.2x the synthetic Cu fcc density (0.1016 atoms/A^3) with a 2.0 A hard core: a liquid tile
    # of 32,000 atoms (synth.liquid_packing) repeated (cells/20)^3 times, 4 * cells^3 atoms in
    # all. With the 2.0 A skin about half the listed pairs fall outside rc.
    "c5": {"cells": 80, "strong": False, "elements": ("Cu", "Zr"), "fractions": (0.64, 0.36),
           "newton": False, "half": False, "scaling": "weak", "liquid": 1.2 * 4 / A_CU ** 3,
           "edges_per_atom": 160, "precision": "float32", "rebuild_every": 1, "one_gpu": True,
           "title": "C5: edge-pack stress test, binary Cu-Zr (64/36) liquid at 1.2x fcc density "
                    "with a 2.0 A core, {c}^3-cell equivalent, synthetic EAM rc 6.5 A skin 2.0 A, "
                    "full list, newton off, fresh list every step"},
}


def package():
    name = "lammps_jax_b200"
    if name in sys.modules:
        return sys.modules[name]
    pkg_dir = ROOT / "lammps-jax_b200"
    spec = importlib.util.spec_from_file_location(
        name, pkg_dir / "__init__.py", submodule_search_locations=[str(pkg_dir)])
    module = importlib.util.module_from_spec(spec)
    sys.modules[name] = module
    spec.loader.exec_module(module)
    return module


def peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons during the timed region."""

    def __init__(self, index: int, path: Path):
        self.path = path
        self.proc = None
        self.index = index

    def _gpu_id(self):
        """nvidia-smi's name for torch device `index`: its UUID (CUDA_VISIBLE_DEVICES renumbers
        the devices torch sees, nvidia-smi does not)."""
        try:
            import torch
            uuid = str(torch.cuda.get_device_properties(self.index).uuid)
            return uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        except Exception:
            return str(self.index)

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.path.parent.mkdir(parents=True, exist_ok=True)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self._gpu_id()}",
                                          f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                          "-lms", "100"],
                                         stdout=self.fh, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
            return self
        # nvidia-smi takes a few hundred ms to print its first sample; a timed region of a few
        # hundred ms would otherwise end before it. Wait (at most 5 s) for that sample.
        deadline = time.time() + 5.0
        while time.time() < deadline and self.proc.poll() is None:
            self.fh.flush()
            if self.path.stat().st_size > 0:
                break
            time.sleep(0.05)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self):
        if self.proc is None or not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def profile_entry(name: str, kernel: str):
    """Value of `kernel` in the committed ncu summary profiles/<name>, or None. These figures
    come from an earlier one-kernel capture of a smaller case, not from this run."""
    path = ROOT / "profiles" / name
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        parts = line.split()
        if len(parts) >= 2 and parts[0] == kernel:
            try:
                return float(parts[1])
            except ValueError:
                return None
    return None


class Case:
    """One configuration set up on this rank: the LAMMPS stand-in state, the pair style and the
    exchange (SelfComm on one GPU, libljx's NCCL halo across GPUs)."""

    def __init__(self, ljx, name, precision, world, rank, local, cells=None):
        import torch
        cfg = CONFIGS[name]
        self.name, self.cfg, self.precision = name, cfg, precision
        self.world, self.rank = world, rank
        if cfg["strong"]:
            total = cells or cfg["cells"]
            if total % world:
                raise SystemExit(f"--config {name}: {total} z-cells do not split over {world} GPUs")
            self.cells = (total, total, total // world)
        else:
            n = cells or cfg["cells"]
            self.cells = (n, n, n)
        if world > 1:
            setup = setup_decomposed(ljx, cfg, self.cells, rank, world, precision, local)
        else:
            setup = setup_single(ljx, cfg, self.cells, precision)
        self.system, self.nlocal, self.nall, self.decomp = setup
        self.pair = self.decomp["pair"]
        self.plan = self.pair.plan
        self.eng = self.pair.engine
        self.atoms = self.system.atoms()
        self.nl = self.system.list.struct()
        self.fp_rows, self.width, self.elem = self.eng.feature_rows(1)
        self.rho_rows = self.eng.feature_rows(0)[0]
        self.halo = self.decomp.get("halo")
        self.stream = torch.cuda.current_stream()
        self.tick = 0
        self.fp_overlap = False

    def streams_rows(self):
        """Whether the force pass can stream its rows to the host (each list row holds its
        atom's whole force: full list, newton off)."""
        return not self.system.newton_pair and not self.system.list.half

    def core(self, ago, mark=lambda k: None, f_host=None, pieces=8, ev=True):
        """One pair-style step on device data, with the exchanges the engine's plan asks for.
        With f_host (pinned, nlocal x 3) the force pass streams the owned force rows to it
        piece by piece (ljx_force_to_host). Without ev the step computes forces alone
        (ljx_force_only: LAMMPS's steps between thermo output). Returns (energy, virial, kept
        edges, overflow) over all ranks."""
        s, eng, atoms, nl = self.system, self.eng, self.atoms, self.nl
        newton = s.newton_pair
        nl.ago = ago
        mark(0)
        eng.pack_atoms(atoms)
        mark(1)
        eng.density(atoms, nl, newton)
        if self.plan.reverse_density:
            s.comm.reverse(self.rho_rows, self.width, self.elem)
        mark(2)
        eng.embed(atoms)
        mark(3)
        # Across GPUs the F' exchange can run on a side stream under the force pass's rows that
        # keep no ghost neighbor (NcclHalo.forward_under_force); the halo_fp phase is then only
        # the launch, and the force phase holds any wait for the exchange.
        overlap = (self.fp_overlap and self.halo is not None and self.plan.forward_fp and
                   f_host is None and ev)
        if self.plan.forward_fp and not overlap:
            s.comm.forward(self.fp_rows, self.width, self.elem)
        mark(4)
        if overlap:
            self.halo.forward_under_force(eng, atoms, nl, newton, self.fp_rows, self.width,
                                          self.elem)
        elif f_host is not None:
            eng.force_to_host(atoms, nl, newton, f_host, 1.0, pieces)
        elif not ev:
            eng.force_only(atoms, nl, newton, 1.0)
        else:
            eng.force(atoms, nl, newton, 1.0)
        if self.plan.reverse_force:
            s.comm.reverse_forces(s.f)  # LAMMPS's own reverse comm of ghost forces
        mark(5)
        if self.halo is not None:
            # The collective capacity check and step totals: one NCCL all-reduce on the stream
            # and one host wait (the pair style's MPI_Allreduce after execution).
            res = self.halo.result_all(eng)
        else:
            res = eng.read_result()
        out = (res.energy, list(res.virial), res.edge_count, res.overflow)
        if out[3]:
            raise RuntimeError("LAMMPS-JAX edge capacity exceeded")
        mark(6)
        return out

    def step(self, rebuild_every, events=None, ev=True):
        def mark(k):
            if events is not None:
                events[k].record(self.stream)
        # neighbor->ago as LAMMPS reports it with a rebuild every `rebuild_every` steps; the
        # engine rebuilds its candidate cache on ago == 0 (-1: cache off).
        ago = self.tick % rebuild_every if rebuild_every > 0 else -1
        self.tick += 1
        return self.core(ago, mark, ev=ev)

    def launches(self):
        return self.eng.launches + (self.halo.launches if self.halo is not None else 0)

    def time(self, steps, warmup, rebuild_every, ev=True):
        """Warm up, then time `steps` steps with CUDA events on the launching stream, bracketed
        by a barrier and a device synchronize; the max over ranks. Without ev: force-only
        steps."""
        import torch
        import torch.distributed as dist
        names = ["pack_atoms", "density", "embed", "halo_fp", "force", "result"]
        self.system.f.zero_()
        kevents = [[torch.cuda.Event(enable_timing=True) for _ in range(7)] for _ in range(steps)]
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        out = None
        for _ in range(warmup):
            out = self.step(rebuild_every, ev=ev)
        torch.cuda.synchronize()
        if self.world > 1:
            dist.barrier()
        launches0 = self.launches()
        start.record(self.stream)
        for k in range(steps):
            out = self.step(rebuild_every, kevents[k], ev=ev)
        stop.record(self.stream)
        torch.cuda.synchronize()
        elapsed = start.elapsed_time(stop) / 1e3
        if self.world > 1:
            t = torch.tensor([elapsed], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            elapsed = float(t.item())
        launches = self.launches() - launches0 + steps * self.decomp["extra_launches"]
        phase = {n: 0.0 for n in names}
        for ev in kevents:
            for k, n in enumerate(names):
                phase[n] += ev[k].elapsed_time(ev[k + 1]) / 1e3
        return {"elapsed": elapsed, "launches": launches, "result": out,
                "phase": {n: v / steps for n, v in phase.items()}}

    def total_atoms(self):
        import torch
        import torch.distributed as dist
        if self.world == 1:
            return self.nlocal
        t = torch.tensor([self.nlocal], dtype=torch.int64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return int(t.item())

    def clean_forces(self, sample_ids, rebuild_every):
        """One step from zeroed forces; returns (energy, virial, max |F| over all owned atoms,
        {global id: force} for the owned atoms among `sample_ids`)."""
        import torch
        import torch.distributed as dist
        self.system.f.zero_()
        energy, virial, _, _ = self.step(rebuild_every)
        torch.cuda.synchronize()
        f = self.system.f[:self.nlocal]
        fmax = f.abs().max().reshape(1)
        if self.world > 1:
            dist.all_reduce(fmax, op=dist.ReduceOp.MAX)
        ids = self.decomp["ids"]
        where = np.nonzero(np.isin(ids, sample_ids))[0]
        rows = (f[torch.as_tensor(where, device="cuda")].cpu().numpy() if len(where)
                else np.zeros((0, 3)))
        mine = {int(ids[w]): [float(v) for v in rows[k]] for k, w in enumerate(where)}
        if self.world > 1:
            parts = [None] * self.world
            dist.all_gather_object(parts, mine)
            mine = {k: v for p in parts for k, v in p.items()}
        return energy, virial, float(fmax.item()), mine

    def close(self):
        self.pair.engine.close()
        if self.halo is not None:
            self.halo.close()


def init_ranks():
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=datetime.timedelta(seconds=180))
    return world, rank, local


def algorithmic_bytes(listed, nlocal, nall, kept, precision, newton):
    """Algorithmic bytes of one step on one rank: (density phase, force pass, whole step).

    Density phase: every row's list slots read (4 B each), ilist and numneigh, each atom's
    staged position once, the kept edges written (4 B), the kept count and rho. Force pass: the
    row's atom and count, the kept edges read, each atom's position and F' once, f read and
    written. Whole step: the list slots and counts, each kept edge written once and its index read
    twice (density and force passes), and per owned atom x read by three passes (24 B each),
    type, rho written, F' written and read, f read-modify-written (double); per ghost x three
    times, type and F' (newton on adds the ghost's rho and f round trips)."""
    real = 8 if precision == "float64" else 4
    pos_bytes = 32 if precision == "float64" else 16
    density = 4 * listed + 4 * nlocal * 2 + 32 * nall + 4 * kept + 4 * nlocal + real * nlocal
    force = 8 * nlocal + 4 * kept + pos_bytes * nall + real * nall + 48 * nlocal
    b_own = 3 * 24 + 4 + real + 2 * real + 48
    b_ghost = 3 * 24 + 4 + real + ((2 * real + 48) if newton else 0)
    step = 4 * listed + 4 * nlocal + 12 * kept + nlocal * b_own + (nall - nlocal) * b_ghost
    return density, force, step


def run_ljx(args):
    import tempfile

    import torch
    import torch.distributed as dist

    ljx = package()
    world, rank, local = init_ranks()
    cfg = CONFIGS[args.config]
    precision = args.precision or cfg.get("precision", "float64")
    if args.rebuild_every is None:
        args.rebuild_every = cfg.get("rebuild_every", 10)
    if cfg.get("one_gpu") and world > 1:
        raise SystemExit(f"--config {args.config} runs on one GPU")
    case = Case(ljx, args.config, precision, world, rank, local, args.cells)
    case.fp_overlap = args.fp_overlap == "on"
    system, nlocal, nall, decomp = case.system, case.nlocal, case.nall, case.decomp

    # The clock samples span the warm-up and the timed steps (both under load); they go to a
    # temporary file, read back for the line's "clocks".
    clock_file = Path(tempfile.mkdtemp(prefix="ljx_clocks_")) / f"clocks_rank{rank}.csv"
    with ClockSampler(local, clock_file) as clocks:
        timing = case.time(args.steps, args.warmup, args.rebuild_every)
    elapsed, phase, launches = timing["elapsed"], timing["phase"], timing["launches"]
    energy_total, _, kept_total, _ = timing["result"]

    # Algorithmic bytes per launch (per step) of the two row kernels, for this rank.
    nn = system.list.numneigh[:nlocal].to(torch.int64)
    listed = int(nn.sum().item())
    kept_local = kept_total // world
    bytes_density, bytes_force, bytes_step = algorithmic_bytes(
        listed, nlocal, nall, kept_local, precision, bool(system.newton_pair))
    # The line's roofline is the phase that moves most of the step's algorithmic bytes: the
    # density phase, which carries the list read. (By time the density and force phases are
    # about equal at C3, so a choice by time would flip between runs.) Both phases and the whole
    # step are reported beside it.
    kernel = "density" if bytes_density >= bytes_force else "force"
    kbytes = bytes_density if kernel == "density" else bytes_force
    achieved = kbytes / phase[kernel] / 1e9
    peak, peak_kind = peaks()
    # The engine caches candidates only for lists that live at least 4 steps (kCacheMinPeriod in
    # csrc/engine.cu); shorter-lived lists take the list pass.
    cached = args.rebuild_every >= 4
    # EAM full lists with newton off hold each owned pair once unless LJX_OWNED_HALF=0
    # (kDensityHalfOwned / kRowsHalfOwned in csrc/kernels.cuh).
    owned = (not system.newton_pair and not system.list.half and
             os.environ.get("LJX_OWNED_HALF", "1") != "0")
    rows = "owned" if owned else "full"
    kname = {"density": (f"k_density_groups_{rows}_{precision}" if cached
                         else f"k_density_{rows}_{precision}"),
             "force": f"k_force_rows_{rows}_{precision}"}[kernel]
    # DRAM bytes and L1 utilisation of this kernel come from committed one-kernel ncu captures
    # (C3 kernels by name, C5 ones as "c5:<name>"), labelled as such: no profiler runs here.
    key = {"c3": kname, "c5": f"c5:{kname}"}.get(args.config)
    traffic = profile_entry("dram_traffic.txt", key) if key else None
    l1 = profile_entry("l1_wavefronts.txt", key) if key else None

    total_atoms = case.total_atoms()
    neigh_ms = time_list_build(torch, decomp["lists"], system.x, case.stream)
    e2e = None if args.skip_extras else run_e2e(torch, case, args, world, total_atoms)
    force_only = None
    if not args.skip_extras:
        # LAMMPS asks for energy and virial on thermo steps only; the steps between run the
        # forces alone (ljx_force_only, the reference's force program).
        fo = case.time(args.steps, args.warmup, args.rebuild_every, ev=False)
        force_only = {"what": "steps without energy or virial (LAMMPS steps between thermo "
                              "output; ljx_force_only)",
                      "value": total_atoms * args.steps / fo["elapsed"], "unit": UNIT,
                      "ms_per_step": fo["elapsed"] / args.steps * 1e3,
                      "phase_ms": {n: v * 1e3 for n, v in fo["phase"].items()}}
    value = total_atoms * args.steps / elapsed
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": elapsed / args.steps * 1e3,
        "higher_is_better": True, "scaling": cfg["scaling"], "vs_baseline": None,
        "dtype": "f64" if precision == "float64" else "f32", "data": "synthetic",
        "config": {
            "workload": cfg["title"].format(c=case.cells[0]) + f" ({total_atoms:,} atoms in all)",
            "name": args.config, "total_atoms": total_atoms,
            "atoms_per_gpu": nlocal, "ghosts_per_gpu": nall - nlocal,
            "listed_pairs_per_atom": listed / nlocal,
            "kept_edges_per_atom": kept_total / total_atoms,
            "precision": precision, "l2": "inputs larger than L2 (neighbor list "
                                           f"{system.list.neighbors.numel() * 4 / 1e9:.2f} GB)",
            "list": ("built once on the device, fixed over timed steps; the engine is told "
                     "neighbor->ago = 0 every step, so every step compacts the whole list as "
                     "after a rebuild; the device rebuild itself is timed apart (neigh_build_ms)"
                     if args.rebuild_every == 1 else
                     "built once on the device, fixed over timed steps"),
            "neigh_build_ms": neigh_ms,
            "rebuild_every": args.rebuild_every,
            "candidate_cache": ("rebuilt when neighbor->ago == 0, every "
                                f"{args.rebuild_every} steps, inside the timed region"
                                if cached else "not used: every step filters the whole list "
                                "(lists living under 4 steps, or the cache turned off)"),
            "parallelism": decomp["parallelism"],
            "phase_ms": {n: v * 1e3 for n, v in phase.items()},
        },
        "roofline": {"bound": "hbm", "kernel": kname, "achieved": achieved, "peak": peak,
                     "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / peak,
                     "algorithmic_bytes": kbytes, "traffic": traffic,
                     "traffic_source": ("profiles/dram_traffic.txt: dram__bytes_read.sum + "
                                        "dram__bytes_write.sum of a committed one-kernel ncu "
                                        "capture of the 256,000-atom case, scaled x8 by owned "
                                        "atoms to the full launch; not measured in this run"
                                        if traffic is not None else None),
                     "limiter": {"resource": "L1 data pipe (LSU wavefronts): random gathers of "
                                             "positions and spline rows",
                                 "frac": l1,
                                 "source": "profiles/l1_wavefronts.txt: committed one-kernel ncu "
                                           "capture of the same kernel on its 256,000-atom case; "
                                           "not measured in this run"},
                     "bytes_basis": "per-step algorithmic bytes of the reference's data flow "
                                    "(list read every step); with the candidate cache the list "
                                    "is read only at rebuilds, so this is an effective bandwidth"
                                    if kernel == "density" and cached else
                                    "per-launch algorithmic bytes",
                     "why_this_kernel": "the phase with the larger algorithmic bytes per step "
                                        "(the density phase carries the list read)",
                     "phases": {
                         n: {"ms": phase[n] * 1e3, "algorithmic_bytes": b,
                             "achieved": b / phase[n] / 1e9,
                             "frac": b / phase[n] / 1e9 / peak}
                         for n, b in (("density", bytes_density), ("force", bytes_force))},
                     "step": {"ms": elapsed / args.steps * 1e3,
                              "algorithmic_bytes": bytes_step,
                              "achieved": bytes_step / (elapsed / args.steps) / 1e9,
                              "frac": bytes_step / (elapsed / args.steps) / 1e9 / peak,
                              "basis": "whole step: list slots and counts read, kept edges "
                                       "written once and read twice, per-atom x, type, rho, "
                                       "F' and f traffic"}},
        "gpu_launches": launches,
        "e2e": e2e,
        "energy_per_atom": energy_total / total_atoms,
    }
    if force_only is not None:
        line["force_only"] = force_only
    extras = not args.skip_extras and not args.quick
    if world == 1 and extras and args.config == "c3":
        line["md"] = run_md(torch, ljx, cfg, case.cells, precision, args.steps, args.warmup)
    line["clocks"] = clocks.summary()
    case.close()
    del case, system, decomp
    torch.cuda.empty_cache()
    if world == 1 and extras and args.config == "c3" and precision == "float64":
        line["c3_f32"] = run_c3_f32(ljx, args, local)
    if extras and not args.no_c4 and args.config == "c3":
        line["c4"] = run_c4(ljx, args, world, rank, local)
    if world == 1 and extras and args.config == "c3":
        line["cpu_baseline"] = cpu_baseline(args)
    if world > 1:
        dist.barrier()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_c3_f32(ljx, args, local):
    """C3 in float32, the other precision the configuration names: the same crystal, list and
    step, timed the same way on the device."""
    import torch
    case = Case(ljx, "c3", "float32", 1, 0, local, args.cells)
    timing = case.time(args.steps, args.warmup, args.rebuild_every)
    energy = timing["result"][0]
    out = {"precision": "float32", "total_atoms": case.nlocal, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": timing["elapsed"] / args.steps * 1e3,
           "value": case.nlocal * args.steps / timing["elapsed"], "unit": UNIT,
           "gpu_launches": timing["launches"],
           "phase_ms": {n: v * 1e3 for n, v in timing["phase"].items()},
           "energy_per_atom": energy / case.nlocal}
    case.close()
    del case
    torch.cuda.empty_cache()
    return out


C4_SAMPLES = 16


def run_c4(ljx, args, world, rank, local):
    """The north-star strong-scaling case beside the headline: C4's 16,384,000-atom binary
    crystal (160^3 cells, one identical system at every GPU count, fcc_layers) split into
    z-slabs over the GPUs of this run, timed like the headline, with the totals and a sample of
    forces that let runs at different GPU counts be compared atom by atom."""
    import torch
    case = Case(ljx, "c4", "float64", world, rank, local)
    case.fp_overlap = args.fp_overlap == "on"
    timing = case.time(args.steps, args.warmup, 10)
    total = case.total_atoms()
    sample_ids = np.linspace(0, total - 1, C4_SAMPLES).astype(np.int64)
    energy, virial, fmax, forces = case.clean_forces(sample_ids, 10)
    elapsed = timing["elapsed"]
    out = {
        "workload": CONFIGS["c4"]["title"].format(c=CONFIGS["c4"]["cells"]),
        "total_atoms": total, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": elapsed / args.steps * 1e3, "value": total * args.steps / elapsed,
        "unit": UNIT, "scaling": "strong", "gpu_launches": timing["launches"],
        "phase_ms": {n: v * 1e3 for n, v in timing["phase"].items()},
        "parallelism": case.decomp["parallelism"],
        "energy": energy, "virial": virial, "max_abs_force": fmax,
        "force_sample": {"ids": [int(i) for i in sample_ids],
                         "f": [forces.get(int(i)) for i in sample_ids]},
        "system": "one crystal at every GPU count: each unit-cell z-layer draws its jitter and "
                  "species from its own seed (synth.fcc_layers), so energy, virial and the "
                  "sampled forces compare across runs",
    }
    case.close()
    del case
    torch.cuda.empty_cache()
    return out


def _bundle(ljx, cfg, path, max_atoms, precision):
    text = ljx.synth.synthetic_setfl(cfg["elements"])
    per_atom = cfg["edges_per_atom"]
    ljx.write_bundle(path, potential=ljx.eam_potential(text), max_atoms=max_atoms,
                     max_edges=max_atoms * per_atom, cutoff=CUTOFF, unit_style="metal",
                     precision=precision, force_output="atom-force",
                     newton="on" if cfg["newton"] else "off", comm=True, half_edges=cfg["half"],
                     n_species=len(cfg["elements"]))


def liquid_atoms(ljx, cfg, cells):
    """C5 positions: a 20^3-cell-equivalent liquid tile repeated (cells/20)^3 times (one tile of
    4 * cells^3 atoms when cells is not a multiple of 20)."""
    tiles, edge = (cells // 20, 20) if cells % 20 == 0 else (1, cells)
    n_tile = 4 * edge ** 3
    types = ljx.synth.substitutional(n_tile, cfg["fractions"], seed=2025)
    return ljx.synth.liquid_packing(n_tile, cfg["liquid"], 2.0, seed=2024, tiles=tiles,
                                    types=types)


def crystal_atoms(ljx, cfg, cells):
    """The C3 / C4 crystal of `cells` unit cells: fcc_layers, wrapped and sorted as LAMMPS does
    (the same atoms as every slab decomposition of it)."""
    return ljx.synth.layered_crystal(cells, cfg["lattice"], JITTER, 2024, cfg["fractions"])


def setup_single(ljx, cfg, cells, precision):
    import tempfile

    import torch
    atoms = (liquid_atoms(ljx, cfg, cells[0]) if cfg.get("liquid")
             else crystal_atoms(ljx, cfg, cells))
    x_all, owner = ljx.synth.periodic_ghosts(atoms.x, atoms.box, CUTOFF + SKIN)
    types_all = np.concatenate([atoms.types, atoms.types[owner]]).astype(np.int32)
    nlocal, nall = len(atoms.x), len(x_all)
    path = Path(tempfile.mkdtemp()) / "bench.json"
    _bundle(ljx, cfg, path, nall + 1024, precision)
    x = torch.as_tensor(x_all, device="cuda")
    system = ljx.System(x=x, type=torch.as_tensor(types_all, device="cuda"),
                        f=torch.zeros_like(x), nlocal=nlocal, nghost=nall - nlocal,
                        newton_pair=cfg["newton"], unit_style="metal",
                        ntypes=len(cfg["elements"]))
    pair = ljx.PairJax()
    pair.coeff(system, "*", "*", str(path))
    pair.init_style(system)
    builder = ljx.synth.DeviceListBuilder(x_all, nlocal, CUTOFF + SKIN, half=cfg["half"])
    system.list = builder.build(x)
    system.comm = ljx.SelfComm(torch.as_tensor(owner, device="cuda"), nlocal)
    # Ghost rows as images of owned rows: whole box lengths per dimension (LAMMPS's pbc shift).
    shift = np.round((x_all[nlocal:] - x_all[owner]) / atoms.box) * atoms.box
    ghosts = (system.comm.owner, torch.as_tensor(shift, device="cuda"))
    ids = atoms.ids if atoms.ids is not None else np.arange(nlocal)
    exchanges = "reverse rho, forward F'(rho) and reverse forces" if cfg["newton"] else "F'(rho)"
    # SelfComm's kernels (one per exchange) are libljx's but not counted by the engine.
    return system, nlocal, nall, {"pair": pair,
                                  "parallelism": "single GPU (periodic self-images; "
                                                 f"{exchanges} by ljx_halo_*_self)",
                                  "extra_launches": 3 if cfg["newton"] else 1,
                                  "lists": builder, "ghosts": ghosts, "ids": ids}


def setup_decomposed(ljx, cfg, cells, rank, world, precision, local):
    """Rank `rank` of a z-slab decomposition of `cells` per rank, exchanging over libljx's NCCL
    halo (ljx_halo)."""
    import tempfile

    import torch
    from importlib import import_module
    halo = import_module("lammps_jax_b200.halo")
    slab = ljx.synth.slab_decomposition(cells, cfg["lattice"], JITTER, 2024, rank, world,
                                        CUTOFF + SKIN, fractions=cfg["fractions"])
    nlocal, nall = slab.nlocal, len(slab.x)
    path = Path(tempfile.mkdtemp()) / f"bench_rank{rank}.json"
    _bundle(ljx, cfg, path, nall + 1024, precision)
    x = torch.as_tensor(slab.x, device="cuda")
    system = ljx.System(x=x, type=torch.as_tensor(slab.types, device="cuda"),
                        f=torch.zeros_like(x), nlocal=nlocal, nghost=nall - nlocal,
                        newton_pair=cfg["newton"], unit_style="metal",
                        ntypes=len(cfg["elements"]))
    pair = ljx.PairJax(device=local)
    pair.coeff(system, "*", "*", str(path))
    pair.init_style(system)
    builder = ljx.synth.DeviceListBuilder(slab.x, nlocal, CUTOFF + SKIN, half=cfg["half"])
    system.list = builder.build(x)
    nccl = halo.NcclHalo(halo.slab_swaps(slab, rank, world), rank, world, local, timeout_ms=60000)
    system.comm = nccl
    exchanges = "reverse rho, forward F'(rho) and reverse forces" if cfg["newton"] else "F'(rho)"
    return system, nlocal, nall, {
        "pair": pair, "extra_launches": 0, "lists": builder, "halo": nccl, "ids": slab.ids,
        "parallelism": f"z-slab spatial decomposition over {world} GPUs; {exchanges} by libljx's "
                       "NCCL halo (ljx_halo: gather kernel, grouped ncclSend/ncclRecv with both "
                       "z-neighbors, x/y periodic images on the device); step totals by one "
                       "on-stream NCCL all-reduce (ljx_read_result_all)"}


def run_md(torch, ljx, cfg, cells, precision, steps, warmup):
    """C3's own run: NVE at dt = 1 fs with a neighbor rebuild every 10 steps, through the pair
    style (ljx_pair_compute) with the device MD step around it (lammps-jax_b200/md.py: fix nve
    integration, forward comm of positions to the periodic images, the device list rebuild every
    10th step). Seeded Gaussian velocities at 300 K. Times `steps` full MD steps after `warmup`."""
    import tempfile
    from importlib import import_module
    md = import_module("lammps_jax_b200.md")
    atoms = ljx.synth.fcc(cells, cfg["lattice"], jitter=JITTER, seed=2024)
    n = len(atoms.x)
    mass = np.array([ljx.synth.ELEMENTS[e]["mass"] for e in cfg["elements"]])
    v0 = md.maxwell_velocities(mass[atoms.types - 1], 300.0, "metal", seed=2026)
    nall = len(ljx.synth.periodic_ghosts(atoms.x, atoms.box, CUTOFF + SKIN)[0])
    path = Path(tempfile.mkdtemp()) / "md.json"
    _bundle(ljx, cfg, path, int(1.05 * nall) + 1024, precision)
    pair = ljx.PairJax()
    run = md.NVE(pair, atoms.x, atoms.types, atoms.box, mass, cutoff=CUTOFF, skin=SKIN, dt=0.001,
                 units="metal", newton_pair=cfg["newton"], half_list=cfg["half"], v=v0,
                 every=10, check=False, borders="when-needed")
    pair.coeff(run.system, "*", "*", str(path))
    pair.init_style(run.system)
    t0 = run.thermo(run.setup())
    for _ in range(warmup):
        run.step()
    stream = torch.cuda.current_stream()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for k in range(steps):
        res = run.step(eflag=(k == steps - 1))
    stop.record(stream)
    torch.cuda.synchronize()
    elapsed = start.elapsed_time(stop) / 1e3
    t1 = run.thermo(res)
    return {"value": n * steps / elapsed, "unit": UNIT, "ms_per_step": elapsed / steps * 1e3,
            "steps": steps, "warmup": warmup, "dt_fs": 1.0, "rebuild_every": 10,
            "list_builds": run.builds, "border_builds": run.border_builds,
            "temp_start_K": t0.temp, "temp_end_K": t1.temp,
            "etotal_drift_ev_per_atom": (t1.etotal - t0.etotal) / n,
            "what": "full MD step on the device: fix nve initial/final integrate, forward comm "
                    "of positions to the periodic images (the device list rebuild every 10th "
                    "step), pair style compute through ljx_pair_compute (energy at the last "
                    "step); velocities at 300 K"}


def time_list_build(torch, lists, x, stream, reps=5):
    """Device neighbor-list rebuild (ljx_neigh_bin + ljx_neigh_build) in ms, the mean of `reps`
    rebuilds into the same buffers after one untimed."""
    lists.launch(x, stream)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(reps):
        lists.launch(x, stream)
    stop.record(stream)
    torch.cuda.synchronize()
    return start.elapsed_time(stop) / reps


def run_e2e(torch, case, args, world, total_atoms):
    """Same step through the C ABI with host buffers: H2D of x and D2H of the forces and the
    result every step. Every `rebuild_every`-th step (10 for C3 and C4, every step for C5) the
    neighbor list is rebuilt on the device from the uploaded positions (ljx_neigh_bin +
    ljx_neigh_build into the same buffers), as LAMMPS-Kokkos builds it on the device."""
    import ctypes

    system, lists, ghosts = case.system, case.decomp["lists"], case.decomp.get("ghosts")
    period = args.rebuild_every if args.rebuild_every > 0 else 10
    nlocal, nghost = system.nlocal, system.nghost
    # One rank owning the whole box: upload the owned positions and fill their periodic images on
    # the device, as LAMMPS's comm does. Slabs (N > 1) upload every row: their ghosts come from
    # the neighbors. Only owned forces come back (ghost forces are folded into them with newton
    # on, unused with newton off).
    owned_only = ghosts is not None
    x_host = (system.x[:nlocal] if owned_only else system.x).cpu().pin_memory()
    f_host = torch.empty_like(system.f[:nlocal], device="cpu").pin_memory()
    stream = case.stream
    steps = max(3, min(args.steps, 10))
    lib = package().abi.load()
    streamed = args.e2e_pieces > 0 and case.streams_rows()

    def one(k):
        if owned_only:
            system.x[:nlocal].copy_(x_host, non_blocking=True)
            owner, shift = ghosts
            st = lib.ljx_ghost_positions(ctypes.c_void_p(stream.cuda_stream),
                                         ctypes.c_void_p(system.x.data_ptr()), nlocal, nghost,
                                         ctypes.c_void_p(owner.data_ptr()),
                                         ctypes.c_void_p(shift.data_ptr()))
            if st != 0:
                raise RuntimeError(f"ljx_ghost_positions failed ({st})")
        else:
            system.x.copy_(x_host, non_blocking=True)
        if k % period == 0:
            lists.launch(system.x, stream)
        ago = k % period if args.rebuild_every > 0 else -1
        if streamed:
            # The force rows go to the host piece by piece under the force pass; the result
            # read that ends the step waits for the last piece.
            case.core(ago, f_host=f_host, pieces=args.e2e_pieces)
        else:
            case.core(ago)  # ends with the result read
            f_host.copy_(system.f[:nlocal], non_blocking=True)
            stream.synchronize()                                # forces on the host
        return x_host.numel() * 8

    one(1)
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    h2d = 0
    for k in range(steps):
        h2d += one(k)
    stop.record(stream)
    torch.cuda.synchronize()
    elapsed = start.elapsed_time(stop) / 1e3
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([elapsed], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed = float(t.item())
    value = total_atoms * steps / elapsed
    return {"value": value, "unit": UNIT, "h2d_bytes_per_step": h2d / steps,
            "d2h_bytes_per_step": f_host.numel() * 8 + (12 if world > 1 else 9) * 8,
            "steps": steps,
            "x_upload": ("owned rows; periodic images filled on the device (ljx_ghost_positions)"
                         if owned_only else "owned and ghost rows"),
            "list": ("rebuilt on the device every step from the uploaded positions" if period == 1
                     else f"rebuilt on the device every {period}th step from the uploaded "
                          "positions"),
            "f_download": (f"streamed under the force pass in {args.e2e_pieces} row pieces "
                           "(ljx_force_to_host)" if streamed
                           else "one copy after the step")}


def reference_sample(ljx, oracle, args):
    """The bench workload for the CPU oracle (the restatement of the reference's path): the
    C3 crystal of one GPU's share (2,048,000 atoms, the same atoms as the N=1 GPU run), the full
    C5 liquid, or for C4 (16.4 M atoms, minutes per CPU step) a 40^3-cell replica of its crystal.
    Returns (one_step, atoms, workload text, same_config)."""
    cfg = CONFIGS[args.config]
    cells = args.cells or cfg["cells"]
    if cfg.get("liquid"):
        atoms = liquid_atoms(ljx, cfg, cells)
        same = True
    elif cfg["strong"]:
        atoms = crystal_atoms(ljx, cfg, (40, 40, 40))
        same = False
    else:
        atoms = crystal_atoms(ljx, cfg, (cells, cells, cells))
        same = True
    x_all, owner = ljx.synth.periodic_ghosts(atoms.x, atoms.box, CUTOFF + SKIN)
    types_all = np.concatenate([atoms.types, atoms.types[owner]]).astype(np.int32)
    nlocal = len(atoms.x)
    tables = oracle.parse_setfl_text(ljx.synth.synthetic_setfl(cfg["elements"]))
    lst = oracle.build_list(x_all, nlocal, CUTOFF + SKIN, half=cfg["half"])
    mode = "half-unique" if cfg["half"] else "rows-full"
    workload = cfg["title"].format(c=cells if same else 40) + f" ({nlocal:,} atoms in all)"

    def one_step():
        oracle.eam_step(tables, x_all, types_all, nlocal, owner, lst, mode=mode,
                        precision=args.precision)

    return one_step, nlocal, workload, same


CPU_STEP_BUDGET_S = 420.0


def cpu_baseline(args, steps=2):
    """The CPU restatement (oracle, all host threads) on the workload of one GPU, a bounded
    number of steps."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle
    oracle.lib()
    threads = os.cpu_count() or 1
    oracle.set_threads(threads)
    one_step, nlocal, workload, _ = reference_sample(package(), oracle, args)
    t0 = time.perf_counter()
    for _ in range(steps):
        one_step()
    dt = time.perf_counter() - t0
    return {"value": nlocal * steps / dt, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{workload}: {steps} full steps (pack from the list + density + "
                      "embedding + exchange + forces + virial), oracle/eam_oracle.c with "
                      f"OpenMP on {threads} threads"}


def run_reference(args):
    """The reference's path on the host cores: the CPU restatement of its per-step work
    (oracle/, OpenMP on every host thread) on the bench's own workload, `warmup` untimed and
    `steps` timed steps. Under torchrun only rank 0 runs it; the others exit without work."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle
    oracle.lib()
    threads = os.cpu_count() or 1
    oracle.set_threads(threads)
    cfg = CONFIGS[args.config]
    one_step, nlocal, workload, same = reference_sample(package(), oracle, args)
    t0 = time.perf_counter()
    for _ in range(args.warmup):
        one_step()
    per_step = (time.perf_counter() - t0) / max(1, args.warmup)
    # All the requested steps when they fit the budget (the driver's runs do); otherwise as many
    # as fit, said in the line.
    steps = (args.steps if args.warmup == 0 or per_step * args.steps <= CPU_STEP_BUDGET_S
             else max(1, int(CPU_STEP_BUDGET_S / per_step)))
    t0 = time.perf_counter()
    for _ in range(steps):
        one_step()
    dt = time.perf_counter() - t0
    value = nlocal * steps / dt
    share = "" if world == 1 else (f"; the GPU run's {world} ranks each own a share of this size "
                                   "(weak scaling), the CPU runs one share")
    sample = (f"{workload}, {args.warmup} warm-up and {steps} timed steps on {threads} threads"
              + ("" if same else "; a 40^3-cell replica of the C4 crystal") + share)
    print(json.dumps({
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": steps, "warmup": args.warmup, "ms_per_step": dt / steps * 1e3,
        "higher_is_better": True, "scaling": cfg["scaling"], "vs_baseline": None,
        "dtype": "f64" if args.precision == "float64" else "f32", "data": "synthetic",
        "impl": "reference",
        "config": {"workload": workload, "name": args.config, "total_atoms": nlocal,
                   "precision": args.precision},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference's own CPU path (LAMMPS Kokkos-OpenMP + XLA CPU PJRT) cannot be "
                "installed offline (no LAMMPS, MPI, jaxlib or PJRT plugin on the box); this "
                "times oracle/eam_oracle.c, the CPU restatement of that path's per-step work",
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ljx", "reference"), default="ljx")
    ap.add_argument("--precision", choices=("float64", "float32"), default=None,
                    help="default: float64 (c3, c4), float32 (c5)")
    ap.add_argument("--rebuild-every", type=int, default=None,
                    help="neighbor rebuild period the engine is told (neighbor->ago); C3 and C4 "
                         "rebuild every 10 steps (the default), C5 every step. 0 turns the "
                         "candidate cache off")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="c3",
                    help="c3: weak scaling (the default bench line); c4: strong scaling of the "
                         "16.4 M-atom binary crystal; c5: the edge-pack stress test (one GPU)")
    ap.add_argument("--cells", type=int, default=None,
                    help="fcc cells per edge: of each rank's box for c3 (default 80, the "
                         "2,048,000-atom config), of the whole box for c4 (default 160); the "
                         "fcc-cell equivalent of the liquid box for c5 (default 80)")
    ap.add_argument("--skip-extras", action="store_true",
                    help="time the device path only (no e2e, MD, C4 or CPU-baseline legs); for "
                         "profiling")
    ap.add_argument("--no-c4", action="store_true",
                    help="leave out the C4 strong-scaling object of the c3 line")
    ap.add_argument("--e2e-pieces", type=int, default=8,
                    help="row pieces of the e2e force pass whose force rows are copied to the "
                         "host as each finishes (ljx_force_to_host); 0: one copy after the step")
    ap.add_argument("--fp-overlap", choices=("on", "off"), default="off",
                    help="across GPUs, run the F' exchange under the force pass's rows without "
                         "ghost neighbors (ljx_force_rows); measured slower at 2 GPUs (force "
                         "phase 1.85 -> 2.19 ms against a 0.04 ms exchange), so off by default")
    ap.add_argument("--quick", action="store_true",
                    help="time the device path, the e2e and the force-only legs only (no MD, "
                         "C4, float32 or CPU-baseline legs)")
    args = ap.parse_args()
    if args.precision is None:
        args.precision = CONFIGS[args.config].get("precision", "float64")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ljx(args)


if __name__ == "__main__":
    main()
