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
threads) on a bounded sample of the same workload (a 40^3-cell replica) and prints the same line
with "impl": "reference".

Multi-GPU runs (torchrun, one rank per GPU) use spatial decomposition along z: every rank owns a
2,048,000-atom slab of a larger crystal (weak scaling) and exchanges F'(rho) of its boundary
atoms with its two z-neighbors over NCCL each step.

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


def profile_l1(kernel: str):
    """Measured L1 data-pipe (LSU wavefront) utilisation of `kernel` from the committed ncu
    summary, if present: the resource that bounds the gather kernels."""
    path = ROOT / "profiles" / "l1_wavefronts.txt"
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


def profile_traffic(kernel: str):
    """DRAM bytes per launch of `kernel` from the committed ncu summary, if present."""
    path = ROOT / "profiles" / "dram_traffic.txt"
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


def run_ljx(args):
    import torch
    import torch.distributed as dist

    ljx = package()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=datetime.timedelta(seconds=180))
    cfg = CONFIGS[args.config]
    precision = args.precision or cfg.get("precision", "float64")
    if args.rebuild_every is None:
        args.rebuild_every = cfg.get("rebuild_every", 10)
    if cfg.get("one_gpu") and world > 1:
        raise SystemExit(f"--config {args.config} runs on one GPU")
    if cfg["strong"]:
        total = args.cells or cfg["cells"]
        if total % world:
            raise SystemExit(f"--config {args.config}: {total} z-cells do not split over {world} GPUs")
        cells = (total, total, total // world)
    else:
        n = args.cells or cfg["cells"]
        cells = (n, n, n)
    if world > 1:
        system, nlocal, nall, decomp = setup_decomposed(ljx, cfg, cells, rank, world, precision,
                                                        local)
    else:
        system, nlocal, nall, decomp = setup_single(ljx, cfg, cells, precision)
    pair = decomp["pair"]
    plan = pair.plan
    newton = system.newton_pair
    stream = torch.cuda.current_stream()
    eng = pair.engine
    atoms = system.atoms()
    nl = system.list.struct()
    fp_rows, width, elem = eng.feature_rows(1)
    rho_rows = eng.feature_rows(0)[0]

    names = ["pack_atoms", "density", "embed", "halo_fp", "force", "result"]
    tick = [0]

    def core(ago, mark=lambda k: None):
        """One pair-style step on device data, with the exchanges the engine's plan asks for."""
        nl.ago = ago
        mark(0)
        eng.pack_atoms(atoms)
        mark(1)
        eng.density(atoms, nl, newton)
        if plan.reverse_density:
            system.comm.reverse(rho_rows, width, elem)
        mark(2)
        eng.embed(atoms)
        mark(3)
        if plan.forward_fp:
            system.comm.forward(fp_rows, width, elem)
        mark(4)
        eng.force(atoms, nl, newton, 1.0)
        if plan.reverse_force:
            system.comm.reverse_forces(system.f)  # LAMMPS's own reverse comm of ghost forces
        mark(5)
        res = eng.read_result()
        if world > 1:
            # Collective capacity check, as the pair style's MPI_Allreduce after execution.
            flags = torch.tensor([res.edge_count, res.overflow], device="cuda")
            dist.all_reduce(flags, op=dist.ReduceOp.MAX)
            if int(flags[1].item()):
                raise RuntimeError("LAMMPS-JAX edge capacity exceeded")
        mark(6)
        return res

    def step(events=None):
        def mark(k):
            if events is not None:
                events[k].record(stream)
        # neighbor->ago as LAMMPS reports it with a rebuild every `rebuild_every` steps; the
        # engine rebuilds its candidate cache on ago == 0 (-1: cache off).
        ago = tick[0] % args.rebuild_every if args.rebuild_every > 0 else -1
        tick[0] += 1
        return core(ago, mark)

    system.f.zero_()
    kevents = [[torch.cuda.Event(enable_timing=True) for _ in range(7)] for _ in range(args.steps)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # The clock samples span the warm-up and the timed steps (both under load).
    with ClockSampler(local, ROOT / "gpurun_out" / f"clocks_rank{rank}.csv") as clocks:
        for _ in range(args.warmup):
            res = step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        launches0 = eng.launches
        start.record(stream)
        for k in range(args.steps):
            res = step(kevents[k])
        stop.record(stream)
        torch.cuda.synchronize()
    elapsed = start.elapsed_time(stop) / 1e3
    if world > 1:
        t = torch.tensor([elapsed], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed = float(t.item())
    # Our kernels per step: pack_atoms, density, embed, forward exchange, force, finalize.
    launches = (eng.launches - launches0) + args.steps * decomp["comm_launches"]
    phase = {n: 0.0 for n in names}
    for ev in kevents:
        for k, n in enumerate(names):
            phase[n] += ev[k].elapsed_time(ev[k + 1]) / 1e3
    phase = {n: v / args.steps for n, v in phase.items()}

    # Algorithmic bytes per launch (per step) of the two row kernels.
    nn = system.list.numneigh[:nlocal].to(torch.int64)
    listed = int(nn.sum().item())
    kept = int(res.edge_count)
    real = 8 if precision == "float64" else 4
    bytes_density = 4 * listed + 4 * nlocal * 2 + 32 * nall + 4 * kept + 4 * nlocal + real * nlocal
    pos_bytes = 32 if precision == "float64" else 16
    bytes_force = 8 * nlocal + 4 * kept + pos_bytes * nall + real * nall + 48 * nlocal
    kernel = max(("density", "force"), key=lambda n: phase[n])
    kbytes = bytes_density if kernel == "density" else bytes_force
    achieved = kbytes / phase[kernel] / 1e9
    peak, peak_kind = peaks()
    # The engine caches candidates only for lists that live at least 4 steps (kCacheMinPeriod in
    # csrc/engine.cu); shorter-lived lists take the list pass.
    cached = args.rebuild_every >= 4
    kname = {"density": (f"k_density_groups_full_{precision}" if cached
                         else f"k_density_full_{precision}"),
             "force": f"k_force_rows_full_{precision}"}[kernel]
    # Committed DRAM captures: the C3 kernels by name, the C5 ones as "c5:<name>".
    traffic = {"c3": profile_traffic(kname),
               "c5": profile_traffic(f"c5:{kname}")}.get(args.config)
    l1 = {"c3": profile_l1(kname), "c5": profile_l1(f"c5:{kname}")}.get(args.config)

    total_atoms, energy_total = nlocal, res.energy
    if world > 1:
        t = torch.tensor([nlocal], dtype=torch.int64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        total_atoms = int(t.item())
        t = torch.tensor([res.energy], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        energy_total = float(t.item())
    neigh_ms = time_list_build(torch, decomp["lists"], system.x, stream)
    e2e = None if args.skip_extras else run_e2e(torch, system, core, args, world,
                                                 decomp["lists"], total_atoms,
                                                 decomp.get("ghosts"))
    value = total_atoms * args.steps / elapsed
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": elapsed / args.steps * 1e3,
        "higher_is_better": True, "scaling": cfg["scaling"], "vs_baseline": None,
        "dtype": "f64" if precision == "float64" else "f32", "data": "synthetic",
        "config": {
            "workload": cfg["title"].format(c=cells[0]) + f" ({total_atoms:,} atoms in all)",
            "name": args.config, "total_atoms": total_atoms,
            "atoms_per_gpu": nlocal, "ghosts_per_gpu": nall - nlocal,
            "listed_pairs_per_atom": listed / nlocal, "kept_edges_per_atom": kept / nlocal,
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
                     "limiter": {"resource": "L1 data pipe (LSU wavefronts): random gathers of "
                                             "positions and spline rows",
                                 "frac": l1, "source": "ncu capture of the same kernel on its "
                                                       "small case (profiles/l1_wavefronts.txt)"},
                     "bytes_basis": "per-step algorithmic bytes of the reference's data flow "
                                    "(list read every step); with the candidate cache the list "
                                    "is read only at rebuilds, so this is an effective bandwidth"
                                    if kernel == "density" and cached else
                                    "per-launch algorithmic bytes"},
        "gpu_launches": launches,
        "e2e": e2e,
        "energy_per_atom": energy_total / total_atoms,
    }
    if world == 1 and not args.skip_extras and args.config == "c3":
        line["md"] = run_md(torch, ljx, cfg, cells, precision, args.steps, args.warmup)
        line["cpu_baseline"] = cpu_baseline(args)
    clocks_summary = clocks.summary()
    line["clocks"] = clocks_summary
    if world > 1:
        dist.barrier()
    if rank == 0:
        print(json.dumps(line), flush=True)
    pair.engine.close()
    if world > 1:
        decomp["close"]()
        dist.destroy_process_group()


def _types_fn(cfg):
    if cfg["fractions"] is None:
        return None
    ljx = package()
    return lambda n, seed: ljx.synth.substitutional(n, cfg["fractions"], seed=seed)


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
    types = _types_fn(cfg)(n_tile, 2025)
    return ljx.synth.liquid_packing(n_tile, cfg["liquid"], 2.0, seed=2024, tiles=tiles,
                                    types=types)


def setup_single(ljx, cfg, cells, precision):
    import tempfile

    import torch
    types_fn = _types_fn(cfg)
    if cfg.get("liquid"):
        atoms = liquid_atoms(ljx, cfg, cells[0])
    else:
        n = 4 * cells[0] * cells[1] * cells[2]
        types = types_fn(n, 2025) if types_fn else None
        atoms = ljx.synth.fcc(cells, cfg["lattice"], jitter=JITTER, seed=2024, types=types)
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
    return system, nlocal, nall, {"pair": pair, "parallelism": "single GPU (periodic self-images)",
                                  "comm_launches": 1, "lists": builder, "ghosts": ghosts}


def setup_decomposed(ljx, cfg, cells, rank, world, precision, local):
    """Rank `rank` of a z-slab decomposition of `cells` per rank."""
    import tempfile

    import torch
    from importlib import import_module
    halo = import_module("lammps_jax_b200.halo")
    slab = ljx.synth.slab_decomposition(cells, cfg["lattice"], JITTER, 2024, rank, world,
                                        CUTOFF + SKIN, types_fn=_types_fn(cfg))
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
    elem = 8 if precision == "float64" else 4
    system.comm = halo.SlabExchange(slab, 1, elem)
    exchanges = "reverse rho, forward F'(rho) and reverse forces" if cfg["newton"] else "F'(rho)"
    return system, nlocal, nall, {
        "pair": pair, "comm_launches": system.comm.launches_per_exchange, "lists": builder,
        "parallelism": f"z-slab spatial decomposition over {world} GPUs; {exchanges} by grouped "
                       "NCCL send/recv with both z-neighbors + x/y periodic images",
        "close": lambda: None}


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


def run_e2e(torch, system, core, args, world, lists, total_atoms, ghosts=None):
    """Same step through the C ABI with host buffers: H2D of x and D2H of the forces and the
    result every step. Every `rebuild_every`-th step (10 for C3 and C4, every step for C5) the
    neighbor list is rebuilt on the device from the uploaded positions (ljx_neigh_bin +
    ljx_neigh_build into the same buffers), as LAMMPS-Kokkos builds it on the device."""
    import ctypes

    period = args.rebuild_every if args.rebuild_every > 0 else 10
    nlocal, nghost = system.nlocal, system.nghost
    # One rank owning the whole box: upload the owned positions and fill their periodic images on
    # the device, as LAMMPS's comm does. Slabs (N > 1) upload every row: their ghosts come from
    # the neighbors. Only owned forces come back (ghost forces are folded into them with newton
    # on, unused with newton off).
    owned_only = ghosts is not None
    x_host = (system.x[:nlocal] if owned_only else system.x).cpu().pin_memory()
    f_host = torch.empty_like(system.f[:nlocal], device="cpu").pin_memory()
    stream = torch.cuda.current_stream()
    steps = max(3, min(args.steps, 10))
    lib = package().abi.load()

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
        core(k % period if args.rebuild_every > 0 else -1)  # ends with the result read (a sync)
        f_host.copy_(system.f[:nlocal], non_blocking=True)
        torch.cuda.current_stream().synchronize()        # forces on the host
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
            "d2h_bytes_per_step": f_host.numel() * 8 + 9 * 8, "steps": steps,
            "x_upload": ("owned rows; periodic images filled on the device (ljx_ghost_positions)"
                         if owned_only else "owned and ghost rows"),
            "list": ("rebuilt on the device every step from the uploaded positions" if period == 1
                     else f"rebuilt on the device every {period}th step from the uploaded "
                          "positions")}


def reference_sample(ljx, oracle, args):
    """A bounded CPU sample of the bench workload for the oracle: a 40^3-cell replica of the C3 or
    C4 crystal (the same lattice, species, potential, cutoffs and list kind) or one 32,000-atom
    tile of the C5 liquid. Returns (one_step, atoms, description)."""
    cfg = CONFIGS[args.config]
    if cfg.get("liquid"):
        atoms = liquid_atoms(ljx, cfg, 20)
        what = "one 32,000-atom tile of the C5 liquid"
    else:
        n = 40
        tf = _types_fn(cfg)
        atoms = ljx.synth.fcc((n, n, n), cfg["lattice"], jitter=JITTER, seed=7,
                              types=tf(4 * n ** 3, 2025) if tf else None)
        what = f"{n}^3-cell replica of the {args.config.upper()} crystal"
    x_all, owner = ljx.synth.periodic_ghosts(atoms.x, atoms.box, CUTOFF + SKIN)
    types_all = np.concatenate([atoms.types, atoms.types[owner]]).astype(np.int32)
    nlocal = len(atoms.x)
    tables = oracle.parse_setfl_text(ljx.synth.synthetic_setfl(cfg["elements"]))
    lst = oracle.build_list(x_all, nlocal, CUTOFF + SKIN, half=cfg["half"])
    mode = "half-unique" if cfg["half"] else "rows-full"

    def one_step():
        oracle.eam_step(tables, x_all, types_all, nlocal, owner, lst, mode=mode,
                        precision=args.precision)

    return one_step, nlocal, f"{what} ({nlocal} atoms, {mode}, {args.precision})"


def cpu_baseline(args, steps=2):
    """The CPU restatement (oracle, all host threads) on a bounded replica of the workload."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle
    oracle.lib()
    threads = os.cpu_count() or 1
    oracle.set_threads(threads)
    one_step, nlocal, what = reference_sample(package(), oracle, args)
    one_step()
    t0 = time.perf_counter()
    for _ in range(steps):
        one_step()
    dt = time.perf_counter() - t0
    return {"value": nlocal * steps / dt, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{what}: {steps} full steps (pack + density + embedding + exchange + "
                      "forces + virial), oracle/eam_oracle.c with OpenMP"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle
    oracle.lib()
    threads = os.cpu_count() or 1
    oracle.set_threads(threads)
    cfg = CONFIGS[args.config]
    one_step, nlocal, what = reference_sample(package(), oracle, args)
    steps = max(1, min(args.steps, 5))
    for _ in range(min(args.warmup, 1)):
        one_step()
    t0 = time.perf_counter()
    for _ in range(steps):
        one_step()
    dt = time.perf_counter() - t0
    value = nlocal * steps / dt
    sample = f"{what}, {steps} timed steps"
    print(json.dumps({
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": int(os.environ.get("WORLD_SIZE", "1")),
        "steps": steps, "warmup": min(args.warmup, 1), "ms_per_step": dt / steps * 1e3,
        "higher_is_better": True, "scaling": cfg["scaling"], "vs_baseline": None,
        "dtype": "f64" if args.precision == "float64" else "f32", "data": "synthetic",
        "impl": "reference",
        "config": {"workload": cfg["title"].format(c=cfg["cells"]) + " (CPU sample)",
                   "name": args.config, "precision": args.precision},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference's own CPU path (LAMMPS Kokkos-OpenMP + XLA CPU PJRT) is not "
                "installable offline; this times the CPU restatement of that path",
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
                    help="time the device path only (no e2e or CPU-baseline legs); for profiling")
    args = ap.parse_args()
    if args.precision is None:
        args.precision = CONFIGS[args.config].get("precision", "float64")
    (ROOT / "gpurun_out").mkdir(exist_ok=True)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ljx(args)


if __name__ == "__main__":
    main()
