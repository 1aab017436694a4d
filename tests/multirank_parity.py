"""Parity of the NCCL-decomposed engine against the CPU oracle on one crystal, N ranks.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node 2 --master-addr 127.0.0.1 \
        --master-port P tests/multirank_parity.py --out result.json

Every rank owns a z-slab of one binary Cu-Zr crystal (synth.fcc_layers: the same atoms at every
rank count) and runs one EAM step in each exchange pattern of the benchmark through libljx's
engine and NCCL halo (include/ljx_halo.h):
  rows-full    full list, newton off: forward F'(rho) (C3);
  half-unique  half list, newton on: reverse rho, forward F'(rho), reverse forces (C4).
Each pattern runs twice: with the F' exchange before the force pass, and with it on a side
stream under the force pass's rows that keep no ghost neighbor (NcclHalo.forward_under_force,
ljx_force_rows). Rank 0 gathers the owned forces by global site id and compares them, and the
collective energy and virial of ljx_read_result_all, with the CPU oracle (oracle/) on the whole
periodic crystal:
forces within 1e-10 of the largest |F|, energy and virial within 1e-12 relative. It writes a
JSON summary and exits non-zero on a mismatch. tests/test_gpu_multirank.py launches it when a
box has two GPUs or more.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
from conftest import ROOT, load_package  # noqa: E402

sys.path.insert(0, str(ROOT / "oracle"))

A, JITTER, SEED, CUT, RC = 0.64 * 3.615 + 0.36 * 4.525, 0.08, 17, 8.5, 6.5
FRACTIONS = (0.64, 0.36)
FORCE_REL, TOTAL_REL = 1e-10, 1e-12


def rank_step(ljx, mode, cells, rank, world, local, text, tmp, overlap=False):
    from lammps_jax_b200.halo import NcclHalo, slab_swaps
    newton, half = (False, False) if mode == "rows-full" else (True, True)
    s = ljx.synth.slab_decomposition(cells, A, JITTER, SEED, rank, world, CUT, fractions=FRACTIONS)
    nall = len(s.x)
    path = Path(tmp) / f"{mode}_{rank}.json"
    ljx.write_bundle(path, potential=ljx.eam_potential(text), max_atoms=nall + 64,
                     max_edges=(nall + 64) * 128, cutoff=RC, unit_style="metal",
                     precision="float64", force_output="atom-force",
                     newton="on" if newton else "off", comm=True, half_edges=half, n_species=2)
    x = torch.as_tensor(s.x, device="cuda")
    system = ljx.System(x=x, type=torch.as_tensor(s.types, device="cuda"), f=torch.zeros_like(x),
                        nlocal=s.nlocal, nghost=nall - s.nlocal, newton_pair=newton,
                        unit_style="metal", ntypes=2)
    system.list = ljx.synth.neighbor_list(s.x, s.nlocal, CUT, half=half)
    pair = ljx.PairJax(device=local)
    pair.coeff(system, "*", "*", str(path))
    pair.init_style(system)
    plan, eng = pair.plan, pair.engine
    halo = NcclHalo(slab_swaps(s, rank, world), rank, world, local, timeout_ms=60000)
    try:
        atoms, nl = system.atoms(), system.list.struct()
        fp_rows, width, elem = eng.feature_rows(1)
        rho_rows = eng.feature_rows(0)[0]
        eng.pack_atoms(atoms)
        eng.density(atoms, nl, newton)
        if plan.reverse_density:
            halo.reverse(rho_rows, width, elem)
        eng.embed(atoms)
        if plan.forward_fp and overlap:
            # The F' exchange on a side stream under the force pass's rows without ghosts.
            halo.forward_under_force(eng, atoms, nl, newton, fp_rows, width, elem)
        else:
            if plan.forward_fp:
                halo.forward(fp_rows, width, elem)
            eng.force(atoms, nl, newton, 1.0)
        if plan.reverse_force:
            halo.reverse_forces(system.f)
        res = halo.result_all(eng)
        torch.cuda.synchronize()
        forces = system.f[:s.nlocal].cpu().numpy()
    finally:
        halo.close()
        pair.close()
    return s.ids, forces, res


def whole_crystal(ljx, oracle, mode, cells_total, text):
    whole = ljx.synth.layered_crystal(cells_total, A, JITTER, SEED, FRACTIONS)
    x_all, owner = ljx.synth.periodic_ghosts(whole.x, whole.box, CUT)
    types_all = np.concatenate([whole.types, whole.types[owner]]).astype(np.int32)
    lst = oracle.build_list(x_all, len(whole.x), CUT, half=(mode == "half-unique"))
    ref = oracle.eam_step(oracle.parse_setfl_text(text), x_all, types_all, len(whole.x), owner,
                          lst, mode=mode, precision="float64")
    return whole.ids, ref


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    ap.add_argument("--cells", type=int, nargs=3, default=(6, 6, 4),
                    help="unit cells of each rank's slab")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                            timeout=datetime.timedelta(seconds=120))
    ljx = load_package()
    import oracle
    oracle.lib()
    text = ljx.synth.synthetic_setfl(("Cu", "Zr"), nr=2000, nrho=2000)
    cells = tuple(args.cells)
    cells_total = (cells[0], cells[1], cells[2] * world)
    summary, ok = {"ranks": world, "cells_per_rank": cells, "modes": {}}, True
    with tempfile.TemporaryDirectory() as tmp:
        for mode, overlap in (("rows-full", False), ("half-unique", False),
                              ("rows-full", True), ("half-unique", True)):
            ids, forces, res = rank_step(ljx, mode, cells, rank, world, local, text, tmp, overlap)
            name = mode + ("+overlap" if overlap else "")
            parts = [None] * world
            dist.all_gather_object(parts, (ids, forces))
            if rank == 0:
                g_ids = np.concatenate([p[0] for p in parts])
                g_f = np.concatenate([p[1] for p in parts])
                w_ids, ref = whole_crystal(ljx, oracle, mode, cells_total, text)
                same_atoms = bool(np.array_equal(np.sort(g_ids), np.sort(w_ids)))
                mine = g_f[np.argsort(g_ids)]
                theirs = ref.forces[np.argsort(w_ids)]
                fmax = float(np.max(np.abs(theirs)))
                ferr = float(np.max(np.abs(mine - theirs))) / fmax if same_atoms else float("inf")
                eerr = abs(res.energy - ref.energy) / abs(ref.energy)
                vscale = float(np.max(np.abs(ref.virial)))
                verr = float(np.max(np.abs(np.array(res.virial) - ref.virial))) / vscale
                good = (same_atoms and ferr <= FORCE_REL and eerr <= TOTAL_REL and
                        verr <= TOTAL_REL and res.edge_count == ref.count and not res.overflow)
                ok &= good
                summary["modes"][name] = {
                    "atoms": int(len(g_ids)), "kept_edges": int(res.edge_count),
                    "oracle_edges": int(ref.count), "force_err_rel_max": ferr,
                    "energy": res.energy, "oracle_energy": float(ref.energy),
                    "energy_err_rel": eerr, "virial_err_rel": verr, "pass": bool(good)}
            dist.barrier()
    if rank == 0:
        summary["pass"] = bool(ok)
        Path(args.out).write_text(json.dumps(summary, indent=1))
        print(json.dumps(summary), flush=True)
    ok_t = torch.tensor([1 if ok else 0], device="cuda")
    dist.broadcast(ok_t, 0)
    dist.destroy_process_group()
    sys.exit(0 if int(ok_t.item()) else 1)


if __name__ == "__main__":
    main()
