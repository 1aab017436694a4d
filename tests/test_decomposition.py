"""z-slab spatial decomposition (the multi-GPU layout) on CPU.

1. Geometry: each rank's ghost rows are exactly its neighbors' send lists, in order.
2. Physics: every rank's rows-full evaluation, with ghost F' taken from the true owners across
   ranks, reproduces the all-pairs minimum-image forces and energy of the whole periodic crystal
   (the oracle runs the ranks as one combined system whose ghost rows point at owners on any rank).
3. Transport: SlabExchange over a real 2-rank gloo process group fills every ghost row with its
   owner's value (forward) and adds every ghost row back into its owner (reverse), with host
   stand-ins for the row operations (on GPUs the ljx_comm_* kernels do them).
4. Identity: the slabs of every rank count own exactly the atoms of the whole crystal.
5. The swap table of libljx's NCCL halo, applied with the host restatement of its semantics,
   fills and folds every ghost row for 1, 2 and 3 ranks.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cases import F64_FORCE_REL, F64_TOTAL_REL, Case
from conftest import load_package
from test_oracle_modes import minimum_image_reference

CELLS, A, JITTER, SEED, CUT = (4, 4, 4), 3.615, 0.08, 7, 8.5


def slabs(ljx, nranks):
    return [ljx.synth.slab_decomposition(CELLS, A, JITTER, SEED, r, nranks, CUT)
            for r in range(nranks)]


@pytest.mark.parametrize("nranks", [2, 3])
def test_ghost_rows_are_neighbor_send_lists(ljx, nranks):
    parts = slabs(ljx, nranks)
    for r, s in enumerate(parts):
        low, up = parts[(r - 1) % nranks], parts[(r + 1) % nranks]
        got_low = s.x[s.nlocal:s.nlocal + s.n_low]
        exp_low = low.x[low.send_up].copy()
        if r == 0:
            exp_low[:, 2] -= s.box[2]
        np.testing.assert_array_equal(got_low, exp_low)
        got_up = s.x[s.nlocal + s.n_low:s.nlocal + s.n_low + s.n_up]
        exp_up = up.x[up.send_down].copy()
        if r == nranks - 1:
            exp_up[:, 2] += s.box[2]
        np.testing.assert_array_equal(got_up, exp_up)
        assert np.all(s.x[:s.nlocal, 2] >= s.zlo) and np.all(s.x[:s.nlocal, 2] < s.zhi)


def test_slabs_tile_the_crystal_without_overlap(ljx):
    """Owned atoms of all ranks form one physical crystal: no site duplicated across a face."""
    from scipy.spatial import cKDTree
    parts = slabs(ljx, 3)
    x = np.concatenate([p.x[:p.nlocal] for p in parts])
    assert len(x) == 3 * 4 * np.prod(CELLS)
    tree = cKDTree(x, boxsize=parts[0].box)
    assert not tree.query_pairs(1.5)


def combined_owner(parts):
    """Owner (in the combined owned index space) of every ghost row of every rank."""
    nranks = len(parts)
    offsets = np.cumsum([0] + [p.nlocal for p in parts])
    owners = []
    for r, s in enumerate(parts):
        low, up = parts[(r - 1) % nranks], parts[(r + 1) % nranks]
        base_rows = np.concatenate([offsets[r] + np.arange(s.nlocal),
                                    offsets[(r - 1) % nranks] + low.send_up,
                                    offsets[(r + 1) % nranks] + up.send_down])
        owners.append(np.concatenate([base_rows[s.nlocal:], base_rows[s.xy_owner]]))
    return owners, offsets


def test_decomposed_physics_matches_whole_crystal(ljx, oracle):
    parts = slabs(ljx, 2)
    text = ljx.synth.synthetic_setfl(("Cu",), nr=800, nrho=800)
    tables = oracle.parse_setfl_text(text)
    owners, offsets = combined_owner(parts)
    n_owned = int(offsets[-1])
    # Combined rows: all owned atoms (rank order), then every rank's ghosts.
    x_rows = [p.x[:p.nlocal] for p in parts] + [p.x[p.nlocal:] for p in parts]
    x_all = np.concatenate(x_rows)
    ghost_base = n_owned + np.cumsum([0] + [p.nghost for p in parts])
    senders, receivers = [], []
    for r, s in enumerate(parts):
        lst = oracle.build_list(s.x, s.nlocal, CUT, half=False)
        snd, rcv, msk, count, _ = oracle.pack_edges(
            s.x, lst[0], lst[1], lst[2], 1, lst[3], s.nlocal, lst[4], len(s.x),
            int(lst[1][:s.nlocal].sum()) + 1, 6.5, nlocal=s.nlocal)
        remap = np.concatenate([offsets[r] + np.arange(s.nlocal),
                                ghost_base[r] + np.arange(s.nghost)])
        senders.append(remap[snd[:count]])
        receivers.append(remap[rcv[:count]])
    senders = np.concatenate(senders).astype(np.int32)
    receivers = np.concatenate(receivers).astype(np.int32)
    order = np.argsort(senders, kind="stable")
    senders, receivers = senders[order], receivers[order]
    owner_all = np.concatenate(owners).astype(np.int32)
    out = oracle.eam_model(tables, x_all, np.zeros(len(x_all), np.int32), n_owned,
                           len(x_all) - n_owned, senders, receivers,
                           np.ones(len(senders), np.uint8), "rows-full", owner=owner_all)
    box = parts[0].box
    glob = Case(text, x_all[:n_owned], np.ones(n_owned, np.int32), n_owned, np.zeros(0, int),
                box, 6.5, 2.0, 1)
    e_ref, f_ref, v_ref = minimum_image_reference(oracle, glob)
    fmax = np.max(np.abs(f_ref))
    assert np.max(np.abs(out.model_force[:n_owned] - f_ref)) <= F64_FORCE_REL * fmax
    assert out.energy == pytest.approx(e_ref, rel=F64_TOTAL_REL)
    assert np.max(np.abs(out.virial - v_ref)) <= 1e-11 * np.max(np.abs(v_ref))


class HostRowOps:
    """The row operations of halo.GpuRowOps on CPU tensors (width-1 double rows), so the
    transport runs over a real gloo process group without a GPU."""

    def pack_forward(self, rows, w, e, sendlist, buf):
        buf[: sendlist.numel()] = rows[sendlist.long()]

    def unpack_forward(self, rows, w, e, first, n, buf):
        rows[first:first + n] = buf[:n]

    def self_forward(self, rows, w, e, owner, first):
        rows[first:first + owner.numel()] = rows[owner.long()]

    def self_reverse(self, rows, w, e, owner, first):
        n = owner.numel()
        rows.index_add_(0, owner.long(), rows[first:first + n].clone())
        rows[first:first + n] = 0

    def pack_reverse(self, rows, w, e, first, n, buf):
        buf[:n] = rows[first:first + n]

    def unpack_reverse(self, rows, w, e, sendlist, buf):
        rows.index_add_(0, sendlist.long(), buf[: sendlist.numel()].clone())

    def zero_rows(self, rows, w, e, first, n):
        rows[first:first + n] = 0


def _exchange_worker(rank, nranks, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=nranks)
    try:
        ljx = load_package()
        from lammps_jax_b200.halo import SlabExchange
        parts = slabs(ljx, nranks)
        s = parts[rank]
        owners, offsets = combined_owner(parts)
        ex = SlabExchange(s, 1, 8, device="cpu", ops=HostRowOps())
        # Forward: every ghost row takes its owner's value (the owner's combined index).
        rows = torch.full((len(s.x),), -1.0, dtype=torch.float64)
        rows[:s.nlocal] = torch.arange(s.nlocal, dtype=torch.float64) + float(offsets[rank])
        ex.forward(rows)
        forward_ok = bool(np.array_equal(rows[s.nlocal:].numpy(), owners[rank].astype(float)))
        # Reverse: every ghost row carries 1; each owned row must end up with the number of its
        # ghost copies on all ranks, and every ghost row with 0.
        rows = torch.zeros(len(s.x), dtype=torch.float64)
        rows[s.nlocal:] = 1.0
        ex.reverse(rows)
        counts = np.bincount(np.concatenate(owners), minlength=int(offsets[-1]))
        mine = counts[offsets[rank]:offsets[rank] + s.nlocal].astype(float)
        reverse_ok = bool(np.array_equal(rows[:s.nlocal].numpy(), mine) and
                          not np.any(rows[s.nlocal:].numpy()))
        results[rank] = (forward_ok, reverse_ok)
    finally:
        dist.destroy_process_group()


def free_port():
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


@pytest.mark.parametrize("nranks", [2])
def test_slab_exchange_over_gloo(nranks):
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    mp.spawn(_exchange_worker, args=(nranks, free_port(), results), nprocs=nranks, join=True)
    assert dict(results) == {r: (True, True) for r in range(nranks)}


@pytest.mark.parametrize("nranks", [1, 2, 3])
def test_slabs_are_one_crystal_at_every_rank_count(ljx, nranks):
    """Per-layer seeding: every decomposition owns exactly the atoms of the whole crystal (same
    coordinates, species and global ids), so runs at different GPU counts compare atom by atom."""
    cells = (4, 4, 6)
    whole = ljx.synth.layered_crystal(cells, A, JITTER, SEED, (0.64, 0.36))
    per = (cells[0], cells[1], cells[2] // nranks)
    parts = [ljx.synth.slab_decomposition(per, A, JITTER, SEED, r, nranks, CUT,
                                          fractions=(0.64, 0.36)) for r in range(nranks)]
    ids = np.concatenate([p.ids for p in parts])
    x = np.concatenate([p.x[:p.nlocal] for p in parts])
    t = np.concatenate([p.types[:p.nlocal] for p in parts])
    o, ow = np.argsort(ids), np.argsort(whole.ids)
    np.testing.assert_array_equal(ids[o], whole.ids[ow])
    np.testing.assert_array_equal(x[o], whole.x[ow])
    np.testing.assert_array_equal(t[o], whole.types[ow])


@pytest.mark.parametrize("nranks", [1, 2, 3])
def test_swap_table_fills_and_folds_every_ghost(ljx, nranks):
    """The swap table libljx's NCCL halo runs (halo.slab_swaps), applied with the host
    restatement of ljx_halo_forward/_reverse: forward fills every ghost row with its owner's
    value; reverse adds every ghost row into its owner and zeroes it."""
    from lammps_jax_b200.halo import apply_swaps, slab_swaps
    parts = slabs(ljx, nranks)
    owners, offsets = combined_owner(parts)
    swaps = [slab_swaps(p, r, nranks) for r, p in enumerate(parts)]
    rows = []
    for r, p in enumerate(parts):
        v = np.full((len(p.x), 2), -1.0)
        v[:p.nlocal, 0] = np.arange(p.nlocal) + offsets[r]
        v[:p.nlocal, 1] = 2.0 * (np.arange(p.nlocal) + offsets[r])
        rows.append(v)
    apply_swaps(rows, swaps, forward=True)
    for r, p in enumerate(parts):
        np.testing.assert_array_equal(rows[r][p.nlocal:, 0], owners[r])
        np.testing.assert_array_equal(rows[r][p.nlocal:, 1], 2.0 * owners[r])
    rows = []
    for p in parts:
        v = np.zeros((len(p.x), 2))
        v[p.nlocal:] = 1.0
        rows.append(v)
    apply_swaps(rows, swaps, forward=False)
    counts = np.bincount(np.concatenate(owners), minlength=int(offsets[-1]))
    for r, p in enumerate(parts):
        mine = counts[offsets[r]:offsets[r] + p.nlocal]
        np.testing.assert_array_equal(rows[r][:p.nlocal, 0], mine)
        np.testing.assert_array_equal(rows[r][:p.nlocal, 1], mine)
        assert not np.any(rows[r][p.nlocal:])
