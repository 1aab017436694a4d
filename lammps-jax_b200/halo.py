"""Halo exchange of per-atom rows between z-slab neighbors over torch.distributed.

This is the standalone harness's stand-in for LAMMPS's comm on a brick decomposition along z.
Forward (owners to ghosts: F'(rho)):
  pack the rows each neighbor needs (by sendlist), one grouped NCCL send/recv with both
  z-neighbors, unpack into the ghost rows, then fill the x/y periodic images on the same rank.
Reverse (ghosts to owners, adding: rho partials, force rows):
  fold the x/y images into their owners on the same rank, pack the z-ghost rows, one grouped
  NCCL send/recv, add them into the sendlist rows they came from, and zero the z-ghost rows.
The message order is the same on every rank, so two ranks that are each other's upper and lower
neighbor (two slabs) match their messages in posting order.

Two transports:
  NcclHalo      the product path: libljx's ljx_halo (include/ljx_halo.h) with the slab's swap
                table (slab_swaps); every pack, grouped ncclSend/ncclRecv and unpack is issued
                by the library on the caller's stream, and the step result is one on-stream
                NCCL all-reduce (ljx_read_result_all).
  SlabExchange  the same exchange over a torch.distributed group (any backend, gloo on CPU in the
                tests), with the row operations behind a small interface (GpuRowOps: libljx's
                ljx_comm_* / ljx_halo_*_self kernels; host stand-ins in the CPU tests).
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch
import torch.distributed as dist

from . import abi


def _slots(width, elem):
    return (width * elem + 7) // 8


class GpuRowOps:
    """Row packing and unpacking with libljx's comm kernels (`rows` is a device address)."""

    def __init__(self):
        self.lib = abi.load()

    @staticmethod
    def _s():
        return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    @staticmethod
    def _check(st, what):
        if st != abi.OK:
            raise RuntimeError(f"{what} failed ({st})")

    def pack_forward(self, rows, width, elem, sendlist, buf):
        self._check(self.lib.ljx_comm_pack_forward(
            self._s(), ctypes.c_void_p(rows), width * elem // 4,
            ctypes.c_void_p(sendlist.data_ptr()), int(sendlist.numel()),
            ctypes.c_void_p(buf.data_ptr()), _slots(width, elem)), "ljx_comm_pack_forward")

    def unpack_forward(self, rows, width, elem, first, n, buf):
        self._check(self.lib.ljx_comm_unpack_forward(
            self._s(), ctypes.c_void_p(rows), width * elem // 4, first, n,
            ctypes.c_void_p(buf.data_ptr()), _slots(width, elem)), "ljx_comm_unpack_forward")

    def self_forward(self, rows, width, elem, owner, first):
        self._check(self.lib.ljx_halo_forward_self(
            self._s(), ctypes.c_void_p(rows), width, elem, ctypes.c_void_p(owner.data_ptr()),
            first, int(owner.numel())), "ljx_halo_forward_self")

    def self_reverse(self, rows, width, elem, owner, first):
        self._check(self.lib.ljx_halo_reverse_self(
            self._s(), ctypes.c_void_p(rows), width, elem, ctypes.c_void_p(owner.data_ptr()),
            first, int(owner.numel())), "ljx_halo_reverse_self")

    def pack_reverse(self, rows, width, elem, first, n, buf):
        self._check(self.lib.ljx_comm_pack_reverse(
            self._s(), ctypes.c_void_p(rows), width * elem // 4, first, n,
            ctypes.c_void_p(buf.data_ptr()), _slots(width, elem)), "ljx_comm_pack_reverse")

    def unpack_reverse(self, rows, width, elem, sendlist, buf):
        self._check(self.lib.ljx_comm_unpack_reverse(
            self._s(), ctypes.c_void_p(rows), width, elem, ctypes.c_void_p(sendlist.data_ptr()),
            int(sendlist.numel()), ctypes.c_void_p(buf.data_ptr()), _slots(width, elem)),
            "ljx_comm_unpack_reverse")

    def zero_rows(self, rows, width, elem, first, n):
        self._check(self.lib.ljx_comm_zero_rows(self._s(), ctypes.c_void_p(rows), width, elem,
                                                first, n), "ljx_comm_zero_rows")


class SlabExchange:
    """Forward and reverse exchange of feature rows for one rank of a slab decomposition.

    `width` / `elem_bytes` are the default row shape (the engine's feature rows); each call may
    pass another (forces: width 3, 8-byte elements). `ops` performs the row operations
    (GpuRowOps unless given)."""

    def __init__(self, slab, width: int, elem_bytes: int, device="cuda", group=None, ops=None):
        self.rank = dist.get_rank(group)
        self.nranks = dist.get_world_size(group)
        self.group = group
        self.device = device
        self.up = (self.rank + 1) % self.nranks
        self.down = (self.rank - 1) % self.nranks
        self.nlocal, self.n_low, self.n_up = slab.nlocal, slab.n_low, slab.n_up
        self.width, self.elem = width, elem_bytes
        self.send_up = torch.as_tensor(slab.send_up, device=device)
        self.send_down = torch.as_tensor(slab.send_down, device=device)
        self.xy_owner = torch.as_tensor(slab.xy_owner, device=device)
        self.ops = ops or GpuRowOps()
        self._buffers: dict = {}
        self.launches_per_exchange = 5

    @property
    def first_image(self) -> int:
        return self.nlocal + self.n_low + self.n_up

    def _bufs(self, width, elem):
        key = (width, elem)
        if key not in self._buffers:
            slots = _slots(width, elem)
            mk = lambda n: torch.zeros(max(n, 1) * slots, dtype=torch.float64,  # noqa: E731
                                       device=self.device)
            self._buffers[key] = {
                "send_up": mk(len(self.send_up)), "send_down": mk(len(self.send_down)),
                "low": mk(self.n_low), "up": mk(self.n_up)}
        return self._buffers[key]

    def _exchange(self, sends, recvs):
        ops = [dist.P2POp(dist.isend, buf, peer, self.group) for buf, peer in sends]
        ops += [dist.P2POp(dist.irecv, buf, peer, self.group) for buf, peer in recvs]
        for work in dist.batch_isend_irecv(ops):
            work.wait()

    def forward(self, rows, width=None, elem_bytes=None, stream=None):
        """Fill every ghost row of `rows` from its owner."""
        w, e = width or self.width, elem_bytes or self.elem
        b, ops = self._bufs(w, e), self.ops
        ops.pack_forward(rows, w, e, self.send_up, b["send_up"])
        ops.pack_forward(rows, w, e, self.send_down, b["send_down"])
        self._exchange([(b["send_up"], self.up), (b["send_down"], self.down)],
                       [(b["low"], self.down), (b["up"], self.up)])
        ops.unpack_forward(rows, w, e, self.nlocal, self.n_low, b["low"])
        ops.unpack_forward(rows, w, e, self.nlocal + self.n_low, self.n_up, b["up"])
        ops.self_forward(rows, w, e, self.xy_owner, self.first_image)

    def reverse(self, rows, width=None, elem_bytes=None, stream=None):
        """Add every ghost row of `rows` into its owner's row, then zero the ghost rows."""
        w, e = width or self.width, elem_bytes or self.elem
        b, ops = self._bufs(w, e), self.ops
        # x/y images first: their owners may be z-ghost rows, which go on to the neighbors.
        ops.self_reverse(rows, w, e, self.xy_owner, self.first_image)
        ops.pack_reverse(rows, w, e, self.nlocal, self.n_low, b["low"])
        ops.pack_reverse(rows, w, e, self.nlocal + self.n_low, self.n_up, b["up"])
        # Ghosts from below go back down, ghosts from above go back up; what comes back from
        # above lines up with send_up, what comes back from below with send_down.
        self._exchange([(b["low"], self.down), (b["up"], self.up)],
                       [(b["send_up"], self.up), (b["send_down"], self.down)])
        ops.unpack_reverse(rows, w, e, self.send_up, b["send_up"])
        ops.unpack_reverse(rows, w, e, self.send_down, b["send_down"])
        ops.zero_rows(rows, w, e, self.nlocal, self.n_low + self.n_up)

    def reverse_forces(self, f: torch.Tensor, stream=None):
        """LAMMPS's own reverse comm of ghost force rows (newton on)."""
        self.reverse(f.data_ptr(), 3, 8, stream)

    def allreduce_max(self, values):
        t = torch.tensor(list(values), dtype=torch.int64, device=self.device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
        return [int(v) for v in t.tolist()]


def slab_swaps(slab, rank: int, nranks: int):
    """LAMMPS-style swap table of one slab rank (include/ljx_halo.h), as dicts with host send
    lists. Stage 0 holds the two z swaps: this rank's top rows (send_up) go to the upper
    neighbor while the lower neighbor's top rows arrive as the low ghosts, and the mirror
    image. Stage 1 holds the x/y periodic images of owned and z-ghost rows, a self swap. With
    one rank both z swaps are self swaps too (the slab is its own neighbor along z)."""
    up, down = (rank + 1) % nranks, (rank - 1) % nranks
    first_image = slab.nlocal + slab.n_low + slab.n_up
    return [
        dict(stage=0, send_rank=up, recv_rank=down, sendlist=np.asarray(slab.send_up, np.int32),
             firstrecv=slab.nlocal, recvnum=slab.n_low),
        dict(stage=0, send_rank=down, recv_rank=up, sendlist=np.asarray(slab.send_down, np.int32),
             firstrecv=slab.nlocal + slab.n_low, recvnum=slab.n_up),
        dict(stage=1, send_rank=rank, recv_rank=rank, sendlist=np.asarray(slab.xy_owner, np.int32),
             firstrecv=first_image, recvnum=len(slab.xy_owner)),
    ]


def apply_swaps(rows_by_rank, swaps_by_rank, forward: bool, zero_ghosts: bool = True):
    """Host restatement of ljx_halo_forward / ljx_halo_reverse over every rank at once (numpy
    rows, first axis = atom rows): the semantics the library implements, for tests. Messages
    from one rank to another within a stage match in posting order."""
    nranks = len(rows_by_rank)
    stages = sorted({sw["stage"] for sws in swaps_by_rank for sw in sws})

    def inbox(stage, r, q, src, direction):
        """Position of swap q among rank r's swaps of `stage` that talk to `src`, and the
        matching message of `src` (its k-th swap of the stage aimed at r)."""
        mine = [qq for qq, sw in enumerate(swaps_by_rank[r])
                if sw["stage"] == stage and sw[direction[0]] == src]
        theirs = [qq for qq, sw in enumerate(swaps_by_rank[src])
                  if sw["stage"] == stage and sw[direction[1]] == r]
        return theirs[mine.index(q)]

    for stage in (stages if forward else stages[::-1]):
        if forward:
            sent = {(r, q): rows_by_rank[r][sw["sendlist"]].copy()
                    for r in range(nranks) for q, sw in enumerate(swaps_by_rank[r])
                    if sw["stage"] == stage}
            for r in range(nranks):
                for q, sw in enumerate(swaps_by_rank[r]):
                    if sw["stage"] != stage:
                        continue
                    src = sw["recv_rank"]
                    msg = sent[(src, inbox(stage, r, q, src, ("recv_rank", "send_rank")))]
                    rows_by_rank[r][sw["firstrecv"]:sw["firstrecv"] + sw["recvnum"]] = msg
        else:
            back = {}
            for r in range(nranks):
                for q, sw in enumerate(swaps_by_rank[r]):
                    if sw["stage"] != stage:
                        continue
                    lo, hi = sw["firstrecv"], sw["firstrecv"] + sw["recvnum"]
                    back[(r, q)] = rows_by_rank[r][lo:hi].copy()
                    if zero_ghosts:
                        rows_by_rank[r][lo:hi] = 0
            for r in range(nranks):
                for q, sw in enumerate(swaps_by_rank[r]):
                    if sw["stage"] != stage:
                        continue
                    src = sw["send_rank"]
                    msg = back[(src, inbox(stage, r, q, src, ("send_rank", "recv_rank")))]
                    np.add.at(rows_by_rank[r], sw["sendlist"], msg)
    return rows_by_rank


def _broadcast_id(group=None) -> bytes:
    """One NCCL unique id made on rank 0 and broadcast over the torch.distributed group."""
    lib = abi.load()
    payload = [None]
    if dist.get_rank(group) == 0:
        buf = (ctypes.c_ubyte * abi.HALO_ID_BYTES)()
        st = lib.ljx_halo_unique_id(buf)
        if st != abi.OK:
            raise abi.LjxError(st, lib.ljx_halo_create_error().decode())
        payload = [bytes(buf)]
    dist.broadcast_object_list(payload, src=0, group=group)
    return payload[0]


class NcclHalo:
    """A libljx NCCL halo (ljx_halo) with a swap table: the multi-GPU exchange of the harness.

    `unique_id` is the NCCL id every rank shares (made and broadcast over the torch.distributed
    group when omitted). The send lists live on the device for the halo's lifetime."""

    def __init__(self, swaps, rank: int, nranks: int, device: int, unique_id: bytes | None = None,
                 group=None, timeout_ms: int = 60000, flags: int = 0, max_row_bytes: int = 24):
        self.lib = abi.load()
        uid = unique_id if unique_id is not None else _broadcast_id(group)
        idbuf = (ctypes.c_ubyte * abi.HALO_ID_BYTES).from_buffer_copy(uid)
        out = ctypes.c_void_p()
        st = self.lib.ljx_halo_create(idbuf, nranks, rank, device, timeout_ms, flags,
                                      ctypes.byref(out))
        if st != abi.OK:
            raise abi.LjxError(st, self.lib.ljx_halo_create_error().decode())
        self._h = out
        self.rank, self.nranks = rank, nranks
        self.set_swaps(swaps, max_row_bytes)

    def _check(self, st):
        if st != abi.OK:
            raise abi.LjxError(st, self.lib.ljx_halo_error(self._h).decode())

    def set_swaps(self, swaps, max_row_bytes: int = 24):
        self._lists = [torch.as_tensor(np.ascontiguousarray(sw["sendlist"], np.int32),
                                       device="cuda") for sw in swaps]
        table = (abi.Swap * max(1, len(swaps)))()
        for k, (sw, lst) in enumerate(zip(swaps, self._lists)):
            table[k] = abi.Swap(sw["stage"], sw["send_rank"], sw["recv_rank"], lst.data_ptr(),
                                int(lst.numel()), sw["firstrecv"], sw["recvnum"])
        self._check(self.lib.ljx_halo_set_swaps(self._h, table, len(swaps), max_row_bytes))

    @staticmethod
    def _s(stream=None):
        return ctypes.c_void_p((stream or torch.cuda.current_stream()).cuda_stream)

    def forward(self, rows, width: int, elem_bytes: int, stream=None):
        """Fill every ghost row of `rows` (a device address) from its owner."""
        self._check(self.lib.ljx_halo_forward(self._h, self._s(stream), ctypes.c_void_p(rows),
                                              width, elem_bytes))

    def reverse(self, rows, width: int, elem_bytes: int, stream=None):
        """Add every ghost row into its owner's row, then zero the ghost rows."""
        self._check(self.lib.ljx_halo_reverse(self._h, self._s(stream), ctypes.c_void_p(rows),
                                              width, elem_bytes, 1))

    def forward_under_force(self, engine, atoms, nl, newton_pair, rows, width: int,
                            elem_bytes: int, scale: float = 1.0):
        """The forward exchange of `rows` (F'(rho)) overlapped with the force pass: the
        exchange runs on a side stream while the current stream runs the force pass over the
        list rows without a ghost neighbor (ljx_force_rows, ROWS_LOCAL); the rows with one
        (ROWS_GHOST) follow once the exchange is done. Leaves what forward() then
        engine.force() would, with the current stream ordered after both."""
        if not hasattr(self, "_side"):
            self._side = torch.cuda.Stream()
            self._ready = torch.cuda.Event()
            self._done = torch.cuda.Event()
        main = torch.cuda.current_stream()
        self._ready.record(main)
        self._side.wait_event(self._ready)
        self.forward(rows, width, elem_bytes, stream=self._side)
        self._done.record(self._side)
        engine.force_rows(atoms, nl, newton_pair, abi.ROWS_LOCAL, scale)
        main.wait_event(self._done)
        engine.force_rows(atoms, nl, newton_pair, abi.ROWS_GHOST, scale)

    def reverse_forces(self, f: torch.Tensor, stream=None):
        """LAMMPS's own reverse comm of ghost force rows (newton on)."""
        self.reverse(f.data_ptr(), 3, 8, stream)

    def result_all(self, engine, stream=None) -> abi.ResultAll:
        """The step result over all ranks (ljx_read_result_all)."""
        out = abi.ResultAll()
        st = self.lib.ljx_read_result_all(engine._h, self._h, self._s(stream), ctypes.byref(out))
        if st != abi.OK:
            raise abi.LjxError(st, self.lib.ljx_engine_error(engine._h).decode())
        return out

    def allreduce_sum(self, t: torch.Tensor, stream=None):
        """In-place sum over ranks of a float64 device tensor."""
        self._check(self.lib.ljx_halo_allreduce_sum(self._h, self._s(stream),
                                                    ctypes.c_void_p(t.data_ptr()), t.numel()))

    @property
    def launches(self) -> int:
        return int(self.lib.ljx_halo_launches(self._h))

    def close(self):
        if getattr(self, "_h", None):
            self.lib.ljx_halo_destroy(self._h)
        self._h = None
