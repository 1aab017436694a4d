"""Halo exchange of per-atom rows between z-slab neighbors over torch.distributed.

This is the standalone harness's stand-in for LAMMPS's comm on a brick decomposition along z.
Forward (owners to ghosts: F'(rho)):
  pack the rows each neighbor needs (by sendlist), one grouped NCCL send/recv with both
  z-neighbors, unpack into the ghost rows, then fill the x/y periodic images on the same rank.
Reverse (ghosts to owners, adding: rho partials, force rows):
  fold the x/y images into their owners on the same rank, pack the z-ghost rows, one grouped
  NCCL send/recv, add them into the sendlist rows they came from, and zero the z-ghost rows.
The message order is the same on every rank, so two ranks that are each other's upper and lower
neighbor (two slabs) match their messages in posting order. The row operations are libljx's
ljx_comm_* / ljx_halo_*_self kernels (GpuRowOps).
"""

from __future__ import annotations

import ctypes

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
