"""Halo exchange of per-atom feature rows between z-slab neighbors over torch.distributed.

Per exchange: pack the rows each neighbor needs (ljx_comm_pack_forward, by sendlist), one
grouped NCCL send/recv with both z-neighbors, unpack into the ghost rows
(ljx_comm_unpack_forward), then fill the x/y periodic images on the same rank
(ljx_halo_forward_self). The message order is the same on every rank: send up, send down,
receive from below, receive from above, so two ranks that are each other's upper and lower
neighbor (two slabs) match their messages in posting order.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import abi


class SlabExchange:
    """Forward exchange of width-`width` feature rows for one rank of a slab decomposition."""

    def __init__(self, slab, width: int, elem_bytes: int, device="cuda", group=None,
                 pack=None, unpack=None, self_fill=None):
        self.rank = dist.get_rank(group)
        self.nranks = dist.get_world_size(group)
        self.group = group
        self.up = (self.rank + 1) % self.nranks
        self.down = (self.rank - 1) % self.nranks
        self.nlocal, self.n_low, self.n_up = slab.nlocal, slab.n_low, slab.n_up
        self.width, self.elem = width, elem_bytes
        self.words = width * elem_bytes // 4
        self.slots = (width * elem_bytes + 7) // 8
        self.send_up = torch.as_tensor(slab.send_up, device=device)
        self.send_down = torch.as_tensor(slab.send_down, device=device)
        self.xy_owner = torch.as_tensor(slab.xy_owner, device=device)
        self.n_xy = int(slab.xy_owner.size)
        mk = lambda n: torch.zeros(max(n, 1) * self.slots, dtype=torch.float64, device=device)  # noqa: E731
        self.sbuf_up, self.sbuf_down = mk(len(slab.send_up)), mk(len(slab.send_down))
        self.rbuf_low, self.rbuf_up = mk(self.n_low), mk(self.n_up)
        self._pack = pack or self._gpu_pack
        self._unpack = unpack or self._gpu_unpack
        self._self_fill = self_fill or self._gpu_self_fill
        self.launches_per_exchange = 5

    def _stream(self):
        return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def _gpu_pack(self, rows: int, sendlist: torch.Tensor, buf: torch.Tensor):
        st = abi.load().ljx_comm_pack_forward(self._stream(), ctypes.c_void_p(rows), self.words,
                                              ctypes.c_void_p(sendlist.data_ptr()),
                                              int(sendlist.numel()),
                                              ctypes.c_void_p(buf.data_ptr()), self.slots)
        if st != abi.OK:
            raise RuntimeError(f"ljx_comm_pack_forward failed ({st})")

    def _gpu_unpack(self, rows: int, first: int, n: int, buf: torch.Tensor):
        st = abi.load().ljx_comm_unpack_forward(self._stream(), ctypes.c_void_p(rows), self.words,
                                                first, n, ctypes.c_void_p(buf.data_ptr()),
                                                self.slots)
        if st != abi.OK:
            raise RuntimeError(f"ljx_comm_unpack_forward failed ({st})")

    def _gpu_self_fill(self, rows: int):
        st = abi.load().ljx_halo_forward_self(self._stream(), ctypes.c_void_p(rows), self.width,
                                              self.elem, ctypes.c_void_p(self.xy_owner.data_ptr()),
                                              self.nlocal + self.n_low + self.n_up, self.n_xy)
        if st != abi.OK:
            raise RuntimeError(f"ljx_halo_forward_self failed ({st})")

    def forward(self, rows, width=None, elem_bytes=None, stream=None):
        """Fill every ghost row of `rows` (a device address) from its owner."""
        self._pack(rows, self.send_up, self.sbuf_up)
        self._pack(rows, self.send_down, self.sbuf_down)
        ops = [dist.P2POp(dist.isend, self.sbuf_up, self.up, self.group),
               dist.P2POp(dist.isend, self.sbuf_down, self.down, self.group),
               dist.P2POp(dist.irecv, self.rbuf_low, self.down, self.group),
               dist.P2POp(dist.irecv, self.rbuf_up, self.up, self.group)]
        for work in dist.batch_isend_irecv(ops):
            work.wait()
        self._unpack(rows, self.nlocal, self.n_low, self.rbuf_low)
        self._unpack(rows, self.nlocal + self.n_low, self.n_up, self.rbuf_up)
        self._self_fill(rows)
