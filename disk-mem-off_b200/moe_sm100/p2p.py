"""Buffers of the peer-memory exchange (``ExpertParallelMoe(small_exchange="p2p")``).

Each rank allocates its receive, partial-sum and flag buffers with cudaMalloc
(``moe_rt_malloc``: CUDA IPC needs the allocation's own base pointer), and maps every
other rank's through CUDA IPC handles exchanged once with ``all_gather_object``.
Layers of a stack that share a ``DeviceEPOps`` pool share one set of buffers and one
epoch counter (the exchange's ordering makes a buffer free again before any rank
writes the next forward's data into it).  The kernels and the protocol are
libmoe_sm100's ``moe_ep_p2p_*`` entry points.
"""
from __future__ import annotations

from ctypes import byref, c_void_p, create_string_buffer
from typing import Any

from ._lib import check, lib

IPC_HANDLE_BYTES = 64
WAIT_LIMIT_CYCLES = 1_000_000_000  # ~0.5 s at B200 clocks, per wait


class _DeviceView:
    """A CUDA array interface over a raw device pointer (for torch.as_tensor)."""

    def __init__(self, ptr: int, shape: tuple[int, ...], typestr: str) -> None:
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr,
                                         "data": (int(ptr), False), "version": 3, "strides": None}


class PeerExchange:
    """One rank's mapped view of every rank's exchange buffers."""

    def __init__(self, rank: int, world: int, cap: int, hidden: int, row_halves: int,
                 device: int, group: Any = None) -> None:
        import torch.distributed as dist
        if not 1 <= world <= 8:
            raise ValueError("the peer-memory exchange runs on 1 to 8 ranks")
        self.rank, self.world, self.cap, self.hidden = rank, world, cap, hidden
        self.row_halves = row_halves
        self.device = device
        self.epoch = 0
        self.users = 0
        self.recv_bytes = world * cap * row_halves * 2
        self.part_bytes = world * cap * hidden * 4
        self._own: list[int] = []
        self._opened: list[int] = []
        lib().moe_rt_set_device(device)
        self.recv = self._malloc(self.recv_bytes)
        self.part = self._malloc(self.part_bytes)
        self.flags = self._malloc(256)  # [2][world] int32 epochs, then 2 launch counters
        zeros = bytes(256)
        check(lib().moe_rt_memcpy_h2d_async(c_void_p(self.flags), zeros, 256, c_void_p(0)))
        check(lib().moe_rt_stream_synchronize(c_void_p(0)))
        mine = [self._handle(self.recv), self._handle(self.part), self._handle(self.flags)]
        everyone: list[Any] = [None] * world
        dist.all_gather_object(everyone, (rank, mine), group=group)
        recv, part, flags = [0] * world, [0] * world, [0] * world
        for r, handles in everyone:
            if r == rank:
                recv[r], part[r], flags[r] = self.recv, self.part, self.flags
                continue
            recv[r], part[r], flags[r] = (self._open(h) for h in handles)
        self.recv_arr = (c_void_p * world)(*recv)
        self.part_arr = (c_void_p * world)(*part)
        self.flags_arr = (c_void_p * world)(*flags)

    def _malloc(self, nbytes: int) -> int:
        p = c_void_p()
        check(lib().moe_rt_malloc(max(int(nbytes), 256), byref(p)))
        self._own.append(int(p.value))
        return int(p.value)

    def _handle(self, ptr: int) -> bytes:
        buf = create_string_buffer(IPC_HANDLE_BYTES)
        check(lib().moe_rt_ipc_get_handle(c_void_p(ptr), buf))
        return buf.raw

    def _open(self, handle: bytes) -> int:
        p = c_void_p()
        check(lib().moe_rt_ipc_open_handle(create_string_buffer(handle, IPC_HANDLE_BYTES), byref(p)))
        self._opened.append(int(p.value))
        return int(p.value)

    @property
    def done_ptr(self) -> int:
        return self.flags + 128  # two int32 launch counters (pack, partials)

    def flags_row(self, which: int) -> int:
        return self.flags + which * self.world * 4

    def recv_ids(self) -> Any:
        """Global expert ids [world*cap, top_k] of the received records (-1: unused)."""
        import torch
        rows = self.world * self.cap
        t = torch.as_tensor(_DeviceView(self.recv, (rows, self.row_halves), "<f2"),
                            device=f"cuda:{self.device}")
        return t[:, self.hidden:].contiguous().view(torch.int32)

    def close(self, group: Any = None) -> None:
        """Unmap the peers' buffers and free this rank's (a collective: no rank frees
        a buffer while another may still write to it)."""
        import torch.distributed as dist
        if not self._own:
            return
        lib().moe_rt_set_device(self.device)
        check(lib().moe_rt_stream_synchronize(c_void_p(0)))
        dist.barrier(group=group)
        for p in self._opened:
            lib().moe_rt_ipc_close_handle(c_void_p(p))
        dist.barrier(group=group)
        for p in self._own:
            lib().moe_rt_free(c_void_p(p))
        self._own, self._opened = [], []
