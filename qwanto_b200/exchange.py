"""Split-KV exchange buffers over the node's NVLink fabric.

One long sequence shards by KV range (:func:`qwanto_b200.sharding.kv_ranges`).
Each rank allocates one exchange buffer (``qwn_kv_exchange_alloc``) and maps
every other rank's buffer through its CUDA IPC handle; the handles travel
through the ``torch.distributed`` process group once, at setup.  From then on
``qwn_kv_decode_split`` needs no collective: the attention kernel stores each
(sequence, kv head) segment's partial (m, l, o) straight into every rank's
buffer, raises the segment's flag there, waits (bounded) for the other ranks'
flags and merges the partials in rank order, so every rank holds the same
output rows when the launch completes.
"""
from __future__ import annotations

import ctypes as C

from . import _lib
from ._lib import check, lib

HANDLE_BYTES = 64


class PeerExchange:
    """This rank's exchange buffer plus the mapped buffers of the other ranks.

    ``max_rows`` bounds the query heads of a call.  Calls must be made in the
    same order on every rank (each call draws the next epoch)."""

    def __init__(self, max_rows: int, device: int = 0, group=None, timeout_ns: int = 0):
        import torch.distributed as dist
        if dist.is_available() and dist.is_initialized():
            rank, world = dist.get_rank(group), dist.get_world_size(group)
        else:
            rank, world = 0, 1
        if world > _lib.MAX_RANKS:
            raise ValueError(f"split-KV exchange supports at most {_lib.MAX_RANKS} ranks")
        self._setup(max_rows, device, rank, world, timeout_ns)
        handles = [bytes(self._handle)] * world
        if world > 1:
            dist.all_gather_object(handles, bytes(self._handle), group=group)
        for p in range(world):
            if p != rank:
                self._map(p, handles[p])

    @classmethod
    def unreachable(cls, max_rows: int, device: int, world: int, timeout_ns: int) -> "PeerExchange":
        """Rank 0 of `world` whose other ranks never run: their buffers are
        local stand-ins that nothing flags, so every wait of a split call runs
        into its limit and the call latches QWN_KV_STATUS_PEER_TIMEOUT."""
        self = cls.__new__(cls)
        self._setup(max_rows, device, 0, world, timeout_ns)
        for p in range(1, world):
            buf, _ = self._alloc()
            self._stand_ins.append(buf)
            self.peers.buffers[p] = buf
        return self

    # -- internals ----------------------------------------------------------
    def _setup(self, max_rows: int, device: int, rank: int, world: int, timeout_ns: int) -> None:
        self.device, self.rank, self.world, self.max_rows = device, rank, world, max_rows
        self.epoch = 0
        self._opened: list[int] = []
        self._stand_ins: list[int] = []
        nbytes = C.c_uint64(0)
        check("qwn_kv_exchange_bytes", lib().qwn_kv_exchange_bytes(max_rows, C.byref(nbytes)))
        self.nbytes = int(nbytes.value)
        self.own, self._handle = self._alloc()
        ps = _lib.init(_lib.PeerSet())
        ps.rank, ps.world, ps.max_rows, ps.timeout_ns = rank, world, max_rows, timeout_ns
        ps.buffers[rank] = self.own
        self.peers = ps

    def _alloc(self):
        buf = C.c_void_p()
        handle = (C.c_uint8 * HANDLE_BYTES)()
        check("qwn_kv_exchange_alloc", lib().qwn_kv_exchange_alloc(self.device, self.nbytes, C.byref(buf), handle))
        return buf.value, handle

    def _map(self, p: int, handle: bytes) -> None:
        h = (C.c_uint8 * HANDLE_BYTES).from_buffer_copy(handle)
        buf = C.c_void_p()
        check("qwn_kv_exchange_open", lib().qwn_kv_exchange_open(self.device, h, C.byref(buf)))
        self._opened.append(buf.value)
        self.peers.buffers[p] = buf.value

    # -- use ------------------------------------------------------------------
    def next_epoch(self) -> int:
        self.epoch = self.epoch % 0xFFFFFFFF + 1
        return self.epoch

    def close(self) -> None:
        """Unmap the other ranks' buffers and free this rank's.  Every rank must
        have finished its last split call first (a barrier on the host)."""
        for b in self._opened:
            lib().qwn_kv_exchange_close(self.device, b)
        for b in self._stand_ins:
            lib().qwn_kv_exchange_free(self.device, b)
        if self.own:
            lib().qwn_kv_exchange_free(self.device, self.own)
        self._opened, self._stand_ins, self.own = [], [], None
