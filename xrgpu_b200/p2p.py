"""All-gather of Y shards over NVLink peer memory (``xrgpu_p2p_*`` in the C ABI).

One process per GPU on one node. ``PeerAllGather(group, slot_bytes)`` allocates this rank's
staging region, exchanges CUDA IPC handles over the ``torch.distributed`` group and maps the other
ranks' regions; ``all_gather(shard, out)`` then enqueues one kernel on the current stream that
leaves every rank's shard in ``out`` -- no NCCL call, so CUDA graphs capture it. Every rank must
make the same sequence of calls. ``close()`` synchronises, waits for all ranks and unmaps.

Fused form (single-row float16 problems of the staged decode GEMV): ``send(problem, S, out)`` runs
this rank's GEMV, whose epilogue also writes each finished pair of output columns to every other
rank as one epoch-tagged 8-byte word; ``recv(S, out, N)`` then waits for the other ranks' words and
writes their columns into ``out``. A send must be followed by its receive before the group's next
call; a send or all-gather issued on another stream than the last receive waits for it.

A peer that does not arrive within 1 s makes the kernel give up, record code 0x401 in the
device's error word and return; every rank's epochs are then out of step, so the group cannot be
used again. ``check()`` (after synchronising) reads and clears that word and raises.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch
import torch.distributed as dist

from . import _native

__all__ = ["PeerAllGather"]


def _capture_id(stream) -> int:
    """The CUDA graph capture `stream` belongs to (0: none)."""
    out = ctypes.c_uint64(0)
    _native.check(_native.load().xrgpu_stream_capture_id(ctypes.c_void_p(stream.cuda_stream), ctypes.byref(out)))
    return out.value


class PeerAllGather:
    def __init__(self, slot_bytes: int, group=None, device: Optional[torch.device] = None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > _native.P2P_MAX_WORLD:
            raise ValueError(f"peer all-gather supports at most {_native.P2P_MAX_WORLD} ranks")
        self.device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.slot_bytes = int(-(-int(slot_bytes) // 256) * 256)
        lib = _native.load()
        handle = ctypes.create_string_buffer(_native.P2P_HANDLE_BYTES)
        ptr = ctypes.c_void_p()
        _native.check(lib.xrgpu_p2p_create(self.device.index, self.world, self.rank, self.slot_bytes,
                                           ctypes.byref(ptr), handle))
        self._g = ptr
        self.broken = False
        self._recv_done = None  # (stream, capture id) of the last fused receive
        self._sent = False      # a fused send is waiting for its receive
        self._recv_seq = 0
        handles = [None] * self.world
        dist.all_gather_object(handles, handle.raw, group=group)
        try:
            _native.check(lib.xrgpu_p2p_connect(self._g, b"".join(handles)))
        except Exception:
            lib.xrgpu_p2p_destroy(self._g)
            self._g = None
            raise

    def all_gather(self, shard: torch.Tensor, out: torch.Tensor, valid_cols: int) -> torch.Tensor:
        """out[m, q * S + j] = shard of rank q [m, j] for j with q * S + j < valid_cols.

        shard: this rank's [M, S] (contiguous); out: [M, >= valid_cols] with a unit inner stride.
        """
        if self._g is None:
            raise RuntimeError("peer all-gather group is closed")
        if self.broken:
            raise RuntimeError("peer all-gather group gave up waiting for a peer earlier; close it")
        if shard.dim() != 2 or not shard.is_contiguous() or out.dim() != 2 or out.stride(1) != 1:
            raise ValueError("shard must be a contiguous [M, S] tensor and out an [M, >= N] row-major view")
        if self._sent:
            raise RuntimeError("peer group: a fused send is waiting for its receive (recv before the next call)")
        es = shard.element_size()
        cur = torch.cuda.current_stream(self.device)
        self._order_after_recv(cur)
        stream = cur.cuda_stream
        _native.check(_native.load().xrgpu_p2p_allgather(
            self._g, ctypes.c_void_p(shard.data_ptr()), shard.shape[0], shard.shape[1] * es,
            ctypes.c_void_p(out.data_ptr()), out.stride(0) * es, valid_cols * es, ctypes.c_void_p(stream)))
        return out

    # ---- fused form (single-row float16 problems of the staged decode GEMV)
    def forward_supported(self, problem, shard_cols: int) -> bool:
        """Whether ``send`` accepts this rank's problem (a ``_native.Problem_``) with shard_cols."""
        if self._g is None or self.broken:
            return False
        yes = ctypes.c_int32(0)
        _native.check(_native.load().xrgpu_p2p_forward_supported(self._g, ctypes.byref(problem), int(shard_cols),
                                                                 ctypes.byref(yes)))
        return bool(yes.value)

    def send(self, problem, shard_cols: int, out: torch.Tensor) -> None:
        """Enqueue on the current stream this rank's GEMV (``problem``, its y ignored) writing its
        columns to out[rank * shard_cols:] and sending them to every other rank. ``recv`` must follow
        before the group's next call; a receive left on another stream is waited for here."""
        if self._g is None:
            raise RuntimeError("peer all-gather group is closed")
        if self.broken:
            raise RuntimeError("peer all-gather group gave up waiting for a peer earlier; close it")
        if self._sent:
            raise RuntimeError("peer group: the previous fused send has no receive yet (recv before the next call)")
        stream = torch.cuda.current_stream(self.device)
        self._order_after_recv(stream)
        self._sent = True
        _native.check(_native.load().xrgpu_p2p_forward_send(self._g, ctypes.byref(problem), int(shard_cols),
                                                            ctypes.c_void_p(out.data_ptr()),
                                                            ctypes.c_void_p(stream.cuda_stream)))

    def recv(self, shard_cols: int, out: torch.Tensor, valid_cols: int) -> None:
        """Enqueue on the current stream the receive of the other ranks' columns of the last
        ``send`` into out (bounded wait; 0x401 on expiry)."""
        PeerAllGather.recv_many([(self, shard_cols, out, valid_cols)])

    @staticmethod
    def recv_many(items) -> None:
        """The receives of several groups [(group, shard_cols, out, valid_cols), ...] (each after its
        own send, all on one device) in one kernel on the current stream."""
        groups = [it[0] for it in items]
        for g in groups:
            if g._g is None:
                raise RuntimeError("peer all-gather group is closed")
            if not g._sent:
                raise RuntimeError("peer group: recv without a preceding fused send")
        n = len(items)
        arr = lambda ct, vals: (ct * n)(*vals)  # noqa: E731
        stream = torch.cuda.current_stream(groups[0].device)
        _native.check(_native.load().xrgpu_p2p_forward_recv_many(
            n, arr(ctypes.c_void_p, [g._g for g in groups]), arr(ctypes.c_int64, [int(it[1]) for it in items]),
            arr(ctypes.c_void_p, [it[2].data_ptr() for it in items]), arr(ctypes.c_int64, [int(it[3]) for it in items]),
            ctypes.c_void_p(stream.cuda_stream)))
        capture = _capture_id(stream)
        for g in groups:
            g._sent = False
            g._recv_seq += 1
            g._recv_done = (stream, capture)

    def _order_after_recv(self, stream) -> None:
        """Make `stream` wait for the stream of the group's last fused receive when that is another
        stream of the same graph capture (or both are outside capture). A receive in another capture
        is ordered by the graphs' own order of replay, one outside capture by the synchronisation
        that begins a capture. No event is recorded when the receive and the next call share a
        stream, so consecutive kernels keep their early launch."""
        if self._recv_done is None or self._recv_done[0] == stream:
            return
        if self._recv_done[1] != _capture_id(stream):
            return
        stream.wait_stream(self._recv_done[0])

    def joined(self, seq: int) -> None:
        """The caller's stream now waits for this group's receive number `seq` (``recv_seq`` after
        it was enqueued): if no receive followed it, later calls need no further ordering."""
        if seq == self._recv_seq:
            self._recv_done = None

    @property
    def recv_seq(self) -> int:
        """Number of fused receives enqueued on this group so far."""
        return self._recv_seq

    PEER_WAIT_EXPIRED = 0x401

    def check(self) -> None:
        """Synchronise this device, then raise ``XrgpuError`` if a call on it gave up waiting for a
        peer (device error word 0x401, read and cleared). The group is marked unusable."""
        if self._g is None:
            return
        torch.cuda.synchronize(self.device)
        import ctypes as _ct
        code = _ct.c_uint32(0)
        _native.check(_native.load().xrgpu_device_error(self.device.index, _ct.byref(code), 1))
        if code.value:
            self.broken = True
            raise _native.XrgpuError(_native.DEVICE_ERROR,
                                     f"peer all-gather: device error 0x{code.value:x} (a peer did not arrive); "
                                     "the group is out of step and must be closed")

    def close(self):
        """Unmap after every rank's last call: synchronise this device, host barrier, destroy."""
        if self._g is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        st = _native.load().xrgpu_p2p_destroy(self._g)
        self._g = None
        _native.check(st)
