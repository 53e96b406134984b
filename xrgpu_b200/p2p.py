"""All-gather of Y shards over NVLink peer memory (``xrgpu_p2p_*`` in the C ABI).

One process per GPU on one node. ``PeerAllGather(group, slot_bytes)`` allocates this rank's
staging region, exchanges CUDA IPC handles over the ``torch.distributed`` group and maps the other
ranks' regions; ``all_gather(shard, out)`` then enqueues one kernel on the current stream that
leaves every rank's shard in ``out`` -- no NCCL call, so CUDA graphs capture it. Every rank must
make the same sequence of calls. ``close()`` synchronises, waits for all ranks and unmaps.

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
        es = shard.element_size()
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _native.check(_native.load().xrgpu_p2p_allgather(
            self._g, ctypes.c_void_p(shard.data_ptr()), shard.shape[0], shard.shape[1] * es,
            ctypes.c_void_p(out.data_ptr()), out.stride(0) * es, valid_cols * es, ctypes.c_void_p(stream)))
        return out

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
