"""N-column sharding of MatMulNBits over the GPUs of one node, with one all-gather of Y.

Every output column of Y = A . dequant(B)^T depends only on its own row of B, scales, zero
points and bias, all of which are N-major: rank r of a ``torch.distributed`` group owns the
contiguous column range ``shard_bounds(N, world, r)`` and the matching contiguous slices of those
tensors, computes its columns of Y with this package's kernels (A is replicated), and one
all-gather (NCCL over NVLink/NVSwitch) assembles Y. The reference backend is single-device;
the contract (inputs, attributes, output shape and values) is unchanged.

Shards are equal (``ceil(N / world)`` columns, the last one padded). On NCCL groups of one node,
shards up to ``peer_max_bytes`` (64 MB) are exchanged by this package's peer-memory all-gather (one
kernel over NVLink that writes Y in place, no NCCL call, so a step can be captured in a CUDA graph);
larger shards and gloo groups use ``all_gather_into_tensor`` / ``all_gather`` (for M == 1 the
gathered buffer already is Y, for M > 1 one permute copy turns ``[world, M, S]`` into
``[M, world * S]``).
"""
from __future__ import annotations

import os
from typing import Callable, Optional

import torch
import torch.distributed as dist

from . import functional as F

__all__ = ["shard_bounds", "shard_tensor", "ShardedMatMulNBits"]


def shard_bounds(N: int, world: int, rank: int) -> tuple[int, int]:
    """Columns [n0, n1) owned by `rank`: equal shards of ceil(N / world) columns (the last ones
    may be short or empty)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a group of {world}")
    S = -(-N // world)
    n0 = min(N, rank * S)
    return n0, min(N, n0 + S)


def shard_tensor(t: Optional[torch.Tensor], N: int, world: int, rank: int) -> Optional[torch.Tensor]:
    """This rank's contiguous slice of an N-major tensor (B, scales, zero points, bias)."""
    if t is None:
        return None
    if t.shape[0] != N:
        raise ValueError(f"expected an N-major tensor with {N} rows, got shape {tuple(t.shape)}")
    n0, n1 = shard_bounds(N, world, rank)
    return t[n0:n1].contiguous()


class ShardedMatMulNBits:
    """MatMulNBits with B split by output column across the ranks of a process group.

    Construct with the full tensors (each rank keeps only its slice) or with this rank's shard
    (``from_shard``); ``forward(a)`` returns the full Y [*, N] on every rank. ``compute`` replaces
    the per-shard kernel call (default ``functional.matmul_nbits``); its signature is that of
    ``matmul_nbits`` with ``out`` given.
    """

    def __init__(self, b: torch.Tensor, scales: torch.Tensor, zero_points: Optional[torch.Tensor] = None,
                 bias: Optional[torch.Tensor] = None, *, K: int, N: int, bits: int = 4, block_size: int,
                 group=None, compute: Optional[Callable] = None, peer_gather: Optional[bool] = None,
                 peer_max_bytes: int = 64 << 20, peer_group=None, peer_slot_bytes: int = 0,
                 fuse: Optional[bool] = None, _presharded: bool = False):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.K, self.N, self.bits, self.block_size = int(K), int(N), int(bits), int(block_size)
        self.n0, self.n1 = shard_bounds(self.N, self.world, self.rank)
        self.S = -(-self.N // self.world)
        if _presharded:
            self.b, self.scales, self.zero_points, self.bias = b, scales, zero_points, bias
        else:
            self.b = shard_tensor(b, self.N, self.world, self.rank)
            self.scales = shard_tensor(scales, self.N, self.world, self.rank)
            self.zero_points = shard_tensor(zero_points, self.N, self.world, self.rank)
            self.bias = shard_tensor(bias, self.N, self.world, self.rank)
        if self.b.shape[0] != self.n1 - self.n0:
            raise ValueError(f"rank {self.rank} shard has {self.b.shape[0]} columns, expected {self.n1 - self.n0}")
        self.compute = compute or F.matmul_nbits
        # Peer-memory all-gather: NCCL groups whose ranks all live on this node (torchrun's
        # LOCAL_WORLD_SIZE), unless disabled; created lazily by the first eligible forward, which
        # every rank makes with the same shapes.
        same_node = int(os.environ.get("LOCAL_WORLD_SIZE", self.world)) == self.world
        auto = (self.world > 1 and dist.is_initialized() and dist.get_backend(group) == "nccl" and same_node)
        self.peer_gather = auto if peer_gather is None else (bool(peer_gather) and self.world > 1)
        self.peer_max_bytes = int(peer_max_bytes)
        self._peer_slot_bytes = int(peer_slot_bytes)  # minimum slot of this module's own group
        # A PeerAllGather shared with other modules (owned by the caller), or this module's own.
        self._shared_peer = peer_group
        self._peer = None
        self._y_buf = None        # shard buffer of the overlapped form (see forward)
        self._gather_done = None  # event of the last overlapped gather
        # Fused form for single-row float16 calls on the staged decode GEMV: the GEMV's epilogue sends
        # its columns to the other ranks itself and only a receive kernel remains (XRGPU_FUSED_GATHER=0
        # turns it off, e.g. to compare with the separate all-gather).
        self.fuse = bool(fuse) if fuse is not None else os.environ.get("XRGPU_FUSED_GATHER", "1") != "0"
        self._fused_ok = None
        self._fused_group = None  # group of a fused receive left on a gather stream
        self._pending = None       # deferred exchange (forward(..., defer=True)), run by wait_gather
        self._pending_copy = None  # (caller's out, aligned buffer) when out was not 16-byte aligned

    @classmethod
    def from_shard(cls, b_shard: torch.Tensor, scales_shard: torch.Tensor, zero_points_shard=None, bias_shard=None,
                   *, K: int, N: int, bits: int = 4, block_size: int, group=None, compute=None, **kw):
        """Build from this rank's slices (rows shard_bounds(N, world, rank) of each tensor)."""
        return cls(b_shard, scales_shard, zero_points_shard, bias_shard, K=K, N=N, bits=bits,
                   block_size=block_size, group=group, compute=compute, _presharded=True, **kw)

    def uses_peer_gather(self, M: int, element_size: int = 2) -> bool:
        """Whether forward with M rows exchanges Y through peer memory (no NCCL call).

        Mirrors the checks of ``xrgpu_p2p_allgather``: 16-byte shard rows (and output rows when
        M > 1), a non-empty last shard (N > (world - 1) * S) and a shard within ``peer_max_bytes``.
        """
        return (self.peer_gather and M * self.S * element_size <= self.peer_max_bytes
                and self.N > (self.world - 1) * self.S
                and (self.S * element_size) % 16 == 0 and (M == 1 or (self.N * element_size) % 16 == 0))

    def set_peer_group(self, peer_group) -> None:
        """Use a PeerAllGather shared with other modules (the caller closes it)."""
        self._shared_peer = peer_group

    def _peer_group(self, nbytes: int):
        from .p2p import PeerAllGather
        if self._shared_peer is not None:
            if self._shared_peer.slot_bytes < nbytes:
                raise ValueError(f"shared peer group slot ({self._shared_peer.slot_bytes} B) < shard ({nbytes} B)")
            return self._shared_peer
        if self._peer is None or self._peer.slot_bytes < nbytes:
            # Creating (or growing) the group allocates device memory, synchronises and exchanges IPC
            # handles over the process group: none of that can be recorded into a CUDA graph.
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError(
                    "ShardedMatMulNBits: the peer-memory group must exist before CUDA graph capture; run one "
                    "forward with the largest M outside capture first, or pass peer_slot_bytes to the constructor")
            if self._peer is not None:
                self._peer.close()
            self._peer = PeerAllGather(max(nbytes, self._peer_slot_bytes, 1 << 16), group=self.group)
        return self._peer

    def prepare_peer_group(self, max_rows: int, element_size: int = 2) -> None:
        """Create this module's peer-memory group for up to ``max_rows`` rows now (collective), so
        that later forwards -- including ones recorded into CUDA graphs -- allocate nothing."""
        if self.world > 1 and self.uses_peer_gather(max_rows, element_size):
            self._peer_group(max_rows * self.S * element_size)

    def check_device_error(self) -> None:
        """Raise if a peer-memory all-gather of this module gave up waiting for a peer (device code
        0x401, after synchronising); the group is then out of step and is closed."""
        for g in (self._shared_peer, self._peer):
            if g is not None:
                g.check()

    def close(self):
        """Release this module's own peer-memory group (collective: every rank calls it)."""
        if self._peer is not None:
            self._peer.close()
            self._peer = None

    def local(self, a: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """This rank's columns of Y into out[..., :n1 - n0] (out is [M, S], S >= n1 - n0)."""
        n_local = self.n1 - self.n0
        if n_local > 0:
            self.compute(a, self.b, self.scales, self.zero_points, self.bias, K=self.K, N=n_local,
                         bits=self.bits, block_size=self.block_size, out=out[:, :n_local])
        if n_local < self.S:
            out[:, n_local:].zero_()
        return out

    def forward(self, a: torch.Tensor, out: Optional[torch.Tensor] = None,
                gather_stream: Optional[torch.cuda.Stream] = None, defer: bool = False) -> torch.Tensor:
        """Full Y [*, N] on every rank. `out` (contiguous, Y's shape) receives it without an extra
        copy when M == 1 and N is a multiple of the group size.

        gather_stream (peer-memory all-gather only): the all-gather runs on that stream after the
        local kernel, so the calling stream can go on with independent work; Y is complete once
        the caller has made its stream wait with ``wait_gather()``. The shard buffer is then this
        module's own and is reused by its next call, so call ``wait_gather()`` before calling the
        module again. Every rank must issue its gathers in the same order on its group.

        defer (peer-memory all-gather only): the exchange is left pending and ``wait_gather()``
        enqueues it on the stream that joins, so independent kernels can run first on one stream
        (no cross-stream event between them, and each kernel launches early behind the previous one);
        Y is complete after ``wait_gather()``."""
        lead = tuple(a.shape[:-1])
        M = a.numel() // self.K
        a2 = a.reshape(M, self.K)
        if self._pending is not None:
            raise RuntimeError("ShardedMatMulNBits: call wait_gather() for the deferred exchange before the next call")
        fused = self._fused_form(a2)
        if fused is not None:
            return self._forward_fused(a2, fused, out, gather_stream, lead, defer)
        overlap = (gather_stream is not None or defer) and self.world > 1 and self.uses_peer_gather(M, a.element_size())
        if overlap:
            key = (M, a.dtype, a.device)
            if self._y_buf is None or self._y_buf[0] != key:
                self._y_buf = (key, torch.empty((M, self.S), dtype=a.dtype, device=a.device))
            y_local = self._y_buf[1]
        else:
            y_local = torch.empty((M, self.S), dtype=a.dtype, device=a.device)
        self.local(a2, y_local)
        if self.world == 1:
            y = y_local[:, :self.N]
            if out is not None:
                out.view(M, self.N).copy_(y)
                return out
            return y.reshape(*lead, self.N)
        if self.uses_peer_gather(M, y_local.element_size()):
            es = y_local.element_size()
            direct = out is not None and out.data_ptr() % 16 == 0 and (M == 1 or (out.view(M, self.N).stride(0) * es) % 16 == 0)
            dst = out.view(M, self.N) if direct else torch.empty((M, self.N), dtype=a.dtype, device=a.device)
            group = self._peer_group(M * self.S * es)
            if defer:
                self._pending = ("call", lambda: group.all_gather(y_local, dst, self.N))
                if out is not None and not direct:
                    self._pending_copy = (out.view(M, self.N), dst)
                return out if out is not None else dst.reshape(*lead, self.N)
            if overlap:
                ready = torch.cuda.Event()
                ready.record()
                gather_stream.wait_event(ready)
                with torch.cuda.stream(gather_stream):
                    group.all_gather(y_local, dst, self.N)
                    self._gather_done = torch.cuda.Event()
                    self._gather_done.record()
            else:
                group.all_gather(y_local, dst, self.N)
            if out is not None and not direct:  # caller's buffer not 16-byte aligned: one copy
                if overlap:
                    self.wait_gather()
                out.view(M, self.N).copy_(dst)
            return out if out is not None else dst.reshape(*lead, self.N)
        direct = out is not None and M == 1 and self.world * self.S == self.N and out.is_contiguous()
        gathered = (out.view(self.world, 1, self.S) if direct
                    else torch.empty((self.world, M, self.S), dtype=a.dtype, device=a.device))
        if dist.get_backend(self.group) == "nccl":
            dist.all_gather_into_tensor(gathered, y_local, group=self.group)
        else:  # gloo (host tests): list form
            dist.all_gather(list(gathered.unbind(0)), y_local, group=self.group)
        if direct:
            return out
        if M == 1:
            y = gathered.view(1, self.world * self.S)[:, :self.N]
        else:
            y = gathered.permute(1, 0, 2).reshape(M, self.world * self.S)[:, :self.N]
        if out is not None:
            out.view(M, self.N).copy_(y)
            return out
        return y.reshape(*lead, self.N)

    # ---- fused form: the decode GEMV sends its columns itself (peer all-gather, flag-in-word words)
    def _fused_form(self, a2: torch.Tensor):
        """(group, problem) when this call can run as one fused GEMV send plus a receive: more than
        one rank, peer all-gather, one float16 row, the package's own kernel as the shard compute, and
        a problem the staged decode GEMV takes (asked of the library once per module)."""
        if (self.world < 2 or not self.fuse or a2.shape[0] != 1 or a2.dtype != torch.float16
                or self.compute is not F.matmul_nbits or not self.uses_peer_gather(1, 2)):
            return None
        group = self._peer_group(self.S * 2)
        prob = F._problem(a2, self.b, self.scales, self.zero_points, self.bias, None, K=self.K,
                          N=self.n1 - self.n0, bits=self.bits, block_size=self.block_size, path="auto")
        key = (id(group), a2.data_ptr() % 16 == 0)
        if self._fused_ok is None or self._fused_ok[0] != key:
            self._fused_ok = (key, group.forward_supported(prob, self.S))
        return (group, prob) if self._fused_ok[1] else None

    def _forward_fused(self, a2, fused, out, gather_stream, lead, defer=False):
        group, prob = fused
        direct = out is not None and out.is_contiguous() and out.data_ptr() % 16 == 0
        dst = out.view(1, self.N) if direct else torch.empty((1, self.N), dtype=a2.dtype, device=a2.device)
        group.send(prob, self.S, dst)
        if defer:
            self._pending = ("recv", (group, self.S, dst, self.N))
            if out is not None and not direct:
                self._pending_copy = (out.view(1, self.N), dst)
            return out if out is not None else dst.reshape(*lead, self.N)
        if gather_stream is not None:
            ready = torch.cuda.Event()
            ready.record()
            gather_stream.wait_event(ready)
            with torch.cuda.stream(gather_stream):
                group.recv(self.S, dst, self.N)
                self._gather_done = torch.cuda.Event()
                self._gather_done.record()
            self._fused_group = (group, group.recv_seq)
        else:
            group.recv(self.S, dst, self.N)
        if out is not None and not direct:
            if gather_stream is not None:
                self.wait_gather()
            out.view(1, self.N).copy_(dst)
            return out
        return out if out is not None else dst.reshape(*lead, self.N)

    def wait_gather(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        """Make `stream` (default: the current one) wait for the last gather issued on a
        gather_stream, or enqueue a deferred exchange on it; a no-op when none is pending."""
        if self._pending is not None:
            ShardedMatMulNBits.wait_gather_all([self], stream)
            return
        if self._gather_done is not None:
            (stream or torch.cuda.current_stream()).wait_event(self._gather_done)
            if self._fused_group is not None:
                self._fused_group[0].joined(self._fused_group[1])
                self._fused_group = None
            self._gather_done = None

    @staticmethod
    def wait_gather_all(mods, stream: Optional[torch.cuda.Stream] = None) -> None:
        """``wait_gather()`` of several modules; their deferred fused receives (at most 8 per kernel)
        run as one kernel on `stream` (default: the current one)."""
        from .p2p import PeerAllGather
        with torch.cuda.stream(stream or torch.cuda.current_stream()):
            recvs = [m for m in mods if m._pending is not None and m._pending[0] == "recv"]
            for i in range(0, len(recvs), 8):
                PeerAllGather.recv_many([m._pending[1] for m in recvs[i:i + 8]])
            for m in mods:
                if m._pending is None:
                    m.wait_gather()
                    continue
                kind, what = m._pending
                m._pending = None
                if kind == "call":
                    what()
                if m._pending_copy is not None:
                    dst_out, src = m._pending_copy
                    m._pending_copy = None
                    dst_out.copy_(src)

    __call__ = forward
