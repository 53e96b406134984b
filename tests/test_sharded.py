"""N-column sharding with one all-gather of Y.

Host logic (shard bounds, slicing, gather and reassembly) runs as world-size-2 gloo ranks on CPU
with the oracle as the per-shard compute; the NCCL path runs the CUDA kernels on 2 GPUs when the
machine has them.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import mmnb_oracle as O
from xrgpu_b200.sharded import ShardedMatMulNBits, shard_bounds, shard_tensor


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("N", [1, 7, 8, 100, 4096, 14336])
def test_shard_bounds_cover_columns_once(world, N):
    seen = []
    S = -(-N // world)
    for r in range(world):
        n0, n1 = shard_bounds(N, world, r)
        assert 0 <= n0 <= n1 <= N and n1 - n0 <= S
        seen.extend(range(n0, n1))
    assert seen == list(range(N))


def test_shard_bounds_rejects_bad_rank():
    with pytest.raises(ValueError):
        shard_bounds(16, 2, 2)


def _case(seed, M, K, N, bs, zp_kind, bias):
    rng = np.random.default_rng(seed)
    kb = K // bs
    a = rng.standard_normal((M, K)).astype(np.float16)
    b = rng.integers(0, 256, (N, kb, bs // 2), dtype=np.uint8)
    s = rng.uniform(0.005, 0.02, (N, kb)).astype(np.float16)
    zp = rng.integers(0, 256, (N, (kb + 1) // 2), dtype=np.uint8) if zp_kind == "packed" else None
    bb = rng.standard_normal(N).astype(np.float16) if bias else None
    return a, b, s, zp, bb


def _oracle_compute(a, b, scales, zero_points, bias, *, K, N, bits, block_size, out):
    npy = lambda t: None if t is None else t.numpy()  # noqa: E731
    y = O.matmul_nbits(npy(a), npy(b), npy(scales), npy(zero_points), npy(bias), K=K, N=N, bits=bits,
                       block_size=block_size)
    out.copy_(torch.from_numpy(y))
    return out


CASES = [(1, 256, 37, 32, "packed", True), (3, 128, 64, 64, None, False), (5, 512, 9, 128, "packed", False)]


def _gloo_rank(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        for i, (M, K, N, bs, zk, bias) in enumerate(CASES):
            a, b, s, zp, bb = _case(i, M, K, N, bs, zk, bias)
            t = lambda x: None if x is None else torch.from_numpy(x)  # noqa: E731
            mod = ShardedMatMulNBits(t(b), t(s), t(zp), t(bb), K=K, N=N, block_size=bs, compute=_oracle_compute)
            y = mod(torch.from_numpy(a))
            # the same module built from this rank's shards alone
            mod2 = ShardedMatMulNBits.from_shard(shard_tensor(t(b), N, world, rank), shard_tensor(t(s), N, world, rank),
                                                 shard_tensor(t(zp), N, world, rank), shard_tensor(t(bb), N, world, rank),
                                                 K=K, N=N, block_size=bs, compute=_oracle_compute)
            y2 = mod2(torch.from_numpy(a))
            ref = O.matmul_nbits(a, b, s, zp, bb, K=K, N=N, bits=4, block_size=bs)
            # defer only applies to the peer-memory exchange: on a gloo group Y is complete at once
            y3 = mod(torch.from_numpy(a), defer=True)
            mod.wait_gather()
            same = bool(torch.equal(y, y2)) and bool(torch.equal(y, y3)) and mod._pending is None
            results[(rank, i)] = (bool(np.array_equal(y.numpy(), ref)), same, tuple(y.shape))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_gloo_ranks_reassemble_the_full_output(world):
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    mp.start_processes(_gloo_rank, args=(world, _free_port(), results), nprocs=world, start_method="spawn")
    for r in range(world):
        for i, (M, K, N, *_rest) in enumerate(CASES):
            exact, same, shape = results[(r, i)]
            assert exact, (r, i)          # the gathered Y equals the oracle's full Y bit for bit
            assert same, (r, i)           # full-tensor and from_shard construction agree
            assert shape == (M, N)


def test_single_process_is_a_plain_call():
    a, b, s, zp, bb = _case(7, 2, 128, 40, 32, "packed", True)
    t = lambda x: None if x is None else torch.from_numpy(x)  # noqa: E731
    mod = ShardedMatMulNBits(t(b), t(s), t(zp), t(bb), K=128, N=40, block_size=32, compute=_oracle_compute)
    y = mod(torch.from_numpy(a))
    assert np.array_equal(y.numpy(), O.matmul_nbits(a, b, s, zp, bb, K=128, N=40, bits=4, block_size=32))


# ----------------------------------------------------------------- NCCL on 2 GPUs
def _nccl_rank(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        from xrgpu_b200 import functional as F
        for i, (M, K, N, bs) in enumerate([(1, 4096, 4100, 32), (4, 4096, 1024, 128), (64, 1024, 1000, 64)]):
            a, b, s, zp, bb = _case(100 + i, M, K, N, bs, "packed", True)
            d = lambda x: None if x is None else torch.from_numpy(x).cuda()  # noqa: E731
            y = ShardedMatMulNBits(d(b), d(s), d(zp), d(bb), K=K, N=N, block_size=bs)(d(a))
            y_one = F.matmul_nbits(d(a), d(b), d(s), d(zp), d(bb), K=K, N=N, block_size=bs)
            torch.cuda.synchronize()
            # different per-call shapes may split K differently: compare within the tolerance
            d_max = (y.float() - y_one.float()).abs().max().item()
            scale = y_one.float().abs().max().item()
            results[(rank, i)] = bool(y.shape == y_one.shape and d_max <= 2e-3 * scale)
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_nccl_two_gpus_match_one_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    mp.start_processes(_nccl_rank, args=(2, _free_port(), results), nprocs=2, start_method="spawn")
    assert all(results[(r, i)] for r in range(2) for i in range(3)), dict(results)


# ----------------------------------------------------------------- peer-memory all-gather on 2 GPUs
def _peer_rank(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    mods = []
    try:
        from xrgpu_b200 import functional as F
        # (M, K, N, bs): shards of 2048 / 2056 columns (16-byte rows); N = 4111 pads the last shard;
        # M = 512 gives 2 MB shards, cut into 8 chunks per peer
        for i, (M, K, N, bs) in enumerate([(1, 4096, 4096, 32), (1, 4096, 4111, 32), (4, 2048, 1024, 64),
                                           (512, 1024, 4096, 64)]):
            a, b, s, zp, bb = _case(200 + i, M, K, N, bs, "packed", True)
            d = lambda x: None if x is None else torch.from_numpy(x).cuda()  # noqa: E731
            peer = ShardedMatMulNBits(d(b), d(s), d(zp), d(bb), K=K, N=N, block_size=bs, peer_gather=True)
            nccl = ShardedMatMulNBits(d(b), d(s), d(zp), d(bb), K=K, N=N, block_size=bs, peer_gather=False)
            mods.append(peer)
            assert peer.uses_peer_gather(M) and not nccl.uses_peer_gather(M)
            ok = True
            if M == 1:  # single-row float16 decode shards take the fused GEMV send
                peer(d(a))
                ok &= peer._fused_ok is not None and peer._fused_ok[1]
            # repeated calls: the epochs advance and the double-buffered staging alternates
            for rep in range(5):
                x = d(a) * (1.0 + 0.25 * rep)
                ok &= torch.equal(peer(x), nccl(x))
            # captured in a CUDA graph and replayed with new inputs (no NCCL call inside the graph)
            x_in = d(a).clone()
            y_out = torch.empty((M, N), dtype=torch.float16, device="cuda")
            peer(x_in, out=y_out)
            torch.cuda.synchronize()
            s_ = torch.cuda.Stream()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.stream(s_):
                with torch.cuda.graph(g, stream=s_):
                    peer(x_in, out=y_out)
            for rep in range(3):
                x_in.copy_(d(a) * (0.5 + rep))
                g.replay()
                torch.cuda.synchronize()
                ok &= torch.equal(y_out, nccl(x_in))
            del g
            # overlapped form: the gather runs on a side stream; Y is complete after wait_gather()
            side = torch.cuda.Stream()
            for rep in range(2):
                x = d(a) * (0.75 + rep)
                y_side = peer(x, gather_stream=side)
                peer.wait_gather()
                ok &= torch.equal(y_side, nccl(x))
            # the single-GPU kernel agrees to the tolerance (its K split may differ)
            y_one = F.matmul_nbits(d(a), d(b), d(s), d(zp), d(bb), K=K, N=N, block_size=bs)
            ok &= bool((peer(d(a)).float() - y_one.float()).abs().max().item() <= 2e-3 * y_one.float().abs().max().item())
            torch.cuda.synchronize()
            results[(rank, i)] = bool(ok) and F.device_error(rank) == 0
    finally:
        for m in mods:
            m.close()
        dist.destroy_process_group()


@pytest.mark.gpu
def test_peer_allgather_two_gpus_matches_nccl():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    mp.start_processes(_peer_rank, args=(2, _free_port(), results), nprocs=2, start_method="spawn")
    assert all(results.get((r, i), False) for r in range(2) for i in range(4)), dict(results)


# ----------------------------------------------------------------- fused GEMV send, mixed with other calls
# (K, N, block_size, zero points): shards of 2048, 504 and 1024 columns on one shared group
FUSED_SPECS = [(4096, 4096, 32, "packed"), (4096, 1008, 64, None), (14336, 2048, 32, "packed")]


def _fused_rank(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    group = None
    try:
        from xrgpu_b200 import functional as F
        from xrgpu_b200.p2p import PeerAllGather
        F.device_error(rank, clear=True)
        group = PeerAllGather(1 << 20)
        d = lambda x: None if x is None else torch.from_numpy(x).cuda()  # noqa: E731
        fused, plain, acts = [], [], []
        for i, (K, N, bs, zk) in enumerate(FUSED_SPECS):
            a, b, s, zp, bb = _case(300 + i, 4, K, N, bs, zk, True)
            fused.append(ShardedMatMulNBits(d(b), d(s), d(zp), d(bb), K=K, N=N, block_size=bs, peer_group=group))
            plain.append(ShardedMatMulNBits(d(b), d(s), d(zp), d(bb), K=K, N=N, block_size=bs, peer_gather=False))
            acts.append(d(a))
        ok = True
        for rep in range(3):  # fused calls of three shard sizes, each followed by a 4-row call (a
            for f, p, a in zip(fused, plain, acts):  # separate all-gather) on the same group
                x1 = a[:1] * (1.0 + 0.5 * rep)
                ok &= torch.equal(f(x1), p(x1)) and bool(f._fused_ok[1])
                ok &= torch.equal(f(a), p(a))
        side = torch.cuda.Stream()
        for rep in range(2):  # overlapped: receives on a side stream, the next send ordered after them
            ys = [f(a[1:2] * (0.5 + rep), gather_stream=side) for f, a in zip(fused, acts)]
            for f in fused:
                f.wait_gather()
            ok &= all(torch.equal(y, p(a[1:2] * (0.5 + rep))) for y, p, a in zip(ys, plain, acts))
        # deferred: the receive is enqueued by wait_gather on the joining stream
        for rep in range(2):
            for f, p, a in zip(fused, plain, acts):
                x1 = a[3:4] * (1.5 + rep)
                y = f(x1, defer=True)
                f.wait_gather()
                ok &= torch.equal(y, p(x1))
        # deferred sends of three modules with their own groups, received by one kernel
        own = [ShardedMatMulNBits(f.b, f.scales, f.zero_points, f.bias, K=f.K, N=f.N, block_size=f.block_size,
                                  _presharded=True) for f in fused]
        for rep in range(3):
            xs = [a[rep:rep + 1] * (0.75 + rep) for a in acts]
            ys = [m(x, defer=True) for m, x in zip(own, xs)]
            ShardedMatMulNBits.wait_gather_all(own)
            ok &= all(torch.equal(y, p(x)) for y, p, x in zip(ys, plain, xs))
        for m in own:
            m.close()
        # two fused sends on one group without the first one's receive in between are refused
        fused[0](acts[0][:1], defer=True)
        try:
            fused[1](acts[1][:1], defer=True)
            ok = False
        except RuntimeError:
            pass
        fused[0].wait_gather()
        # captured in a CUDA graph with its receive, replayed with new inputs
        x_in = acts[0][:1].clone()
        y_out = torch.empty((1, FUSED_SPECS[0][1]), dtype=torch.float16, device="cuda")
        fused[0](x_in, out=y_out)
        torch.cuda.synchronize()
        s_ = torch.cuda.Stream()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s_):
            with torch.cuda.graph(g, stream=s_):
                fused[0](x_in, out=y_out)
        for rep in range(4):
            x_in.copy_(acts[0][2:3] * (0.25 + rep))
            g.replay()
            torch.cuda.synchronize()
            ok &= torch.equal(y_out, plain[0](x_in))
        del g
        torch.cuda.synchronize()
        results[rank] = bool(ok) and F.device_error(rank) == 0
    finally:
        if group is not None:
            group.close()
        dist.destroy_process_group()


@pytest.mark.gpu
def test_fused_gemv_send_two_gpus_matches_nccl():
    """Single-row calls whose GEMV sends its columns to the other rank itself (flag-in-word words)
    and a receive kernel assembles Y: bit-exact against NCCL's all-gather of the same shards, on one
    group shared with separate all-gathers of other sizes, overlapped, and replayed in a graph."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    mp.start_processes(_fused_rank, args=(2, _free_port(), results), nprocs=2, start_method="spawn")
    assert results.get(0) and results.get(1), dict(results)


# ----------------------------------------------------------------- shards of changing size on one group
# (rows, shard columns) of float16 shards: 4 KB, 1 MB and 1 MB + 16 B (4 and 5 chunks per peer), prefill
# shards of 7.3, 8 and 16 MB (28, 32 and 64 chunks), back to a decode shard, then the same again.
ALTERNATING = [(1, 2048), (512, 1024), (1, 524296), (2048, 1792), (1, 2048), (4096, 1024), (1, 524296),
               (1024, 8192), (512, 1024), (1, 4096)]


def _alternating_rank(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    group = None
    try:
        from xrgpu_b200 import functional as F
        from xrgpu_b200.p2p import PeerAllGather
        group = PeerAllGather(max(r * c * 2 for r, c in ALTERNATING))
        gen = torch.Generator(device="cuda")
        ok = True
        for rep in range(2):
            for i, (M, S) in enumerate(ALTERNATING):
                gen.manual_seed(1000 * rep + 10 * i + rank)
                shard = torch.randn((M, S), generator=gen, device="cuda").to(torch.float16)
                N = world * S - (8 if i % 3 == 1 else 0)  # a padded last shard on some calls
                out = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
                group.all_gather(shard, out, N)
                ref = torch.empty((world, M, S), dtype=torch.float16, device="cuda")
                dist.all_gather_into_tensor(ref, shard)
                ref = ref.permute(1, 0, 2).reshape(M, world * S)[:, :N]
                ok &= torch.equal(out, ref)
        torch.cuda.synchronize()
        results[rank] = bool(ok) and F.device_error(rank) == 0
    finally:
        if group is not None:
            group.close()
        dist.destroy_process_group()


@pytest.mark.gpu
def test_peer_allgather_shards_of_changing_size_on_one_group():
    """One group, successive calls whose shards fall in different chunk counts (the staging
    parity must follow the call, not the chunk index): every call equals NCCL's all-gather."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    mp.start_processes(_alternating_rank, args=(2, _free_port(), results), nprocs=2, start_method="spawn")
    assert results.get(0) and results.get(1), dict(results)


def test_epoch_slots_advance_once_per_call_for_any_chunk_count():
    """Host model of the kernel's epoch bookkeeping: the CTA of chunk c advances slots
    c, c + chunks, ... of its peer, so all 64 slots stay equal whatever the chunk counts."""
    rng = np.random.default_rng(3)
    slots = np.zeros(64, dtype=np.int64)
    for call in range(1, 400):
        chunks = int(rng.integers(4, 65))
        e = {c: slots[c] + 1 for c in range(chunks)}  # every chunk CTA reads its own slot
        assert len(set(e.values())) == 1 and e[0] == call
        for c in range(chunks):
            for s in range(c, 64, chunks):
                slots[s] = e[c]
        assert (slots == call).all()


# ----------------------------------------------------------------- a peer that never arrives
def _absent_peer(conn):
    """Rank 1 of a two-rank group on the same GPU that exports its region and never calls."""
    import ctypes
    from xrgpu_b200 import _native
    lib = _native.load()
    handle = ctypes.create_string_buffer(_native.P2P_HANDLE_BYTES)
    g = ctypes.c_void_p()
    st = lib.xrgpu_p2p_create(0, 2, 1, 1 << 16, ctypes.byref(g), handle)
    conn.send((st, handle.raw))
    conn.recv()  # the other rank has finished
    lib.xrgpu_p2p_destroy(g)
    conn.close()


@pytest.mark.gpu
def test_peer_wait_gives_up_and_reports_0x401():
    """A bounded device-side wait that runs out: rank 0's all-gather waits for a flag that rank 1
    (another process, same GPU, never calling) does not set. The kernel gives up after 1 s,
    records 0x401 in the device error word and returns; the context stays usable."""
    import ctypes
    from xrgpu_b200 import _native
    from xrgpu_b200 import functional as F
    lib = _native.load()
    ctx = mp.get_context("spawn")
    parent, child = ctx.Pipe()
    proc = ctx.Process(target=_absent_peer, args=(child,))
    proc.start()
    g = ctypes.c_void_p()
    try:
        st, other = parent.recv()
        assert st == 0
        torch.cuda.set_device(0)
        F.device_error(0, clear=True)
        mine = ctypes.create_string_buffer(_native.P2P_HANDLE_BYTES)
        _native.check(lib.xrgpu_p2p_create(0, 2, 0, 1 << 16, ctypes.byref(g), mine))
        _native.check(lib.xrgpu_p2p_connect(g, mine.raw + other))
        shard = torch.ones((1, 256), dtype=torch.float16, device="cuda")
        out = torch.zeros((1, 512), dtype=torch.float16, device="cuda")
        stream = torch.cuda.current_stream().cuda_stream
        _native.check(lib.xrgpu_p2p_allgather(g, ctypes.c_void_p(shard.data_ptr()), 1, 512,
                                              ctypes.c_void_p(out.data_ptr()), 1024, 1024, ctypes.c_void_p(stream)))
        torch.cuda.synchronize()
        assert F.device_error(0, clear=True) == 0x401
        assert torch.equal(out[:, :256], shard)          # this rank's own block was still written
        assert torch.equal(out[:, 256:], torch.zeros_like(out[:, 256:]))  # the absent peer's was not
        # the context is still usable: a GEMV runs and the word stays clear
        a = torch.randn((1, 512), device="cuda").half()
        b = torch.randint(0, 256, (64, 16, 16), dtype=torch.uint8, device="cuda")
        s = torch.full((64, 16), 0.01, dtype=torch.float16, device="cuda")
        F.matmul_nbits(a, b, s, K=512, N=64, block_size=32)
        torch.cuda.synchronize()
        assert F.device_error(0) == 0
    finally:
        if g.value:
            torch.cuda.synchronize()
            lib.xrgpu_p2p_destroy(g)
        parent.send("done")
        proc.join(timeout=60)
    assert proc.exitcode == 0


def _skipping_rank(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    group = None
    try:
        from xrgpu_b200 import _native
        from xrgpu_b200 import functional as F
        from xrgpu_b200.p2p import PeerAllGather
        F.device_error(rank, clear=True)
        group = PeerAllGather(1 << 16)
        shard = torch.full((1, 1024), float(rank + 1), dtype=torch.float16, device="cuda")
        out = torch.zeros((1, 2048), dtype=torch.float16, device="cuda")
        group.all_gather(shard, out, 2048)  # both ranks: a normal call
        group.check()
        first_ok = torch.equal(out[:, 1024:], torch.full_like(out[:, 1024:], 2.0)) if rank == 0 else True
        if rank == 0:  # rank 1 leaves out the second call, between steps
            group.all_gather(shard, out, 2048)
        try:
            group.check()
            raised = False
        except _native.XrgpuError:
            raised = True
        results[rank] = (bool(first_ok), raised, group.broken)
    finally:
        if group is not None:
            group.close()
        dist.destroy_process_group()


@pytest.mark.gpu
def test_peer_wait_expires_when_a_rank_skips_a_call_two_gpus():
    """On 2 GPUs rank 1 skips one all-gather: rank 0's kernel gives up after 1 s, records 0x401 and
    returns; ``check()`` raises on rank 0 only and marks the group unusable."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    mp.start_processes(_skipping_rank, args=(2, _free_port(), results), nprocs=2, start_method="spawn")
    assert results.get(0) == (True, True, True) and results.get(1) == (True, False, False), dict(results)
