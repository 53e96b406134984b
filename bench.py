#!/usr/bin/env python
"""MatMulNBits benchmark on B200: decode GB/s and prefill TFLOP/s through this repo's C ABI.

Contract (one JSON line from rank 0):
  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

Workloads (synthetic seeded data of their shapes/distributions):
  llama3_8b_decode (default, config 2): one Llama-3-8B layer of decode GEMVs per step -- q, k, v,
      o, gate, up, down with (K, N) = (4096,4096) x2, (4096,1024) x2, (4096,14336) x2,
      (14336,4096); M=1, A fp16 ~N(0,1), bits 4, block 32, scales fp16 ~U(0.005,0.02), packed
      uint8 zero points (nibbles uniform in [0,15]). metric GB/s of algorithmic bytes
      (B + scales + zero points + A + Y).
  batched_decode_m{4,16,64} (config 3), prefill_m2048 (config 4, TFLOP/s), oracle_case (config 1).
  llama70b_shard_decode / llama70b_shard_prefill (config 5): one GPU's 1/8 column shard of the
      70B-scale projections (K, N) = (8192, 28672), (28672, 8192), (8192, 128256), i.e. (8192,3584),
      (28672,1024), (8192,16032), at M=1 (GB/s) and M=4096 (TFLOP/s); bs 32, packed zero points.
      With --gpus 8 the weak-scaled step is exactly the full config-5 problem.
Each step uses a different copy ("layer") of the weights; the copies total > 3x the 126 MB L2,
so every step streams its weights from HBM (config: "l2": "rotating weight copies > L2").

The line for the default workload also carries a "prefill" object: config 4 (M=2048, K=4096,
N=14336, bs 64, no zero points) measured in the same run with its own roofline, e2e and CPU
baseline, so both halves of the metric are in one record. On one GPU it also carries
"batched_decode": config 3 (M = 4, 16, 64; K=4096, N=14336, bs 128, packed zero points), each
with its step time and roofline.

Multi-GPU (torchrun, one process per GPU, NCCL): the headline is weak scaling -- every rank owns a
contiguous 1/N slice of each projection's output columns of an N-times-wider layer (per-GPU work
fixed), and the step ends with one all-gather of Y per projection (the library's peer-memory
all-gather over NVLink; NCCL for shards above 64 MB). Time is the max over ranks. The line adds
  "strong": config 2 decode and config 4 prefill as FIXED problems sharded N ways (step time at N
      GPUs, the same problem on one GPU, speed-up), each checked against the unsharded result;
  "parity": the first step's gathered Y checked against a reference (strong problems: the
      single-GPU kernel on the full problem, BASELINE tolerances; weak headline: an NCCL
      all-gather of the same shards, bit-exact).

--impl reference times the reference's own CPU algorithm (oracle/_ref: packedMatmul/nbitWeight
compiled from the reference sources; the C oracle port when that is absent) on all host threads,
on a bounded column sample of the same workload, on rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
import zlib
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PEAKS_FILE = ROOT / "MEASURED_PEAKS.json"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

LLAMA_LAYER = [("q", 4096, 4096), ("k", 4096, 1024), ("v", 4096, 1024), ("o", 4096, 4096),
               ("gate", 4096, 14336), ("up", 4096, 14336), ("down", 14336, 4096)]
# Dependencies of a decoder layer: q, k, v share their input; o needs attention over all three;
# gate and up share their input; down needs both.
LLAMA_GROUPS = [["q", "k", "v"], ["o"], ["gate", "up"], ["down"]]

WORKLOADS = {
    "llama3_8b_decode": dict(config=2, M=1, bs=32, zp=True, scale=(0.005, 0.02), proj=LLAMA_LAYER, kind="decode"),
    "batched_decode_m4": dict(config=3, M=4, bs=128, zp=True, scale=(0.002, 0.01), proj=[("ffn", 4096, 14336)], kind="decode"),
    "batched_decode_m16": dict(config=3, M=16, bs=128, zp=True, scale=(0.002, 0.01), proj=[("ffn", 4096, 14336)], kind="decode"),
    "batched_decode_m64": dict(config=3, M=64, bs=128, zp=True, scale=(0.002, 0.01), proj=[("ffn", 4096, 14336)], kind="decode"),
    "prefill_m2048": dict(config=4, M=2048, bs=64, zp=False, scale=(0.005, 0.02), proj=[("ffn", 4096, 14336)], kind="prefill"),
    "llama70b_shard_decode": dict(config=5, M=1, bs=32, zp=True, scale=(0.005, 0.02), kind="decode",
                                  proj=[("up", 8192, 3584), ("down", 28672, 1024), ("lm_head", 8192, 16032)]),
    "llama70b_shard_prefill": dict(config=5, M=4096, bs=32, zp=True, scale=(0.005, 0.02), kind="prefill",
                                   proj=[("up", 8192, 3584), ("down", 28672, 1024), ("lm_head", 8192, 16032)]),
    "oracle_case": dict(config=1, M=1, bs=32, zp=False, scale=(0.005, 0.02), proj=[("proj", 4096, 4096)], kind="decode",
                        dtype="float32"),
}
TOL_MAX, TOL_FROB = 1e-2, 2e-3  # max|dY| <= 1e-2 max|Y_ref|, relative Frobenius <= 2e-3


def upload_graph(g) -> None:
    """cuGraphUpload of a captured torch CUDA graph on the current stream (driver API): a graph's
    first launch otherwise includes its upload to the device."""
    import ctypes
    import torch
    drv = ctypes.CDLL("libcuda.so.1")
    drv.cuGraphUpload.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    st = drv.cuGraphUpload(ctypes.c_void_p(g.raw_cuda_graph_exec()), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    if st != 0:
        raise RuntimeError(f"cuGraphUpload failed with CUresult {st}")


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def peaks():
    if PEAKS_FILE.exists():
        d = json.loads(PEAKS_FILE.read_text())
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def proj_bytes(M, K, N, bs, zp, act_bytes, zp_bytes=None):
    """Algorithmic bytes of one projection: B + scales + zero points + A + Y at their stored widths.
    zp_bytes: bytes per zero point in the float form ([N, kb]); None = packed uint8 ([N, ceil(kb/2)])."""
    kb = K // bs
    z = 0
    if zp:
        z = N * kb * zp_bytes if zp_bytes else N * ((kb + 1) // 2)
    return N * K // 2 + N * kb * act_bytes + z + M * K * act_bytes + M * N * act_bytes


def groups_for(wl):
    names = [n for (n, _, _) in wl["proj"]]
    if sorted(names) == sorted(n for g in LLAMA_GROUPS for n in g):
        return [list(g) for g in LLAMA_GROUPS]
    return [[n] for n in names]  # other workloads: each projection depends on the last


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampled every 200 ms during the timed region (read-only queries)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200", "-f", self.path],
                                         stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        except Exception as e:  # pragma: no cover
            log("clock sampling unavailable:", e)
            self.proc = None

    def stop(self):
        out = {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        if not self.proc:
            return out
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        try:
            for line in Path(self.path).read_text().splitlines():
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
            os.unlink(self.path)
        except Exception:
            pass
        if not rows:
            return out
        num = lambda v: v.replace(".", "").isdigit()  # noqa: E731
        sm = [float(r[1]) for r in rows if num(r[1])]
        mx = [float(r[2]) for r in rows if num(r[2])]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        power = [float(r[3]) for r in rows if num(r[3])]
        out.update(sm_mhz=statistics.median(sm) if sm else None, sm_max_mhz=max(mx) if mx else None,
                   reasons=reasons, samples=len(rows), power_w_max=max(power) if power else None)
        return out


# ----------------------------------------------------------------------------- distributed
def dist_init():
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    import torch
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(world, value):
    if world == 1:
        return value
    import torch
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def min_over_ranks(world, value):
    return -max_over_ranks(world, -value)


# ----------------------------------------------------------------------------- data
def seed_of(seed, layer, name, rank):
    return seed * 1000003 + layer * 1009 + zlib.crc32(name.encode()) % 997 + 7919 * rank


def gen_projection(wl, name, K, N, key, device, dtype):
    """B, scales and (packed) zero points of one projection, seeded by `key` (BASELINE distributions)."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(key)
    kb = K // wl["bs"]
    lo, hi = wl["scale"]
    b = torch.randint(0, 256, (N, kb, wl["bs"] // 2), dtype=torch.uint8, device=device, generator=g)
    s = (torch.rand((N, kb), device=device, generator=g) * (hi - lo) + lo).to(torch.float16).to(dtype)
    zp = torch.randint(0, 256, (N, (kb + 1) // 2), dtype=torch.uint8, device=device, generator=g) if wl["zp"] else None
    return dict(name=name, K=K, N=N, b=b, s=s, zp=zp)


def within_tol(got, ref):
    """(ok, max|dY| / max|Y_ref|, relative Frobenius) under BASELINE.json's tolerances."""
    d = (got.double() - ref.double())
    scale = ref.double().abs().max().item()
    rel_max = d.abs().max().item() / max(scale, 1e-30)
    frob = (d.norm() / ref.double().norm().clamp_min(1e-30)).item()
    return rel_max <= TOL_MAX and frob <= TOL_FROB, rel_max, frob


class Runner:
    """One workload's decode or prefill step on this rank.

    mode "weak": this rank owns N columns of an (N * world)-wide projection (its own seeded shard).
    mode "strong": every rank generates the same full projection and keeps its 1/world column slice
    (ShardedMatMulNBits); the first `keep_full` layers keep the full weights for the single-GPU
    comparison. With world == 1 a step is plain ``functional.matmul_nbits`` calls.
    """

    def __init__(self, wl, args, world, rank, device, mode="weak", max_layers=64):
        import torch
        from xrgpu_b200 import functional as F
        self.F = F
        self.wl, self.args, self.world, self.rank, self.device, self.mode = wl, args, world, rank, device, mode
        self.M = wl["M"]
        self.dt = torch.float32 if wl.get("dtype") == "float32" else torch.float16
        self.act_bytes = 4 if self.dt == torch.float32 else 2
        props = torch.cuda.get_device_properties(device)
        l2 = getattr(props, "L2_cache_size", 126 * 2**20) or 126 * 2**20
        # bytes this rank streams per step, and the whole job's algorithmic bytes / FLOPs per step
        if mode == "weak":
            self.rank_proj = [(n, K, N) for (n, K, N) in wl["proj"]]
            self.full_proj = [(n, K, N * world) for (n, K, N) in wl["proj"]]
        else:
            self.full_proj = [(n, K, N) for (n, K, N) in wl["proj"]]
            self.rank_proj = [(n, K, -(-N // world)) for (n, K, N) in wl["proj"]]
        pb = lambda projs: sum(proj_bytes(self.M, K, N, wl["bs"], wl["zp"], self.act_bytes) for (_, K, N) in projs)  # noqa: E731
        self.bytes_rank, self.bytes_job = pb(self.rank_proj), pb(self.full_proj)
        self.flops_job = sum(2 * self.M * K * N for (_, K, N) in self.full_proj)
        self.layers = args.layers or min(max_layers, max(2, math.ceil(3 * l2 / self.bytes_rank) + 1))
        self.groups = groups_for(wl)
        self.keep_full = 0
        self._build()

    def _build(self):
        import torch
        wl, dev, F = self.wl, self.device, self.F
        g = torch.Generator(device=dev)
        g.manual_seed(self.args.seed)
        # Activations and outputs are views into one buffer each (offsets padded to 64 elements), so
        # the end-to-end step moves them with one host-to-device and one device-to-host copy.
        pad = lambda n: -(-n // 64) * 64  # noqa: E731
        ks = sorted({K for (_, K, _) in wl["proj"]})
        self.act_flat = torch.empty(sum(pad(self.M * K) for K in ks), device=dev, dtype=self.dt)
        self.acts, off = {}, 0
        for K in ks:
            self.acts[K] = self.act_flat[off:off + self.M * K].view(self.M, K)
            self.acts[K].copy_(torch.randn((self.M, K), generator=g, device=dev, dtype=torch.float32))
            off += pad(self.M * K)
        self.y_flat = torch.empty(sum(pad(self.M * N) for (_, _, N) in self.full_proj), device=dev, dtype=self.dt)
        self.ys, off = {}, 0
        for (n, K, N) in self.full_proj:
            self.ys[n] = self.y_flat[off:off + self.M * N].view(self.M, N)
            off += pad(self.M * N)
        self.weights, self.full = [], []
        self.keep_full = min(self.layers, 4) if (self.mode == "strong" and self.world > 1) else 0
        shard_bytes = {}
        for layer in range(self.layers):
            projs = []
            for (name, K, N) in wl["proj"]:
                if self.mode == "weak":
                    p = gen_projection(wl, name, K, N, seed_of(self.args.seed, layer, name, self.rank), dev, self.dt)
                else:
                    p = gen_projection(wl, name, K, N, seed_of(self.args.seed, layer, name, 0), dev, self.dt)
                projs.append(p)
            if self.world > 1:
                from xrgpu_b200.sharded import ShardedMatMulNBits
                mods = []
                for p, (name, K, Nf) in zip(projs, self.full_proj):
                    if self.mode == "weak":
                        mod = ShardedMatMulNBits.from_shard(p["b"], p["s"], p["zp"], None, K=K, N=Nf, block_size=wl["bs"])
                    else:
                        mod = ShardedMatMulNBits(p["b"], p["s"], p["zp"], None, K=K, N=Nf, block_size=wl["bs"])
                    shard_bytes[name] = self.M * mod.S * self.act_bytes
                    mods.append(dict(name=name, K=K, N=Nf, mod=mod))
                if layer < self.keep_full:
                    self.full.append(projs)  # full weights of this layer, for the single-GPU comparison
                projs = mods
            self.weights.append(projs)
        self.paths = sorted({self._path(K, N) for (_, K, N) in self.rank_proj})
        self.shared = None
        self.peer = self.world > 1 and all(p["mod"].uses_peer_gather(self.M, self.act_bytes)
                                           for layer in self.weights for p in layer)
        if self.peer:
            from xrgpu_b200.p2p import PeerAllGather
            # one peer-memory group per projection, shared by its copies in every layer and created
            # before any capture: a projection's calls alternate send and receive on its own group,
            # so the gathers of different projections may be in flight together
            self.shared = {name: PeerAllGather(nbytes) for name, nbytes in shard_bytes.items()}
            for layer in self.weights:
                for p in layer:
                    p["mod"].set_peer_group(self.shared[p["name"]])
        # How the peer-memory exchanges of a step are ordered (N > 1): "defer" enqueues each exchange
        # on the compute stream just before the first kernel that needs its Y (one stream, every
        # launch early behind the previous one); "stream" runs them on a side stream joined by events;
        # "inline" puts each right after its own GEMV.
        mode = "inline" if self.args.no_overlap else self.args.gather_mode
        self.gather_mode = mode if self.peer else "inline"
        self.overlap = self.gather_mode != "inline"
        self.comm = torch.cuda.Stream(dev) if self.gather_mode == "stream" else None
        self.graphs = []

    def _path(self, K, N):
        import torch
        dev = self.device
        kb = K // self.wl["bs"]
        b = torch.empty((N, kb, self.wl["bs"] // 2), dtype=torch.uint8, device=dev)
        s = torch.empty((N, kb), dtype=self.dt, device=dev)
        zp = torch.empty((N, (kb + 1) // 2), dtype=torch.uint8, device=dev) if self.wl["zp"] else None
        return self.F.select_path(self.acts[K], b, s, zp, K=K, N=N, block_size=self.wl["bs"])

    # ------------------------------------------------------------------ execution
    def step(self, layer):
        """One step over layer `layer`: the projections in dependency-group order."""
        projs = {p["name"]: p for p in self.weights[layer]}
        bs = self.wl["bs"]
        for grp in self.groups:
            for name in grp:
                p = projs[name]
                x = self.acts[p["K"]]
                if self.world == 1:
                    self.F.matmul_nbits(x, p["b"], p["s"], p["zp"], K=p["K"], N=p["N"], block_size=bs, out=self.ys[name])
                elif self.gather_mode == "stream":  # the gather runs beside the group's other kernels
                    p["mod"](x, out=self.ys[name], gather_stream=self.comm)
                elif self.gather_mode == "defer":  # the gather waits on this stream until the group ends
                    p["mod"](x, out=self.ys[name], defer=True)
                else:
                    p["mod"](x, out=self.ys[name])
            if self.world > 1 and self.overlap:
                from xrgpu_b200.sharded import ShardedMatMulNBits
                ShardedMatMulNBits.wait_gather_all([projs[name]["mod"] for name in grp])

    def step_full(self, layer):
        """The unsharded problem of a kept layer on this GPU alone (strong-scaling comparison)."""
        for p in self.full[layer]:
            self.F.matmul_nbits(self.acts[p["K"]], p["b"], p["s"], p["zp"], K=p["K"], N=p["N"],
                                block_size=self.wl["bs"], out=self.ys_full[p["name"]])

    @property
    def graphable(self):
        return (self.world == 1 or self.peer) and not self.args.no_graphs

    def capture(self, fn, count):
        """One CUDA graph per layer of fn(layer) (only for steps without NCCL calls)."""
        import torch
        graphs = []
        s = torch.cuda.Stream(self.device)
        with torch.cuda.stream(s):
            for layer in range(count):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=s):
                    fn(layer)
                graphs.append(g)
        torch.cuda.synchronize()
        return graphs

    def capture_seq(self, fn, layers):
        """One CUDA graph of fn(layer) for every layer in `layers`, in order (every capture of a
        runner on one stream)."""
        import torch
        if getattr(self, "_cap_stream", None) is None:
            self._cap_stream = torch.cuda.Stream(self.device)
        s = self._cap_stream
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                for layer in layers:
                    fn(layer)
        torch.cuda.synchronize()
        return g

    def timed(self, fn, count, graphs, steps, warmup, clocks=None):
        """Device time per step (ms, max over ranks) of `steps` steps after `warmup` untimed ones,
        bracketed by a barrier and a synchronize on both sides. With graphs, the timed steps are one
        CUDA graph holding all of them (step i on weight copy i mod count), so a step's time is the
        device's and not the host's launch rate; the warm-up replays its own graph."""
        import torch

        seq = {}
        if graphs:
            seq[max(3, warmup)] = self.capture_seq(fn, [i % count for i in range(max(3, warmup))])
            seq[steps] = seq.get(steps) or self.capture_seq(fn, [i % count for i in range(steps)])
            for g in seq.values():  # set-up: upload now, so that no timed launch pays for it
                upload_graph(g)
            torch.cuda.synchronize()

        def run(n, offset=0):
            if graphs:
                seq[n].replay()
                return
            for i in range(n):
                fn((offset + i) % count)

        run(max(3, warmup))
        barrier(self.world)
        if clocks is not None:
            clocks.start()
            time.sleep(0.25)
        barrier(self.world)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        run(steps)
        t1.record()
        torch.cuda.synchronize()
        barrier(self.world)
        ms = max_over_ranks(self.world, t0.elapsed_time(t1))
        clock = None
        if clocks is not None:
            # keep the sampler running for a few samples: every rank runs the same extra steps
            # (ms is the same on every rank after the max)
            reps = max(1, int(600 / max(ms, 1e-3))) if ms < 600 else 0
            for _ in range(reps):
                run(steps)
            torch.cuda.synchronize()
            clock = clocks.stop()
        return ms / steps, clock

    def kernel_times(self):
        """Each projection alone: a CUDA graph of back-to-back launches over the rotating copies
        (one GPU only)."""
        import torch
        out = {}
        bs = self.wl["bs"]
        for (name, K, N) in self.rank_proj:
            reps = 4 * self.layers
            gs = torch.cuda.Stream(self.device)
            gk = torch.cuda.CUDAGraph()
            with torch.cuda.stream(gs):
                with torch.cuda.graph(gk, stream=gs):
                    for r in range(reps):
                        p = [q for q in self.weights[r % self.layers] if q["name"] == name][0]
                        self.F.matmul_nbits(self.acts[K], p["b"], p["s"], p["zp"], K=K, N=N, block_size=bs,
                                            out=self.ys[name])
            torch.cuda.synchronize()
            gk.replay()
            torch.cuda.synchronize()
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record()
            for _ in range(5):
                gk.replay()
            ev1.record()
            torch.cuda.synchronize()
            per = ev0.elapsed_time(ev1) / (5 * reps)
            kb = proj_bytes(self.M, K, N, bs, self.wl["zp"], self.act_bytes)
            out[name] = dict(K=K, N=N, us=round(per * 1e3, 3), gbs=round(kb / (per * 1e-3) / 1e9, 1),
                             tflops=round(2 * self.M * K * N / (per * 1e-3) / 1e12, 3))
            del gk
        return out

    def value_of(self, ms):
        if self.wl["kind"] == "decode":
            return self.bytes_job / (ms * 1e-3) / 1e9
        return self.flops_job / (ms * 1e-3) / 1e12

    def e2e(self, steps, warmup):
        """End to end through the public call: every step copies its activations in from pinned host
        memory (one copy: they share one buffer), runs the step's library calls and copies every Y out
        to pinned host memory (one copy), then synchronises. Steps without NCCL calls replay one CUDA
        graph holding the copies and the calls (recorded through the same public API); the eager form
        is timed too (e2e_eager_ms)."""
        import torch
        host_a = self.act_flat.cpu().pin_memory()
        host_y = torch.empty(self.y_flat.shape, dtype=self.y_flat.dtype).pin_memory()
        h2d = host_a.numel() * host_a.element_size()
        d2h = host_y.numel() * host_y.element_size()

        def body(layer):
            self.act_flat.copy_(host_a, non_blocking=True)
            self.step(layer)
            host_y.copy_(self.y_flat, non_blocking=True)

        def timed_e2e(graphs):
            for i in range(max(3, warmup)):
                graphs[i % len(graphs)].replay() if graphs else body(i % self.layers)
                torch.cuda.synchronize()
            barrier(self.world)
            w0 = time.perf_counter()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for i in range(steps):
                if graphs:
                    graphs[i % len(graphs)].replay()
                else:
                    body(i % self.layers)
                torch.cuda.synchronize()
            e1.record()
            torch.cuda.synchronize()
            wall = time.perf_counter() - w0
            return max_over_ranks(self.world, max(e0.elapsed_time(e1), wall * 1e3) / steps)

        eager_ms = timed_e2e(None)
        graphs = self.capture(body, self.layers) if self.graphable else None
        e_ms = timed_e2e(graphs) if graphs else eager_ms
        del graphs
        unit = "GB/s" if self.wl["kind"] == "decode" else "TFLOP/s"
        api = "functional.matmul_nbits -> xrgpu_mmnb_forward (C ABI)"
        if self.world > 1:
            api = "ShardedMatMulNBits -> " + api + " + peer-memory all-gather"
        return dict(value=round(self.value_of(e_ms), 2), unit=unit, h2d_bytes_per_step=h2d, d2h_bytes_per_step=d2h,
                    ms_per_step=round(e_ms, 4), e2e_eager_ms=round(eager_ms, 4),
                    path=api + ("; one CUDA graph per step holding the host copies and the calls, one sync per step"
                                if self.graphable else "; eager calls, one sync per step"))

    # ------------------------------------------------------------------ checks
    def parity(self):
        """Check the first step's gathered Y (world > 1). strong: against the single-GPU kernel on the
        full problem (BASELINE tolerances); weak: against an NCCL all-gather of the same shards
        (bit-exact). Every rank checks; the verdict is the AND over ranks."""
        import torch
        import torch.distributed as dist
        self.step(0)
        torch.cuda.synchronize()
        ok, worst_max, worst_frob = True, 0.0, 0.0
        if self.mode == "strong":
            self.ys_full = {n: torch.empty_like(y) for n, y in self.ys.items()}
            self.step_full(0)
            torch.cuda.synchronize()
            for n in self.ys:
                good, rel_max, frob = within_tol(self.ys[n], self.ys_full[n])
                ok &= good
                worst_max, worst_frob = max(worst_max, rel_max), max(worst_frob, frob)
            kind = "gathered Y vs the single-GPU kernel on the full problem (BASELINE tolerances)"
        else:
            for p in self.weights[0]:
                mod, n = p["mod"], p["name"]
                y_local = torch.empty((self.M, mod.S), dtype=self.dt, device=self.device)
                mod.local(self.acts[p["K"]], y_local)
                g = torch.empty((self.world, self.M, mod.S), dtype=self.dt, device=self.device)
                dist.all_gather_into_tensor(g, y_local)
                ref = g.permute(1, 0, 2).reshape(self.M, self.world * mod.S)[:, :p["N"]]
                ok &= torch.equal(self.ys[n], ref)
            kind = "gathered Y vs an NCCL all-gather of the same shards (bit-exact)"
        ok = min_over_ranks(self.world, 1.0 if ok else 0.0) > 0.5
        out = dict(ok=bool(ok), check=kind, ranks=self.world, projections=[n for (n, _, _) in self.full_proj])
        if self.mode == "strong":
            out.update(max_rel=float(f"{max_over_ranks(self.world, worst_max):.3e}"),
                       rel_frobenius=float(f"{max_over_ranks(self.world, worst_frob):.3e}"), tol_max=TOL_MAX,
                       tol_frobenius=TOL_FROB)
        return out

    def close(self):
        self.graphs = []
        if self.world > 1:
            import torch
            torch.cuda.synchronize()
            for layer in self.weights:
                for p in layer:
                    p["mod"].close()
            for name in sorted(self.shared or {}):
                self.shared[name].close()  # collective: every rank closes them in the same order


def roofline_of(runner, step_ms, pk, pk_kind, clock=None):
    wl = runner.wl
    if wl["kind"] == "decode":
        achieved = runner.bytes_rank / (step_ms * 1e-3) / 1e9
        peak = pk["hbm_gbs"]
        r = dict(bound="hbm", achieved=round(achieved, 1), peak=peak, unit="GB/s", frac=round(achieved / peak, 4),
                 traffic=None, peak_source=f"{pk_kind} hbm_gbs",
                 note="achieved = algorithmic bytes this GPU streams per step / device time per step (CUDA graph "
                      "of the step's launches, rotating weight copies); per-projection kernel times in kernels_us")
    else:
        flops_rank = sum(2 * runner.M * K * N for (_, K, N) in runner.rank_proj)
        achieved = flops_rank / (step_ms * 1e-3) / 1e12
        # The timed region is a graph of back-to-back GEMMs: when the power cap acted during it, the
        # sustained GEMM figure is the denominator, else the burst one.
        capped = bool(clock) and "sw_power_cap" in (clock.get("reasons") or [])
        key = "bf16_tflops_sustained" if capped else "bf16_tflops"
        peak = pk.get(key, FALLBACK_PEAKS[key])
        r = dict(bound="tensor", achieved=round(achieved, 1), peak=peak, unit="TFLOP/s", frac=round(achieved / peak, 4),
                 traffic=None, peak_source=f"{pk_kind} {key} (" + ("sw_power_cap active during the timed GEMMs)"
                                                                  if capped else "burst: no power capping seen)"))
    return r


def attach_traffic(roofline, workload):
    traffic_file = ROOT / "profiles" / "traffic.json"
    if traffic_file.exists():
        tr = json.loads(traffic_file.read_text()).get(workload)
        if tr:
            roofline["traffic"] = tr.get("bytes_per_step")
            roofline["traffic_source"] = tr.get("source")


# ----------------------------------------------------------------------------- our arm
def measure(name, args, world, rank, local, device, *, mode="weak", headline=False, cpu=False):
    """Time one workload; returns the pieces of a JSON line (rank 0 uses them)."""
    wl = WORKLOADS[name]
    pk, pk_kind = peaks()
    runner = Runner(wl, args, world, rank, device, mode=mode, max_layers=64 if wl["kind"] == "decode" else 16)
    log(f"[rank {rank}] {name} ({mode}): {runner.layers} weight copies, paths {runner.paths}")
    for layer in range(runner.layers):  # warm-up outside capture (kernel attributes, peer group)
        runner.step(layer)
    import torch
    torch.cuda.synchronize()
    res = dict(workload=name, config=wl["config"], mode=mode, layers=runner.layers, paths=runner.paths)
    if world > 1:
        res["parity"] = runner.parity()
    graphs = runner.graphable
    clocks = ClockSampler(local) if (headline or wl["kind"] == "prefill") else None
    step_ms, clock = runner.timed(runner.step, runner.layers, graphs, args.steps, args.warmup, clocks)
    res.update(step_ms=step_ms, value=runner.value_of(step_ms), clocks=clock,
               unit="GB/s" if wl["kind"] == "decode" else "TFLOP/s",
               metric="MatMulNBits decode GB/s" if wl["kind"] == "decode" else "MatMulNBits prefill TFLOP/s",
               roofline=roofline_of(runner, step_ms, pk, pk_kind, clock), graphs=runner.graphable,
               overlap=runner.overlap, gather_mode=runner.gather_mode, peer=runner.peer, launches=len(wl["proj"]))
    attach_traffic(res["roofline"], name)
    if world == 1:
        res["kernels_us"] = runner.kernel_times()
    if mode == "strong" and world > 1:
        runner.ys_full = {n: torch.empty_like(y) for n, y in runner.ys.items()}
        g1 = not args.no_graphs
        one_ms, _ = runner.timed(runner.step_full, len(runner.full), g1, args.steps, args.warmup)
        res.update(one_gpu_ms=one_ms, speedup=one_ms / step_ms, efficiency=one_ms / step_ms / world)
    if not args.no_e2e and mode == "weak":
        res["e2e"] = runner.e2e(args.steps, args.warmup)
    if cpu and rank == 0 and world == 1 and not args.no_cpu:
        res["cpu_baseline"] = cpu_reference_time(wl, budget_s=args.cpu_seconds, kind_pref="reference")
    runner.close()
    del runner
    torch.cuda.empty_cache()
    return res


def run_ours(args):
    import torch
    from xrgpu_b200 import _native

    world, rank, local = dist_init()
    _native.load()
    device = torch.device("cuda", local)
    head = measure(args.workload, args, world, rank, local, device, mode="weak", headline=True, cpu=True)
    wl = WORKLOADS[args.workload]
    extra = {}
    if args.workload == "llama3_8b_decode" and not args.no_prefill:
        pre = measure("prefill_m2048", args, world, rank, local, device, mode="weak", cpu=True)
        extra["prefill"] = {k: pre[k] for k in ("metric", "unit", "config", "paths", "layers", "roofline", "graphs",
                                                "clocks") if k in pre}
        extra["prefill"].update(value=round(pre["value"], 2), ms_per_step=round(pre["step_ms"], 5),
                                workload="prefill_m2048", M=2048, K=4096, N=14336, block_size=64, zero_points="none",
                                e2e=pre.get("e2e"), cpu_baseline=pre.get("cpu_baseline"),
                                kernels_us=pre.get("kernels_us"), parity=pre.get("parity"))
    if args.workload == "llama3_8b_decode" and world == 1 and not args.no_batched:
        batched = {}
        for name in ("batched_decode_m4", "batched_decode_m16", "batched_decode_m64"):
            r = measure(name, args, world, rank, local, device, mode="weak")
            w = WORKLOADS[name]
            batched[name] = dict(value=round(r["value"], 2), unit=r["unit"], ms_per_step=round(r["step_ms"], 5),
                                 M=w["M"], K=4096, N=14336, block_size=w["bs"], zero_points="packed uint8",
                                 paths=r["paths"], roofline=r["roofline"], kernels_us=r.get("kernels_us"))
        extra["batched_decode"] = batched
    if world > 1 and not args.no_strong:
        strong = {}
        for name in ("llama3_8b_decode", "prefill_m2048"):
            r = measure(name, args, world, rank, local, device, mode="strong")
            strong[name] = dict(unit=r["unit"], value=round(r["value"], 2), ms_per_step=round(r["step_ms"], 5),
                                one_gpu_ms_per_step=round(r["one_gpu_ms"], 5), speedup=round(r["speedup"], 3),
                                parallel_efficiency=round(r["efficiency"], 3), parity=r["parity"],
                                roofline_per_gpu=r["roofline"], graphs=r["graphs"])
        extra["strong"] = strong
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    step_ms = head["step_ms"]
    dt = "fp32" if wl.get("dtype") == "float32" else "fp16 activations x 4-bit weights, fp32 accumulate"
    proj = wl["proj"] if world == 1 else [[n, K, N * world] for (n, K, N) in wl["proj"]]
    line = {
        "metric": head["metric"], "value": round(head["value"], 2), "unit": head["unit"], "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": dt,
        "data": "synthetic (seeded torch RNG; BASELINE.json distributions)",
        "config": {"workload": args.workload, "baseline_config": wl["config"], "M": wl["M"],
                   "projections": [list(p) for p in proj], "bits": 4, "block_size": wl["bs"],
                   "zero_points": "packed uint8" if wl["zp"] else "none",
                   "l2": f"{head['layers']} rotating weight copies (> 3x L2)",
                   "parallelism": f"column-shard x{world}" + (
                       (" + peer-memory all-gather of Y" + (f" ({head['gather_mode']}: exchanges of q/k/v and gate/up "
                                                            "joined before their consumers)" if head["overlap"] else "")
                        if head["peer"] else " + NCCL all-gather of Y") if world > 1 else ""),
                   "cuda_graphs": head["graphs"], "paths": head["paths"]},
        "roofline": head["roofline"], "kernels_us": head.get("kernels_us", {}),
        "gpu_launches": head["launches"] * args.steps * (2 if world > 1 else 1),
        "clocks": head["clocks"], "e2e": head.get("e2e"), "cpu_baseline": head.get("cpu_baseline"),
    }
    if world > 1:
        line["parity"] = head["parity"]
    line.update(extra)
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- CPU / reference arm
def cpu_reference_time(wl, budget_s=15.0, kind_pref="reference", steps=None, warmup=0):
    """Time the reference's algorithm on host cores over a bounded column sample of one step."""
    import numpy as np
    from oracle.native import OracleC, ReferenceC, host_threads

    threads = host_threads()
    try:
        impl, kind = (ReferenceC(), "reference") if kind_pref == "reference" else (OracleC(), "port")
    except FileNotFoundError:
        impl, kind = OracleC(), "port"
    rng = np.random.default_rng(1)
    M = min(wl["M"], 16)
    lo, hi = wl["scale"]
    dt = np.float32 if wl.get("dtype") == "float32" else np.float16
    act = 2 if dt == np.float16 else 4
    probs = []
    for (name, K, N) in wl["proj"]:
        kb = K // wl["bs"]
        cols = min(max(threads * 4, 64), N)
        a = rng.standard_normal((M, K)).astype(dt)
        b = rng.integers(0, 256, (cols, kb, wl["bs"] // 2), dtype=np.uint8)
        s = rng.uniform(lo, hi, (cols, kb)).astype(dt)
        zp = rng.integers(0, 16, (cols, kb)).astype(dt) if wl["zp"] else None  # reference contract: float form
        probs.append((name, K, cols, a, b, s, zp))

    def one():
        for (name, K, cols, a, b, s, zp) in probs:
            impl.matmul(a, b, s, zp, K=K, N=cols, bits=4, block_size=wl["bs"], threads=threads)

    t = time.perf_counter()
    one()
    first = time.perf_counter() - t
    reps = steps if steps else max(1, min(50, int(budget_s / max(first, 1e-4))))
    for _ in range(warmup):
        one()
    t = time.perf_counter()
    for _ in range(reps):
        one()
    dt_s = (time.perf_counter() - t) / reps
    # bytes as read: the reference contract's float zero points ([N, kb] in A's dtype)
    nbytes = sum(proj_bytes(M, K, cols, wl["bs"], wl["zp"], act, zp_bytes=act) for (_, K, cols, *_r) in probs)
    flops = sum(2 * M * K * cols for (_, K, cols, *_r) in probs)
    if wl["kind"] == "decode":
        value, unit = nbytes / dt_s / 1e9, "GB/s"
    else:
        value, unit = flops / dt_s / 1e12, "TFLOP/s"
    sample = (f"{len(probs)} projections x {probs[0][2]} output columns each, M={M}, full K; "
              f"{reps} timed repetitions of {dt_s * 1e3:.1f} ms")
    return dict(value=round(value, 6), unit=unit, cores=threads, kind=kind, sample=sample,
                impl="oracle/_ref (reference packedMatmul compiled as C++)" if kind == "reference" else "oracle/mmnb_oracle.c")


def run_reference(args, wl):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    res = cpu_reference_time(wl, budget_s=args.cpu_seconds, kind_pref="reference", steps=args.steps, warmup=args.warmup)
    line = {"impl": "reference", "metric": "MatMulNBits decode GB/s" if wl["kind"] == "decode" else "MatMulNBits prefill TFLOP/s",
            "value": res["value"], "unit": res["unit"], "n_gpus": int(os.environ.get("WORLD_SIZE", "1")),
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp32 accumulate (reference serial loop)", "data": "synthetic (seeded)",
            "config": {"workload": args.workload, "baseline_config": wl["config"]},
            "cpu_baseline": res, "e2e": {"value": res["value"], "unit": res["unit"], "h2d_bytes_per_step": 0,
                                         "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="llama3_8b_decode")
    ap.add_argument("--layers", type=int, default=0, help="weight copies (default: > 3x L2)")
    ap.add_argument("--seed", type=int, default=2024)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-graphs", action="store_true")
    ap.add_argument("--no-overlap", action="store_true",
                    help="N > 1: run every all-gather right after its own GEMV (same as --gather-mode inline)")
    ap.add_argument("--gather-mode", choices=["defer", "stream", "inline"], default="defer",
                    help="N > 1: order of the peer-memory exchanges within a step (see Runner._build)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-prefill", action="store_true", help="omit the config-4 prefill object")
    ap.add_argument("--no-strong", action="store_true", help="N > 1: omit the fixed-problem (strong) objects")
    ap.add_argument("--no-batched", action="store_true", help="omit the config-3 batched-decode objects (N = 1)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    wl = WORKLOADS[args.workload]
    if args.impl == "reference":
        run_reference(args, wl)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
