#!/usr/bin/env python
"""MatMulNBits benchmark on B200: decode GB/s (and prefill TFLOP/s) through this repo's C ABI.

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

Multi-GPU (torchrun, one process per GPU, NCCL): every rank owns a contiguous 1/N slice of each
projection's output columns (weak scaling: the model is N times wider, per-GPU work fixed) and the
step ends with one all-gather of Y per projection: the library's peer-memory all-gather over NVLink
for decode shards (the whole step is then one CUDA graph), NCCL for large prefill shards. Time is
the max over ranks.

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
import threading
import time
import zlib
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PEAKS_FILE = ROOT / "MEASURED_PEAKS.json"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

LLAMA_LAYER = [("q", 4096, 4096), ("k", 4096, 1024), ("v", 4096, 1024), ("o", 4096, 4096),
               ("gate", 4096, 14336), ("up", 4096, 14336), ("down", 14336, 4096)]

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


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def peaks():
    if PEAKS_FILE.exists():
        d = json.loads(PEAKS_FILE.read_text())
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def proj_bytes(M, K, N, bs, zp, act_bytes):
    kb = K // bs
    b = N * K // 2 + N * kb * act_bytes + (N * ((kb + 1) // 2) if zp else 0) + M * K * act_bytes + M * N * act_bytes
    return b


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
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        out.update(sm_mhz=statistics.median(sm) if sm else None, sm_max_mhz=max(mx) if mx else None,
                   reasons=reasons, samples=len(rows),
                   power_w_max=max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit()) if rows else None)
        return out


# ----------------------------------------------------------------------------- distributed
def dist_init(n_gpus):
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
    if world > 1:
        import torch
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


# ----------------------------------------------------------------------------- data
def make_weights(wl, world, rank, layers, seed, device):
    """Per layer and projection: this rank's column shard of B, scales, zero points."""
    import torch
    g = torch.Generator(device=device)
    out = []
    lo, hi = wl["scale"]
    for layer in range(layers):
        projs = []
        for (name, K, N) in wl["proj"]:
            n_local = N  # weak scaling: each rank owns N columns of an N*world-wide projection
            g.manual_seed(seed * 1000003 + layer * 1009 + zlib.crc32(name.encode()) % 997 + 7919 * rank)
            kb = K // wl["bs"]
            b = torch.randint(0, 256, (n_local, kb, wl["bs"] // 2), dtype=torch.uint8, device=device, generator=g)
            s = (torch.rand((n_local, kb), device=device, generator=g) * (hi - lo) + lo).to(torch.float16)
            zp = (torch.randint(0, 256, (n_local, (kb + 1) // 2), dtype=torch.uint8, device=device, generator=g)
                  if wl["zp"] else None)
            projs.append(dict(name=name, K=K, N=n_local, b=b, s=s, zp=zp))
        out.append(projs)
    return out


def layers_for_l2(wl, l2_bytes):
    per_layer = sum(proj_bytes(wl["M"], K, N, wl["bs"], wl["zp"], 2) for (_, K, N) in wl["proj"])
    return max(2, math.ceil(3 * l2_bytes / per_layer) + 1), per_layer


# ----------------------------------------------------------------------------- our arm
def run_ours(args, wl):
    import torch
    from xrgpu_b200 import functional as F
    from xrgpu_b200 import _native

    world, rank, local = dist_init(args.gpus)
    lib = _native.load()
    device = torch.device("cuda", local)
    props = torch.cuda.get_device_properties(device)
    l2 = getattr(props, "L2_cache_size", 126 * 2**20) or 126 * 2**20
    layers, per_layer = layers_for_l2(wl, l2)
    if args.layers:
        layers = args.layers
    M = wl["M"]
    dt = torch.float32 if wl.get("dtype") == "float32" else torch.float16
    act_bytes = 4 if dt == torch.float32 else 2
    weights = make_weights(wl, world, rank, layers, args.seed, device)
    if dt == torch.float32:
        for layer in weights:
            for p in layer:
                p["s"] = p["s"].float()
    g = torch.Generator(device=device)
    g.manual_seed(args.seed)
    acts = {K: torch.randn((M, K), generator=g, device=device, dtype=torch.float32).to(dt)
            for K in sorted({K for (_, K, _) in wl["proj"]})}
    ys = {(name, N): torch.empty((M, N), device=device, dtype=dt) for (name, K, N) in wl["proj"]}
    gathered = {(name, N): torch.empty((M, N * world), device=device, dtype=dt) for (name, K, N) in wl["proj"]}
    launches_per_step = len(wl["proj"])
    paths = sorted({F.select_path(acts[p["K"]], p["b"], p["s"], p["zp"], K=p["K"], N=p["N"], block_size=wl["bs"])
                    for p in weights[0]})

    shared = None
    if world > 1:
        # Each rank's shard is one column slice of an (N * world)-wide projection, used through the
        # library's sharded module: local kernel + one all-gather of Y per projection (peer memory
        # for small shards, NCCL otherwise).
        from xrgpu_b200.sharded import ShardedMatMulNBits
        from xrgpu_b200.p2p import PeerAllGather
        for layer in weights:
            for p in layer:
                p["mod"] = ShardedMatMulNBits.from_shard(p["b"], p["s"], p["zp"], None, K=p["K"], N=p["N"] * world,
                                                         block_size=wl["bs"])
        if all(p["mod"].uses_peer_gather(M) for layer in weights for p in layer):
            # one peer-memory group shared by every projection (calls are stream-ordered)
            shared = PeerAllGather(max(M * p["N"] * 2 for p in weights[0]))
            for layer in weights:
                for p in layer:
                    p["mod"].set_peer_group(shared)

    # With N > 1 ranks and peer-memory all-gathers, a projection's all-gather may overlap the GEMVs
    # that do not depend on its Y: in a decoder layer q, k, v share their input, o needs attention
    # over all three, gate and up share their input and down needs both. Each group's gathers are
    # joined before the next group starts, so the gathers of v, o, up and down stay exposed.
    order = [p["name"] for p in weights[0]]
    layer_groups = [["q", "k", "v"], ["o"], ["gate", "up"], ["down"]]
    if sorted(order) != sorted(n for grp in layer_groups for n in grp):
        layer_groups = [[n] for n in order]  # other workloads: each projection depends on the last
    overlap = world > 1 and shared is not None and not args.no_overlap
    comm = torch.cuda.Stream(device) if overlap else None

    def step(layer, gather=True):
        by_name = {p["name"]: p for p in weights[layer]}
        if world > 1 and gather and overlap:
            for grp in layer_groups:
                for name in grp:
                    p = by_name[name]
                    p["mod"](acts[p["K"]], out=gathered[(p["name"], p["N"])], gather_stream=comm)
                for name in grp:
                    by_name[name]["mod"].wait_gather()
            return
        for p in weights[layer]:
            if world > 1 and gather:
                p["mod"](acts[p["K"]], out=gathered[(p["name"], p["N"])])
            else:
                y = ys[(p["name"], p["N"])]
                F.matmul_nbits(acts[p["K"]], p["b"], p["s"], p["zp"], K=p["K"], N=p["N"], block_size=wl["bs"], out=y)

    # Warm-up outside capture (allocates the library workspace, sets kernel attributes).
    for layer in range(layers):
        step(layer)
    torch.cuda.synchronize()
    # Each layer's step is one CUDA graph when it contains no NCCL call: always on one GPU, and with
    # N > 1 ranks when every projection's all-gather goes through peer memory. Steps that hold NCCL
    # all-gathers run eagerly.
    peer = world > 1 and all(p["mod"].uses_peer_gather(M) for layer in weights for p in layer)
    use_graphs = (world == 1 or peer) and not args.no_graphs
    graphs = []
    if use_graphs:
        stream = torch.cuda.Stream(device)
        with torch.cuda.stream(stream):
            for layer in range(layers):
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gr, stream=stream):
                    step(layer)
                graphs.append(gr)
        torch.cuda.synchronize()

    def run_steps(n, offset=0):
        for i in range(n):
            layer = (offset + i) % layers
            if use_graphs:
                graphs[layer].replay()
            else:
                step(layer)

    log(f"[rank {rank}] graphs captured: {len(graphs)}")
    run_steps(max(3, args.warmup))
    log(f"[rank {rank}] warm-up done")
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    barrier(world)
    clocks.start()
    time.sleep(0.25)
    torch.cuda.synchronize()
    barrier(world)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    run_steps(args.steps)
    t1.record()
    torch.cuda.synchronize()
    barrier(world)
    ms_local = t0.elapsed_time(t1)
    # The max over ranks is taken before anything depends on it: every rank must then run the
    # same number of extra steps (each holds collectives).
    ms = max_over_ranks(world, ms_local)
    # Keep the clock sampler running for at least a few samples.
    if ms < 600:
        reps = max(1, int(600 / max(ms, 1e-3)))
        for _ in range(reps):
            run_steps(args.steps)
        torch.cuda.synchronize()
    clock = clocks.stop()
    step_ms = ms / args.steps
    bytes_rank = per_layer if wl["kind"] == "decode" else None
    flops_rank = sum(2 * M * K * N for (_, K, N) in wl["proj"])
    pk, pk_kind = peaks()
    result = {}
    if wl["kind"] == "decode":
        value = bytes_rank * world / (step_ms * 1e-3) / 1e9
        metric, unit = "MatMulNBits decode GB/s", "GB/s"
    else:
        value = flops_rank * world / (step_ms * 1e-3) / 1e12
        metric, unit = "MatMulNBits prefill TFLOP/s", "TFLOP/s"

    # Each projection's kernel alone: a CUDA graph of back-to-back launches over the rotating
    # weight copies (no host launch overhead between them).
    kernel = {}
    # Per-projection kernel times: one GPU only (no collectives inside; with several ranks one
    # rank capturing graphs while the others sit in collectives would only add waiting).
    if world == 1:
        for (name, K, N) in wl["proj"]:
            reps = 4 * layers
            gs = torch.cuda.Stream(device)
            gk = torch.cuda.CUDAGraph()
            with torch.cuda.stream(gs):
                with torch.cuda.graph(gk, stream=gs):
                    for r in range(reps):
                        p = [q for q in weights[r % layers] if q["name"] == name][0]
                        F.matmul_nbits(acts[K], p["b"], p["s"], p["zp"], K=K, N=N, block_size=wl["bs"],
                                       out=ys[(name, N)])
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
            kb = proj_bytes(M, K, N, wl["bs"], wl["zp"], act_bytes)
            kernel[name] = dict(K=K, N=N, us=round(per * 1e3, 3), gbs=round(kb / (per * 1e-3) / 1e9, 1),
                                tflops=round(2 * M * K * N / (per * 1e-3) / 1e12, 3))
            del gk
    if wl["kind"] == "decode":
        achieved = bytes_rank / (step_ms * 1e-3) / 1e9
        peak = pk["hbm_gbs"]
        roofline = dict(bound="hbm", achieved=round(achieved, 1), peak=peak, unit="GB/s", frac=round(achieved / peak, 4),
                        traffic=None, peak_source=f"{pk_kind} hbm_gbs",
                        note="achieved = algorithmic bytes per step / device time per step (CUDA graph of the step's "
                             "launches, rotating weight copies); per-projection kernel times in kernels_us")
    else:
        achieved = flops_rank / (step_ms * 1e-3) / 1e12
        peak = pk.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])
        roofline = dict(bound="tensor", achieved=round(achieved, 1), peak=peak, unit="TFLOP/s",
                        frac=round(achieved / peak, 4), traffic=None, peak_source=f"{pk_kind} bf16_tflops (burst)")
    traffic_file = ROOT / "profiles" / "traffic.json"
    if traffic_file.exists():
        tr = json.loads(traffic_file.read_text()).get(args.workload)
        if tr:
            roofline["traffic"] = tr.get("bytes_per_step")
            roofline["traffic_source"] = tr.get("source")

    log(f"[rank {rank}] timed region done")
    # End to end through the public C-ABI call: pinned host A -> device, the step's C-ABI calls,
    # device -> pinned host Y, synchronise; every step.
    e2e = None
    if not args.no_e2e:
        host_a = {K: acts[K].cpu().pin_memory() for K in acts}
        host_y = {key: torch.empty_like(v, device="cpu").pin_memory() for key, v in
                  (gathered.items() if world > 1 else ys.items())}
        h2d = sum(v.numel() * v.element_size() for v in host_a.values())
        d2h = sum(v.numel() * v.element_size() for v in host_y.values())

        def e2e_step(i):
            for K, h in host_a.items():
                acts[K].copy_(h, non_blocking=True)
            step(i % layers)
            src = gathered if world > 1 else ys
            for key, h in host_y.items():
                h.copy_(src[key], non_blocking=True)
            torch.cuda.synchronize()

        for i in range(max(3, args.warmup)):
            e2e_step(i)
        barrier(world)
        w0 = time.perf_counter()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(args.steps):
            e2e_step(i)
        e1.record()
        torch.cuda.synchronize()
        wall = time.perf_counter() - w0
        e_ms = max_over_ranks(world, max(e0.elapsed_time(e1), wall * 1e3) / args.steps)
        e_val = (bytes_rank * world / (e_ms * 1e-3) / 1e9) if wl["kind"] == "decode" else (flops_rank * world / (e_ms * 1e-3) / 1e12)
        e2e = dict(value=round(e_val, 2), unit=unit, h2d_bytes_per_step=h2d, d2h_bytes_per_step=d2h, ms_per_step=round(e_ms, 4),
                   path=("ShardedMatMulNBits -> " if world > 1 else "") +
                   "functional.matmul_nbits -> xrgpu_mmnb_forward (C ABI), one sync per step")

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_reference_time(wl, budget_s=args.cpu_seconds, kind_pref="reference")

    if world > 1:
        import torch.distributed as dist
        graphs.clear()  # graphs are released before the process group goes
        torch.cuda.synchronize()
        for layer in weights:
            for p in layer:
                p["mod"].close()
        if shared is not None:
            shared.close()  # collective: every rank closes it at the same point
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": metric, "value": round(value, 2), "unit": unit, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(step_ms, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp16 activations x 4-bit weights, fp32 accumulate" if dt == torch.float16 else "fp32",
        "data": "synthetic (seeded torch RNG; BASELINE.json distributions)",
        "config": {"workload": args.workload, "baseline_config": wl["config"], "M": M,
                   "projections": [[n, K, N] for (n, K, N) in wl["proj"]], "bits": 4, "block_size": wl["bs"],
                   "zero_points": "packed uint8" if wl["zp"] else "none", "l2": f"{layers} rotating weight copies "
                   f"({layers * per_layer / 1e6:.0f} MB > 3x L2)", "parallelism": f"column-shard x{world}" +
                   ((" + peer-memory all-gather of Y" + (" overlapped within q/k/v and gate/up" if overlap and any(len(g) > 1 for g in layer_groups) else "")
                    if peer else " + NCCL all-gather of Y") if world > 1 else ""),
                   "cuda_graphs": use_graphs, "paths": paths},
        "roofline": roofline, "kernels_us": kernel, "gpu_launches": launches_per_step * args.steps,
        "clocks": clock, "e2e": e2e, "cpu_baseline": cpu,
    }
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
    probs = []
    for (name, K, N) in wl["proj"]:
        kb = K // wl["bs"]
        cols = max(threads * 4, 64)
        cols = min(cols, N)
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
    nbytes = sum(proj_bytes(M, K, cols, wl["bs"], wl["zp"], 2 if dt == np.float16 else 4) for (_, K, cols, *_r) in probs)
    flops = sum(2 * M * K * cols for (_, K, cols, *_r) in probs)
    if wl["kind"] == "decode":
        value, unit = nbytes / dt_s / 1e9, "GB/s"
    else:
        value, unit = flops / dt_s / 1e12, "TFLOP/s"
    sample = (f"{len(probs)} projections x {probs[0][2]} output columns each, M={M}, full K; "
              f"{reps} timed repetitions of {dt_s * 1e3:.1f} ms")
    return dict(value=round(value, 4), unit=unit, cores=threads, kind=kind, sample=sample,
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
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-graphs", action="store_true")
    ap.add_argument("--no-overlap", action="store_true",
                    help="N > 1: run every all-gather on the compute stream (no overlap with independent GEMVs)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    wl = WORKLOADS[args.workload]
    if args.impl == "reference":
        run_reference(args, wl)
    else:
        run_ours(args, wl)


if __name__ == "__main__":
    main()
