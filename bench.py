#!/usr/bin/env python
"""Benchmark: one OrthoCache decode layer (score -> compact -> attend) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (N = 1): configuration 1 of the baseline — GQA decode, batch 1,
32 query heads / 8 KV heads, head_dim 128, bf16, 65,536-token KV cache
(128 blocks of 512), 75 % union eviction, synthetic seeded keys (smooth /
noise block mixture), values N(0,1), queries N(0, 1/sqrt(128)).  τ is
calibrated per layer for the eviction target, ζ_max = 5.

A step is one decode layer: the fused scorer reads all keys, the compaction
emits the retained block list, the split-KV attention reads the retained K
and V blocks.  The KV caches of 4 layers (1.07 GB) rotate across steps, so
every step reads data that left L2 three steps earlier.

N > 1 (torchrun, one rank per GPU, NCCL): sequence-parallel decode with a
65,536-token shard per GPU (weak scaling; configuration 3 at N = 8, with
per-shard eviction drawn from 60-90 %).  Each rank runs the fused decode
layer on its own shard, producing the partial (max, sum, output) per query
head; the partials (32 x 130 floats per rank, one packed buffer) are
all-gathered over NVLink in one call and merged in log-sum-exp form.  No KV
block crosses NVLink.

Prints one JSON line (rank 0).  The value is µs per decode layer for the
whole job (lower is better).
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode attn µs/layer @64K ctx 75% evict (incl. scoring); scorer HBM GB/s vs peak"
UNIT = "us/layer"
S_SHARD, HQ, HKV, D = 65536, 32, 8, 128
ZETA_MAX = 5.0
LAYERS = 4
FALLBACK_HBM = 6650.0
# DRAM bytes read + written by one launch of the fused decode-layer kernel at
# this workload (75 % eviction), from the ncu capture summarised in
# profiles/decode_fused_config1.md.
FUSED_TRAFFIC = 194310144


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=2000)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--evict", type=float, default=0.75)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--config", type=int, choices=[1, 2], default=1,
                   help="1: decode layer (the headline metric); 2: chunked prefill on the tensor cores")
    return p.parse_args()


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            pk = json.load(f)
        return float(pk["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM, "fallback"


class Clocks:
    """Sample SM clocks and throttle reasons with nvidia-smi during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=2)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# workload
# ---------------------------------------------------------------------------
class Layer:
    pass


def make_layers(rank, evict, device, world=1):
    import torch
    from orthocache_b200 import synthetic as syn, score_blocks
    nb = S_SHARD // 512
    layers = []
    import random
    for l in range(LAYERS):
        seed = 1000 * rank + l
        L = Layer()
        # configuration 3: uneven per-shard eviction, uniform in 60-90 %
        L.evict = evict if world == 1 else random.Random(seed).uniform(0.6, 0.9)
        L.kinds = syn.block_kinds(nb, L.evict, seed=seed)
        L.k = syn.make_keys(nb, HKV, D, L.kinds, seed=seed, device=device)
        L.v = syn.make_values(S_SHARD, HKV, D, seed=seed, device=device)
        L.q = syn.make_queries(1, HQ, D, seed=seed, device=device)
        sc = score_blocks(L.k, L.q, want=("zeta", "bound_max"))
        L.tau, L.kept = syn.calibrate_tau(sc["zeta"], sc["bound_max"], ZETA_MAX, L.evict)
        layers.append(L)
    torch.cuda.synchronize()
    return layers


class Engine:
    """Device buffers and the C-ABI calls of one decode layer."""

    def __init__(self, layers, device, world):
        import torch
        from orthocache_b200 import _lib
        self.torch, self.lib, self.layers, self.world = torch, _lib, layers, world
        nb = S_SHARD // 512
        self.nb = nb
        self.keep = torch.empty((nb, HKV), dtype=torch.uint8, device=device)
        self.perm = torch.empty((nb,), dtype=torch.int32, device=device)
        self.count = torch.empty((1,), dtype=torch.int32, device=device)
        self.out = torch.empty((1, HQ, D), dtype=torch.bfloat16, device=device)
        # one workspace for both paths: the decode step's (whose leading
        # counters must start at zero) covers the partial attention's too
        self.ws_bytes = _lib.query("oc_decode_step_workspace_bytes", 1, 1, HQ, HKV, D, S_SHARD)
        self.ws = torch.zeros(self.ws_bytes, dtype=torch.uint8, device=device)
        # sequence-parallel: this shard's (m, l, o) partial packed in one
        # buffer [m (rows) | l (rows) | o (rows, D)], all-gathered in one call
        rows = HQ
        self.rows = rows
        self.send = torch.empty((rows * (D + 2),), dtype=torch.float32, device=device)
        self.m, self.l = self.send[:rows], self.send[rows:2 * rows]
        self.o = self.send[2 * rows:].view(rows, D)
        self.recv = torch.empty((world * rows * (D + 2),), dtype=torch.float32, device=device)
        # our kernels per layer: one (the fused decode layer: score, block
        # decisions, attention, merge); sequence-parallel: the fused layer
        # writing the shard's partial, then the cross-shard merge
        self.launches_per_step = 1 if world == 1 else 2

    @property
    def stream(self):
        return self.torch.cuda.current_stream().cuda_stream

    def score(self, L, q=None):
        _l = self.lib
        q = L.q if q is None else q
        _l.call("oc_score_blocks", _l.ptr(L.k), _l.ptr(q), 1, 1, S_SHARD, HKV, D, 1, HQ,
                1, 64, 64, 256, 256, 512, L.tau, ZETA_MAX,
                None, None, None, None, None, None, None, _l.ptr(self.keep), 0, self.stream)

    def decode(self, L, q=None):
        """One layer through the one-call C ABI (score -> compact -> attend)."""
        _l = self.lib
        q = L.q if q is None else q
        _l.call("oc_decode_step", _l.ptr(q), _l.ptr(L.k), _l.ptr(L.v), 1, 1, 1, HQ, HKV, D, S_SHARD, L.tau, ZETA_MAX,
                _l.ptr(self.keep), _l.ptr(self.perm), _l.ptr(self.count), _l.ptr(self.out), 1,
                _l.ptr(self.ws), self.ws_bytes, self.stream)

    def decode_sharded(self, L, q=None):
        """One layer of sequence-parallel decode: the fused kernel writes this
        shard's partial, one all-gather over NCCL, one merge."""
        import torch.distributed as dist
        _l = self.lib
        q = L.q if q is None else q
        _l.call("oc_decode_step_partial", _l.ptr(q), _l.ptr(L.k), _l.ptr(L.v), 1, 1, 1, HQ, HKV, D, S_SHARD,
                L.tau, ZETA_MAX, _l.ptr(self.keep), _l.ptr(self.perm), _l.ptr(self.count), _l.ptr(self.m),
                _l.ptr(self.l), _l.ptr(self.o), _l.ptr(self.ws), self.ws_bytes, self.stream)
        dist.all_gather_into_tensor(self.recv, self.send)
        _l.call("oc_merge_partials_packed", _l.ptr(self.recv), self.world, self.rows, D, _l.ptr(self.out), 1,
                self.stream)

    def step(self, L, q=None):
        if self.world == 1:
            self.decode(L, q)
        else:
            self.decode_sharded(L, q)


# ---------------------------------------------------------------------------
# CPU port of the reference path (baseline leg and --impl reference)
# ---------------------------------------------------------------------------
def cpu_port_time(L, min_seconds=10.0, max_reps=20):
    """Time the reference's decode layer on the host cores (oracle/oc_port.c,
    OpenMP on all cores) on a full layer; returns (median µs, threads, reps)."""
    import numpy as np
    import torch
    from oracle import port
    bits = lambda t: t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)
    kb, vb, qb = bits(L.k), bits(L.v), bits(L.q)
    port.decode(kb, vb, qb, L.tau, ZETA_MAX)  # warm-up
    ts = []
    t_end = time.perf_counter() + min_seconds
    while len(ts) < 3 or (time.perf_counter() < t_end and len(ts) < max_reps):
        t0 = time.perf_counter()
        port.decode(kb, vb, qb, L.tau, ZETA_MAX)
        ts.append(time.perf_counter() - t0)
    return statistics.median(ts) * 1e6, port.threads(), len(ts)


def run_reference(args, rank, world):
    """--impl reference: the reference's CPU path (the C port, all host threads), rank 0 only."""
    if rank != 0:
        return
    import torch
    from orthocache_b200 import synthetic as syn
    from oracle import oc_oracle as O, port
    import numpy as np
    nb = S_SHARD // 512
    torch.manual_seed(0)
    kinds = syn.block_kinds(nb, args.evict, seed=0)
    L = Layer()
    L.k = syn.make_keys(nb, HKV, D, kinds, seed=0, device="cpu")
    L.v = syn.make_values(S_SHARD, HKV, D, seed=0, device="cpu")
    L.q = syn.make_queries(1, HQ, D, seed=0, device="cpu")
    sc = O.score_blocks(L.q.float().numpy(), L.k.float().numpy(), -1e30, ZETA_MAX)
    L.tau, _ = syn.calibrate_tau(torch.tensor(sc["zeta"]), torch.tensor(sc["bound_max"]), ZETA_MAX, args.evict)
    bits = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)
    kb, vb, qb = bits(L.k), bits(L.v), bits(L.q)
    steps = max(1, min(args.steps, 200))
    for _ in range(max(1, min(args.warmup, 5))):
        port.decode(kb, vb, qb, L.tau, ZETA_MAX)
    t0 = time.perf_counter()
    for _ in range(steps):
        port.decode(kb, vb, qb, L.tau, ZETA_MAX)
    us = (time.perf_counter() - t0) / steps * 1e6
    cores = port.threads()
    line = {
        "impl": "reference", "metric": METRIC, "value": round(us, 2), "unit": UNIT, "n_gpus": world,
        "steps": steps, "warmup": args.warmup, "ms_per_step": round(us / 1e3, 4), "higher_is_better": False,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "config1: GQA decode B=1, Hq=32/Hkv=8, D=128, S=65536, evict=%.2f" % args.evict,
                   "layers": 1, "l2": "host run"},
        "cpu_baseline": {"value": round(us, 2), "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": "full layer (65536 tokens) per step; reference JAX CPU path unavailable "
                                   "(jax not installed), C/OpenMP port of its algorithm timed instead"},
        "e2e": {"value": round(us, 2), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def warmup_steps(step, min_steps, min_seconds, world, sync, device):
    """Run step(i) for i = 0, 1, ... until at least min_steps steps and
    min_seconds of wall time have passed; returns the number of steps.

    With world > 1 every step is a collective, so every rank must run the same
    number of steps whatever its own clock says: rank 0 decides, and its
    decision is broadcast every 64 steps."""
    import torch
    import torch.distributed as dist
    t0 = time.perf_counter()
    flag = torch.zeros((1,), dtype=torch.int32, device=device)
    i = 0
    while True:
        step(i)
        i += 1
        if world == 1:
            if i >= min_steps and time.perf_counter() - t0 >= min_seconds:
                return i
            if i % 64 == 0:
                sync()
        elif i % 64 == 0:
            sync()
            flag.fill_(int(i >= min_steps and time.perf_counter() - t0 >= min_seconds))
            dist.broadcast(flag, 0)
            if int(flag.item()):
                return i


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    layers = make_layers(rank, args.evict, device, world)
    eng = Engine(layers, device, world)
    nb = S_SHARD // 512

    def barrier():
        if world > 1:
            dist.barrier()

    warmup_steps(lambda i: eng.step(layers[i % LAYERS]), args.warmup, 0.5, world, torch.cuda.synchronize,
                 device)
    torch.cuda.synchronize()

    K = args.steps
    # The timed region replays a CUDA graph of LAYERS consecutive layers (the
    # same C-ABI calls captured), so host launch latency is not on the clock
    # and each kernel may start while the one before it drains (programmatic
    # dependent launch).  Multi-GPU steps run eagerly (NCCL in the step).
    graphs = None
    if world == 1:
        cap = torch.cuda.Stream()
        cap.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(cap):
            for L in layers:
                eng.step(L)
        torch.cuda.current_stream().wait_stream(cap)
        torch.cuda.synchronize()
        g_all = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_all):
            for L in layers:
                eng.step(L)
        g_one = []
        for L in layers:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                eng.step(L)
            g_one.append(g)
        graphs = (g_all, g_one)
        for s in range(2):
            g_all.replay()
        torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local_rank) as clk:
        barrier()
        torch.cuda.synchronize()
        start.record()
        if graphs is not None:
            for s in range(K // LAYERS):
                graphs[0].replay()
            for s in range(K % LAYERS):
                graphs[1][s].replay()
        else:
            for s in range(K):
                eng.step(layers[s % LAYERS])
        stop.record()
        torch.cuda.synchronize()
        barrier()
    ms = start.elapsed_time(stop) / K
    # Launch durations: CUDA events bracketing each launch on the launching
    # stream, eager, inputs rotating past L2.  The scorer alone (oc_score_blocks)
    # and the whole layer (oc_decode_step: at N = 1 a single launch of the
    # fused kernel, the roofline kernel).
    # each launch on the launching stream, eager, inputs rotating past L2.
    Kb = max(LAYERS, min(K, 400))
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(Kb)]
    for s in range(Kb):
        evs[s][0].record()
        eng.score(layers[s % LAYERS])
        evs[s][1].record()
    torch.cuda.synchronize()
    t_score = statistics.median(e[0].elapsed_time(e[1]) for e in evs)
    for s in range(Kb):
        evs[s][0].record()
        eng.step(layers[s % LAYERS])
        evs[s][1].record()
    torch.cuda.synchronize()
    t_step_eager = statistics.median(e[0].elapsed_time(e[1]) for e in evs)
    if world > 1:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())

    # ---- end to end through the public API, host buffers ----
    from orthocache_b200 import _lib  # noqa: F401
    q_host = [L.q.cpu().pin_memory() for L in layers]
    q_dev = torch.empty_like(layers[0].q)
    out_host = torch.empty((1, HQ, D), dtype=torch.bfloat16).pin_memory()
    cnt_host = torch.empty((1,), dtype=torch.int32).pin_memory()
    Ke = max(8, min(K, 2000))
    for s in range(4):
        q_dev.copy_(q_host[s % LAYERS], non_blocking=True)
        eng.step(layers[s % LAYERS], q_dev)
        out_host.copy_(eng.out, non_blocking=True)
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for s in range(Ke):
        L = layers[s % LAYERS]
        q_dev.copy_(q_host[s % LAYERS], non_blocking=True)
        eng.step(L, q_dev)
        out_host.copy_(eng.out, non_blocking=True)
        cnt_host.copy_(eng.count, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / Ke
    if world > 1:
        t = torch.tensor([e2e_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    # correctness guard on the last step: retained count matches the calibration
    assert int(cnt_host[0]) == layers[(Ke - 1) % LAYERS].kept, "retained block count changed"

    if rank != 0:
        return
    hbm, peak_kind = peaks()
    k_bytes = S_SHARD * HKV * D * 2
    kept = statistics.mean(L.kept for L in layers)
    alg_bytes = k_bytes + kept / nb * 2 * k_bytes + HQ * D * 2 * 2
    score_gbs = k_bytes / (t_score * 1e-3) / 1e9
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        us_cpu, cores, reps = cpu_port_time(layers[0])
        cpu = {"value": round(us_cpu, 2), "unit": UNIT, "cores": cores, "kind": "port",
               "sample": f"one full layer of this workload (layer 0), median of {reps} runs; C/OpenMP port of "
                         "the reference's compute_multiband_mask + compaction + online-softmax loop"}
    line = {
        "metric": METRIC, "value": round(ms * 1e3, 3), "unit": UNIT, "n_gpus": world, "steps": K,
        "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": ("config1: GQA decode B=1, Hq=32/Hkv=8, D=128, bf16, %d tokens, evict=%.2f, "
                                "zeta_max=5" % (S_SHARD, args.evict)) if world == 1 else
                               ("config3: sequence-parallel GQA decode B=1, Hq=32/Hkv=8, D=128, bf16, %d tokens per "
                                "GPU (%d total), per-shard eviction U[0.6, 0.9], zeta_max=5" % (S_SHARD, S_SHARD * world)),
                   "l2": "inputs > L2: 4 layers of KV (1.07 GB) rotate per step",
                   "parallelism": "single GPU" if world == 1 else f"sequence-parallel x{world}, LSE merge"},
        "roofline": ({"bound": "hbm", "kernel": "score_tma_kernel<128,true> (fused decode layer)",
                      "achieved": round(alg_bytes / (ms * 1e-3) / 1e9, 1), "peak": hbm, "unit": "GB/s",
                      "frac": round(alg_bytes / (ms * 1e-3) / 1e9 / hbm, 4),
                      "traffic": FUSED_TRAFFIC if abs(args.evict - 0.75) < 1e-9 else None,
                      "peak_kind": peak_kind, "bytes_per_launch": int(alg_bytes),
                      "eager_launch_us": round(t_step_eager * 1e3, 2),
                      "eager_frac": round(alg_bytes / (t_step_eager * 1e-3) / 1e9 / hbm, 4),
                      "how": "algorithmic bytes |K| + kept/nb (|K|+|V|) per launch over the average launch "
                             "duration in the timed region (CUDA events around K graph-replayed launches, one "
                             "kernel per layer); eager_*: one launch alone, bracketed by CUDA events; traffic = "
                             "dram bytes read+written per launch from the ncu capture in profiles/"}
                     if world == 1 else
                     {"bound": "hbm", "kernel": "score_tma_kernel<128,false> (scorer)",
                      "achieved": round(score_gbs, 1), "peak": hbm, "unit": "GB/s",
                      "frac": round(score_gbs / hbm, 4), "traffic": None, "peak_kind": peak_kind,
                      "bytes_per_launch": k_bytes}),
        "scorer_roofline": {"kernel": "score_tma_kernel<128,false> (oc_score_blocks alone)",
                            "achieved": round(score_gbs, 1), "frac": round(score_gbs / hbm, 4),
                            "bytes_per_launch": k_bytes},
        "step_roofline": {"alg_bytes": int(alg_bytes), "achieved_gbs": round(alg_bytes / (ms * 1e-3) / 1e9, 1),
                          "frac": round(alg_bytes / (ms * 1e-3) / 1e9 / hbm, 4)},
        "kernel_us": {"score": round(t_score * 1e3, 2), "step_eager": round(t_step_eager * 1e3, 2),
                      "how": "median of eager launches bracketed by CUDA events"},
        "timed_region": ("CUDA-graph replay of %d consecutive layers" % LAYERS) if world == 1 else "eager launches",
        "cpu_baseline": cpu,
        "e2e": {"value": round(e2e_ms * 1e3, 3), "unit": UNIT, "h2d_bytes_per_step": HQ * D * 2,
                "d2h_bytes_per_step": HQ * D * 2 + 4,
                "note": "public C-ABI calls per step; q copied from pinned host, output + count read back; "
                        "KV cache resident in HBM as in decode"},
        "gpu_launches": K * eng.launches_per_step,
        "clocks": clk.summary(),
        "retained_blocks": kept,
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# configuration 2: chunked prefill (tensor-bound attention)
# ---------------------------------------------------------------------------
P_B, P_SQ, P_S = 4, 2048, 32768
P_LAYERS = 2


def run_prefill(args, rank, world, local_rank):
    """Configuration 2: batch 4, 2048-query chunks against a 32,768-token
    cache, 32/8 heads, D 128, bf16, keys of the 30/40/30 smooth / mid-band /
    noise mixture, 75 % union eviction per batch row.  A step is one layer:
    the fused scorer over all keys (bounds of all 8192 query rows of each KV
    head), the compaction, and the tensor-core attention (oc_prefill_attention)
    over the retained blocks.  With N > 1 every rank runs its own batch
    (replicas: the chunked prefill does not shard across GPUs here)."""
    import torch
    import torch.distributed as dist
    from orthocache_b200 import synthetic as syn, score_blocks, _lib
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    nb = P_S // 512
    layers = []
    for li in range(P_LAYERS):
        L = Layer()
        ks, vs, qs, taus, kept = [], [], [], [], []
        for b in range(P_B):
            seed = 10000 * rank + 100 * li + b
            kinds = syn.block_kinds(nb, 0.3, 0.4, seed=seed)
            ks.append(syn.make_keys(nb, HKV, D, kinds, seed=seed, device=device))
            vs.append(syn.make_values(P_S, HKV, D, seed=seed, device=device))
            qs.append(syn.make_queries(P_SQ, HQ, D, seed=seed, device=device))
        L.k, L.v, L.q = torch.stack(ks), torch.stack(vs), torch.stack(qs)
        del ks, vs, qs
        sc = score_blocks(L.k, L.q, want=("zeta", "bound_max"))
        for b in range(P_B):
            t, kp = syn.calibrate_tau(sc["zeta"][b], sc["bound_max"][b], ZETA_MAX, args.evict)
            taus.append(t)
            kept.append(kp)
        # τ is calibrated per batch row (the reference has no batch
        # dimension) and the scorer takes one τ per call: one call per row
        L.taus, L.kept = taus, kept
        layers.append(L)
    torch.cuda.synchronize()
    keep = torch.empty((P_B, nb, HKV), dtype=torch.uint8, device=device)
    perm = torch.empty((P_B, nb), dtype=torch.int32, device=device)
    count = torch.empty((P_B,), dtype=torch.int32, device=device)
    out = torch.empty((P_B, P_SQ, HQ, D), dtype=torch.bfloat16, device=device)
    st = lambda: torch.cuda.current_stream().cuda_stream
    rows_b = P_SQ * HQ * D * 2
    kv_b = P_S * HKV * D * 2

    f32 = dict(dtype=torch.float32, device=device)
    dc = torch.empty((P_B, nb, HKV, D), **f32)
    e_ac, zeta, bmax = (torch.empty((P_B, nb, HKV), **f32) for _ in range(3))
    cells = nb * HKV

    def score(L):
        # one pass over all keys for the query-independent block metadata
        # (DC, E_AC, zeta), the bounds of all 8192 query rows per KV head as a
        # tiled GEMM, then the two gates with each batch row's own τ (the
        # reference has no batch dimension; the synthetic rows are calibrated
        # one by one)
        _lib.call("oc_block_metadata", L.k.data_ptr(), 1, P_B, P_S, HKV, D, dc.data_ptr(), e_ac.data_ptr(),
                  zeta.data_ptr(), st())
        _lib.call("oc_score_from_metadata", dc.data_ptr(), e_ac.data_ptr(), zeta.data_ptr(), L.q.data_ptr(), 1, P_B,
                  nb, HKV, D, P_SQ, HQ, -math.inf, ZETA_MAX, bmax.data_ptr(), None, None, st())
        for b in range(P_B):
            _lib.call("oc_apply_gates", bmax.data_ptr() + 4 * b * cells, zeta.data_ptr() + 4 * b * cells, cells,
                      None, L.taus[b], ZETA_MAX, keep.data_ptr() + b * cells, st())

    def compact():
        _lib.call("oc_stream_compact", keep.data_ptr(), P_B, nb, HKV, perm.data_ptr(), count.data_ptr(), st())

    def attend(L, q=None):
        q = L.q if q is None else q
        _lib.call("oc_prefill_attention", q.data_ptr(), L.k.data_ptr(), L.v.data_ptr(), 1, perm.data_ptr(), nb, 0,
                  count.data_ptr(), 1, 0, P_B, P_SQ, HQ, HKV, D, P_S, 512, nb, out.data_ptr(), 1, st())

    def step(L, q=None):
        score(L)
        compact()
        attend(L, q)

    for i in range(max(args.warmup, 3)):
        step(layers[i % P_LAYERS])
    torch.cuda.synchronize()
    assert [int(c) for c in count.cpu()] == layers[(max(args.warmup, 3) - 1) % P_LAYERS].kept
    K = max(4, min(args.steps, 200))
    ev = lambda: torch.cuda.Event(enable_timing=True)

    def timed(fn, n):
        a, b = ev(), ev()
        torch.cuda.synchronize()
        a.record()
        for i in range(n):
            fn(i)
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / n

    with Clocks(local_rank) as clk:
        if world > 1:
            dist.barrier()
        ms = timed(lambda i: step(layers[i % P_LAYERS]), K)
        if world > 1:
            dist.barrier()
    # per-kernel launch durations (CUDA events on the launching stream); the
    # retained lists of the last step stay in perm / count for the attention
    ms_score = timed(lambda i: score(layers[i % P_LAYERS]), K)
    step(layers[0])
    ms_attn = timed(lambda i: attend(layers[0]), K)
    if world > 1:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    # end to end: the chunk's queries from pinned host memory, the output back
    q_host = [L.q.cpu().pin_memory() for L in layers]
    out_host = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    q_dev = torch.empty_like(layers[0].q)
    Ke = max(4, min(K, 50))

    def e2e_step(i):
        q_dev.copy_(q_host[i % P_LAYERS], non_blocking=True)
        L = layers[i % P_LAYERS]
        score(L)
        compact()
        attend(L, q_dev)
        out_host.copy_(out, non_blocking=True)

    e2e_step(0)
    e2e_ms = timed(e2e_step, Ke)
    if rank != 0:
        return
    kept = statistics.mean(statistics.mean(L.kept) for L in layers)
    flops = 4.0 * P_B * HQ * P_SQ * (kept * 512) * D
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            pk = json.load(f)
        tf_peak, tf_kind = float(pk["bf16_tflops"]), "measured (burst: the kernel is timed on its own)"
    except Exception:
        tf_peak, tf_kind = 1590.0, "fallback"
    hbm, _ = peaks()
    attn_tf = flops / (ms_attn * 1e-3) / 1e12
    score_bytes = P_B * kv_b + P_B * rows_b
    line = {
        "metric": "chunked-prefill layer ms @32K ctx 75% evict (incl. scoring); attention TFLOP/s vs peak",
        "value": round(ms, 4), "unit": "ms/layer", "n_gpus": world, "steps": K, "warmup": args.warmup,
        "ms_per_step": round(ms, 4), "higher_is_better": False, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "config2: chunked prefill B=4, Sq=2048, Hq=32/Hkv=8, D=128, bf16, 32768 tokens, "
                               "30/40/30 smooth/mid/noise keys, evict=%.2f per batch row, zeta_max=5" % args.evict,
                   "l2": "inputs > L2: 2 layers of KV (2 x 537 MB) alternate per step",
                   "parallelism": "single GPU" if world == 1 else f"{world} independent replicas"},
        "roofline": {"bound": "tensor", "kernel": "prefill_attn_kernel (tcgen05, TMEM accumulators)",
                     "achieved": round(attn_tf, 1), "peak": tf_peak, "unit": "TFLOP/s",
                     "frac": round(attn_tf / tf_peak, 4), "traffic": None, "peak_kind": tf_kind,
                     "flops_per_launch": flops, "launch_ms": round(ms_attn, 4),
                     "how": "4*B*Hq*Sq*(retained tokens)*D FLOPs over the median-free average launch time of K "
                            "back-to-back launches bracketed by CUDA events"},
        "scorer": {"launch_ms": round(ms_score, 4), "bytes": score_bytes,
                   "achieved_gbs": round(score_bytes / (ms_score * 1e-3) / 1e9, 1),
                   "frac": round(score_bytes / (ms_score * 1e-3) / 1e9 / hbm, 4),
                   "note": "oc_block_metadata over all keys + bound GEMM (oc_score_from_metadata) + per-row gates; "
                           "bytes = keys + queries"},
        "cpu_baseline": None,
        "e2e": {"value": round(e2e_ms, 4), "unit": "ms/layer", "h2d_bytes_per_step": P_B * rows_b,
                "d2h_bytes_per_step": P_B * rows_b,
                "note": "queries of the chunk from pinned host memory, attention output back; KV cache resident"},
        "gpu_launches": K * (1 + 3 + P_B + 1 + 1),
        "clocks": clk.summary(),
        "retained_blocks": kept,
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    import torch
    import torch.distributed as dist
    if world > 1:
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
    try:
        if args.config == 2:
            run_prefill(args, rank, world, local_rank)
        else:
            run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
