#!/usr/bin/env python3
"""Benchmark of the B200 GQA attention hot path.

Workload (benchmark config 4, long-context decode): batch 1, a 65,536-token
FP16 KV cache ~N(0, 0.5) per layer, 16 query / 4 KV heads, head_dim 128,
36 layers. One step = one generated token through all 36 layers: per layer
RoPE of the new token (NoPE on every 4th layer) + KV-cache append at
position 65,536 + step, split-KV flash-decode over kv_len = position + 1
(KV_CHUNK 256) and the partial merge.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

value : whole-job KV-read throughput in GB/s with the inputs resident in HBM;
        one captured CUDA graph per step (device-resident positions), CUDA
        events on the launching stream, max over ranks.
e2e   : the same metric through the reference-facing C-ABI calls
        (launch_rope_and_store_kv + launch_causal_attention_decode_vectorized
        per layer) with the step's Q/K/V rows copied from pinned host memory
        and the attention outputs copied back every step.
Algorithmic bytes per layer-step: K+V read 2*kv_len*512*2 + Q 4 KiB +
output 4 KiB + appended K/V row 2 KiB (partial-workspace traffic excluded).

--impl reference times the reference algorithm's CPU implementation (the
C oracle restating it, all host threads) on a bounded sample of the same
workload (one layer-step at the same kv_len per step) and prints the same line.

N > 1 (torchrun): the 64K KV range of every layer is split into N contiguous
ranges, one per rank; the rank holding the tail appends the new token; each
rank reduces its range to one (o, m, l) partial per head, the partials are
all-gathered over NCCL and merged on every rank (strong scaling: total work
fixed).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "llm-inference_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

H, KVH, D, LAYERS, PAST = 16, 4, 128, 36, 65536
KV_DIM = KVH * D
Q_DIM = H * D
QKV = Q_DIM + 2 * KV_DIM
SEED = 2024
METRIC = "GQA attn: decode KV-read HBM GB/s, prefill TFLOP/s, % B200 roofline @1-8 GPU"
WORKLOAD = ("config4: long-context decode, batch 1, KV 65536 tokens ~N(0,0.5) FP16, 16/4 heads, head_dim 128, "
            "36 layers x 1 token per step (RoPE+append+split-KV decode+merge), KV_CHUNK 256")


# benchmark config 3 (prefill): 4 sequences x 8192 tokens, 36 layers, NoPE every 4th layer
PF_B, PF_S = 4, 8192
PF_WORKLOAD = ("config3: causal GQA prefill, batch 4 x 8192 tokens, 16/4 heads, head_dim 128, N(0,1) FP16, "
               "36 layers x (RoPE theta 5e6 / NoPE every 4th layer + KV append + causal attention)")


# benchmark config 5 (ragged decode): 64 sequences, per-sequence caches of 16384 rows
RG_B, RG_MAX = 64, 16384
RG_WORKLOAD = ("config5: ragged decode, 64 sequences, KV lengths numpy default_rng(2024).integers(512, 16385, 64) "
               "(length after the new token's append), per-sequence cache of 16384 rows, N(0,1) FP16, 16/4 heads, "
               "head_dim 128, 36 layers x 1 new token per sequence per step (RoPE / NoPE + append + ragged "
               "split-KV decode + merge)")


def prefill_flops(batch: int, seq: int, heads: int = 16) -> int:
    """Causal exact count for QK^T + PV: 2 * B * H * d * S * (S + 1)."""
    return 2 * batch * heads * D * seq * (seq + 1)


def layer_bytes(kv_len: int) -> int:
    return 2 * kv_len * KV_DIM * 2 + Q_DIM * 2 + Q_DIM * 2 + 2 * KV_DIM * 2


def step_bytes(kv_len: int) -> int:
    return LAYERS * layer_bytes(kv_len)


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """NVML sampling of SM clock and throttle reasons during the timed region."""

    REASONS = {
        "hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
        "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, device_index: int, interval: float = 0.01):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self.interval = interval
        self._stop = threading.Event()
        self.ok = False
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            self.nv = pynvml
            p = torch.cuda.get_device_properties(device_index)
            try:  # NVML numbers all GPUs; match the CUDA device by PCI address
                bus = f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0"
                self.h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:
                self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.reason_fn = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                getattr(pynvml, "nvmlDeviceGetCurrentClocksThrottleReasons")
            self.ok = True
        except Exception as e:  # NVML absent: report no clocks rather than fail the bench
            self.err = str(e)

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                r = self.reason_fn(self.h)
                for name, bit in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.interval)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *exc):
        if self.ok:
            self._stop.set()
            self.t.join()
        return False

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": len(self.samples)}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# --------------------------------------------------------------------------- CPU baseline
def cpu_decode_sample(kv_len: int, threads: int, rng_seed: int = 7, budget_s: float = 12.0, min_reps: int = 2):
    """Oracle RoPE+append + decode attention for one layer-step at kv_len, repeated
    until budget_s; returns (GB/s, reps, seconds)."""
    import numpy as np
    import oracle
    rng = np.random.default_rng(rng_seed)
    k = (rng.standard_normal((kv_len, KV_DIM), dtype=np.float32) * 0.5).astype(np.float16)
    v = (rng.standard_normal((kv_len, KV_DIM), dtype=np.float32) * 0.5).astype(np.float16)
    qkv = rng.standard_normal(QKV, dtype=np.float32).astype(np.float16)
    cos, sin = oracle.rope_tables(kv_len, D, 5.0e6)
    reps, t0 = 0, time.perf_counter()
    while True:
        q = qkv[:Q_DIM].copy()
        kn = qkv[Q_DIM:Q_DIM + KV_DIM].copy()
        vn = qkv[Q_DIM + KV_DIM:].copy()
        oracle.rope_and_store_kv(q, kn, vn, k, v, cos, sin, 1, H, KVH, D, Q_DIM, KV_DIM, kv_len - 1, True)
        oracle.decode_attention(q, k, v, kv_len, H, KVH, D, threads=threads)
        reps += 1
        el = time.perf_counter() - t0
        if reps >= min_reps and el >= budget_s:
            break
    return layer_bytes(kv_len) * reps / el / 1e9, reps, el


def run_reference(args, rank, world):
    """--impl reference: the reference algorithm's CPU implementation (C oracle)."""
    if rank != 0:
        return
    import numpy as np
    import oracle
    threads = os.cpu_count() or 1
    kv_len = PAST + 1
    rng = np.random.default_rng(7)
    k = (rng.standard_normal((kv_len + args.warmup + args.steps, KV_DIM), dtype=np.float32) * 0.5).astype(np.float16)
    v = (rng.standard_normal(k.shape, dtype=np.float32) * 0.5).astype(np.float16)
    qkv = rng.standard_normal(QKV, dtype=np.float32).astype(np.float16)
    cos, sin = oracle.rope_tables(k.shape[0], D, 5.0e6)

    def one(step):
        pos = PAST + step
        q = qkv[:Q_DIM].copy()
        kn = qkv[Q_DIM:Q_DIM + KV_DIM].copy()
        vn = qkv[Q_DIM + KV_DIM:].copy()
        oracle.rope_and_store_kv(q, kn, vn, k, v, cos, sin, 1, H, KVH, D, Q_DIM, KV_DIM, pos, (step + 1) % 4 != 0)
        oracle.decode_attention(q, k, v, pos + 1, H, KVH, D, threads=threads)
        return layer_bytes(pos + 1)

    for s in range(args.warmup):
        one(s)
    total, t0 = 0, time.perf_counter()
    for s in range(args.steps):
        total += one(s)
    el = time.perf_counter() - t0
    val = total / el / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(val, 3), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16 in, f64 accumulate",
        "data": "synthetic (seeded numpy), KV ~N(0,0.5)",
        "config": {"workload": WORKLOAD, "sample": "one layer-step per step (RoPE+append+decode at kv_len "
                   "65537+step) instead of 36 layers", "l2": "n/a (CPU)"},
        "cpu_baseline": {"value": round(val, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{args.steps} layer-steps of the 64K decode, C oracle, {threads} OpenMP threads"},
        "e2e": {"value": round(val, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------- prefill (config 3)
def run_prefill(args, rank, world, dev):
    """36 layers of RoPE/append + causal prefill for the (sequence, KV head)
    units this rank owns; returns a dict for the JSON line (rank 0)."""
    import numpy as np
    import torch
    import b200attn
    from b200attn import dist as bdist
    shard = bdist.prefill_shard(PF_B, KVH, world, rank)
    units = shard.units() if shard is not None else bdist.prefill_units(PF_B, KVH, world, rank)
    seqs = sorted({b for b, _ in units})
    gen = torch.Generator(device=dev).manual_seed(SEED + 100 + rank)
    qkv = torch.empty((PF_B, PF_S, QKV), dtype=torch.float16, device=dev).normal_(0.0, 1.0, generator=gen)
    cache = torch.empty((PF_B, LAYERS, 2, PF_S, KV_DIM), dtype=torch.float16, device=dev)
    out = torch.empty((PF_B, PF_S, Q_DIM), dtype=torch.float16, device=dev)
    cos, sin = b200attn.rope_tables_host(PF_S, D, 5.0e6)
    d_cos, d_sin = torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev)
    stream = torch.cuda.Stream(device=dev)
    G = H // KVH

    def layer(l, t_attn=None):
        rotate = (l + 1) % 4 != 0
        for b in seqs:
            row = qkv[b]
            b200attn.launch_rope_and_store_kv(row, row[:, Q_DIM:], row[:, Q_DIM + KV_DIM:], cache[b, l, 0],
                                              cache[b, l, 1], d_cos, d_sin, PF_S, H, KVH, D, QKV, QKV, 0, rotate,
                                              stream=stream)
        if t_attn is not None:
            t_attn[0].record(stream)
        if shard is not None:
            # one batched launch over this rank's block of sequences x KV heads
            s0, nb = shard.seq_begin, shard.seq_end - shard.seq_begin
            g0, ng = shard.kvh_begin, shard.kvh_end - shard.kvh_begin
            b200attn.launch_causal_attention_prefill_batched(
                qkv[s0, :, g0 * G * D:], cache[s0, l, 0, :, g0 * D:], cache[s0, l, 1, :, g0 * D:],
                out[s0, :, g0 * G * D:], nb, PF_S, ng * G, ng, D, QKV, KV_DIM, PF_S * QKV,
                LAYERS * 2 * PF_S * KV_DIM, PF_S * Q_DIM, stream=stream, out_stride=Q_DIM)
        else:
            for b, g in units:
                g0 = g * G
                b200attn.launch_causal_attention_prefill(
                    qkv[b, :, g0 * D:], cache[b, l, 0, :, g * D:], cache[b, l, 1, :, g * D:], out[b, :, g0 * D:],
                    PF_S, H // KVH, 1, D, QKV, KV_DIM, stream=stream)
        if t_attn is not None:
            t_attn[1].record(stream)

    steps = max(1, min(args.steps, args.prefill_steps))
    with torch.cuda.stream(stream):
        for _ in range(max(1, args.warmup // 2)):
            for l in range(LAYERS):
                layer(l)
    torch.cuda.synchronize()
    n0 = b200attn.kernel_launch_count()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    attn_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(LAYERS)]
    if world > 1:
        import torch.distributed as tdist
        tdist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(dev.index) as clocks, torch.cuda.stream(stream):
        ev[0].record(stream)
        for s_ in range(steps):
            for l in range(LAYERS):
                layer(l, attn_ev[l] if s_ == steps - 1 else None)
        ev[1].record(stream)
        torch.cuda.synchronize()
    launches = b200attn.kernel_launch_count() - n0
    ms = ev[0].elapsed_time(ev[1])
    attn_ms = sum(a.elapsed_time(b) for a, b in attn_ev) / LAYERS
    if world > 1:
        ms = bdist.max_over_ranks(ms, dev)
    total_flops = prefill_flops(PF_B, PF_S) * LAYERS * steps       # whole job, all ranks
    unit_flops = prefill_flops(1, PF_S, H // KVH) * len(units)     # this rank, one layer
    tf = total_flops / (ms / 1e3) / 1e12
    achieved = unit_flops / (attn_ms / 1e3) / 1e12
    # the attention launches are timed inside a long (power-capped) step: the
    # sustained tensor peak is the denominator, the burst one is reported beside
    peak, burst = 1400.0, 1590.0
    pk = os.path.join(ROOT, "MEASURED_PEAKS.json")
    kind = "fallback (sustained)"
    if os.path.exists(pk):
        with open(pk) as f:
            pj = json.load(f)
        peak = float(pj.get("bf16_tflops_sustained", pj["bf16_tflops"]))
        burst = float(pj["bf16_tflops"])
        kind = "measured (bf16 sustained, back-to-back GEMMs under the power cap; fp16 runs at the same rate)"
    return {"metric": "prefill TFLOP/s", "value": round(tf, 2), "unit": "TFLOP/s", "workload": PF_WORKLOAD,
            "clocks": clocks.summary(),
            "steps": steps, "ms_per_step": round(ms / steps, 3), "gpu_launches": launches,
            "units_per_rank": len(units), "parallelism": f"batch x kv-head units over {world} GPU(s)" + (
                f", one batched launch per layer for sequences [{shard.seq_begin}, {shard.seq_end}) x kv heads "
                f"[{shard.kvh_begin}, {shard.kvh_end})" if shard is not None else ""),
            "roofline": {"bound": "tensor", "kernel": "prefill_pair_kernel", "achieved": round(achieved, 1),
                         "peak": peak, "unit": "TFLOP/s", "frac": round(achieved / peak, 4), "peak_kind": kind,
                         "frac_of_burst": round(achieved / burst, 4),
                         "frac_of_nominal_2250": round(achieved / 2250.0, 4), "avg_launch_ms": round(attn_ms, 4),
                         "algorithmic_flops_per_launch": unit_flops}}


# --------------------------------------------------------------------------- ragged decode (config 5)
def run_ragged(args, rank, world, dev):
    """36 layers of ragged RoPE/append + ragged decode for the sequences this
    rank owns (greedy longest-first assignment), one captured CUDA graph per
    step; returns a dict for the JSON line (rank 0)."""
    import numpy as np
    import torch
    import b200attn
    from b200attn import dist as bdist
    lens_all = [int(x) for x in np.random.default_rng(SEED).integers(512, RG_MAX + 1, RG_B)]
    mine = bdist.assign_sequences(lens_all, world)[rank]
    B = len(mine)
    lens = [lens_all[i] for i in mine]
    gen = torch.Generator(device=dev).manual_seed(SEED + 200 + rank)
    cache = torch.empty((LAYERS, 2, B, RG_MAX, KV_DIM), dtype=torch.float16, device=dev)
    for l in range(LAYERS):
        for kv in range(2):
            for b in range(B):
                cache[l, kv, b, :lens[b]].normal_(0.0, 1.0, generator=gen)
    qkv = torch.empty((LAYERS, B, QKV), dtype=torch.float16, device=dev).normal_(0.0, 1.0, generator=gen)
    out = torch.empty((LAYERS, B, Q_DIM), dtype=torch.float16, device=dev)
    cos, sin = b200attn.rope_tables_host(RG_MAX, D, 5.0e6)
    d_cos, d_sin = torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev)
    pos = torch.tensor([n - 1 for n in lens], dtype=torch.int32, device=dev)   # the new token's row
    ws_bytes = b200attn.decode_ragged_workspace_bytes(B, H, KVH, RG_MAX)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev)
    stream = torch.cuda.Stream(device=dev)

    def step(st):
        for l in range(LAYERS):
            row = qkv[l]
            rotate = (l + 1) % 4 != 0
            if args.unfused:
                # the two-launch form: ragged RoPE/append, then the ragged decode
                b200attn.launch_rope_and_store_kv_ragged(row, row[:, Q_DIM:], row[:, Q_DIM + KV_DIM:], cache[l, 0],
                                                         cache[l, 1], RG_MAX * KV_DIM, d_cos, d_sin, B, H, KVH, D,
                                                         QKV, QKV, pos, RG_MAX, rotate, stream=st)
                b200attn.launch_causal_attention_decode_ragged(row, QKV, cache[l, 0], cache[l, 1], RG_MAX * KV_DIM,
                                                               pos, 1, RG_MAX, out[l], 0, B, H, KVH, D, ws, ws_bytes,
                                                               stream=st)
            else:
                b200attn.launch_decode_step_ragged_fused(row, QKV, row[:, Q_DIM:], row[:, Q_DIM + KV_DIM:], QKV,
                                                         cache[l, 0], cache[l, 1], RG_MAX * KV_DIM, d_cos, d_sin,
                                                         RG_MAX, rotate, pos, RG_MAX, out[l], 0, B, H, KVH, D, ws,
                                                         ws_bytes, stream=st)

    with torch.cuda.stream(stream):
        step(stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    n0 = b200attn.kernel_launch_count()
    with torch.cuda.graph(graph, stream=stream):
        step(torch.cuda.current_stream())
    per_step = b200attn.kernel_launch_count() - n0
    torch.cuda.synchronize()
    steps = max(1, min(args.steps, args.ragged_steps))
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as tdist
        tdist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        ev0.record(stream)
        for _ in range(steps):
            graph.replay()
        ev1.record(stream)
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        ms = bdist.max_over_ranks(ms, dev)
    graph.reset()
    # K+V rows read + Q + output + appended row, every sequence, every layer
    seq_bytes = lambda n: 2 * n * KV_DIM * 2 + Q_DIM * 2 + Q_DIM * 2 + 2 * KV_DIM * 2
    total = sum(seq_bytes(n) for n in lens_all) * LAYERS * steps
    mine_layer = sum(seq_bytes(n) for n in lens)
    peak, peak_kind = load_peaks()
    launch_ms = ms / steps / LAYERS
    achieved = mine_layer / (launch_ms / 1e3) / 1e9
    # ncu DRAM bytes of one config-5-shape launch, scaled by this layer's algorithmic bytes
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "ragged_traffic.json")
    if os.path.exists(tpath):
        with open(tpath) as f:
            t = json.load(f)
        traffic = int(round(mine_layer * t["bytes_per_launch"] / t["algorithmic_bytes"]))
    return {"metric": "ragged decode KV-read GB/s", "value": round(total / (ms / 1e3) / 1e9, 2), "unit": "GB/s",
            "workload": RG_WORKLOAD, "steps": steps, "ms_per_step": round(ms / steps, 4),
            "gpu_launches": per_step * steps, "sequences_per_rank": B,
            "parallelism": f"sequences over {world} GPU(s), greedy longest-first",
            "roofline": {"bound": "hbm",
                         "kernel": ("decode_ragged_kernel + merge_ragged_kernel (+ ragged RoPE/append kernel)"
                                    if args.unfused else
                                    "decode_ragged_kernel<fused step> (RoPE + append + split attention) + "
                                    "merge_ragged_kernel"),
                         "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind, "traffic": traffic,
                         "avg_layer_us": round(launch_ms * 1e3, 3), "algorithmic_bytes_per_layer": mine_layer,
                         "timing": "timed region (graph replays) / 36 layers per step"}}


# --------------------------------------------------------------------------- GPU arm
def run_b200(args, rank, world):
    import numpy as np
    import torch
    import b200attn
    from b200attn import dist as bdist

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    plan = bdist.split_kv_plan(PAST, world, rank)
    capacity = plan.local_capacity(args.warmup + args.steps + 1)   # local cache rows
    max_global = PAST + args.warmup + args.steps + 1

    # ---- state: KV cache (local slice), RoPE tables, per-layer QKV rows, outputs
    gen = torch.Generator(device=dev).manual_seed(SEED + rank)
    cache = b200attn.KVCache(LAYERS, capacity, KVH, D, device=dev)
    for l in range(LAYERS):
        for t in (cache.get_k_cache(l), cache.get_v_cache(l)):
            t.normal_(0.0, 0.5, generator=gen)
    cos, sin = b200attn.rope_tables_host(max_global, D, 5.0e6)
    d_cos, d_sin = torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev)
    hgen = np.random.default_rng(SEED)     # identical Q/K/V rows on every rank
    qkv_host = torch.from_numpy(hgen.standard_normal((LAYERS, QKV), dtype=np.float32).astype(np.float16)).pin_memory()
    qkv = qkv_host.to(dev)
    out = torch.zeros((LAYERS, Q_DIM), dtype=torch.float16, device=dev)
    out_host = torch.zeros_like(out, device="cpu").pin_memory()
    step_state = bdist.DecodeStepState(plan, H, KVH, D, LAYERS, capacity, max_global, dev, fused=not args.unfused,
                                       exchange=args.exchange)

    stream = torch.cuda.Stream(device=dev)
    group = None
    if world > 1:
        import torch.distributed as tdist
        group = tdist.group.WORLD

    def enqueue_step(s):
        bdist.enqueue_decode_step(step_state, cache, qkv, out, d_cos, d_sin, s, group)

    # ---- capture one step as a CUDA graph (device-resident positions)
    step_state.reset_position(PAST)
    with torch.cuda.stream(stream):
        enqueue_step(stream)         # eager warm-up of every launch (and NCCL) once
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    n0 = b200attn.kernel_launch_count()
    with torch.cuda.graph(graph, stream=stream):
        enqueue_step(torch.cuda.current_stream())
    launches_per_step = b200attn.kernel_launch_count() - n0
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            import torch.distributed as tdist
            tdist.barrier()

    # ---- value: graph replays, inputs resident
    # graph.replay() launches on the current stream: make it `stream` and time there
    step_state.reset_position(PAST)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            graph.replay()
    torch.cuda.synchronize()
    step_state.reset_position(PAST)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index) as clocks, torch.cuda.stream(stream):
        ev0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        ev1.record(stream)
        torch.cuda.synchronize()
    barrier()
    ms = ev0.elapsed_time(ev1)
    ms = bdist.max_over_ranks(ms, dev) if world > 1 else ms
    total_bytes = sum(step_bytes(PAST + 1 + s) for s in range(args.steps))
    value = total_bytes / (ms / 1e3) / 1e9

    # ---- roofline: one layer's decode launch(es), CUDA events on its stream
    peak, peak_kind = load_peaks()
    dec_ms = bdist.time_decode_launches(step_state, cache, qkv, out, stream, reps=3, d_cos=d_cos, d_sin=d_sin)
    kv_len_local = plan.local_len(PAST + 1)
    # K/V rows read, Q read, output written (+ the new K/V row read and appended)
    dec_bytes = 2 * kv_len_local * KV_DIM * 2 + Q_DIM * 2 + Q_DIM * 2 + (4 * KV_DIM * 2 if step_state.fused else 0)
    if step_state.fused and (world == 1 or step_state.exchange == "peer"):
        # Inside the captured step consecutive layers overlap (programmatic
        # dependent launch, L2 warm-up of the next layer's first tiles), so the
        # per-launch time is the timed region over its fused launches; the
        # step's one other kernel (position advance) is counted against them.
        launch_ms = ms / args.steps / LAYERS
        timing = (f"timed region (CUDA events around {args.steps} graph replays) / {LAYERS} fused launches per step; "
                  f"isolated launch {dec_ms * 1e3:.1f} us")
    else:
        launch_ms = dec_ms
        timing = "CUDA events around isolated launches on the decode stream"
    achieved = dec_bytes / (launch_ms / 1e3) / 1e9
    # ncu DRAM bytes of one 64K launch, scaled to this rank's launch by its
    # algorithmic bytes (the same on one GPU; a 1/N range of the cache on N)
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "decode_traffic.json")
    if os.path.exists(tpath):
        with open(tpath) as f:
            t = json.load(f)
        traffic = int(round(dec_bytes * t["bytes_per_launch"] / t["algorithmic_bytes"]))

    # ---- e2e: reference-facing C-ABI calls, host buffers in and out every step
    e2e = None
    if world == 1:
        e2e = bdist.e2e_decode(cache, qkv, qkv_host, out, out_host, d_cos, d_sin, PAST, args.warmup, args.steps,
                               stream, step_state, mode="reference" if args.unfused else "fused")
        if not args.unfused:
            ref_calls = bdist.e2e_decode(cache, qkv, qkv_host, out, out_host, d_cos, d_sin, PAST, args.warmup,
                                         args.steps, stream, step_state, mode="reference")
            e2e["reference_launchers"] = {"value": ref_calls["value"], "ms_per_step": ref_calls["ms_per_step"],
                                          "path": ref_calls["path"]}

    # ---- CPU baseline (rank 0, N=1): bounded sample
    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu:
        threads = os.cpu_count() or 1
        gbs, reps, el = cpu_decode_sample(PAST + 1, threads)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
               "sample": f"{reps} layer-steps of the 64K decode (RoPE+append+attention) in {el:.1f} s, "
                         f"C oracle, {threads} OpenMP threads"}

    prefill = None
    del cache
    torch.cuda.empty_cache()
    if not args.no_prefill:
        prefill = run_prefill(args, rank, world, dev)
        torch.cuda.empty_cache()
    ragged = None
    if not args.no_ragged:
        ragged = run_ragged(args, rank, world, dev)
        torch.cuda.empty_cache()

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f16 (f32 accumulate)",
            "data": "synthetic: KV ~N(0,0.5) (torch CUDA generator, seed 2024+rank), Q/K/V rows ~N(0,1) seeded",
            "config": {"workload": WORKLOAD, "global_batch": 1, "seq_len": PAST, "layers": LAYERS,
                       "parallelism": (f"kv-split{world}, " + ("cross-rank merge in the fused kernel over CUDA-IPC "
                                       "peer memory" if step_state.exchange == "peer" else "NCCL all-gather of rank "
                                       "partials + merge kernel")) if world > 1 else "single-gpu",
                       "l2": "inputs larger than L2 (4.8 GB of KV per step)",
                       "step_graph": f"one CUDA graph per step, {launches_per_step} kernels"},
            "gpu_launches": launches_per_step * args.steps,
            "roofline": {"bound": "hbm",
                         "kernel": ("decode_tma_kernel<fused> (RoPE + append + split attention + merge)"
                                    if step_state.fused else "decode_tma_kernel + merge_partials_kernel"),
                         "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "traffic": traffic, "avg_launch_us": round(launch_ms * 1e3, 3),
                         "isolated_launch_us": round(dec_ms * 1e3, 3), "timing": timing,
                         "algorithmic_bytes_per_launch": dec_bytes},
            "clocks": clocks.summary(),
            "e2e": e2e,
            "cpu_baseline": cpu,
            "prefill": prefill,
            "ragged": ragged,
        }
        print(json.dumps(line), flush=True)
    graph.reset()
    step_state.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU-baseline sample")
    ap.add_argument("--no-prefill", action="store_true", help="skip the config-3 prefill sub-measurement")
    ap.add_argument("--no-ragged", action="store_true", help="skip the config-5 ragged decode sub-measurement")
    ap.add_argument("--exchange", default="peer", choices=["peer", "nccl"],
                    help="N > 1 decode: cross-rank merge inside the fused kernel over peer memory, or an NCCL "
                         "all-gather of the rank partials and a merge kernel")
    ap.add_argument("--ragged-steps", type=int, default=8, help="timed ragged steps (36 layers each)")
    ap.add_argument("--unfused", action="store_true",
                    help="decode step as the reference's launch sequence (RoPE/append, split, merge) per layer "
                         "instead of the fused one-kernel-per-layer step")
    ap.add_argument("--prefill-steps", type=int, default=4, help="timed prefill steps (36 layers each)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if world > 1:
        import datetime
        import torch
        import torch.distributed as tdist
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    try:
        run_b200(args, rank, world)
    finally:
        if world > 1:
            import torch.distributed as tdist
            tdist.destroy_process_group()


if __name__ == "__main__":
    main()
