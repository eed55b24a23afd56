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
e2e   : the same metric through the C ABI with host buffers: every step
        copies the step's Q/K/V rows and position in from pinned host memory,
        issues one fused-step call per layer (eager) and copies the attention
        outputs back; e2e.reference_launchers (one GPU) times the reference
        engine's own call sequence (launch_rope_and_store_kv +
        launch_causal_attention_decode_vectorized per layer) the same way.
Algorithmic bytes per layer-step: K+V read 2*kv_len*512*2 + Q 4 KiB +
output 4 KiB + appended K/V row 2 KiB (partial-workspace traffic excluded).

Sub-measurements in the same line: `prefill` (config 3: 36 layers of
RoPE/append + batched causal prefill, TFLOP/s, with its own e2e and CPU
baseline), `ragged` (config 5, GB/s, e2e and CPU baseline) and, on one GPU,
`small` (configs 1 and 2, latency-bound single layers: per-call device time
eager and graphed, e2e, CPU baselines in full) and `out_projection` (the
path's consumer: the o_proj GEMM over config 3's tokens and the decode GEMV). CPU baselines (rank 0, one
GPU) time the C oracle (the double-precision restatement of
tests/test_causal_attention.cpp:176-196) and the python/reference.py:62-92
path on CPU torch (FP16, FP32) with every host thread, on bounded samples.

--impl reference times the reference algorithm's CPU implementation (the
C oracle restating it, all host threads) on a bounded sample of the same
workload (one layer-step at the same kv_len per step), with the
python/reference.py path on the same layer-step reported beside it, and
prints the same line.

N > 1 (torchrun): config-4 decode by KV head (--decode-split heads, the
default when the 4 KV heads divide or are divided by N): each rank owns whole
GQA groups with only their cache and writes their heads' outputs, the layout
a tensor-parallel o_proj consumes, with no exchange; at N = 8 the two ranks
of each KV head also split its range. With --decode-split kv the 64K KV range
of every layer is split into N contiguous ranges, one per rank; the rank
holding the tail appends the new token; each rank reduces its range to one
(o, m, l) partial per head. Partials of a split range are merged across ranks
inside the fused kernel over CUDA-IPC peer memory (--exchange peer, default)
or by an NCCL all-gather and a merge kernel (--exchange nccl). Strong
scaling: total work fixed. Prefill shards
(sequence, KV head) units and the ragged decode shards whole sequences
(weak in units, no exchange).
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


TRAFFIC_NOTE = ("static ncu figure, not measured in this run: dram__bytes_read.sum + dram__bytes_write.sum of {what} "
                "({f}), scaled to this launch by its algorithmic bytes")


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
def cpu_info() -> dict:
    model = None
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return {"cpu_model": model, "logical_cpus": os.cpu_count()}


def _best(variants: dict, unit: str, threads: int, sample: str, scale_note: str | None = None) -> dict:
    """cpu_baseline object: the fastest of the timed CPU implementations is the
    value; every variant is listed beside it."""
    name = max(variants, key=lambda k: variants[k]["value"])
    out = {"value": variants[name]["value"], "unit": unit, "cores": threads, "kind": "port", "best": name,
           "sample": sample, **cpu_info(), "variants": variants}
    if scale_note:
        out["extrapolated"] = scale_note
    return out


def _torch_threads(threads: int):
    import torch
    torch.set_num_threads(threads)


def cpu_decode_sample(kv_len: int, threads: int, rng_seed: int = 7, budget_s: float = 8.0, min_reps: int = 2):
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


def torch_decode_sample(kv_len: int, threads: int, dtype_name: str, budget_s: float = 3.0):
    """The python/reference.py path for one layer-step at kv_len (HF RoPE of
    the new token, append, repeat_interleave + SDPA over the cache); GB/s."""
    import torch
    from oracle import torch_ref
    _torch_threads(threads)
    dt = getattr(torch, dtype_name)
    kc = torch_ref.seeded((kv_len, KV_DIM), 7, 0.5).to(dt)
    vc = torch_ref.seeded((kv_len, KV_DIM), 8, 0.5).to(dt)
    row = torch_ref.seeded(QKV, 9).to(dt)
    q, kn, vn = row[:Q_DIM], row[Q_DIM:Q_DIM + KV_DIM], row[Q_DIM + KV_DIM:]
    per, reps = torch_ref.time_calls(lambda: torch_ref.decode(q, kn, vn, kc, vc, kv_len - 1, H, KVH, D), budget_s, 2)
    return layer_bytes(kv_len) / per / 1e9, reps, per * reps


def cpu_config4(threads: int, budget_s: float = 8.0) -> dict:
    gbs, reps, el = cpu_decode_sample(PAST + 1, threads, budget_s=budget_s)
    var = {"c_oracle_f64": {"value": round(gbs, 3), "reps": reps, "seconds": round(el, 2)}}
    for dt in ("float16", "float32"):
        g, r, e = torch_decode_sample(PAST + 1, threads, dt)
        var[f"python_reference_{dt}"] = {"value": round(g, 3), "reps": r, "seconds": round(e, 2)}
    return _best(var, "GB/s", threads, "one layer-step of the 64K decode (RoPE + append + attention at kv_len "
                 "65537), repeated: the C oracle (test_causal_attention.cpp:176-196 double softmax, OpenMP) and the "
                 "python/reference.py:62-92 path on CPU torch (HF apply_rotary_pos_emb, repeat_interleave, SDPA) in "
                 "FP16 and FP32", "per layer-step; a 36-layer step is 36 of these")


def cpu_prefill_unit(S: int, heads: int, kv_heads: int, threads: int, row_stride: int = 1, budget_s: float = 1.0):
    """Causal prefill of S tokens, `heads` query heads over `kv_heads` KV heads
    (RoPE + attention): TFLOP/s of the C oracle (every row_stride-th query row,
    scaled to all rows by FLOP count) and of the python/reference.py path."""
    import numpy as np
    import torch
    import oracle
    from oracle import torch_ref
    _torch_threads(threads)
    rng = np.random.default_rng(11)
    qd, kd = heads * D, kv_heads * D
    q = rng.standard_normal((S, qd), dtype=np.float32).astype(np.float16)
    k = rng.standard_normal((S, kd), dtype=np.float32).astype(np.float16)
    v = rng.standard_normal((S, kd), dtype=np.float32).astype(np.float16)
    cos, sin = oracle.rope_tables(S, D, 5.0e6)
    rows = None if row_stride == 1 else list(range(row_stride - 1, S, row_stride))
    # FLOPs of the rows computed: 2 * heads * d * (keys per row) * 2
    row_keys = S * (S + 1) // 2 if rows is None else sum(r + 1 for r in rows)
    flops_done = 4 * heads * D * row_keys
    flops_all = prefill_flops(1, S, heads)

    def c_call():
        qq, kk = q.copy(), k.copy()
        oracle.rope_and_store_kv(qq, kk, None, None, None, cos, sin, S, heads, kv_heads, D, qd, kd, 0, True)
        oracle.causal_attention(qq, kk, v, S, heads, kv_heads, D, rows=rows, threads=threads)
    per, reps = torch_ref.time_calls(c_call, budget_s, warm=0)
    var = {"c_oracle_f64": {"value": round(flops_done / per / 1e12, 6), "reps": reps, "seconds": round(per * reps, 2),
                            "rows": "all" if rows is None else f"every {row_stride}th query row"}}
    tq, tk, tv = torch.from_numpy(q), torch.from_numpy(k), torch.from_numpy(v)
    for dt in ("float16", "float32"):
        d_ = getattr(torch, dt)
        per, reps = torch_ref.time_calls(lambda: torch_ref.prefill(tq, tk, tv, heads, kv_heads, D, dtype=d_),
                                         budget_s, 2)
        var[f"python_reference_{dt}"] = {"value": round(flops_all / per / 1e12, 6), "reps": reps,
                                         "seconds": round(per * reps, 2)}
    return var


def cpu_config5(lens, threads: int) -> dict:
    """One layer of the ragged decode on CPU (every sequence: RoPE + append +
    attention at its length); the sequences' caches are windows of one seeded
    pool of rows (timing only). GB/s of algorithmic bytes."""
    import numpy as np
    import torch
    import oracle
    from oracle import torch_ref
    _torch_threads(threads)
    n = max(lens)
    rng = np.random.default_rng(13)
    pool_k = rng.standard_normal((n, KV_DIM), dtype=np.float32).astype(np.float16)
    pool_v = rng.standard_normal((n, KV_DIM), dtype=np.float32).astype(np.float16)
    rows = rng.standard_normal((len(lens), QKV), dtype=np.float32).astype(np.float16)
    cos, sin = oracle.rope_tables(n, D, 5.0e6)
    nbytes = sum(2 * L_ * KV_DIM * 2 + Q_DIM * 4 + 2 * KV_DIM * 2 for L_ in lens)

    def c_layer():
        for i, L_ in enumerate(lens):
            q, kn, vn = rows[i, :Q_DIM].copy(), rows[i, Q_DIM:Q_DIM + KV_DIM].copy(), rows[i, Q_DIM + KV_DIM:].copy()
            oracle.rope_and_store_kv(q, kn, vn, pool_k, pool_v, cos, sin, 1, H, KVH, D, Q_DIM, KV_DIM, L_ - 1, True)
            oracle.decode_attention(q, pool_k, pool_v, L_, H, KVH, D, threads=threads)
    per, reps = torch_ref.time_calls(c_layer, 1.0, warm=0)
    var = {"c_oracle_f64": {"value": round(nbytes / per / 1e9, 3), "reps": reps, "seconds": round(per * reps, 2)}}
    for dt in ("float16", "float32"):
        d_ = getattr(torch, dt)
        kc, vc, tr = torch.from_numpy(pool_k).to(d_), torch.from_numpy(pool_v).to(d_), torch.from_numpy(rows).to(d_)

        def t_layer():
            for i, L_ in enumerate(lens):
                torch_ref.decode(tr[i, :Q_DIM], tr[i, Q_DIM:Q_DIM + KV_DIM], tr[i, Q_DIM + KV_DIM:], kc, vc, L_ - 1,
                                 H, KVH, D)
        per, reps = torch_ref.time_calls(t_layer, 1.0)
        var[f"python_reference_{dt}"] = {"value": round(nbytes / per / 1e9, 3), "reps": reps,
                                         "seconds": round(per * reps, 2)}
    return _best(var, "GB/s", threads, f"one layer of the {len(lens)} sequences (RoPE + append + attention at each "
                 "length): C oracle and the python/reference.py path (FP16, FP32)",
                 "one layer timed; the 36-layer step is 36 of these (GB/s unchanged)")


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
    # the python/reference.py path on the same layer-step, beside the C oracle
    py = {}
    for dt in ("float16", "float32"):
        g, r, e = torch_decode_sample(PAST + 1, threads, dt, budget_s=2.0)
        py[dt] = {"value": round(g, 3), "unit": "GB/s", "reps": r, "seconds": round(e, 2)}
    line = {
        "impl": "reference", "metric": METRIC, "value": round(val, 3), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16 in, f64 accumulate",
        "data": "synthetic (seeded numpy), KV ~N(0,0.5)",
        "config": {"workload": WORKLOAD, "sample": "one layer-step per step (RoPE+append+decode at kv_len "
                   "65537+step) instead of 36 layers", "l2": "n/a (CPU)"},
        "cpu_baseline": {"value": round(val, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{args.steps} layer-steps of the 64K decode, C oracle "
                                   f"(test_causal_attention.cpp:176-196 restated), {threads} OpenMP threads",
                         **cpu_info()},
        "python_reference_path": {"what": "python/reference.py:62-92 on CPU torch (HF apply_rotary_pos_emb, "
                                          "repeat_interleave, SDPA), same layer-step, "
                                          f"torch.set_num_threads({threads})", **py},
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

    def layer(l, t_attn=None, qkv_=qkv, out_=out, st=stream):
        rotate = (l + 1) % 4 != 0
        for b in seqs:
            row = qkv_[b]
            b200attn.launch_rope_and_store_kv(row, row[:, Q_DIM:], row[:, Q_DIM + KV_DIM:], cache[b, l, 0],
                                              cache[b, l, 1], d_cos, d_sin, PF_S, H, KVH, D, QKV, QKV, 0, rotate,
                                              stream=st)
        if t_attn is not None:
            t_attn[0].record(st)
        if shard is not None:
            # one batched launch over this rank's block of sequences x KV heads
            s0, nb = shard.seq_begin, shard.seq_end - shard.seq_begin
            g0, ng = shard.kvh_begin, shard.kvh_end - shard.kvh_begin
            b200attn.launch_causal_attention_prefill_batched(
                qkv_[s0, :, g0 * G * D:], cache[s0, l, 0, :, g0 * D:], cache[s0, l, 1, :, g0 * D:],
                out_[s0, :, g0 * G * D:], nb, PF_S, ng * G, ng, D, QKV, KV_DIM, PF_S * QKV,
                LAYERS * 2 * PF_S * KV_DIM, PF_S * Q_DIM, stream=st, out_stride=Q_DIM)
        else:
            for b, g in units:
                g0 = g * G
                b200attn.launch_causal_attention_prefill(
                    qkv_[b, :, g0 * D:], cache[b, l, 0, :, g * D:], cache[b, l, 1, :, g * D:], out_[b, :, g0 * D:],
                    PF_S, H // KVH, 1, D, QKV, KV_DIM, stream=st)
        if t_attn is not None:
            t_attn[1].record(st)

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

    # ---- e2e: the same 36 layers with this rank's [Q|K|V] rows copied in from
    # pinned host memory before every layer and its outputs copied back after
    # it, through the C-ABI launchers; copies on their own streams, two device
    # buffers, so layer l's copies overlap layers l +- 1's compute
    s0, s1 = seqs[0], seqs[-1] + 1
    nseq = s1 - s0
    qkv_host = qkv[s0:s1].cpu().pin_memory()
    out_host = torch.empty((nseq, PF_S, Q_DIM), dtype=torch.float16).pin_memory()
    qkv_b = [qkv, torch.empty_like(qkv)]
    out_b = [out, torch.empty_like(out)]
    h2d_s, d2h_s = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    ev_h = [torch.cuda.Event() for _ in range(2)]
    ev_c = [torch.cuda.Event() for _ in range(2)]
    ev_d = [torch.cuda.Event() for _ in range(2)]

    def e2e_steps(n):
        i = 0
        for _ in range(n):
            for l in range(LAYERS):
                bf = i & 1
                if i >= 2:
                    h2d_s.wait_event(ev_c[bf])          # layer i - 2 is done reading this buffer
                with torch.cuda.stream(h2d_s):
                    qkv_b[bf][s0:s1].copy_(qkv_host, non_blocking=True)
                ev_h[bf].record(h2d_s)
                stream.wait_event(ev_h[bf])
                if i >= 2:
                    stream.wait_event(ev_d[bf])         # its outputs have left the device
                layer(l, None, qkv_b[bf], out_b[bf], stream)
                ev_c[bf].record(stream)
                d2h_s.wait_event(ev_c[bf])
                with torch.cuda.stream(d2h_s):
                    out_host.copy_(out_b[bf][s0:s1], non_blocking=True)
                ev_d[bf].record(d2h_s)
                i += 1
        stream.wait_stream(h2d_s)
        stream.wait_stream(d2h_s)

    e2e_steps(1)
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as tdist
        tdist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    e2e_steps(steps)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        e2e_ms = bdist.max_over_ranks(e2e_ms, dev)
    e2e = {"value": round(total_flops / (e2e_ms / 1e3) / 1e12, 2), "unit": "TFLOP/s",
           "h2d_bytes_per_step": LAYERS * qkv_host.numel() * 2, "d2h_bytes_per_step": LAYERS * out_host.numel() * 2,
           "ms_per_step": round(e2e_ms / steps, 3),
           "path": "per layer: this rank's [Q|K|V] rows H2D from pinned memory (own stream), C-ABI "
                   "launch_rope_and_store_kv + launch_causal_attention_prefill_batched, outputs D2H (own stream); "
                   "two device buffers so copies overlap the neighbouring layers' compute"}
    del qkv_b, out_b

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

    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu:
        threads = os.cpu_count() or 1
        var = cpu_prefill_unit(PF_S, H // KVH, 1, threads, row_stride=8)
        cpu = _best(var, "TFLOP/s", threads,
                    "one (sequence, KV head) unit of config 3 (8192 tokens, 4 query heads over 1 KV head, RoPE + "
                    "causal attention): C oracle on every 8th query row (FLOP-scaled) and the python/reference.py "
                    "path (FP16, FP32) on the whole unit",
                    "the rate of one unit stands for the 16 units x 36 layers of a step (equal causal work per unit)")
        cpu["ms_per_step_extrapolated"] = round(prefill_flops(PF_B, PF_S) * LAYERS / (cpu["value"] * 1e12) * 1e3, 1)
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
                         "algorithmic_flops_per_launch": unit_flops},
            "e2e": e2e, "cpu_baseline": cpu}


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
    split = args.ragged_split
    # by KV head: every rank decodes every sequence for its KV heads (its own
    # cache of those heads); ranks sharing heads (world > KVH) split the
    # sequences among themselves. By sequence: whole sequences per rank.
    hs = (bdist.head_split_plan(KVH, world, rank) if split == "heads"
          else bdist.HeadSplit(world, rank, KVH, 0, KVH, tuple(range(world))))
    share = tp_share(args, world)
    if share > 1:  # one GPU running rank 0's share of a `share`-way KV-head split
        hs = bdist.HeadSplit(1, 0, KVH, 0, KVH // share, (0,))
        split = "heads"
    kvh_l = hs.local_kv_heads
    h_l = kvh_l * (H // KVH)
    q_l, kv_l = h_l * D, kvh_l * D
    qkv_l = q_l + 2 * kv_l
    mine = bdist.assign_sequences(lens_all, hs.group_world)[hs.group_rank]
    B = len(mine)
    lens = [lens_all[i] for i in mine]
    gen = torch.Generator(device=dev).manual_seed(SEED + 200 + rank)
    cache = torch.empty((LAYERS, 2, B, RG_MAX, kv_l), dtype=torch.float16, device=dev)
    for l in range(LAYERS):
        for kv in range(2):
            for b in range(B):
                cache[l, kv, b, :lens[b]].normal_(0.0, 1.0, generator=gen)
    qkv = torch.empty((LAYERS, B, qkv_l), dtype=torch.float16, device=dev).normal_(0.0, 1.0, generator=gen)
    out = torch.empty((LAYERS, B, q_l), dtype=torch.float16, device=dev)
    cos, sin = b200attn.rope_tables_host(RG_MAX, D, 5.0e6)
    d_cos, d_sin = torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev)
    pos = torch.tensor([n - 1 for n in lens], dtype=torch.int32, device=dev)   # the new token's row
    ws_bytes = b200attn.decode_ragged_workspace_bytes(B, h_l, kvh_l, RG_MAX)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev)
    stream = torch.cuda.Stream(device=dev)

    def step(st):
        for l in range(LAYERS):
            row = qkv[l]
            rotate = (l + 1) % 4 != 0
            if args.unfused:
                # the two-launch form: ragged RoPE/append, then the ragged decode
                b200attn.launch_rope_and_store_kv_ragged(row, row[:, q_l:], row[:, q_l + kv_l:], cache[l, 0],
                                                         cache[l, 1], RG_MAX * kv_l, d_cos, d_sin, B, h_l, kvh_l, D,
                                                         qkv_l, qkv_l, pos, RG_MAX, rotate, stream=st)
                b200attn.launch_causal_attention_decode_ragged(row, qkv_l, cache[l, 0], cache[l, 1], RG_MAX * kv_l,
                                                               pos, 1, RG_MAX, out[l], 0, B, h_l, kvh_l, D, ws,
                                                               ws_bytes, stream=st)
            else:
                b200attn.launch_decode_step_ragged_fused(row, qkv_l, row[:, q_l:], row[:, q_l + kv_l:], qkv_l,
                                                         cache[l, 0], cache[l, 1], RG_MAX * kv_l, d_cos, d_sin,
                                                         RG_MAX, rotate, pos, RG_MAX, out[l], 0, B, h_l, kvh_l, D,
                                                         ws, ws_bytes, stream=st)

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
    total = sum(seq_bytes(n) for n in lens_all) * LAYERS * steps // share

    # ---- e2e: every step copies this rank's 36 x B new [Q|K|V] rows and the
    # positions in from pinned host memory, issues the 36 fused ragged calls
    # through the C ABI (eager) and copies the 36 x B outputs back
    qkv_host = qkv.cpu().pin_memory()
    pos_host = pos.cpu().pin_memory()
    out_host = torch.empty(out.shape, dtype=out.dtype).pin_memory()

    def e2e_step():
        qkv.copy_(qkv_host, non_blocking=True)
        pos.copy_(pos_host, non_blocking=True)
        step(stream)
        out_host.copy_(out, non_blocking=True)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as tdist
        tdist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(steps):
            e2e_step()
        e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        e2e_ms = bdist.max_over_ranks(e2e_ms, dev)
    e2e = {"value": round(total / (e2e_ms / 1e3) / 1e9, 2), "unit": "GB/s",
           "h2d_bytes_per_step": qkv_host.numel() * 2 + pos_host.numel() * 4,
           "d2h_bytes_per_step": out_host.numel() * 2, "ms_per_step": round(e2e_ms / steps, 4),
           "path": "per step: this rank's new rows and positions H2D from pinned memory, 36 eager C-ABI "
                   + ("launch_rope_and_store_kv_ragged + launch_causal_attention_decode_ragged pairs"
                      if args.unfused else "b2_launch_decode_step_ragged_fused calls") + ", outputs D2H"}
    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu:
        cpu = cpu_config5(lens_all, os.cpu_count() or 1)
    seq_bytes_l = lambda n: 2 * n * kv_l * 2 + q_l * 2 + q_l * 2 + 2 * kv_l * 2
    mine_layer = sum(seq_bytes_l(n) for n in lens)
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
            "parallelism": (f"one GPU running rank 0's share of a {share}-way KV-head split ({kvh_l} KV head(s) / "
                            f"{h_l} query heads of every sequence): per-rank work, not a whole-job number"
                            if share > 1 else
                            f"sequences over {world} GPU(s), greedy longest-first" if split != "heads" else
                            f"kv-heads over {world} GPU(s): {kvh_l} KV head(s) / {h_l} query heads of every "
                            "sequence per rank (own cache of those heads, head-sharded output)"
                            + (f", sequences split greedily over the {hs.group_world} ranks of each head"
                               if hs.group_world > 1 else "")),
            "roofline": {"bound": "hbm",
                         "kernel": ("decode_ragged_kernel + merge_ragged_kernel (+ ragged RoPE/append kernel)"
                                    if args.unfused else
                                    "decode_ragged_kernel<fused step> (RoPE + append + split attention) + "
                                    "merge_ragged_kernel"),
                         "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind, "traffic": traffic,
                         "traffic_source": TRAFFIC_NOTE.format(f="profiles/ragged_traffic.json",
                                                               what="one config-5 launch"),
                         "avg_layer_us": round(launch_ms * 1e3, 3), "algorithmic_bytes_per_layer": mine_layer,
                         "timing": "timed region (graph replays) / 36 layers per step"},
            "e2e": e2e, "cpu_baseline": cpu}


# --------------------------------------------------------------------------- configs 1 and 2 (latency-bound)
C1_S = 254          # config 1: one prefill layer of the benchmark prompt length
C2_PAST = 4096      # config 2: one decode layer, new token at position 4096
C1_WORKLOAD = ("config1: one causal GQA prefill layer, batch 1, 254 tokens, 16/4 heads, head_dim 128, N(0,1) FP16, "
               "RoPE theta 5e6 (launch_rope_and_store_kv + launch_causal_attention_prefill)")
C2_WORKLOAD = ("config2: one decode layer, batch 1, KV cache 4096 tokens N(0,1) FP16, new token RoPE'd at 4096 and "
               "appended (kv_len 4097), 16/4 heads, head_dim 128, KV_CHUNK 256 partials + merge")


def _per_call_ms(fn, calls: int, stream, graph: bool):
    """Device time per call of fn(i) over `calls` back-to-back calls, CUDA
    events on `stream`: eager launches, or one captured graph of all calls."""
    import torch
    if graph:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(calls):
                fn(i, torch.cuda.current_stream())
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            g.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            g.replay()
            e1.record(stream)
        torch.cuda.synchronize()
        g.reset()
        return e0.elapsed_time(e1) / calls
    with torch.cuda.stream(stream):
        for i in range(calls):
            fn(i, stream)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(calls):
            fn(i, stream)
        e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / calls


def run_small(args, dev):
    """Configs 1 and 2 on one GPU: per-call device time of the reference
    launch sequence (and of the fused decode step) cycling through enough
    copies of the inputs to exceed L2, eager and as one captured graph; e2e
    through the C ABI with host buffers; CPU baselines in full."""
    import numpy as np
    import torch
    import b200attn
    stream = torch.cuda.Stream(device=dev)
    gen = torch.Generator(device=dev).manual_seed(SEED + 300)
    res = {}

    # ---- config 1: RoPE/append + prefill of 254 tokens, 96 input copies (200 MB)
    n1 = 96
    qkv = torch.empty((n1, C1_S, QKV), dtype=torch.float16, device=dev).normal_(0.0, 1.0, generator=gen)
    cache = torch.zeros((n1, 2, C1_S, KV_DIM), dtype=torch.float16, device=dev)
    out = torch.empty((n1, C1_S, Q_DIM), dtype=torch.float16, device=dev)
    cos, sin = b200attn.rope_tables_host(C2_PAST + 8, D, 5.0e6)
    d_cos, d_sin = torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev)

    def c1(i, st):
        row = qkv[i]
        b200attn.launch_rope_and_store_kv(row, row[:, Q_DIM:], row[:, Q_DIM + KV_DIM:], cache[i, 0], cache[i, 1],
                                          d_cos, d_sin, C1_S, H, KVH, D, QKV, QKV, 0, True, stream=st)
        b200attn.launch_causal_attention_prefill(row, cache[i, 0], cache[i, 1], out[i], C1_S, H, KVH, D, QKV, KV_DIM,
                                                 stream=st)
    fl = prefill_flops(1, C1_S)
    eager = _per_call_ms(c1, n1, stream, False)
    graphed = _per_call_ms(c1, n1, stream, True)
    # e2e: each call copies its [Q|K|V] rows in from pinned memory and its output back
    h_in = qkv[0].cpu().pin_memory()
    h_out = torch.empty((C1_S, Q_DIM), dtype=torch.float16).pin_memory()

    def c1_e2e(i, st):
        qkv[i].copy_(h_in, non_blocking=True)
        c1(i, st)
        h_out.copy_(out[i], non_blocking=True)
    e2e = _per_call_ms(c1_e2e, n1, stream, False)
    res["config1"] = {
        "workload": C1_WORKLOAD, "unit": "TFLOP/s", "algorithmic_flops_per_call": fl,
        "eager": {"us_per_call": round(eager * 1e3, 2), "value": round(fl / (eager / 1e3) / 1e12, 2)},
        "graph": {"us_per_call": round(graphed * 1e3, 2), "value": round(fl / (graphed / 1e3) / 1e12, 2)},
        "e2e": {"value": round(fl / (e2e / 1e3) / 1e12, 2), "unit": "TFLOP/s", "us_per_call": round(e2e * 1e3, 2),
                "h2d_bytes_per_step": h_in.numel() * 2, "d2h_bytes_per_step": h_out.numel() * 2},
        "timing": f"CUDA events around {n1} back-to-back calls cycling through {n1} input copies (> L2)",
        "gpu_launches_per_call": 2}
    del qkv, cache, out

    # ---- config 2: one decode layer at kv_len 4097, 24 caches (200 MB)
    n2 = 24
    rows = C2_PAST + 8
    kc = torch.empty((n2, 2, rows, KV_DIM), dtype=torch.float16, device=dev).normal_(0.0, 1.0, generator=gen)
    new = torch.empty((n2, QKV), dtype=torch.float16, device=dev).normal_(0.0, 1.0, generator=gen)
    o2 = torch.empty((n2, Q_DIM), dtype=torch.float16, device=dev)
    pos = torch.tensor([C2_PAST], dtype=torch.int32, device=dev)
    sws_bytes = b200attn.decode_step_workspace_bytes(H, KVH)
    sws = torch.zeros(sws_bytes, dtype=torch.uint8, device=dev)
    nfl = b200attn.decode_workspace_floats(H, D, rows)
    ws = torch.empty(nfl, dtype=torch.float32, device=dev)
    ch = (rows + 255) // 256
    po, pm, pl = ws[:H * ch * D], ws[H * ch * D:H * ch * (D + 1)], ws[H * ch * (D + 1):]

    def c2_ref(i, st):
        row = new[i]
        b200attn.launch_rope_and_store_kv(row, row[Q_DIM:], row[Q_DIM + KV_DIM:], kc[i, 0], kc[i, 1], d_cos, d_sin,
                                          1, H, KVH, D, QKV, QKV, C2_PAST, True, stream=st)
        b200attn.launch_causal_attention_decode_vectorized(row, kc[i, 0], kc[i, 1], o2[i], po, pm, pl, 1, C2_PAST + 1,
                                                           C2_PAST, H, KVH, D, QKV, KV_DIM, stream=st)

    def c2_fused(i, st):
        row = new[i]
        b200attn.launch_decode_step_fused(row, row[Q_DIM:], row[Q_DIM + KV_DIM:], kc[i, 0], kc[i, 1], d_cos, d_sin,
                                          rows, True, pos, pos, 1, rows, o2[i], sws, sws_bytes, H, KVH, D, stream=st)
    nb = layer_bytes(C2_PAST + 1)
    t = {name: {"eager": _per_call_ms(fn, n2, stream, False), "graph": _per_call_ms(fn, n2, stream, True)}
         for name, fn in (("reference_launchers", c2_ref), ("fused_step", c2_fused))}
    h_row = new[0].cpu().pin_memory()
    h_o = torch.empty(Q_DIM, dtype=torch.float16).pin_memory()

    def c2_e2e(i, st):
        new[i].copy_(h_row, non_blocking=True)
        c2_fused(i, st)
        h_o.copy_(o2[i], non_blocking=True)
    e2e2 = _per_call_ms(c2_e2e, n2, stream, False)
    res["config2"] = {
        "workload": C2_WORKLOAD, "unit": "GB/s", "algorithmic_bytes_per_call": nb,
        **{name: {mode: {"us_per_call": round(v * 1e3, 2), "value": round(nb / (v / 1e3) / 1e9, 1)}
                  for mode, v in d_.items()} for name, d_ in t.items()},
        "e2e": {"value": round(nb / (e2e2 / 1e3) / 1e9, 1), "unit": "GB/s", "us_per_call": round(e2e2 * 1e3, 2),
                "h2d_bytes_per_step": h_row.numel() * 2, "d2h_bytes_per_step": h_o.numel() * 2,
                "path": "new [Q|K|V] row H2D, b2_launch_decode_step_fused, output D2H"},
        "timing": f"CUDA events around {n2} back-to-back calls cycling through {n2} caches (> L2)",
        "gpu_launches_per_call": {"reference_launchers": 3, "fused_step": 1}}
    del kc, new, ws, sws
    torch.cuda.empty_cache()

    if not args.no_cpu:
        threads = os.cpu_count() or 1
        var = cpu_prefill_unit(C1_S, H, KVH, threads)
        res["config1"]["cpu_baseline"] = _best(var, "TFLOP/s", threads, "config 1 in full (RoPE + causal attention "
                                               "of 254 tokens): C oracle and the python/reference.py path (FP16, "
                                               "FP32)")
        g, r, e = cpu_decode_sample(C2_PAST + 1, threads, budget_s=1.0)
        var2 = {"c_oracle_f64": {"value": round(g, 3), "reps": r, "seconds": round(e, 2)}}
        for dt in ("float16", "float32"):
            g, r, e = torch_decode_sample(C2_PAST + 1, threads, dt, budget_s=1.0)
            var2[f"python_reference_{dt}"] = {"value": round(g, 3), "reps": r, "seconds": round(e, 2)}
        res["config2"]["cpu_baseline"] = _best(var2, "GB/s", threads, "config 2 in full (RoPE + append + decode at "
                                               "kv_len 4097): C oracle and the python/reference.py path (FP16, FP32)")
    return res


# --------------------------------------------------------------------------- out projection (the consumer)
OP_HIDDEN = 2048


def run_out_proj(args, dev):
    """The attention output projection at the benchmark shapes, one GPU:
    prefill GEMM over config 3's 4 x 8192 tokens per layer (36 layers, a
    distinct weight matrix per layer, fused residual add), and the decode GEMV
    of config 4 (36 layers' weights, 302 MB, larger than L2)."""
    import torch
    import b200attn
    stream = torch.cuda.Stream(device=dev)
    gen = torch.Generator(device=dev).manual_seed(SEED + 400)
    M, N, K = PF_B * PF_S, OP_HIDDEN, Q_DIM
    x = torch.empty((M, K), dtype=torch.float16, device=dev).normal_(0.0, 1.0, generator=gen)
    w = torch.empty((LAYERS, N, K), dtype=torch.float16, device=dev).normal_(0.0, 0.02, generator=gen)
    y = torch.empty((M, N), dtype=torch.float16, device=dev).normal_(0.0, 1.0, generator=gen)
    n0 = b200attn.kernel_launch_count()

    def gemm_step(st):
        for l in range(LAYERS):
            b200attn.launch_attention_out_projection(x, y, w[l], M, N, H, D, 1.0, stream=st)
    with torch.cuda.stream(stream):
        gemm_step(stream)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        steps = max(1, min(args.steps, args.prefill_steps))
        with ClockSampler(dev.index) as clocks:
            e0.record(stream)
            for _ in range(steps):
                gemm_step(stream)
            e1.record(stream)
            torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps / LAYERS
    flops = 2 * M * N * K
    tf = flops / (ms / 1e3) / 1e12
    peak = 1400.0
    pk = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(pk):
        with open(pk) as f:
            peak = float(json.load(f).get("bf16_tflops_sustained", peak))
    del x, y
    torch.cuda.empty_cache()

    # decode GEMV: one token per layer, weights of all 36 layers cycled
    xv = torch.empty((LAYERS, K), dtype=torch.float16, device=dev).normal_(0.0, 1.0, generator=gen)
    yv = torch.empty((LAYERS, N), dtype=torch.float16, device=dev).normal_(0.0, 1.0, generator=gen)

    def gemv_step(st):
        for l in range(LAYERS):
            b200attn.launch_attention_out_projection_decode(xv[l], yv[l], w[l], N, H, D, 1.0, stream=st)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        gemv_step(stream)
        torch.cuda.synchronize()
    with torch.cuda.graph(g, stream=stream):
        gemv_step(torch.cuda.current_stream())
    torch.cuda.synchronize()
    reps = 20
    with torch.cuda.stream(stream):
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            g.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    g.reset()
    us = e0.elapsed_time(e1) / reps / LAYERS * 1e3
    vbytes = N * K * 2 + K * 2 + 2 * N * 2
    hbm, hbm_kind = load_peaks()
    launches = b200attn.kernel_launch_count() - n0
    del w, xv, yv
    torch.cuda.empty_cache()
    return {"workload": f"o_proj: prefill GEMM [{M} x {K}] @ W^T [{K} x {N}] + residual per layer (config 3 tokens), "
                        f"decode GEMV W [{N} x {K}] per layer (config 4), 36 layers' weights, FP16 in/out, FP32 "
                        "accumulate",
            "prefill": {"value": round(tf, 1), "unit": "TFLOP/s", "ms_per_layer": round(ms, 4),
                        "roofline": {"bound": "tensor", "kernel": "out_proj_gemm_pair_kernel (CTA pairs)",
                                     "achieved": round(tf, 1),
                                     "peak": peak, "unit": "TFLOP/s", "frac": round(tf / peak, 4),
                                     "frac_of_nominal_2250": round(tf / 2250.0, 4),
                                     "algorithmic_flops_per_launch": flops, "peak_kind": "measured bf16 sustained"},
                        "clocks": clocks.summary()},
            "decode": {"value": round(vbytes / us / 1e3, 1), "unit": "GB/s", "us_per_layer": round(us, 3),
                       "roofline": {"bound": "hbm", "kernel": "out_proj_gemv_kernel",
                                    "achieved": round(vbytes / us / 1e3, 1), "peak": hbm, "unit": "GB/s",
                                    "frac": round(vbytes / us / 1e3 / hbm, 4), "peak_kind": hbm_kind,
                                    "algorithmic_bytes_per_launch": vbytes,
                                    "timing": f"one CUDA graph of 36 launches (distinct weights), {reps} replays"}},
            "gpu_launches": launches}


def run_qkv_proj(args, dev):
    """The QKV projection with RoPE and the KV append in its epilogue, at the
    benchmark shapes, one GPU: per layer and per config-3 sequence, [8192 x
    2048] @ W_qkv^T [2048 x 3072] into the [Q | K | V] rows, Q rotated in
    place, rotated K and V into the sequence's cache rows (NoPE every 4th
    layer), 36 layers' weights. Timed beside the two launches it replaces
    (the GEMM, then the RoPE/append kernel over its rows)."""
    import torch
    import b200attn
    stream = torch.cuda.Stream(device=dev)
    gen = torch.Generator(device=dev).manual_seed(SEED + 500)
    M, N, K = PF_S, QKV, OP_HIDDEN
    x = torch.empty((PF_B, M, K), dtype=torch.float16, device=dev).normal_(0.0, 1.0, generator=gen)
    w = torch.empty((LAYERS, N, K), dtype=torch.float16, device=dev).normal_(0.0, 0.02, generator=gen)
    qkv = torch.empty((PF_B, M, N), dtype=torch.float16, device=dev)
    # one cache pair per sequence, reused by every layer (the write traffic is the same)
    cache = torch.empty((PF_B, 2, M, KV_DIM), dtype=torch.float16, device=dev)
    cos, sin = b200attn.rope_tables_host(M, D, 5.0e6)
    dcos, dsin = torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev)
    n0 = b200attn.kernel_launch_count()

    def fused_step(st):
        for l in range(LAYERS):
            for b in range(PF_B):
                b200attn.launch_qkv_gemm_rope_store_kv(x[b], qkv[b], w[l], cache[b, 0], cache[b, 1], dcos, dsin, M,
                                                       K, H, KVH, D, 0, (l + 1) % 4 != 0, stream=st)

    def two_launch_step(st):
        for l in range(LAYERS):
            for b in range(PF_B):
                q = qkv[b]
                b200attn.launch_qkv_gemm(x[b], q, w[l], M, K, N, stream=st)
                b200attn.launch_rope_and_store_kv(q, q[:, Q_DIM:], q[:, Q_DIM + KV_DIM:], cache[b, 0], cache[b, 1],
                                                  dcos, dsin, M, H, KVH, D, N, N, 0, (l + 1) % 4 != 0, stream=st)

    steps = max(1, min(args.steps, args.prefill_steps))
    res = {}
    for name, fn in (("fused", fused_step), ("two_launches", two_launch_step)):
        with torch.cuda.stream(stream):
            fn(stream)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with ClockSampler(dev.index) as clocks:
                e0.record(stream)
                for _ in range(steps):
                    fn(stream)
                e1.record(stream)
                torch.cuda.synchronize()
        res[name] = (e0.elapsed_time(e1) / steps / LAYERS, clocks.summary())
    launches = b200attn.kernel_launch_count() - n0
    flops = 2 * PF_B * M * N * K
    ms, clk = res["fused"]
    tf = flops / (ms / 1e3) / 1e12
    peak = 1400.0
    pk = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(pk):
        with open(pk) as f:
            peak = float(json.load(f).get("bf16_tflops_sustained", peak))
    del x, w, qkv, cache
    torch.cuda.empty_cache()
    return {"workload": f"QKV projection per layer: {PF_B} sequences x [{M} x {K}] @ W_qkv^T [{K} x {N}] (config 3 "
                        "tokens), RoPE (NoPE every 4th layer) and the KV append in the GEMM epilogue, 36 layers' "
                        "weights, FP16 in/out, FP32 accumulate",
            "value": round(tf, 1), "unit": "TFLOP/s", "ms_per_layer": round(ms, 4),
            "two_launches_ms_per_layer": round(res["two_launches"][0], 4),
            "speedup_vs_two_launches": round(res["two_launches"][0] / ms, 3),
            "roofline": {"bound": "tensor", "kernel": "qkv_rope_gemm_pair_kernel (CTA pairs)",
                         "achieved": round(tf, 1),
                         "peak": peak, "unit": "TFLOP/s", "frac": round(tf / peak, 4),
                         "frac_of_nominal_2250": round(tf / 2250.0, 4),
                         "algorithmic_flops_per_launch": flops // PF_B, "peak_kind": "measured bf16 sustained"},
            "clocks": clk, "gpu_launches": launches}


def tp_share(args, world):
    """--tp-share S (one GPU only): run rank 0's share of an S-way KV-head
    split, to measure a tensor-parallel rank's work without the other ranks."""
    share = int(getattr(args, "tp_share", 1) or 1)
    if share > 1 and (world != 1 or KVH % share != 0):
        raise SystemExit(f"--tp-share {share} needs one GPU and a divisor of the {KVH} KV heads")
    return share


def decode_parallelism(split, hs, h_l, exchange):
    xch = ("cross-rank merge in the fused kernel over CUDA-IPC peer memory" if exchange == "peer"
           else "NCCL all-gather of rank partials + merge kernel")
    if split != "heads":
        return f"kv-split{hs.world}, {xch}"
    txt = (f"kv-heads over {hs.world} ranks: {hs.local_kv_heads} KV head(s) / {h_l} query heads per rank with only "
           "those heads' cache, output head-sharded (the layout a tensor-parallel o_proj takes)")
    if hs.group_world > 1:
        txt += f"; each KV head's range split over {hs.group_world} ranks, {xch}"
    else:
        txt += ", no exchange"
    return txt


# --------------------------------------------------------------------------- GPU arm
def run_b200(args, rank, world):
    import numpy as np
    import torch
    import b200attn
    from b200attn import dist as bdist

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    split = args.decode_split
    if split == "auto":
        split = "heads" if world > 1 and (KVH % world == 0 or world % KVH == 0) else "kv"
    # this rank's KV heads (all of them for the KV-range split) and the ranks
    # that share them, which split the KV range among themselves
    hs = (bdist.head_split_plan(KVH, world, rank) if split == "heads"
          else bdist.HeadSplit(world, rank, KVH, 0, KVH, tuple(range(world))))
    share = tp_share(args, world)
    if share > 1:  # one GPU running rank 0's share of a `share`-way KV-head split
        hs = bdist.HeadSplit(1, 0, KVH, 0, KVH // share, (0,))
    kvh_l = hs.local_kv_heads
    h_l = kvh_l * (H // KVH)
    q_l, kv_l = h_l * D, kvh_l * D
    plan = bdist.split_kv_plan(PAST, hs.group_world, hs.group_rank)
    capacity = plan.local_capacity(args.warmup + args.steps + 1)   # local cache rows
    max_global = PAST + args.warmup + args.steps + 1

    # ---- state: KV cache (local slice), RoPE tables, per-layer QKV rows, outputs
    gen = torch.Generator(device=dev).manual_seed(SEED + rank)
    cache = b200attn.KVCache(LAYERS, capacity, kvh_l, D, device=dev)
    for l in range(LAYERS):
        for t in (cache.get_k_cache(l), cache.get_v_cache(l)):
            t.normal_(0.0, 0.5, generator=gen)
    cos, sin = b200attn.rope_tables_host(max_global, D, 5.0e6)
    d_cos, d_sin = torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev)
    hgen = np.random.default_rng(SEED)     # identical Q/K/V rows on every rank; each takes its heads' slice
    rows_full = hgen.standard_normal((LAYERS, QKV), dtype=np.float32).astype(np.float16)
    qkv_host = torch.from_numpy(bdist.head_split_rows(rows_full, hs, H, D)).pin_memory()
    qkv = qkv_host.to(dev)
    out = torch.zeros((LAYERS, q_l), dtype=torch.float16, device=dev)
    out_host = torch.zeros_like(out, device="cpu").pin_memory()
    step_state = bdist.DecodeStepState(plan, h_l, kvh_l, D, LAYERS, capacity, max_global, dev, fused=not args.unfused,
                                       exchange=args.exchange, members=hs.group, job_world=world,
                                       job_kv_dim=KV_DIM // share, job_q_dim=Q_DIM // share,
                                       pipeline=args.pipeline_exchange)

    stream = torch.cuda.Stream(device=dev)
    group = None
    if world > 1:
        import torch.distributed as tdist
        group = tdist.group.WORLD
        if hs.group_world < world:
            # one process group per set of ranks sharing KV heads (every rank
            # creates every group, in the same order)
            for g0 in range(0, world, hs.group_world):
                g = tdist.new_group(list(range(g0, g0 + hs.group_world)))
                if rank in range(g0, g0 + hs.group_world):
                    group = g

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
    # N > 1: one untimed step right before the start event lines the ranks up
    # on the device (every layer waits for all ranks' partials), so the host
    # skew after the barrier is not timed as a wait inside the first step
    align = 1 if world > 1 else 0
    with ClockSampler(dev.index) as clocks, torch.cuda.stream(stream):
        for _ in range(align):
            graph.replay()
        ev0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        ev1.record(stream)
        torch.cuda.synchronize()
    barrier()
    ms = ev0.elapsed_time(ev1)
    ms = bdist.max_over_ranks(ms, dev) if world > 1 else ms
    total_bytes = sum(step_bytes(PAST + 1 + align + s) for s in range(args.steps)) // share
    value = total_bytes / (ms / 1e3) / 1e9

    # ---- roofline: one layer's decode launch(es), CUDA events on its stream
    peak, peak_kind = load_peaks()
    dec_ms = bdist.time_decode_launches(step_state, cache, qkv, out, stream, reps=3, d_cos=d_cos, d_sin=d_sin)
    kv_len_local = plan.local_len(PAST + 1)
    # K/V rows read, Q read, output written (+ the new K/V row read and appended)
    dec_bytes = 2 * kv_len_local * kv_l * 2 + q_l * 2 + q_l * 2 + (4 * kv_l * 2 if step_state.fused else 0)
    if step_state.fused and (plan.world == 1 or step_state.exchange == "peer"):
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
    if world == 1 and args.unfused:
        e2e = bdist.e2e_decode(cache, qkv, qkv_host, out, out_host, d_cos, d_sin, PAST, args.warmup, args.steps,
                               stream, step_state, mode="reference")
    else:
        e2e = bdist.e2e_decode(cache, qkv, qkv_host, out, out_host, d_cos, d_sin, PAST, args.warmup, args.steps,
                               stream, step_state, mode="graph", group=group)
        eager = bdist.e2e_decode(cache, qkv, qkv_host, out, out_host, d_cos, d_sin, PAST, args.warmup,
                                 args.steps, stream, step_state, mode="fused", group=group)
        e2e["eager"] = {"value": eager["value"], "ms_per_step": eager["ms_per_step"], "path": eager["path"]}
        if world == 1:
            ref_calls = bdist.e2e_decode(cache, qkv, qkv_host, out, out_host, d_cos, d_sin, PAST, args.warmup,
                                         args.steps, stream, step_state, mode="reference")
            e2e["reference_launchers"] = {"value": ref_calls["value"], "ms_per_step": ref_calls["ms_per_step"],
                                          "path": ref_calls["path"]}

    # ---- CPU baseline (rank 0, N=1): bounded sample
    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu:
        cpu = cpu_config4(os.cpu_count() or 1)

    prefill = None
    del cache
    torch.cuda.empty_cache()
    small = None
    if world == 1 and not args.no_small:
        small = run_small(args, dev)
        torch.cuda.empty_cache()
    out_proj = None
    if world == 1 and not args.no_out_proj:
        out_proj = run_out_proj(args, dev)
        torch.cuda.empty_cache()
    qkv_proj = None
    if world == 1 and not args.no_qkv_proj:
        qkv_proj = run_qkv_proj(args, dev)
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
            "data": "synthetic: KV ~N(0,0.5) (torch CUDA generator, seed 2024+rank), Q/K/V rows ~N(0,1) seeded"
                    + ("; layers pipelined across the exchange (not valid for a model)" if step_state.pipeline
                       else ""),
            "config": {"workload": WORKLOAD, "global_batch": 1, "seq_len": PAST, "layers": LAYERS,
                       "parallelism": (f"one GPU running rank 0's share of a {share}-way KV-head split ({kvh_l} KV "
                                       f"head(s) / {h_l} query heads): per-rank work, not a whole-job number"
                                       if share > 1 else
                                       decode_parallelism(split, hs, h_l, step_state.exchange) +
                                       ("; SYNTHETIC: layer l's all-gather + merge on a second stream under layer "
                                        "l+1's kernel, valid only because this benchmark's Q rows do not depend on "
                                        "the previous layer" if step_state.pipeline else "")) if world > 1
                       else "single-gpu",
                       "l2": "inputs larger than L2 (4.8 GB of KV per step)",
                       "step_graph": f"one CUDA graph per step, {launches_per_step} kernels"},
            "gpu_launches": launches_per_step * args.steps,
            "roofline": {"bound": "hbm",
                         "kernel": ("decode_tma_kernel<fused> (RoPE + append + split attention + merge)"
                                    if step_state.fused else "decode_tma_kernel + merge_partials_kernel"),
                         "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "traffic": traffic,
                         "traffic_source": TRAFFIC_NOTE.format(f="profiles/decode_traffic.json",
                                                               what="one 64K fused launch"),
                         "avg_launch_us": round(launch_ms * 1e3, 3),
                         "isolated_launch_us": round(dec_ms * 1e3, 3), "timing": timing,
                         "algorithmic_bytes_per_launch": dec_bytes},
            "clocks": clocks.summary(),
            "e2e": e2e,
            "cpu_baseline": cpu,
            "prefill": prefill,
            "ragged": ragged,
            "small": small,
            "out_projection": out_proj,
            "qkv_projection": qkv_proj,
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
    ap.add_argument("--no-small", action="store_true", help="skip the config-1/2 (latency-bound) sub-measurement")
    ap.add_argument("--no-out-proj", action="store_true", help="skip the attention output projection measurement")
    ap.add_argument("--no-qkv-proj", action="store_true", help="skip the QKV projection (+ RoPE/append) measurement")
    ap.add_argument("--tp-share", type=int, default=1,
                    help="one GPU: run rank 0's share of an S-way KV-head split of the decode and ragged legs "
                         "(per-rank work; the line says so)")
    ap.add_argument("--ragged-split", default="seqs", choices=["seqs", "heads"],
                    help="N > 1 ragged decode: whole sequences per rank, or KV heads per rank (tensor-parallel layout)")
    ap.add_argument("--decode-split", default="auto", choices=["auto", "heads", "kv"],
                    help="N > 1 decode: KV heads per rank (tensor-parallel layout; auto when the KV heads divide or "
                         "are divided by N) or KV range per rank")
    ap.add_argument("--pipeline-exchange", action="store_true",
                    help="N > 1 with --exchange nccl: overlap layer l's exchange with layer l+1 (synthetic only: "
                         "a model's next layer needs this layer's output)")
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
