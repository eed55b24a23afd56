"""KV-split decode across GPUs (benchmark config 4's multi-GPU path), one
process per GPU: each rank attends over its contiguous KV range, the tail rank
appends the new token, and the per-head (o, m, l) partials are merged across
ranks -- inside the fused kernel over CUDA-IPC peer memory ("peer") or by an
NCCL all-gather and a merge kernel ("nccl"). Every rank's output must match
the oracle's attention over the whole cache. Skipped with fewer than 2 GPUs
(ranks that wait on one another are never emulated on one GPU)."""
import os
import socket
import traceback

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
H, KVH, D = 16, 4, 128
PAST, LAYERS, STEPS = 9000, 2, 3


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, exchange, q):
    try:
        import sys
        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        for p in (root, os.path.join(root, "llm-inference_b200"), os.path.join(root, "tests")):
            sys.path.insert(0, p)
        import datetime
        import torch
        import torch.distributed as tdist
        import b200attn
        import oracle
        from b200attn import dist as bdist
        from _util import assert_attention_close, seeded_f16
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        backend = "nccl" if exchange == "nccl" else "gloo"
        tdist.init_process_group(backend, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                 device_id=dev if backend == "nccl" else None)
        plan = bdist.split_kv_plan(PAST, world, rank)
        capacity = plan.local_capacity(STEPS + 1)
        max_global = PAST + STEPS + 1
        total = H * D + 2 * KVH * D
        cos, sin = b200attn.rope_tables_host(max_global, D, 5.0e6)
        d_cos, d_sin = torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev)
        gk = [seeded_f16((max_global, KVH * D), 10 + l, std=0.5) for l in range(LAYERS)]
        gv = [seeded_f16((max_global, KVH * D), 20 + l, std=0.5) for l in range(LAYERS)]
        cache = b200attn.KVCache(LAYERS, capacity, KVH, D, device=dev)
        for l in range(LAYERS):
            cache.get_k_cache(l)[:plan.local_past] = torch.from_numpy(gk[l][plan.begin:plan.end]).to(dev)
            cache.get_v_cache(l)[:plan.local_past] = torch.from_numpy(gv[l][plan.begin:plan.end]).to(dev)
        qkv = torch.empty((LAYERS, total), dtype=torch.float16, device=dev)
        out = torch.empty((LAYERS, H * D), dtype=torch.float16, device=dev)
        st = bdist.DecodeStepState(plan, H, KVH, D, LAYERS, capacity, max_global, dev, fused=True,
                                   exchange=exchange)
        st.reset_position(PAST)
        stream = torch.cuda.Stream(device=dev)
        group = tdist.group.WORLD if exchange == "nccl" else None
        for t in range(STEPS):
            p = PAST + t
            news = [seeded_f16(total, 500 + 10 * t + l) for l in range(LAYERS)]
            for l in range(LAYERS):
                qkv[l].copy_(torch.from_numpy(news[l]).to(dev))
            torch.cuda.synchronize()
            with torch.cuda.stream(stream):
                bdist.enqueue_decode_step(st, cache, qkv, out, d_cos, d_sin, stream, group)
            torch.cuda.synchronize()
            for l in range(LAYERS):
                qd, kd = H * D, KVH * D
                oq, ok, ov = news[l][:qd].copy(), news[l][qd:qd + kd].copy(), news[l][qd + kd:].copy()
                rotate = (l + 1) % 4 != 0
                oracle.rope_and_store_kv(oq, ok, ov, gk[l], gv[l], cos, sin, 1, H, KVH, D, qd, kd, p, rotate)
                _, o32 = oracle.decode_attention(oq, gk[l], gv[l], p + 1, H, KVH, D)
                assert_attention_close(out[l].cpu().numpy(), o32.reshape(-1))
        assert b200attn.lib().b2_device_error_word() == 0
        tdist.barrier()
        st.close()
        tdist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception:
        q.put((rank, traceback.format_exc()))


def _run(exchange):
    import torch
    import multiprocessing as mp
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 or more GPUs (one process per GPU)")
    world = min(n, 4)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, exchange, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            r, msg = q.get(timeout=300)
            results[r] = msg
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    bad = {r: m for r, m in results.items() if m != "ok"}
    assert not bad, bad


def test_kv_split_decode_peer_exchange(cuda):
    _run("peer")


def test_kv_split_decode_nccl_exchange(cuda):
    _run("nccl")
