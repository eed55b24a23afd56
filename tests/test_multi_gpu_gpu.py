"""Decode across GPUs (benchmark config 4's multi-GPU paths), one process per
GPU, against the oracle's attention over the whole cache.

KV split: each rank attends over its contiguous KV range, the tail rank
appends the new token, and the per-head (o, m, l) partials are merged across
ranks -- inside the fused kernel over CUDA-IPC peer memory ("peer") or by an
NCCL all-gather and a merge kernel ("nccl"); every rank's output is the whole
output. Head split: each rank owns whole GQA groups (its KV heads' cache only)
and writes its query heads' outputs; with more ranks than KV heads the ranks
of a KV head also split its range and merge among themselves. Skipped with
fewer than 2 GPUs (ranks that wait on one another are never emulated on one
GPU)."""
import os
import socket
import traceback

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
H_ALL, KVH_ALL, D = 16, 4, 128
PAST, LAYERS, STEPS = 9000, 2, 3


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, exchange, split, q, pipeline=False, heads=None):
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
        H, KVH = heads if heads is not None else (H_ALL, KVH_ALL)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        backend = "nccl" if exchange == "nccl" else "gloo"
        tdist.init_process_group(backend, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                 device_id=dev if backend == "nccl" else None)
        hs = (bdist.head_split_plan(KVH, world, rank) if split == "heads"
              else bdist.HeadSplit(world, rank, KVH, 0, KVH, tuple(range(world))))
        kvh_l = hs.local_kv_heads
        h_l = kvh_l * (H // KVH)
        q0, q1 = hs.query_heads(H)
        c0, c1 = hs.kvh_begin * D, hs.kvh_end * D
        plan = bdist.split_kv_plan(PAST, hs.group_world, hs.group_rank)
        capacity = plan.local_capacity(STEPS + 1)
        max_global = PAST + STEPS + 1
        total = H * D + 2 * KVH * D
        cos, sin = b200attn.rope_tables_host(max_global, D, 5.0e6)
        d_cos, d_sin = torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev)
        gk = [seeded_f16((max_global, KVH * D), 10 + l, std=0.5) for l in range(LAYERS)]
        gv = [seeded_f16((max_global, KVH * D), 20 + l, std=0.5) for l in range(LAYERS)]
        cache = b200attn.KVCache(LAYERS, capacity, kvh_l, D, device=dev)
        for l in range(LAYERS):
            cache.get_k_cache(l)[:plan.local_past] = torch.from_numpy(
                np.ascontiguousarray(gk[l][plan.begin:plan.end, c0:c1])).to(dev)
            cache.get_v_cache(l)[:plan.local_past] = torch.from_numpy(
                np.ascontiguousarray(gv[l][plan.begin:plan.end, c0:c1])).to(dev)
        qkv = torch.empty((LAYERS, h_l * D + 2 * kvh_l * D), dtype=torch.float16, device=dev)
        out = torch.empty((LAYERS, h_l * D), dtype=torch.float16, device=dev)
        st = bdist.DecodeStepState(plan, h_l, kvh_l, D, LAYERS, capacity, max_global, dev, fused=True,
                                   exchange=exchange, members=hs.group, job_world=world, pipeline=pipeline)
        st.reset_position(PAST)
        stream = torch.cuda.Stream(device=dev)
        group = None
        if exchange == "nccl":
            group = tdist.group.WORLD
            if hs.group_world < world:
                for g0 in range(0, world, hs.group_world):
                    g = tdist.new_group(list(range(g0, g0 + hs.group_world)))
                    if g0 <= rank < g0 + hs.group_world:
                        group = g
        for t in range(STEPS):
            p = PAST + t
            news = [seeded_f16(total, 500 + 10 * t + l) for l in range(LAYERS)]
            for l in range(LAYERS):
                qkv[l].copy_(torch.from_numpy(bdist.head_split_rows(news[l], hs, H, D)).to(dev))
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
                assert_attention_close(out[l].cpu().numpy(), o32.reshape(H, D)[q0:q1].reshape(-1))
        assert b200attn.lib().b2_device_error_word() == 0
        tdist.barrier()
        st.close()
        tdist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception:
        q.put((rank, traceback.format_exc()))


def _run(exchange, split="kv", max_world=4, pipeline=False, heads=None):
    import torch
    import multiprocessing as mp
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 or more GPUs (one process per GPU)")
    world = min(n, max_world)
    kvh = heads[1] if heads is not None else KVH_ALL
    if split == "heads" and kvh % world != 0 and world % kvh != 0:
        world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, exchange, split, q, pipeline, heads))
             for r in range(world)]
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


def test_kv_split_decode_nccl_exchange_pipelined(cuda):
    """Each layer's all-gather + merge on a second stream under the next
    layer's kernel (the synthetic benchmark's mode): same outputs."""
    _run("nccl", pipeline=True)


def test_head_split_decode(cuda):
    """KV heads over up to 4 ranks: no exchange, head-sharded output."""
    _run("peer", "heads")


def test_head_split_decode_with_range_split_peer(cuda):
    """8 ranks over 4 KV heads: rank pairs split each head's range and merge
    over peer memory (runs at the 2 or 4 GPUs there are as the plain head
    split when fewer than 8)."""
    _run("peer", "heads", max_world=8)


def test_head_split_decode_with_range_split_nccl(cuda):
    _run("nccl", "heads", max_world=8)


@pytest.mark.parametrize("exchange", ["peer", "nccl"])
def test_one_kv_head_range_split_across_all_ranks(cuda, exchange):
    """A model with one KV head (4 query heads): the head split gives every
    rank the same head, so all ranks split its range and exchange -- the
    sub-tiled one-head stages together with the cross-rank merge, on as many
    GPUs as there are (up to 8)."""
    _run(exchange, "heads", max_world=8, heads=(4, 1))
