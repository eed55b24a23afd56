"""Multi-GPU host logic on CPU: work partitions, and the KV-split decode
exchange (partial per rank -> all-gather -> merge) run as 2 gloo ranks.
The per-rank compute here is the CPU oracle; on GPUs it is
b2_launch_decode_rank_partial_devlen + NCCL + b2_launch_merge_partials_strided."""
import os
import socket

import numpy as np
import pytest

from b200attn import dist as bdist


@pytest.mark.parametrize("past,world", [(65536, 1), (65536, 2), (65536, 8), (1000, 3), (7, 4), (5, 8)])
def test_split_kv_plan_covers_range(past, world):
    plans = [bdist.split_kv_plan(past, world, r) for r in range(world)]
    assert plans[0].begin == 0 and plans[-1].end == past
    for a, b in zip(plans, plans[1:]):
        assert a.end == b.begin
    sizes = [p.local_past for p in plans]
    assert max(sizes) - min(sizes) <= 1
    assert [p.is_tail for p in plans] == [False] * (world - 1) + [True]
    # the tail owns every appended token; the others are fixed
    for p in plans:
        assert p.local_len(past + 5) == p.local_past + (5 if p.is_tail else 0)
        assert p.local_capacity(9) == p.local_past + (9 if p.is_tail else 0)


def test_assign_sequences_balanced_and_complete():
    rng = np.random.default_rng(0)
    lens = rng.integers(512, 16385, 64)   # benchmark config 5
    for world in (1, 2, 4, 8):
        parts = bdist.assign_sequences(lens, world)
        got = sorted(i for p in parts for i in p)
        assert got == list(range(64))
        loads = [int(sum(lens[i] for i in p)) for p in parts]
        assert max(loads) - min(loads) <= int(lens.max())


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_prefill_shard_blocks_partition(world):
    """Config 3 (4 sequences x 4 KV heads): every (sequence, KV head) unit
    belongs to exactly one rank's contiguous block, equal work per rank."""
    shards = [bdist.prefill_shard(4, 4, world, r) for r in range(world)]
    assert all(sh is not None for sh in shards)
    units = [u for sh in shards for u in sh.units()]
    assert sorted(units) == [(b, g) for b in range(4) for g in range(4)]
    assert len({len(sh.units()) for sh in shards}) == 1
    assert bdist.prefill_shard(4, 4, 3, 0) is None


def test_prefill_units_partition():
    for world in (1, 2, 4, 8):
        units = [bdist.prefill_units(4, 4, world, r) for r in range(world)]
        flat = sorted(u for us in units for u in us)
        assert flat == [(b, h) for b in range(4) for h in range(4)]
        assert len({len(u) for u in units}) == 1   # 16 equal units: 16/8/4/2 per rank


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q, k, v, L, H, KVH, d, out):
    import torch
    import torch.distributed as tdist
    import oracle
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    tdist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        plan = bdist.split_kv_plan(L, world, rank)
        n = plan.end - plan.begin
        po, pm, pl = oracle.decode_partials(q, np.ascontiguousarray(k[plan.begin:plan.end]),
                                            np.ascontiguousarray(v[plan.begin:plan.end]), n, H, KVH, d, 0, 256)
        # reduce the rank's chunks to one partial per head (what the merge kernel writes)
        M = pm.max(axis=1)
        w = np.exp(pm - M[:, None])
        o = (w[:, :, None] * po).sum(axis=1)
        l_ = (w * pl).sum(axis=1)
        part = torch.from_numpy(np.concatenate([o.ravel(), M, l_]).astype(np.float32))
        gathered = torch.zeros(world * part.numel(), dtype=torch.float32)
        tdist.all_gather_into_tensor(gathered, part)
        g = gathered.numpy().reshape(world, -1)
        parts = [(g[r, :H * d].reshape(H, d), g[r, H * d:H * d + H], g[r, H * d + H:]) for r in range(world)]
        res = bdist.merge_rank_partials_reference(parts)
        out[rank] = res.astype(np.float32).ravel().tolist()
    finally:
        tdist.destroy_process_group()


def test_kv_split_exchange_two_gloo_ranks():
    import torch.multiprocessing as mp
    import oracle
    H, KVH, d, L, world = 16, 4, 128, 3000, 2
    rng = np.random.default_rng(5)
    q = rng.standard_normal(H * d, dtype=np.float32).astype(np.float16)
    k = (rng.standard_normal((L, KVH * d), dtype=np.float32) * 0.5).astype(np.float16)
    v = (rng.standard_normal((L, KVH * d), dtype=np.float32) * 0.5).astype(np.float16)
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    out = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q, k, v, L, H, KVH, d, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    _, ref = oracle.decode_attention(q, k, v, L, H, KVH, d)
    for r in range(world):
        got = np.asarray(out[r], np.float32)
        assert np.max(np.abs(got - ref.ravel())) <= 1e-3
