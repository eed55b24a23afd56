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


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_head_split_plan_partitions(world):
    KVH, H = 4, 16
    plans = [bdist.head_split_plan(KVH, world, r) for r in range(world)]
    # every rank's group contains it, groups are equal and disjoint
    groups = {p.group for p in plans}
    assert all(p.rank in p.group for p in plans)
    assert sorted(r for g in groups for r in g) == list(range(world))
    # each group owns a distinct block of KV heads, the blocks cover all heads
    heads = sorted((p.kvh_begin, p.kvh_end) for p in plans if p.group_rank == 0)
    assert heads[0][0] == 0 and heads[-1][1] == KVH
    assert all(a[1] == b[0] for a, b in zip(heads, heads[1:]))
    for p in plans:
        q0, q1 = p.query_heads(H)
        assert (q1 - q0) == p.local_kv_heads * (H // KVH)
        assert p.group_world * len(groups) == world


def test_head_split_plan_rejects_uneven():
    with pytest.raises(ValueError):
        bdist.head_split_plan(4, 3, 0)


def test_head_split_rows_slices_qkv():
    H, KVH, d = 16, 4, 8
    rows = np.arange(2 * (H + 2 * KVH) * d, dtype=np.float32).reshape(2, -1)
    qd, kd = H * d, KVH * d
    for world in (2, 4):
        got = [bdist.head_split_rows(rows, bdist.head_split_plan(KVH, world, r), H, d) for r in range(world)]
        assert np.array_equal(np.concatenate([g[:, :qd // world] for g in got], axis=1), rows[:, :qd])
        assert np.array_equal(np.concatenate([g[:, qd // world:qd // world + kd // world] for g in got], axis=1),
                              rows[:, qd:qd + kd])
        assert np.array_equal(np.concatenate([g[:, qd // world + kd // world:] for g in got], axis=1),
                              rows[:, qd + kd:])


def _head_rank_main(rank, world, port, q, k, v, L, H, KVH, d, out):
    """Head split with a range split inside each head group (world > KVH):
    the rank's heads over its range, partials all-gathered within the group."""
    import torch
    import torch.distributed as tdist
    import oracle
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    tdist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        hs = bdist.head_split_plan(KVH, world, rank)
        groups = [tdist.new_group(list(range(g0, g0 + hs.group_world))) for g0 in range(0, world, hs.group_world)]
        group = groups[rank // hs.group_world]
        plan = bdist.split_kv_plan(L, hs.group_world, hs.group_rank)
        q0, q1 = hs.query_heads(H)
        c0, c1 = hs.kvh_begin * d, hs.kvh_end * d
        hl, kvl = q1 - q0, hs.local_kv_heads
        n = plan.end - plan.begin
        po, pm, pl = oracle.decode_partials(np.ascontiguousarray(q[q0 * d:q1 * d]),
                                            np.ascontiguousarray(k[plan.begin:plan.end, c0:c1]),
                                            np.ascontiguousarray(v[plan.begin:plan.end, c0:c1]), n, hl, kvl, d, 0,
                                            256)
        M = pm.max(axis=1)
        w = np.exp(pm - M[:, None])
        part = torch.from_numpy(np.concatenate([(w[:, :, None] * po).sum(axis=1).ravel(), M,
                                                (w * pl).sum(axis=1)]).astype(np.float32))
        gathered = torch.zeros(hs.group_world * part.numel(), dtype=torch.float32)
        tdist.all_gather_into_tensor(gathered, part, group=group)
        g = gathered.numpy().reshape(hs.group_world, -1)
        parts = [(g[r, :hl * d].reshape(hl, d), g[r, hl * d:hl * d + hl], g[r, hl * d + hl:])
                 for r in range(hs.group_world)]
        out[rank] = (q0, bdist.merge_rank_partials_reference(parts).astype(np.float32).ravel().tolist())
    finally:
        tdist.destroy_process_group()


def test_head_split_with_range_split_four_gloo_ranks():
    """4 ranks over 2 KV heads: two groups of two ranks, each group one KV head
    (its 4 query heads) split over its two ranks; every rank's heads against
    the oracle's attention over the whole cache."""
    import torch.multiprocessing as mp
    import oracle
    H, KVH, d, L, world = 8, 2, 64, 2000, 4
    rng = np.random.default_rng(6)
    q = rng.standard_normal(H * d, dtype=np.float32).astype(np.float16)
    k = (rng.standard_normal((L, KVH * d), dtype=np.float32) * 0.5).astype(np.float16)
    v = (rng.standard_normal((L, KVH * d), dtype=np.float32) * 0.5).astype(np.float16)
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    out = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_head_rank_main, args=(r, world, port, q, k, v, L, H, KVH, d, out))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    _, ref = oracle.decode_attention(q, k, v, L, H, KVH, d)
    ref = ref.reshape(H, d)
    for r in range(world):
        q0, got = out[r]
        got = np.asarray(got, np.float32).reshape(-1, d)
        assert np.max(np.abs(got - ref[q0:q0 + got.shape[0]])) <= 1e-3


def test_head_split_rows_torch_matches_numpy():
    import torch
    H, KVH, d = 16, 4, 8
    rows = np.random.default_rng(3).standard_normal((3, (H + 2 * KVH) * d)).astype(np.float32)
    for world in (1, 2, 4, 8):
        for r in range(world):
            hs = bdist.head_split_plan(KVH, world, r)
            a = bdist.head_split_rows(rows, hs, H, d)
            b = bdist.head_split_rows(torch.from_numpy(rows), hs, H, d)
            assert isinstance(b, torch.Tensor) and b.is_contiguous()
            np.testing.assert_array_equal(a, b.numpy())
            assert a.shape[-1] == hs.local_kv_heads * (H // KVH + 2) * d
