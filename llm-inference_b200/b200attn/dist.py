"""Work partitioning across GPUs and the decode-step driver.

The reference engine is single-GPU (include/model_inference.hpp). Across the
GPUs of one box the attention path shards where it naturally does:

* long-context decode -- by KV head (`head_split_plan`: each rank owns whole
  GQA groups and their cache, no exchange, the output head-sharded as a
  tensor-parallel o_proj takes it), or by KV range (`split_kv_plan`: contiguous
  ranges, the rank that holds the tail appends the new token, every rank
  reduces its range to one (o, m, l) partial per head, the partials are
  exchanged and merged with the reference's chunk-merge algebra), or both
  when there are more ranks than KV heads;
* batched prefill -- independent (sequence, KV head) units (`prefill_units`);
* ragged decode -- whole sequences, longest first (`assign_sequences`).

The partition functions are pure host logic; `enqueue_decode_step` issues one
decode step (all layers) on a stream so it can be captured in a CUDA graph.
"""
from __future__ import annotations

import dataclasses

H_DEFAULT = 16


@dataclasses.dataclass(frozen=True)
class SplitPlan:
    """Rank `rank` of `world` owns global KV rows [begin, end) of the first
    `past` tokens; the last rank also owns every appended token."""
    past: int
    world: int
    rank: int
    begin: int
    end: int

    @property
    def is_tail(self) -> bool:
        return self.rank == self.world - 1

    @property
    def local_past(self) -> int:
        return self.end - self.begin

    def local_capacity(self, extra: int) -> int:
        """Rows this rank's cache needs for `extra` appended tokens."""
        return self.local_past + (extra if self.is_tail else 0)

    def local_len(self, global_len: int) -> int:
        """Rows of this rank's range inside a cache of global_len tokens."""
        return max(0, min(global_len, self.end if not self.is_tail else global_len) - self.begin)


def split_kv_plan(past: int, world: int, rank: int) -> SplitPlan:
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    base, rem = divmod(past, world)
    begin = rank * base + min(rank, rem)
    end = begin + base + (1 if rank < rem else 0)
    return SplitPlan(past, world, rank, begin, end)


@dataclasses.dataclass(frozen=True)
class HeadSplit:
    """Rank `rank` of `world` decodes KV heads [kvh_begin, kvh_end) and their
    query heads (GQA keeps each KV head's query group together), with its own
    cache holding only those heads, as a tensor-parallel engine shards them.
    When there are more ranks than KV heads, the `group` of ranks that share a
    KV head also splits its KV range (split_kv_plan over the group) and merges
    across the group."""
    world: int
    rank: int
    num_kv_heads: int
    kvh_begin: int
    kvh_end: int
    group: tuple

    @property
    def local_kv_heads(self) -> int:
        return self.kvh_end - self.kvh_begin

    @property
    def group_world(self) -> int:
        return len(self.group)

    @property
    def group_rank(self) -> int:
        return self.group.index(self.rank)

    def query_heads(self, num_heads: int) -> tuple[int, int]:
        """Query heads [begin, end) of this rank's KV heads."""
        per = num_heads // self.num_kv_heads
        return self.kvh_begin * per, self.kvh_end * per


def head_split_plan(num_kv_heads: int, world: int, rank: int) -> HeadSplit:
    """KV heads over ranks: KVH / world heads each when world divides KVH;
    one head per world / KVH ranks (which then split its KV range) when KVH
    divides world."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    if num_kv_heads % world == 0:
        per = num_kv_heads // world
        return HeadSplit(world, rank, num_kv_heads, rank * per, (rank + 1) * per, (rank,))
    if world % num_kv_heads == 0:
        parts = world // num_kv_heads
        g = rank // parts
        return HeadSplit(world, rank, num_kv_heads, g, g + 1, tuple(g * parts + i for i in range(parts)))
    raise ValueError(f"{num_kv_heads} KV heads cannot be split evenly over {world} ranks")


def head_split_rows(rows, hs: HeadSplit, num_heads: int, head_dim: int):
    """This rank's slice of [..][Q | K | V] rows (the row a tensor-parallel QKV
    projection produces on it): its query heads, then its K heads, then its V
    heads. Works on numpy arrays and torch tensors (last axis)."""
    q0, q1 = hs.query_heads(num_heads)
    kv = hs.num_kv_heads * head_dim
    qd = num_heads * head_dim
    k0, k1 = hs.kvh_begin * head_dim, hs.kvh_end * head_dim
    parts = [rows[..., q0 * head_dim:q1 * head_dim], rows[..., qd + k0:qd + k1], rows[..., qd + kv + k0:qd + kv + k1]]
    try:
        import torch
        if isinstance(rows, torch.Tensor):
            return torch.cat(parts, dim=-1).contiguous()
    except ImportError:
        pass
    import numpy as np
    return np.ascontiguousarray(np.concatenate(parts, axis=-1))


@dataclasses.dataclass(frozen=True)
class PrefillShard:
    """Rank's block of a batched prefill: sequences [seq_begin, seq_end) x KV
    heads [kvh_begin, kvh_end), launched as one batched call."""
    seq_begin: int
    seq_end: int
    kvh_begin: int
    kvh_end: int

    def units(self) -> list[tuple[int, int]]:
        return [(b, g) for b in range(self.seq_begin, self.seq_end) for g in range(self.kvh_begin, self.kvh_end)]


def prefill_shard(batch: int, num_kv_heads: int, world: int, rank: int) -> PrefillShard | None:
    """Contiguous (sequence, KV head) block per rank when the batch divides
    evenly: whole sequences while world <= batch, else each sequence's KV heads
    split over world / batch ranks. None when no even block exists (use
    prefill_units)."""
    if world <= batch and batch % world == 0:
        per = batch // world
        return PrefillShard(rank * per, (rank + 1) * per, 0, num_kv_heads)
    if world > batch and world % batch == 0 and num_kv_heads % (world // batch) == 0:
        parts = world // batch
        per = num_kv_heads // parts
        b, p = divmod(rank, parts)
        return PrefillShard(b, b + 1, p * per, (p + 1) * per)
    return None


def prefill_units(batch: int, num_kv_heads: int, world: int, rank: int) -> list[tuple[int, int]]:
    """(sequence, kv_head) units of a batched causal prefill owned by `rank`.
    Every unit has the same causal work, so a round-robin split balances."""
    units = [(b, h) for b in range(batch) for h in range(num_kv_heads)]
    return units[rank::world]


def assign_sequences(kv_lens, world: int) -> list[list[int]]:
    """Greedy longest-first assignment of ragged sequences to ranks, balancing
    the total KV length (the decode cost) per rank."""
    order = sorted(range(len(kv_lens)), key=lambda i: (-int(kv_lens[i]), i))
    loads = [0] * world
    out: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda j: (loads[j], j))
        out[r].append(i)
        loads[r] += int(kv_lens[i])
    return [sorted(x) for x in out]


def merge_rank_partials_reference(parts):
    """Host restatement of the cross-rank merge for CPU tests: parts is a list of
    (o [H][d], m [H], l [H]) numpy arrays; returns out [H][d] float64."""
    import numpy as np
    o = np.stack([p[0] for p in parts]).astype(np.float64)
    m = np.stack([p[1] for p in parts]).astype(np.float64)
    l = np.stack([p[2] for p in parts]).astype(np.float64)
    M = m.max(axis=0)
    w = np.exp(m - M)
    return (w[:, :, None] * o).sum(axis=0) / (w * l).sum(axis=0)[:, None]


# ---------------------------------------------------------------------------
# Decode step driver (GPU). Imported lazily so the partition logic above has
# no torch / CUDA dependency.

class DecodeStepState:
    """Device-resident positions and workspaces for a graph-static decode step."""

    def __init__(self, plan: SplitPlan, num_heads, num_kv_heads, head_dim, num_layers, capacity, max_global,
                 device, fused=True, exchange="peer", members=None, job_world=None, job_kv_dim=None,
                 job_q_dim=None, pipeline=False):
        """plan: the KV split among the ranks that share this rank's heads
        (`members`, global ranks; default all ranks); num_heads / num_kv_heads
        are this rank's. job_*: the whole job's world size and widths, for the
        barrier, the max over ranks and the whole-job byte count (default: the
        plan's world and these heads). pipeline (NCCL exchange only): each
        layer's all-gather and merge run on a second stream, overlapping the
        next layer's kernel -- valid only when a layer's Q does not depend on
        the previous layer's output (the synthetic benchmark), never in a
        model."""
        import torch
        from . import kernels as K
        self.plan = plan
        # fused: one kernel per layer (RoPE + append + split attention + merge);
        # otherwise the reference's sequence of RoPE/append, split, merge launches
        self.fused = fused
        self.step_ws_bytes = K.decode_step_workspace_bytes(num_heads, num_kv_heads)
        self.step_ws = torch.zeros(self.step_ws_bytes, dtype=torch.uint8, device=device)
        # world > 1: "peer" = cross-rank merge inside the fused kernel over
        # CUDA-IPC exchange buffers; "nccl" = rank partials all-gathered by NCCL
        self.exchange = exchange if (fused and plan.world > 1) else None
        self.xbuf = None
        if self.exchange == "peer":
            import torch.distributed as tdist

            def gather(obj):
                out = [None] * tdist.get_world_size()
                tdist.all_gather_object(out, obj)
                return out if members is None else [out[r] for r in members]
            self.xbuf = K.ExchangeBuffers(plan.world, plan.rank, num_heads, gather)
        self.pipeline = bool(pipeline) and self.exchange == "nccl"
        if pipeline and not self.pipeline:
            raise ValueError("the pipelined exchange needs the fused step, N > 1 and the NCCL exchange")
        if self.pipeline:
            self.comm_stream = torch.cuda.Stream(device=device)
            self.layer_events = [torch.cuda.Event() for _ in range(num_layers)]
            self.join_event = torch.cuda.Event()
        self.H, self.KVH, self.D, self.L = num_heads, num_kv_heads, head_dim, num_layers
        self.job_world = job_world or plan.world
        self.job_kv_dim = job_kv_dim or num_kv_heads * head_dim
        self.job_q_dim = job_q_dim or num_heads * head_dim
        self.capacity = capacity
        self.max_global = max_global
        self.device = device
        # global position of the token being decoded (start_pos); kv_len = pos + 1
        self.pos = torch.zeros(1, dtype=torch.int32, device=device)
        self.local_const = torch.tensor([plan.local_past], dtype=torch.int32, device=device)
        nfl = K.decode_workspace_floats(num_heads, head_dim, capacity)
        self.ws = torch.empty(nfl, dtype=torch.float32, device=device)
        chunks = (capacity + K._kv_chunk() - 1) // K._kv_chunk()
        n = num_heads * chunks
        self.po, self.pm, self.pl = self.ws[:n * head_dim], self.ws[n * head_dim:n * (head_dim + 1)], \
            self.ws[n * (head_dim + 1):]
        w = plan.world
        per = num_heads * (head_dim + 2)
        self.rank_part = torch.zeros((num_layers, per), dtype=torch.float32, device=device)
        self.gathered = torch.zeros((num_layers, w * per), dtype=torch.float32, device=device)

    def close(self):
        if self.xbuf is not None:
            self.xbuf.close()
            self.xbuf = None

    def reset_position(self, pos: int):
        self.pos.fill_(pos)

    def kv_len_source(self):
        """(device int, bias) giving this rank's local kv_len for the step."""
        if self.plan.is_tail:
            return self.pos, 1 - self.plan.begin
        return self.local_const, 0


def enqueue_decode_step(st: DecodeStepState, cache, qkv, out, d_cos, d_sin, stream, group=None, advance=True):
    """One token through every layer: RoPE + append (tail rank), decode over the
    local KV range, exchange + merge across ranks, then advance the position
    (unless advance is False: the caller writes st.pos before each step)."""
    import torch
    from . import kernels as K
    H, KVH, D = st.H, st.KVH, st.D
    q_dim, kv_dim = H * D, KVH * D
    total = q_dim + 2 * kv_dim
    plan = st.plan
    src, bias = st.kv_len_source()
    for l in range(st.L):
        rotate = (l + 1) % 4 != 0          # include/model_inference.hpp:272 NoPE rule
        row = qkv[l]
        q, k, v = row, row[q_dim:], row[q_dim + kv_dim:]
        if st.fused:
            kn, vn = (k, v) if plan.is_tail else (None, None)
            kc, vc = cache.get_k_cache(l), cache.get_v_cache(l)
            if plan.world == 1:
                K.launch_decode_step_fused(q, kn, vn, kc, vc, d_cos, d_sin, st.max_global, rotate, st.pos, src, bias,
                                           st.capacity, out[l], st.step_ws, st.step_ws_bytes, H, KVH, D,
                                           stream=stream)
                continue
            if st.exchange == "peer":
                K.launch_decode_step_fused_exchange(q, kn, vn, kc, vc, d_cos, d_sin, st.max_global, rotate, st.pos,
                                                    src, bias, st.capacity, out[l], st.step_ws, st.step_ws_bytes,
                                                    plan.world, plan.rank, st.xbuf.ptrs, H, KVH, D, stream=stream)
                continue
            part = st.rank_part[l]
            K.launch_decode_step_fused_rank_partial(q, kn, vn, kc, vc, d_cos, d_sin, st.max_global, rotate, st.pos,
                                                    src, bias, st.capacity, part[:H * D], part[H * D:H * D + H],
                                                    part[H * D + H:], st.step_ws, st.step_ws_bytes, H, KVH, D,
                                                    stream=stream)
            if st.pipeline:
                # layer l's exchange on the side stream; layer l + 1 goes on
                st.layer_events[l].record(_as_stream(stream))
                st.comm_stream.wait_event(st.layer_events[l])
                _exchange_and_merge(st, l, part, out, group, st.comm_stream)
            else:
                _exchange_and_merge(st, l, part, out, group, stream)
            continue
        if plan.is_tail:
            # cache rows are local: global position p lives at local row p - begin
            kc = cache.get_k_cache(l)
            vc = cache.get_v_cache(l)
            off = plan.begin * kv_dim * 2
            K.launch_rope_and_store_kv_devpos(q, k, v, kc.data_ptr() - off, vc.data_ptr() - off, d_cos, d_sin, 1,
                                              H, KVH, D, total, total, st.pos, plan.begin + st.capacity, rotate,
                                              stream=stream)
        elif rotate:
            # only Q needs rotating on ranks that do not store the new token
            K.launch_rope_and_store_kv_devpos(q, q, None, None, None, d_cos, d_sin, 1, H, 0, D, total, total,
                                              st.pos, st.max_global, True, stream=stream)
        if plan.world == 1:
            K.launch_causal_attention_decode_devlen(q, cache.get_k_cache(l), cache.get_v_cache(l), out[l], st.po,
                                                    st.pm, st.pl, src, bias, st.capacity, H, KVH, D, kv_dim,
                                                    stream=stream)
        else:
            part = st.rank_part[l]
            K.launch_decode_rank_partial_devlen(q, cache.get_k_cache(l), cache.get_v_cache(l), st.po, st.pm, st.pl,
                                                src, bias, st.capacity, H, KVH, D, kv_dim, part[:H * D],
                                                part[H * D:H * D + H], part[H * D + H:], stream=stream)
            _exchange_and_merge(st, l, part, out, group, stream)
    if st.fused and getattr(st, "pipeline", False):
        st.join_event.record(st.comm_stream)
        _as_stream(stream).wait_event(st.join_event)
    if advance:
        K.advance_position(st.pos, 1, stream=stream)


def _as_stream(stream):
    import torch
    if isinstance(stream, torch.cuda.Stream):
        return stream
    return torch.cuda.current_stream()


def _exchange_and_merge(st: DecodeStepState, l, part, out, group, stream):
    """All-gather every rank's (o, m, l) partial of layer l and merge them into out[l]."""
    import torch
    import torch.distributed as tdist
    from . import kernels as K
    H, D = st.H, st.D
    with torch.cuda.stream(stream if isinstance(stream, torch.cuda.Stream) else torch.cuda.current_stream()):
        tdist.all_gather_into_tensor(st.gathered[l], part, group=group)
    per = H * (D + 2)
    g = st.gathered[l]
    K.launch_merge_partials_strided(g, g[H * D:], g[H * D + H:], out[l], H, st.plan.world, D, per, D, per, 1,
                                    stream=stream)


def max_over_ranks(value: float, device) -> float:
    import torch
    import torch.distributed as tdist
    t = torch.tensor([value], dtype=torch.float64, device=device)
    tdist.all_reduce(t, op=tdist.ReduceOp.MAX)
    return float(t.item())


def time_decode_launches(st: DecodeStepState, cache, qkv, out, stream, reps=3, d_cos=None, d_sin=None) -> float:
    """Average device time (ms) of one layer's decode launch over the local
    range at kv_len = past + 1 -- the fused step kernel when st.fused (RoPE,
    append of the same row each time, attention, merge), else split + merge --
    measured with CUDA events on its stream, cycling through the layers so the
    cache is not L2-resident."""
    import torch
    from . import kernels as K
    H, KVH, D = st.H, st.KVH, st.D
    q_dim, kv_dim = H * D, KVH * D
    src, bias = st.kv_len_source()
    st.reset_position(st.plan.past)
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(reps * st.L)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(reps * st.L)]
    i = 0
    for _ in range(reps):
        for l in range(st.L):
            row = qkv[l]
            starts[i].record(stream)
            if st.fused:
                kn, vn = (row[q_dim:], row[q_dim + kv_dim:]) if st.plan.is_tail else (None, None)
                rotate = (l + 1) % 4 != 0
                if st.plan.world == 1:
                    K.launch_decode_step_fused(row, kn, vn, cache.get_k_cache(l), cache.get_v_cache(l), d_cos, d_sin,
                                               st.max_global, rotate, st.pos, src, bias, st.capacity, out[l],
                                               st.step_ws, st.step_ws_bytes, H, KVH, D, stream=stream)
                elif st.exchange == "peer":
                    K.launch_decode_step_fused_exchange(
                        row, kn, vn, cache.get_k_cache(l), cache.get_v_cache(l), d_cos, d_sin, st.max_global, rotate,
                        st.pos, src, bias, st.capacity, out[l], st.step_ws, st.step_ws_bytes, st.plan.world,
                        st.plan.rank, st.xbuf.ptrs, H, KVH, D, stream=stream)
                else:
                    part = st.rank_part[l]
                    K.launch_decode_step_fused_rank_partial(
                        row, kn, vn, cache.get_k_cache(l), cache.get_v_cache(l), d_cos, d_sin, st.max_global, rotate,
                        st.pos, src, bias, st.capacity, part[:H * D], part[H * D:H * D + H], part[H * D + H:],
                        st.step_ws, st.step_ws_bytes, H, KVH, D, stream=stream)
            else:
                K.launch_causal_attention_decode_devlen(row, cache.get_k_cache(l), cache.get_v_cache(l), out[l],
                                                        st.po, st.pm, st.pl, src, bias, st.capacity, H, KVH, D,
                                                        kv_dim, stream=stream)
            ends[i].record(stream)
            i += 1
    torch.cuda.synchronize()
    times = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    return sum(times) / len(times)


def e2e_decode(cache, qkv, qkv_host, out, out_host, d_cos, d_sin, past, warmup, steps, stream, st,
               mode="fused", group=None) -> dict:
    """The decode metric end to end through the C ABI with host buffers: every
    step copies its Q/K/V rows (and position) in from pinned host memory, runs
    36 layers, and copies the attention outputs back.
    mode "fused": one fused-step call per layer, eager (b2_launch_decode_step_fused
    on one GPU; on N GPUs the rank's fused call with the cross-rank exchange,
    peer or NCCL as st.exchange says); the position travels with the step's
    inputs. mode "graph": the same calls and both copies captured once into a
    CUDA graph that is replayed every step, the way the reference engine runs
    its decode (include/model_inference.hpp:96-123), with the position kept on
    the device and advanced inside the graph. mode "reference" (one GPU): the
    reference engine's calls, launch_rope_and_store_kv +
    launch_causal_attention_decode_vectorized per layer with a host start_pos.
    Returns the device time, max over ranks."""
    import torch
    from . import kernels as K
    H, KVH, D, L = st.H, st.KVH, st.D, st.L
    q_dim, kv_dim = H * D, KVH * D
    total = q_dim + 2 * kv_dim
    # one pinned position word per step, written before any copy is queued (a
    # host write into a word an earlier queued copy still reads would race)
    n_pos = max(warmup, steps)
    pos_host = torch.arange(past, past + n_pos, dtype=torch.int32).pin_memory()

    def step(s):
        pos = past + s
        qkv.copy_(qkv_host, non_blocking=True)
        if mode == "fused":
            st.pos.copy_(pos_host[s:s + 1], non_blocking=True)
            enqueue_decode_step(st, cache, qkv, out, d_cos, d_sin, stream, group, advance=False)
        else:
            for l in range(L):
                row = qkv[l]
                K.launch_rope_and_store_kv(row, row[q_dim:], row[q_dim + kv_dim:], cache.get_k_cache(l),
                                           cache.get_v_cache(l), d_cos, d_sin, 1, H, KVH, D, total, total, pos,
                                           (l + 1) % 4 != 0, stream=stream)
                K.launch_causal_attention_decode_vectorized(row, cache.get_k_cache(l), cache.get_v_cache(l), out[l],
                                                            st.po, st.pm, st.pl, 1, pos + 1, pos, H, KVH, D, total,
                                                            kv_dim, stream=stream)
        out_host.copy_(out, non_blocking=True)

    graph = None
    if mode == "graph":
        st.reset_position(past)
        with torch.cuda.stream(stream):
            qkv.copy_(qkv_host, non_blocking=True)
            enqueue_decode_step(st, cache, qkv, out, d_cos, d_sin, stream, group, advance=True)
            out_host.copy_(out, non_blocking=True)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            cur = torch.cuda.current_stream()
            qkv.copy_(qkv_host, non_blocking=True)
            enqueue_decode_step(st, cache, qkv, out, d_cos, d_sin, cur, group, advance=True)
            out_host.copy_(out, non_blocking=True)
        torch.cuda.synchronize()
        st.reset_position(past)
        torch.cuda.synchronize()

        def step(s):  # noqa: F811 -- the graph replaces the eager step
            graph.replay()

    with torch.cuda.stream(stream):
        for s in range(warmup):
            step(s)
        torch.cuda.synchronize()
        if graph is not None:
            st.reset_position(past)
            torch.cuda.synchronize()
        if st.job_world > 1:
            import torch.distributed as tdist
            tdist.barrier()
            torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        # N > 1: one untimed step lines the ranks up on the device first (each
        # layer waits for every rank), so host skew is not timed
        align = 1 if st.job_world > 1 else 0
        for _ in range(align):
            step(0)
        e0.record(stream)
        for s in range(steps):
            step(s)
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if graph is not None:
        graph.reset()
    if st.job_world > 1:
        ms = max_over_ranks(ms, qkv.device)
    # whole-job bytes: every layer's full KV range (all ranks' shares, all heads)
    jkv, jq = st.job_kv_dim, st.job_q_dim
    # the graph advances the position on the device, so after the aligning
    # step the timed steps run one token further
    first = past + 1 + (align if graph is not None else 0)
    nbytes = sum(L * (2 * (first + s) * jkv * 2 + jq * 2 * 2 + 2 * jkv * 2) for s in range(steps))
    h2d = int(qkv_host.numel() * 2) + (4 if mode == "fused" else 0)
    if mode == "graph":
        return {"value": round(nbytes / (ms / 1e3) / 1e9, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": int(out_host.numel() * 2), "ms_per_step": round(ms / steps, 4),
                "path": "one CUDA graph per step replayed through the C ABI (as the reference engine runs decode): "
                        "the step's Q/K/V rows H2D from pinned memory, the " + str(L) + " fused-step calls "
                        "(b2_launch_decode_step_fused" + ("" if st.plan.world == 1 else
                                                          ", cross-rank exchange " + str(st.exchange)) +
                        ") with the position on the device, the outputs D2H"}
    fused_call = ("b2_launch_decode_step_fused" + (" on this rank's KV heads" if st.job_world > 1 else "")
                  if st.plan.world == 1 else
                  "b2_launch_decode_step_fused_exchange (cross-rank merge over peer memory)"
                  if st.exchange == "peer" else
                  "b2_launch_decode_step_fused_rank_partial + NCCL all-gather + b2_launch_merge_partials_strided")
    path = (f"C-ABI {fused_call} per layer (eager launches, device position copied in with the "
            "step's rows), pinned H2D/D2H each step" if mode == "fused" else
            "C-ABI launch_rope_and_store_kv + launch_causal_attention_decode_vectorized per layer (the reference "
            "engine's calls), host start_pos, pinned H2D/D2H each step")
    return {"value": round(nbytes / (ms / 1e3) / 1e9, 2), "unit": "GB/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": int(out_host.numel() * 2),
            "ms_per_step": round(ms / steps, 4), "path": path}
