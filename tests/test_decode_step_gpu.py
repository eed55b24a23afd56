"""Fused decode step (per layer: one split-attention kernel that also rotates the
new token and appends its K/V, with dynamically claimed tiles, then the merge)
on the GPU vs the CPU oracle and vs the reference's launch sequence (rope.hip.cpp:138-196 launch_rope_and_store_kv,
then causal_attention.hip.cpp:840-921 launch_causal_attention_decode)."""
import numpy as np
import pytest

import b200attn
import oracle
from _gpu import Graph, bits, dev, host
from _util import assert_attention_close, seeded_f16

pytestmark = pytest.mark.gpu
H, KVH, D = 16, 4, 128
THETA = 5.0e6
GUARD = np.float16(77.0)


def _sync():
    import torch
    torch.cuda.synchronize()


def _workspace(heads=H, kvh=KVH):
    import torch
    n = b200attn.decode_step_workspace_bytes(heads, kvh)
    return torch.zeros(n, dtype=torch.uint8, device="cuda"), n


def _oracle_step(qkv, hist_k, hist_v, cap, pos, row, cos, sin, rotate, heads=H, kvh=KVH):
    """Oracle: append the new token at cache row `row` (RoPE at `pos`), attend rows [0, row]."""
    qd, kd = heads * D, kvh * D
    oq, ok, ov = qkv[:qd].copy(), qkv[qd:qd + kd].copy(), qkv[qd + kd:].copy()
    kc = np.full((cap, kd), GUARD, np.float16)
    vc = kc.copy()
    kc[:row], vc[:row] = hist_k[:row], hist_v[:row]
    if rotate:
        # rope_and_store_kv appends at start_pos; rotate at pos, then move the row
        tk, tv = np.zeros((pos + 1, kd), np.float16), np.zeros((pos + 1, kd), np.float16)
        oracle.rope_and_store_kv(oq, ok, ov, tk, tv, cos, sin, 1, heads, kvh, D, qd, kd, pos, True)
        kc[row], vc[row] = tk[pos], tv[pos]
    else:
        kc[row], vc[row] = ok, ov
    _, o32 = oracle.decode_attention(oq, kc, vc, row + 1, heads, kvh, D)
    return kc, vc, o32.reshape(-1)


def _fused(qkv_d, kc, vc, cos_d, sin_d, rope_rows, rotate, pos_d, len_d, bias, cap, out, ws, heads=H, kvh=KVH,
           append=True):
    qd, kd = heads * D, kvh * D
    b200attn.launch_decode_step_fused(qkv_d, qkv_d[qd:] if append else None, qkv_d[qd + kd:] if append else None,
                                      kc, vc, cos_d if rotate else None, sin_d if rotate else None, rope_rows,
                                      rotate, pos_d, len_d, bias, cap, out, ws[0], ws[1], heads, kvh, D)


@pytest.mark.parametrize("kv_len", [1, 2, 16, 17, 255, 256, 257, 3000, 4097, 37000])
@pytest.mark.parametrize("rotate", [True, False])
def test_fused_step_matches_oracle(cuda, kv_len, rotate):
    import torch
    cap = kv_len + 40
    hist_k = seeded_f16((cap, KVH * D), 1000 + kv_len)
    hist_v = seeded_f16((cap, KVH * D), 2000 + kv_len)
    qkv = seeded_f16(H * D + 2 * KVH * D, 3000 + kv_len)
    cos, sin = b200attn.rope_tables_host(cap + 8, D, THETA)
    pos = kv_len - 1
    exp_k, exp_v, o32 = _oracle_step(qkv, hist_k, hist_v, cap, pos, pos, cos, sin, rotate)

    init_k = exp_k.copy()
    init_v = exp_v.copy()
    init_k[pos] = GUARD  # the kernel must write the new row
    init_v[pos] = GUARD
    kc, vc = dev(init_k), dev(init_v)
    qkv_d = dev(qkv)
    pos_d = torch.tensor([pos], dtype=torch.int32, device=cuda)
    out = torch.full((H * D,), -123.0, dtype=torch.float16, device=cuda)
    ws = _workspace()
    _fused(qkv_d, kc, vc, dev(cos), dev(sin), cos.shape[0], rotate, pos_d, pos_d, 1, cap, out, ws)
    _sync()
    np.testing.assert_array_equal(bits(host(kc)), bits(exp_k))
    np.testing.assert_array_equal(bits(host(vc)), bits(exp_v))
    np.testing.assert_array_equal(bits(host(qkv_d)), bits(qkv))  # Q is read, not written
    got = host(out)
    assert_attention_close(got, o32)
    # same result as the reference's launch sequence on this library's kernels
    kc2, vc2 = dev(init_k), dev(init_v)
    qkv2 = dev(qkv)
    if rotate:
        b200attn.launch_rope_and_store_kv_devpos(qkv2, qkv2[H * D:], qkv2[H * D + KVH * D:], kc2, vc2, dev(cos),
                                                 dev(sin), 1, H, KVH, D, 0, 0, pos_d, cos.shape[0], True)
    else:
        kc2[pos] = qkv2[H * D:H * D + KVH * D]
        vc2[pos] = qkv2[H * D + KVH * D:]
    wsf = torch.empty(b200attn.decode_workspace_floats(H, D, cap), dtype=torch.float32, device=cuda)
    n = H * ((cap + 255) // 256)
    out2 = torch.empty(H * D, dtype=torch.float16, device=cuda)
    b200attn.launch_causal_attention_decode_devlen(qkv2, kc2, vc2, out2, wsf[:n * D], wsf[n * D:n * (D + 1)],
                                                   wsf[n * (D + 1):], pos_d, 1, cap, H, KVH, D)
    _sync()
    two = host(out2).astype(np.float32)
    assert np.max(np.abs(got.astype(np.float32) - two)) <= 2e-3
    assert b200attn.lib().b2_device_error_word() == 0


def test_fused_step_workspace_counters_return_to_zero(cuda):
    """Many calls on one workspace (lengths spanning 1..148+ splits) each match
    the oracle: a call that left its tile counter non-zero would make the next
    one skip tiles."""
    import torch
    cap = 50000
    hist_k = seeded_f16((cap, KVH * D), 41, std=0.5)
    hist_v = seeded_f16((cap, KVH * D), 42, std=0.5)
    kc, vc = dev(hist_k), dev(hist_v)
    cos, sin = b200attn.rope_tables_host(cap, D, THETA)
    cos_d, sin_d = dev(cos), dev(sin)
    ws = _workspace()
    for i, kv_len in enumerate([5000, 300, 49999, 1, 12 * 256 + 1, 37 * 256, 148 * 256 + 7, 800]):
        qkv = seeded_f16(H * D + 2 * KVH * D, 50 + i, std=0.5)
        # no append: attend the stored history only
        qkv_d = dev(qkv)
        ln = torch.tensor([kv_len], dtype=torch.int32, device=cuda)
        pos = torch.tensor([kv_len - 1], dtype=torch.int32, device=cuda)
        out = torch.empty(H * D, dtype=torch.float16, device=cuda)
        _fused(qkv_d, kc, vc, cos_d, sin_d, cap, True, pos, ln, 0, cap, out, ws, append=False)
        _sync()
        oq = qkv[:H * D].copy()
        ok = qkv[H * D:H * D + KVH * D].copy()
        oracle.rope_and_store_kv(oq, ok, None, None, None, cos, sin, 1, H, KVH, D, H * D, KVH * D, kv_len - 1, True)
        _, o32 = oracle.decode_attention(oq, hist_k, hist_v, kv_len, H, KVH, D)
        assert_attention_close(host(out), o32.reshape(-1))
    assert b200attn.lib().b2_device_error_word() == 0


def test_fused_step_length_written_by_previous_kernel(cuda):
    """The kernel reads the length before its dependency wait to warm its first
    tiles in L2; when the kernel before it on the stream writes that length
    (here: a long fused step on another cache, then the position advance), the
    early read is usually stale. The output must be that of the new length,
    for a longer and a shorter new length."""
    import torch
    cap = 9000
    hist_k = seeded_f16((cap, KVH * D), 141, std=0.5)
    hist_v = seeded_f16((cap, KVH * D), 142, std=0.5)
    kc, vc = dev(hist_k), dev(hist_v)
    cos, sin = b200attn.rope_tables_host(cap, D, THETA)
    cos_d, sin_d = dev(cos), dev(sin)
    # the long kernel in front: a 64K step on its own cache and workspace
    big = 65536 + 8
    fk = torch.zeros((big, KVH * D), dtype=torch.float16, device=cuda)
    fv = torch.zeros_like(fk)
    fq = dev(seeded_f16(H * D + 2 * KVH * D, 143))
    fpos = torch.tensor([65536], dtype=torch.int32, device=cuda)
    fout = torch.empty(H * D, dtype=torch.float16, device=cuda)
    fws = _workspace()
    ws = _workspace()
    for start, delta in ((3000, 1000), (6000, -2500)):
        qkv = seeded_f16(H * D + 2 * KVH * D, 150 + start, std=0.5)
        qkv_d = dev(qkv)
        ln = torch.tensor([start], dtype=torch.int32, device=cuda)  # kv_len = ln, attended history only
        pos = torch.tensor([start + delta - 1], dtype=torch.int32, device=cuda)
        out = torch.empty(H * D, dtype=torch.float16, device=cuda)
        _sync()
        _fused(fq, fk, fv, cos_d, sin_d, big, False, fpos, fpos, 1, big, fout, fws, append=False)
        b200attn.advance_position(ln, delta)
        _fused(qkv_d, kc, vc, cos_d, sin_d, cap, True, pos, ln, 0, cap, out, ws, append=False)
        _sync()
        kv_len = start + delta
        oq = qkv[:H * D].copy()
        ok = qkv[H * D:H * D + KVH * D].copy()
        oracle.rope_and_store_kv(oq, ok, None, None, None, cos, sin, 1, H, KVH, D, H * D, KVH * D, kv_len - 1, True)
        _, o32 = oracle.decode_attention(oq, hist_k, hist_v, kv_len, H, KVH, D)
        assert_attention_close(host(out), o32.reshape(-1))
    assert b200attn.lib().b2_device_error_word() == 0


def test_fused_step_graph_decode_sequence(cuda):
    """A captured 2-layer step replayed for 6 tokens with a device position:
    every token's output of both layers matches the oracle's sequential decode."""
    import torch
    cap, start, steps = 2048, 700, 6
    layers = 2
    cos, sin = b200attn.rope_tables_host(cap, D, THETA)
    cos_d, sin_d = dev(cos), dev(sin)
    hist = [(seeded_f16((cap, KVH * D), 60 + l), seeded_f16((cap, KVH * D), 70 + l)) for l in range(layers)]
    caches = [(dev(k), dev(v)) for k, v in hist]
    qkv_d = [torch.empty(H * D + 2 * KVH * D, dtype=torch.float16, device=cuda) for _ in range(layers)]
    outs = [torch.empty(H * D, dtype=torch.float16, device=cuda) for _ in range(layers)]
    pos = torch.tensor([start], dtype=torch.int32, device=cuda)
    ws = _workspace()
    g = Graph()
    with g:
        for l in range(layers):
            b200attn.launch_decode_step_fused(qkv_d[l], qkv_d[l][H * D:], qkv_d[l][H * D + KVH * D:], caches[l][0],
                                              caches[l][1], cos_d, sin_d, cap, l == 0, pos, pos, 1, cap, outs[l],
                                              ws[0], ws[1], H, KVH, D, stream=g.stream)
        b200attn.advance_position(pos, 1, stream=g.stream)
    ref_k = [k.copy() for k, _ in hist]
    ref_v = [v.copy() for _, v in hist]
    for t in range(steps):
        p = start + t
        news = [seeded_f16(H * D + 2 * KVH * D, 900 + 10 * t + l) for l in range(layers)]
        for l in range(layers):
            qkv_d[l].copy_(dev(news[l]))
        _sync()
        g.launch()
        _sync()
        for l in range(layers):
            qd, kd = H * D, KVH * D
            oq, ok, ov = news[l][:qd].copy(), news[l][qd:qd + kd].copy(), news[l][qd + kd:].copy()
            oracle.rope_and_store_kv(oq, ok, ov, ref_k[l], ref_v[l], cos, sin, 1, H, KVH, D, qd, kd, p, l == 0)
            if l != 0:
                ref_k[l][p], ref_v[l][p] = ok, ov
            _, o32 = oracle.decode_attention(oq, ref_k[l], ref_v[l], p + 1, H, KVH, D)
            assert_attention_close(host(outs[l]), o32.reshape(-1))
            np.testing.assert_array_equal(bits(host(caches[l][0])[:p + 1]), bits(ref_k[l][:p + 1]))
            np.testing.assert_array_equal(bits(host(caches[l][1])[:p + 1]), bits(ref_v[l][:p + 1]))
    assert int(host(pos)[0]) == start + steps
    assert b200attn.lib().b2_device_error_word() == 0


@pytest.mark.parametrize("ranks", [2, 3])
def test_fused_rank_partials_merge_to_oracle(cuda, ranks):
    """KV-split decode across 'ranks' emulated on one GPU: each rank runs the fused
    step over its own range, the tail rank appends the new token, the partials
    are merged with the strided merge."""
    import torch
    from b200attn import dist as bdist
    L = 9001  # tokens after the append
    hist_k = seeded_f16((L, KVH * D), 81, std=0.5)
    hist_v = seeded_f16((L, KVH * D), 82, std=0.5)
    qkv = seeded_f16(H * D + 2 * KVH * D, 83, std=0.5)
    cos, sin = b200attn.rope_tables_host(L + 16, D, THETA)
    cos_d, sin_d = dev(cos), dev(sin)
    exp_k, exp_v, o32 = _oracle_step(qkv, hist_k, hist_v, L, L - 1, L - 1, cos, sin, True)
    qkv_d = dev(qkv)
    per = H * (D + 2)
    gathered = torch.zeros(ranks * per, dtype=torch.float32, device=cuda)
    pos = torch.tensor([L - 1], dtype=torch.int32, device=cuda)
    for r in range(ranks):
        plan = bdist.split_kv_plan(L, ranks, r)
        n = plan.end - plan.begin
        tail = plan.end == L
        init_k = exp_k[plan.begin:plan.end].copy()
        init_v = exp_v[plan.begin:plan.end].copy()
        if tail:
            init_k[-1] = GUARD
            init_v[-1] = GUARD
        kc, vc = dev(init_k), dev(init_v)
        ln = torch.tensor([n], dtype=torch.int32, device=cuda)
        ws = _workspace()
        part = gathered[r * per:(r + 1) * per]
        b200attn.launch_decode_step_fused_rank_partial(
            qkv_d, qkv_d[H * D:] if tail else None, qkv_d[H * D + KVH * D:] if tail else None, kc, vc, cos_d, sin_d,
            cos.shape[0], True, pos, ln, 0, n, part[:H * D], part[H * D:H * D + H], part[H * D + H:], ws[0], ws[1],
            H, KVH, D)
        _sync()
        np.testing.assert_array_equal(bits(host(kc)), bits(exp_k[plan.begin:plan.end]))
        np.testing.assert_array_equal(bits(host(vc)), bits(exp_v[plan.begin:plan.end]))
    out = torch.empty(H * D, dtype=torch.float16, device=cuda)
    b200attn.launch_merge_partials_strided(gathered, gathered[H * D:], gathered[H * D + H:], out, H, ranks, D, per,
                                           D, per, 1)
    _sync()
    assert_attention_close(host(out), o32)


@pytest.mark.parametrize("kvh,heads,kv_len", [
    (1, 8, 5000), (2, 16, 5000), (8, 32, 5000),
    # one or two KV heads (a tensor-parallel rank's share): stages of 64 / 32
    # tokens split into 16-token sub-tiles, partial stages at every boundary
    (1, 4, 1), (1, 4, 17), (1, 4, 63), (1, 4, 64), (1, 4, 65), (1, 4, 1000), (1, 4, 65537),
    (2, 8, 15), (2, 8, 32), (2, 8, 33), (2, 8, 4097),
])
def test_fused_step_other_gqa_shapes(cuda, kvh, heads, kv_len):
    import torch
    cap = kv_len + 10
    hist_k = seeded_f16((cap, kvh * D), 91 + kvh)
    hist_v = seeded_f16((cap, kvh * D), 92 + kvh)
    qkv = seeded_f16(heads * D + 2 * kvh * D, 93 + kvh)
    cos, sin = b200attn.rope_tables_host(cap, D, THETA)
    exp_k, exp_v, o32 = _oracle_step(qkv, hist_k, hist_v, cap, kv_len - 1, kv_len - 1, cos, sin, True, heads, kvh)
    init_k, init_v = exp_k.copy(), exp_v.copy()
    init_k[kv_len - 1] = GUARD
    init_v[kv_len - 1] = GUARD
    kc, vc = dev(init_k), dev(init_v)
    qkv_d = dev(qkv)
    pos = torch.tensor([kv_len - 1], dtype=torch.int32, device=cuda)
    out = torch.empty(heads * D, dtype=torch.float16, device=cuda)
    ws = _workspace(heads, kvh)
    _fused(qkv_d, kc, vc, dev(cos), dev(sin), cap, True, pos, pos, 1, cap, out, ws, heads, kvh)
    _sync()
    np.testing.assert_array_equal(bits(host(kc)), bits(exp_k))
    np.testing.assert_array_equal(bits(host(vc)), bits(exp_v))
    assert_attention_close(host(out), o32)


def test_fused_step_64k(cuda):
    """benchmark config 4 size (65,536 cached tokens + the new one) through the fused step."""
    import torch
    past = 65536
    cap = past + 64
    hist_k = seeded_f16((cap, KVH * D), 31, std=0.5)
    hist_v = seeded_f16((cap, KVH * D), 32, std=0.5)
    qkv = seeded_f16(H * D + 2 * KVH * D, 33, std=0.5)
    cos, sin = b200attn.rope_tables_host(cap, D, THETA)
    exp_k, exp_v, o32 = _oracle_step(qkv, hist_k, hist_v, cap, past, past, cos, sin, True)
    kc, vc = dev(exp_k), dev(exp_v)
    kc[past] = 0
    qkv_d = dev(qkv)
    pos = torch.tensor([past], dtype=torch.int32, device=cuda)
    out = torch.empty(H * D, dtype=torch.float16, device=cuda)
    ws = _workspace()
    _fused(qkv_d, kc, vc, dev(cos), dev(sin), cap, True, pos, pos, 1, cap, out, ws)
    _sync()
    np.testing.assert_array_equal(bits(host(kc)[past]), bits(exp_k[past]))
    assert_attention_close(host(out), o32)


def test_fused_step_empty_and_clamped_lengths(cuda):
    import torch
    cap = 600
    hist_k = seeded_f16((cap, KVH * D), 101)
    hist_v = seeded_f16((cap, KVH * D), 102)
    qkv = seeded_f16(H * D + 2 * KVH * D, 103)
    cos, sin = b200attn.rope_tables_host(cap, D, THETA)
    kc, vc = dev(hist_k), dev(hist_v)
    qkv_d = dev(qkv)
    ws = _workspace()
    out = torch.full((H * D,), 5.0, dtype=torch.float16, device=cuda)
    ln = torch.tensor([-1], dtype=torch.int32, device=cuda)  # kv_len 0
    _fused(qkv_d, kc, vc, dev(cos), dev(sin), cap, True, ln, ln, 1, cap, out, ws, append=False)
    _sync()
    assert np.all(host(out) == 0)
    # past capacity: clamped to cap, no append
    ln.fill_(cap + 100)
    pos = torch.tensor([cap - 1], dtype=torch.int32, device=cuda)
    _fused(qkv_d, kc, vc, dev(cos), dev(sin), cap, True, pos, ln, 0, cap, out, ws, append=False)
    _sync()
    oq = qkv[:H * D].copy()
    oracle.rope_and_store_kv(oq, qkv[H * D:H * D + KVH * D].copy(), None, None, None, cos, sin, 1, H, KVH, D, H * D,
                             KVH * D, cap - 1, True)
    _, o32 = oracle.decode_attention(oq, hist_k, hist_v, cap, H, KVH, D)
    assert_attention_close(host(out), o32.reshape(-1))
    np.testing.assert_array_equal(bits(host(kc)), bits(hist_k))
    assert b200attn.lib().b2_device_error_word() == 0


def test_fused_step_position_outside_table_sets_error_bit(cuda):
    import torch
    cap = 300
    hist_k = seeded_f16((cap, KVH * D), 111)
    hist_v = seeded_f16((cap, KVH * D), 112)
    qkv = seeded_f16(H * D + 2 * KVH * D, 113)
    cos, sin = b200attn.rope_tables_host(64, D, THETA)  # table shorter than the position
    kc, vc = dev(hist_k), dev(hist_v)
    pos = torch.tensor([200], dtype=torch.int32, device=cuda)
    out = torch.empty(H * D, dtype=torch.float16, device=cuda)
    ws = _workspace()
    assert b200attn.lib().b2_device_error_word() == 0
    _fused(dev(qkv), kc, vc, dev(cos), dev(sin), 64, True, pos, pos, 1, cap, out, ws)
    _sync()
    assert b200attn.lib().b2_device_error_word() & 2
    np.testing.assert_array_equal(bits(host(kc)), bits(hist_k))  # nothing appended
    assert b200attn.lib().b2_clear_device_error_word() == 0
    assert b200attn.lib().b2_device_error_word() == 0
