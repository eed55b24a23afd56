"""Split-KV flash-decode + merge on the GPU vs the CPU oracle and the golden
vectors. Restates tests/test_causal_attention.cpp:80-228."""
import numpy as np
import pytest

import b200attn
import oracle
from _gpu import Graph, bits, dev, host
from _util import assert_attention_close, golden, max_abs, seeded_f16, tensor_close_mismatches
from test_oracle import KAT_LENGTHS, _kat_expected, _kat_inputs

pytestmark = pytest.mark.gpu
CHUNK = 256


def _sync():
    import torch
    torch.cuda.synchronize()


def _workspace(heads, kv_len, head_dim):
    import torch
    chunks = (kv_len + CHUNK - 1) // CHUNK
    po = torch.full((heads * chunks * head_dim,), float("nan"), dtype=torch.float32, device="cuda")
    pm = torch.full((heads * chunks,), float("nan"), dtype=torch.float32, device="cuda")
    pl = torch.full((heads * chunks,), float("nan"), dtype=torch.float32, device="cuda")
    return po, pm, pl


def _decode(entry, q, k, v, kv_len, H, KVH, d, kv_stride, guard=1):
    """Run a decode entry point with -123 guards around the output; return output, guards, partials."""
    out = np.full(H * d + 2 * guard, -123.0, np.float16)
    dout = dev(out)
    po, pm, pl = _workspace(H, kv_len, d)
    entry(dev(q), dev(k), dev(v), dout[guard:], po, pm, pl, 1, kv_len, kv_len - 1, H, KVH, d, 0, kv_stride)
    _sync()
    res = host(dout)
    return res[guard:guard + H * d], np.concatenate([res[:guard], res[guard + H * d:]]), (po, pm, pl)


ENTRIES = {
    "decode": lambda *a: b200attn.launch_causal_attention_decode(*a),
    "vectorized": lambda *a: b200attn.launch_causal_attention_decode_vectorized(*a),
}


@pytest.mark.parametrize("entry", ["decode", "vectorized"])
@pytest.mark.parametrize("head_dim", [32, 128])
@pytest.mark.parametrize("kv_heads", [1, 2, 4])
@pytest.mark.parametrize("padded", [False, True])
def test_flash_decode_known_answer(cuda, entry, head_dim, kv_heads, padded):
    """tests/test_causal_attention.cpp:152-228, with KV_CHUNK boundaries added."""
    heads = 4
    for length in KAT_LENGTHS + [255, 511, 1025]:
        q, k, v, stride = _kat_inputs(head_dim, kv_heads, length, padded)
        exp = _kat_expected(q, k, v, heads, kv_heads, head_dim, length, stride)
        got, guards, _ = _decode(ENTRIES[entry], q, k, v, length, heads, kv_heads, head_dim,
                                 stride if padded else 0)
        assert np.all(guards == np.float16(-123.0))
        assert np.all(np.isfinite(got.astype(np.float32)))
        assert tensor_close_mismatches(got, exp, 2e-3, 2e-3) == 0, (length,)


@pytest.mark.parametrize("subset", ["", "sharp"])
@pytest.mark.parametrize("interleaved", [False, True])
def test_decode_matches_golden_prefill_rows(cuda, interleaved, subset):
    """tests/test_causal_attention.cpp:80-150: decode at kv_len p+1 == prefill row p;
    future cache rows hold 123, output guards -123. Both fixture sets (the
    160-token one has a peaked softmax)."""
    meta, g = golden(subset)
    S, H, KVH, d = meta["seq_len"], meta["num_heads"], meta["num_kv_heads"], meta["head_dim"]
    q_dim, kv_dim = H * d, KVH * d
    cache_k = np.full((S + 2, kv_dim), 123.0, np.float16)
    cache_v = cache_k.copy()
    cache_k[:S] = g["k_rope"]
    cache_v[:S] = g["v"]
    dk, dv = dev(cache_k), dev(cache_v)
    for p in range(S):
        stride = q_dim + 2 * kv_dim if interleaved else q_dim
        qin = np.full(stride, -123.0, np.float16)
        qin[:q_dim] = g["q_rope"][p]
        out = np.full(3 * q_dim, -123.0, np.float16)
        dout = dev(out)
        po, pm, pl = _workspace(H, p + 1, d)
        b200attn.launch_causal_attention_decode(dev(qin), dk, dv, dout[q_dim:], po, pm, pl, 1, p + 1, p, H, KVH, d,
                                                stride if interleaved else 0, 0)
        _sync()
        res = host(dout)
        got = res[q_dim:2 * q_dim]
        assert tensor_close_mismatches(got, g["attn"][p], 2e-2, 2e-2) == 0, p
        np.testing.assert_array_equal(bits(res[:q_dim]), bits(out[:q_dim]))
        np.testing.assert_array_equal(bits(res[2 * q_dim:]), bits(out[2 * q_dim:]))
        _, o32 = oracle.decode_attention(g["q_rope"][p], g["k_rope"], g["v"], p + 1, H, KVH, d)
        assert_attention_close(got, o32.reshape(-1))


def _sm_count():
    import torch
    return torch.cuda.get_device_properties(0).multi_processor_count


@pytest.mark.parametrize("L", [1000, 5000, 65536 + 17])
@pytest.mark.parametrize("packed", [True, False])
def test_decode_partials_match_oracle(cuda, L, packed):
    """The workspace holds the reference's partial semantics, one (o, m, l) per
    split: o [H][S][d] unnormalised, m (natural-log units) and l [H][S] with o and
    l relative to m, so o/l and m + ln(l) are the split's attention and LSE. The
    TMA path (packed rows) uses S = min(#SMs, chunks) ranges of a 16-token
    multiple; the strided path uses KV_CHUNK chunks."""
    H, KVH, d = 16, 4, 128
    stride = KVH * d if packed else 3072
    q = seeded_f16(H * d, 1)
    k = seeded_f16(L * stride, 2)
    v = seeded_f16(L * stride, 3)
    _, _, (po, pm, pl) = _decode(ENTRIES["decode"], q, k, v, L, H, KVH, d, 0 if packed else stride)
    chunks = (L + CHUNK - 1) // CHUNK
    if packed:
        S = min(_sm_count(), chunks)
        per = -(-(-(-L // S)) // 16) * 16
    else:
        S, per = chunks, CHUNK
    ro, rm, rl = oracle.decode_partials(q, k, v, L, H, KVH, d, stride, per)
    n = ro.shape[1]
    assert n <= S
    gm = host(pm)[:H * S].reshape(H, S)
    gl = host(pl)[:H * S].reshape(H, S)
    go = host(po)[:H * S * d].reshape(H, S, d)
    # m is a running max that may trail the split's true max by < 8 log2 units
    # (lazy rescaling); o and l are relative to it, so the invariants are the
    # normalised partial o/l and the log-sum-exp m + ln(l).
    assert np.all(gm[:, :n] <= rm + 1e-5) and np.all(gm[:, :n] >= rm - 8 * np.log(2) - 1e-5)
    np.testing.assert_allclose(gm[:, :n] + np.log(gl[:, :n]), rm + np.log(rl), rtol=0, atol=2e-3)
    np.testing.assert_allclose(go[:, :n] / gl[:, :n, None], ro / rl[:, :, None], rtol=0, atol=2e-3)
    assert np.all(gm[:, n:] == -np.inf) and np.all(gl[:, n:] == 0)


def test_devlen_equals_host_length(cuda):
    """Graph-static decode (kv_len read from device memory) == host-length decode."""
    import torch
    H, KVH, d, cap = 16, 4, 128, 3000
    k = dev(seeded_f16((cap, KVH * d), 51))
    v = dev(seeded_f16((cap, KVH * d), 52))
    q = dev(seeded_f16(H * d, 53))
    ws = torch.empty(b200attn.decode_workspace_floats(H, d, cap), dtype=torch.float32, device=cuda)
    n = H * ((cap + 255) // 256)
    po, pm, pl = ws[:n * d], ws[n * d:n * (d + 1)], ws[n * (d + 1):]
    pos = torch.zeros(1, dtype=torch.int32, device=cuda)
    for kv_len in (1, 255, 256, 257, 1234, 2999, 3000):
        a = torch.empty(H * d, dtype=torch.float16, device=cuda)
        b = torch.empty_like(a)
        b200attn.launch_causal_attention_decode(q, k, v, a, po, pm, pl, 1, kv_len, kv_len - 1, H, KVH, d, 0, 0)
        pos.fill_(kv_len - 1)
        b200attn.launch_causal_attention_decode_devlen(q, k, v, b, po, pm, pl, pos, 1, cap, H, KVH, d)
        _sync()
        np.testing.assert_array_equal(bits(host(a)), bits(host(b)))
    # past capacity is clamped to max_kv_len
    pos.fill_(cap + 50)
    b200attn.launch_causal_attention_decode_devlen(q, k, v, b, po, pm, pl, pos, 1, cap, H, KVH, d)
    _sync()
    np.testing.assert_array_equal(bits(host(a)), bits(host(b)))
    assert b200attn.lib().b2_device_error_word() == 0


@pytest.mark.parametrize("ranks", [2, 3, 8])
def test_rank_partials_and_strided_merge(cuda, ranks):
    """KV-split decode as the multi-GPU path runs it, emulated on one GPU: every
    'rank' reduces its contiguous range to one (o, m, l) per head, the partials
    are concatenated like an all-gather and merged with the strided merge."""
    import torch
    from b200attn import dist as bdist
    H, KVH, d, L = 16, 4, 128, 9000
    kh = seeded_f16((L, KVH * d), 61, std=0.5)
    vh = seeded_f16((L, KVH * d), 62, std=0.5)
    qh = seeded_f16(H * d, 63, std=0.5)
    q = dev(qh)
    per = H * (d + 2)
    gathered = torch.zeros(ranks * per, dtype=torch.float32, device=cuda)
    for r in range(ranks):
        plan = bdist.split_kv_plan(L, ranks, r)
        kc = dev(kh[plan.begin:plan.end])
        vc = dev(vh[plan.begin:plan.end])
        n = plan.end - plan.begin
        ws = torch.empty(b200attn.decode_workspace_floats(H, d, n), dtype=torch.float32, device=cuda)
        c = H * ((n + 255) // 256)
        ln = torch.tensor([n], dtype=torch.int32, device=cuda)
        part = gathered[r * per:(r + 1) * per]
        b200attn.launch_decode_rank_partial_devlen(q, kc, vc, ws[:c * d], ws[c * d:c * (d + 1)], ws[c * (d + 1):],
                                                   ln, 0, n, H, KVH, d, KVH * d, part[:H * d], part[H * d:H * d + H],
                                                   part[H * d + H:])
        _sync()
    out = torch.empty(H * d, dtype=torch.float16, device=cuda)
    b200attn.launch_merge_partials_strided(gathered, gathered[H * d:], gathered[H * d + H:], out, H, ranks, d, per,
                                           d, per, 1)
    _sync()
    _, o32 = oracle.decode_attention(qh, kh, vh, L, H, KVH, d)
    assert_attention_close(host(out), o32.reshape(-1))
    # the host restatement of the cross-rank merge agrees
    g = host(gathered).reshape(ranks, per)
    parts = [(g[r, :H * d].reshape(H, d), g[r, H * d:H * d + H], g[r, H * d + H:]) for r in range(ranks)]
    ref = bdist.merge_rank_partials_reference(parts)
    assert_attention_close(ref.reshape(-1), o32.reshape(-1))


def test_config2_append_then_decode(cuda):
    """benchmark config 2: cache 4096 tokens ~N(0,1), the new token RoPE'd at 4096 and
    appended, kv_len 4097, chunk 256 (17 chunks) + merge -- against the oracle."""
    import torch
    H, KVH, d, past = 16, 4, 128, 4096
    total = H * d + 2 * KVH * d
    cos, sin = b200attn.rope_tables_host(past + 64, d, 5.0e6)
    cache = b200attn.KVCache(1, past + 64, KVH, d, device=cuda)
    hist_k = seeded_f16((past, KVH * d), 11)
    hist_v = seeded_f16((past, KVH * d), 12)
    cache.get_k_cache(0)[:past] = dev(hist_k)
    cache.get_v_cache(0)[:past] = dev(hist_v)
    qkv = seeded_f16((1, total), 13)
    dqkv = dev(qkv)
    b200attn.launch_rope_and_store_kv(dqkv, dqkv[:, H * d:], dqkv[:, H * d + KVH * d:], cache.get_k_cache(0),
                                      cache.get_v_cache(0), dev(cos), dev(sin), 1, H, KVH, d, total, total, past, True)
    ws = torch.empty(b200attn.decode_workspace_floats(H, d, past + 64), dtype=torch.float32, device=cuda)
    chunks = (past + 1 + 255) // 256
    po, pm, pl = ws[:H * chunks * d], ws[H * chunks * d:H * chunks * (d + 1)], ws[H * chunks * (d + 1):]
    out = torch.empty(H * d, dtype=torch.float16, device=cuda)
    b200attn.launch_causal_attention_decode_vectorized(dqkv, cache.get_k_cache(0), cache.get_v_cache(0), out, po, pm,
                                                       pl, 1, past + 1, past, H, KVH, d, total, KVH * d)
    _sync()
    # oracle: same append, then attention over 4097 tokens
    oq, ok = qkv[0, :H * d].copy(), qkv[0, H * d:H * d + KVH * d].copy()
    kc = np.zeros((past + 64, KVH * d), np.float16)
    vc = kc.copy()
    kc[:past], vc[:past] = hist_k, hist_v
    oracle.rope_and_store_kv(oq, ok, np.ascontiguousarray(qkv[0, H * d + KVH * d:]), kc, vc, cos, sin, 1, H, KVH, d,
                             H * d, KVH * d, past, True)
    np.testing.assert_array_equal(bits(host(cache.get_k_cache(0))[:past + 1]), bits(kc[:past + 1]))
    np.testing.assert_array_equal(bits(host(dqkv)[0, :H * d]), bits(oq))
    _, o32 = oracle.decode_attention(oq, kc, vc, past + 1, H, KVH, d)
    assert_attention_close(host(out), o32.reshape(-1))


@pytest.mark.parametrize("kv_len", [65536, 65536 + 63])
def test_long_context_64k_one_layer(cuda, kv_len):
    """benchmark config 4 size: 64K cached tokens ~N(0, 0.5), one layer, vs the oracle."""
    import torch
    H, KVH, d = 16, 4, 128
    k = seeded_f16((kv_len, KVH * d), 21, std=0.5)
    v = seeded_f16((kv_len, KVH * d), 22, std=0.5)
    q = seeded_f16(H * d, 23, std=0.5)
    got, guards, _ = _decode(ENTRIES["vectorized"], q, k, v, kv_len, H, KVH, d, 0)
    assert np.all(guards == np.float16(-123.0))
    _, o32 = oracle.decode_attention(q, k, v, kv_len, H, KVH, d)
    assert_attention_close(got, o32.reshape(-1))


def test_decode_group8_and_strided_cache(cuda):
    """Group size 8 (all MMA columns live) and a cache row stride of 3072 (interleaved rows)."""
    H, KVH, d, L = 16, 2, 128, 777
    stride = 3072
    q = seeded_f16(H * d, 31)
    k = seeded_f16(L * stride, 32)
    v = seeded_f16(L * stride, 33)
    got, _, _ = _decode(ENTRIES["decode"], q, k, v, L, H, KVH, d, stride)
    _, o32 = oracle.decode_attention(q, k, v, L, H, KVH, d, stride)
    assert_attention_close(got, o32.reshape(-1))


def test_merge_tiled_on_oracle_partials(cuda):
    """launch_merge_attention_decode_tiled (kernels.hpp:157-166) on caller partials."""
    import torch
    H, d = 16, 128
    for chunks in (1, 3, 17, 257, 1000):
        rng = np.random.default_rng(chunks)
        pm = rng.normal(0, 3, (H, chunks)).astype(np.float32)
        pl = rng.uniform(0.5, 50, (H, chunks)).astype(np.float32)
        po = rng.normal(0, 5, (H, chunks, d)).astype(np.float32)
        out = torch.empty(H * d, dtype=torch.float16, device=cuda)
        b200attn.launch_merge_attention_decode_tiled(dev(po), dev(pm), dev(pl), out, H, chunks, d)
        _sync()
        _, ref32 = oracle.merge_partials(po, pm, pl)
        assert max_abs(host(out), ref32.reshape(-1)) <= 2e-3 * max(1.0, float(np.abs(ref32).max()))


def test_decode_graph_capture_and_node_updates(cuda):
    """include/model_inference.hpp:96-123: capture once at kv_len L0, then patch
    kv_len with update_causal_attention_decode_node / update_merge_attention_decode_node
    (causal_attention.hip.cpp:975-1026) and replay."""
    import torch
    H, KVH, d, max_len = 16, 4, 128, 2000
    k = dev(seeded_f16((max_len, KVH * d), 41))
    v = dev(seeded_f16((max_len, KVH * d), 42))
    q = dev(seeded_f16(H * d, 43))
    ws = torch.empty(b200attn.decode_workspace_floats(H, d, max_len), dtype=torch.float32, device=cuda)
    cmax = (max_len + 255) // 256
    po, pm, pl = ws[:H * cmax * d], ws[H * cmax * d:H * cmax * (d + 1)], ws[H * cmax * (d + 1):]
    out = torch.zeros(H * d, dtype=torch.float16, device=cuda)
    gph = Graph()
    with gph:
        an, mn = b200attn.launch_causal_attention_decode_vectorized(q, k, v, out, po, pm, pl, 1, 300, 299, H, KVH, d,
                                                                    0, 0, stream=gph.stream, capture_nodes=True)
    assert an and mn and an != mn
    for kv_len in (300, 301, 512, 513, 1999, 7):
        b200attn.update_causal_attention_decode_node(gph.exec_handle, an, kv_len)
        b200attn.update_merge_attention_decode_node(gph.exec_handle, mn, kv_len)
        gph.launch()
        _, o32 = oracle.decode_attention(host(q), host(k), host(v), kv_len, H, KVH, d)
        assert_attention_close(host(out), o32.reshape(-1))
    # a node of another kind is rejected, not corrupted
    with pytest.raises(b200attn.B2Error):
        b200attn.update_merge_attention_decode_node(gph.exec_handle, an, 10)
    gph.close()
