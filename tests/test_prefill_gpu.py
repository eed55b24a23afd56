"""Causal GQA prefill on the GPU vs the CPU oracle and the golden vectors.
Restates tests/test_causal_attention.cpp:15-78 and tests/test_qkv_gemm.cpp:87-117."""
import numpy as np
import pytest

import b200attn
import oracle
from _gpu import bits, dev, host
from _util import assert_attention_close, golden, seeded_f16, tensor_close_mismatches

pytestmark = pytest.mark.gpu


def _sync():
    import torch
    torch.cuda.synchronize()


def _prefill(q, k, v, S, H, KVH, d, q_stride=0, kv_stride=0, guard_rows=1):
    """Run prefill with guard rows of -123 above and below the packed output."""
    out = np.full(((S + 2 * guard_rows), H * d), -123.0, np.float16)
    dout = dev(out)
    b200attn.launch_causal_attention_prefill(dev(q), dev(k), dev(v), dout[guard_rows:], S, H, KVH, d, q_stride,
                                             kv_stride)
    _sync()
    res = host(dout)
    np.testing.assert_array_equal(bits(res[:guard_rows]), bits(out[:guard_rows]))
    np.testing.assert_array_equal(bits(res[guard_rows + S:]), bits(out[guard_rows + S:]))
    return res[guard_rows:guard_rows + S]


def test_prefill_matches_golden_from_cache(cuda):
    """K/V in a real KVCache (max_seq = S + 2, trailing rows 123), Q packed (:15-78)."""
    meta, g = golden()
    S, H, KVH, d = meta["seq_len"], meta["num_heads"], meta["num_kv_heads"], meta["head_dim"]
    cache = b200attn.KVCache(1, S + 2, KVH, d, device=cuda)
    cache.buffer.fill_(123.0)
    cache.get_k_cache(0)[:S] = dev(g["k_rope"])
    cache.get_v_cache(0)[:S] = dev(g["v"])
    out = dev(np.zeros((S, H * d), np.float16))
    b200attn.launch_causal_attention_prefill(dev(g["q_rope"]), cache.get_k_cache(0), cache.get_v_cache(0), out, S, H,
                                             KVH, d, H * d, KVH * d)
    _sync()
    got = host(out)
    assert tensor_close_mismatches(got, g["attn"], 2e-2, 2e-2) == 0
    _, o32 = oracle.causal_attention(g["q_rope"], g["k_rope"], g["v"], S, H, KVH, d)
    assert_attention_close(got, o32)


def test_prefill_matches_sharp_golden_from_cache(cuda):
    """The 160-token fixture (peaked softmax, two query tiles) from a cache with
    populated spare rows, against the fixture and the FP32 oracle."""
    meta, g = golden("sharp")
    S, H, KVH, d = meta["seq_len"], meta["num_heads"], meta["num_kv_heads"], meta["head_dim"]
    cache = b200attn.KVCache(1, S + 2, KVH, d, device=cuda)
    cache.buffer.fill_(123.0)
    cache.get_k_cache(0)[:S] = dev(g["k_rope"])
    cache.get_v_cache(0)[:S] = dev(g["v"])
    out = dev(np.zeros((S, H * d), np.float16))
    b200attn.launch_causal_attention_prefill(dev(g["q_rope"]), cache.get_k_cache(0), cache.get_v_cache(0), out, S, H,
                                             KVH, d, H * d, KVH * d)
    _sync()
    got = host(out)
    assert tensor_close_mismatches(got, g["attn"], 2e-2, 2e-2) == 0
    _, o32 = oracle.causal_attention(g["q_rope"], g["k_rope"], g["v"], S, H, KVH, d)
    assert_attention_close(got, o32)


def test_prefill_on_interleaved_qkv_rows(cuda):
    """tests/test_qkv_gemm.cpp:87-117: RoPE then prefill straight on [Q|K|V] rows, stride 3072."""
    meta, g = golden()
    S, H, KVH, d = meta["seq_len"], meta["num_heads"], meta["num_kv_heads"], meta["head_dim"]
    total = H * d + 2 * KVH * d
    qkv = dev(np.concatenate([g["q"], g["k"], g["v"]], axis=1))
    cos, sin = b200attn.rope_tables_host(4096, d, meta["rope_theta"])
    b200attn.launch_rope(qkv, qkv[:, H * d:], dev(cos), dev(sin), S, H, KVH, d, total, total)
    out = dev(np.zeros((S, H * d), np.float16))
    b200attn.launch_causal_attention_prefill(qkv, qkv[:, H * d:], qkv[:, H * d + KVH * d:], out, S, H, KVH, d, total,
                                             total)
    _sync()
    got = host(out)
    assert tensor_close_mismatches(got, g["attn"], 2e-2, 2e-2) == 0
    _, o32 = oracle.causal_attention(g["q_rope"], g["k_rope"], g["v"], S, H, KVH, d)
    assert_attention_close(got, o32)


@pytest.mark.parametrize("S", [1, 2, 17, 127, 128, 129, 254, 255, 256, 257, 300, 1000])
def test_prefill_random_vs_oracle(cuda, S):
    H, KVH, d = 16, 4, 128
    q = seeded_f16((S, H * d), 100 + S)
    k = seeded_f16((S, KVH * d), 200 + S)
    v = seeded_f16((S, KVH * d), 300 + S)
    got = _prefill(q, k, v, S, H, KVH, d)
    _, o32 = oracle.causal_attention(q, k, v, S, H, KVH, d)
    assert_attention_close(got, o32)


@pytest.mark.parametrize("S", [2048, 4097])
def test_prefill_long_sampled_rows(cuda, S):
    """Longer sequences: every row is finite, sampled rows (incl. first/last/tile edges) match."""
    H, KVH, d = 16, 4, 128
    q = seeded_f16((S, H * d), 7 + S)
    k = seeded_f16((S, KVH * d), 8 + S)
    v = seeded_f16((S, KVH * d), 9 + S)
    got = _prefill(q, k, v, S, H, KVH, d)
    assert np.all(np.isfinite(got.astype(np.float32)))
    rng = np.random.default_rng(S)
    rows = sorted(set([0, 1, 127, 128, 129, S // 2, S - 129, S - 128, S - 2, S - 1] +
                      list(rng.integers(0, S, 40))))
    _, o32 = oracle.causal_attention(q, k, v, S, H, KVH, d, rows=rows)
    assert_attention_close(got[rows], o32)


@pytest.mark.parametrize("shape", [
    # (S, H, KVH, d, q_pad, kv_pad): SIMT path shapes
    (37, 4, 2, 32, 0, 0),
    (65, 8, 1, 64, 3, 5),
    (40, 16, 4, 128, 1, 17),
    (33, 6, 3, 96, 0, 0),
])
def test_prefill_other_shapes_vs_oracle(cuda, shape):
    S, H, KVH, d, qp, kp = shape
    qs, ks = H * d + qp, KVH * d + kp
    q = seeded_f16(S * qs, 1 + S)
    k = seeded_f16(S * ks, 2 + S)
    v = seeded_f16(S * ks, 3 + S)
    got = _prefill(q, k, v, S, H, KVH, d, qs, ks)
    _, o32 = oracle.causal_attention(q, k, v, S, H, KVH, d, qs, ks)
    assert_attention_close(got, o32)


def test_prefill_batched_matches_per_sequence(cuda):
    """Config-3 layout: B sequences with per-sequence strides (batched entry point)."""
    import torch
    B, S, H, KVH, d = 3, 300, 16, 4, 128
    q = seeded_f16((B, S, H * d), 71)
    k = seeded_f16((B, S + 5, KVH * d), 72)   # per-sequence cache with spare rows
    v = seeded_f16((B, S + 5, KVH * d), 73)
    out = torch.zeros((B, S, H * d), dtype=torch.float16, device=cuda)
    b200attn.launch_causal_attention_prefill_batched(dev(q), dev(k), dev(v), out, B, S, H, KVH, d, H * d, KVH * d,
                                                     S * H * d, (S + 5) * KVH * d, S * H * d)
    _sync()
    got = host(out)
    for b in range(B):
        _, o32 = oracle.causal_attention(q[b], k[b], v[b], S, H, KVH, d)
        assert_attention_close(got[b], o32)


@pytest.mark.parametrize("S", [8192])
def test_prefill_config3_unit_sampled(cuda, S):
    """One (sequence, KV head) unit of benchmark config 3 at full length, sampled rows."""
    H, KVH, d = 16, 4, 128
    q = seeded_f16((S, H * d), 81)
    k = seeded_f16((S, KVH * d), 82)
    v = seeded_f16((S, KVH * d), 83)
    got = _prefill(q, k, v, S, H, KVH, d)
    assert np.all(np.isfinite(got.astype(np.float32)))
    rng = np.random.default_rng(S)
    rows = sorted(set([0, 127, 128, 4095, 4096, S - 1] + list(rng.integers(0, S, 24))))
    _, o32 = oracle.causal_attention(q, k, v, S, H, KVH, d, rows=rows)
    assert_attention_close(got[rows], o32)


def test_prefill_batched_head_block_into_wider_output(cuda):
    """One rank's block of KV heads (the multi-GPU prefill split): heads of KV
    heads [2, 4) written into the full-width output rows (out_stride), other
    heads' columns untouched."""
    import torch
    B, S, H, KVH, d = 2, 300, 16, 4, 128
    G = H // KVH
    q = seeded_f16((B, S, H * d), 91)
    k = seeded_f16((B, S, KVH * d), 92)
    v = seeded_f16((B, S, KVH * d), 93)
    out = torch.full((B, S, H * d), -5.0, dtype=torch.float16, device=cuda)
    dq, dk, dv = dev(q), dev(k), dev(v)
    g0, ng = 2, 2
    b200attn.launch_causal_attention_prefill_batched(dq[:, :, g0 * G * d:], dk[:, :, g0 * d:], dv[:, :, g0 * d:],
                                                     out[:, :, g0 * G * d:], B, S, ng * G, ng, d, H * d, KVH * d,
                                                     S * H * d, S * KVH * d, S * H * d, out_stride=H * d)
    _sync()
    got = host(out)
    assert np.all(got[:, :, :g0 * G * d] == np.float16(-5.0))
    for b in range(B):
        _, o32 = oracle.causal_attention(q[b], k[b], v[b], S, H, KVH, d)
        assert_attention_close(got[b, :, g0 * G * d:], o32[:, g0 * G * d:])


@pytest.mark.parametrize("layer", [2, 3])
def test_prefill_config3_full_batched_launch(cuda, layer):
    """The bench's config-3 launch as it runs: 4 sequences x 8192 tokens of
    interleaved [Q|K|V] rows (stride 3072), RoPE/append into a 36-layer cache
    per sequence (batch stride 36 * 2 * 8192 * 512; layer 2 rotates, layer 3
    is a NoPE layer, (l + 1) % 4 == 0), then one batched prefill launch over
    all 4 x 4 (sequence, KV head) units. Sampled rows of every sequence and
    every head against the FP32 oracle; sequence 0's cache rows bit-exact
    against the oracle's RoPE/append."""
    import torch
    B, S, H, KVH, d, L = 4, 8192, 16, 4, 128, 36
    QD, KD = H * d, KVH * d
    QKV = QD + 2 * KD
    rotate = (layer + 1) % 4 != 0
    qkv_h = seeded_f16((B, S, QKV), 300 + layer)
    qkv = dev(qkv_h)
    cache = torch.zeros((B, L, 2, S, KD), dtype=torch.float16, device=cuda)
    cos, sin = b200attn.rope_tables_host(S, d, 5.0e6)
    dcos, dsin = dev(cos), dev(sin)
    for b in range(B):
        row = qkv[b]
        b200attn.launch_rope_and_store_kv(row, row[:, QD:], row[:, QD + KD:], cache[b, layer, 0], cache[b, layer, 1],
                                          dcos, dsin, S, H, KVH, d, QKV, QKV, 0, rotate)
    out = torch.full((B, S, QD), float("nan"), dtype=torch.float16, device=cuda)
    b200attn.launch_causal_attention_prefill_batched(qkv, cache[0, layer, 0], cache[0, layer, 1], out, B, S, H, KVH,
                                                     d, QKV, KD, S * QKV, L * 2 * S * KD, S * QD)
    _sync()
    assert b200attn.lib().b2_device_error_word() == 0
    got = host(out)
    assert np.all(np.isfinite(got.astype(np.float32)))
    # the neighbouring layers of the cache stay untouched
    assert not bool(cache[:, layer - 1].any()) and not bool(cache[:, layer + 1].any())
    # sequence 0: RoPE/append bit-exact against the oracle
    q0 = np.ascontiguousarray(qkv_h[0, :, :QD])
    k0 = np.ascontiguousarray(qkv_h[0, :, QD:QD + KD])
    v0 = np.ascontiguousarray(qkv_h[0, :, QD + KD:])
    kc = np.zeros((S, KD), np.float16)
    vc = np.zeros((S, KD), np.float16)
    oracle.rope_and_store_kv(q0, k0, v0, kc, vc, cos, sin, S, H, KVH, d, QD, KD, 0, rotate)
    np.testing.assert_array_equal(bits(host(cache[0, layer, 0])), bits(kc))
    np.testing.assert_array_equal(bits(host(cache[0, layer, 1])), bits(vc))
    # every sequence, every head: sampled rows vs the FP32 oracle on the
    # device's own rotated Q and cache rows
    q_rot = host(qkv[:, :, :QD])
    rng = np.random.default_rng(layer)
    for b in range(B):
        rows = sorted(set([0, 127, 128, 8191 - 128, S - 1] + list(rng.integers(0, S, 11))))
        kb = host(cache[b, layer, 0])
        vb = host(cache[b, layer, 1])
        _, o32 = oracle.causal_attention(np.ascontiguousarray(q_rot[b]), kb, vb, S, H, KVH, d, rows=rows)
        assert_attention_close(got[b][rows], o32)
