"""Pin the CPU oracle before trusting it (CPU only, no GPU).

* golden vectors from the reference's own fixture generator
  (python/reference.py save_activations, see tests/golden/make_golden.py);
* the self-contained known-answer test of tests/test_causal_attention.cpp:152-228;
* the invariants of tests/test_rope.cpp:92-195 on the oracle's append path.
"""
import math

import numpy as np
import pytest

import oracle
from _util import (assert_attention_close, golden, max_abs, rel_l2, seeded_f16,
                   tensor_close_mismatches)


def test_half_conversions_match_numpy():
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    ref = bits.view(np.float16).astype(np.float32)
    L = oracle.lib()
    got = np.array([L.or_half_to_float(int(b)) for b in bits[::7]], np.float32)
    np.testing.assert_array_equal(got.view(np.uint32)[~np.isnan(got)],
                                  ref[::7].view(np.uint32)[~np.isnan(ref[::7])])
    rng = np.random.default_rng(0)
    xs = np.concatenate([rng.standard_normal(20000).astype(np.float32) * s for s in (1e-6, 1e-3, 1, 100, 7e4)])
    xs = np.concatenate([xs, np.float32([0.0, -0.0, 65504, 65520, 65519.99, 6.1e-5, 5.96e-8, 2.98e-8, 2.99e-8])])
    got = np.array([L.or_float_to_half(float(x)) for x in xs], np.uint16)
    with np.errstate(over="ignore"):
        ref16 = xs.astype(np.float16)
    np.testing.assert_array_equal(got, ref16.view(np.uint16))


def test_rope_table_matches_hf_rotary_embedding():
    """rope_cache.hpp tables vs the HF rotary embedding the fixtures used."""
    torch = pytest.importorskip("torch")
    tr = pytest.importorskip("transformers")
    from transformers.models.smollm3.modeling_smollm3 import SmolLM3RotaryEmbedding
    cfg = tr.SmolLM3Config(hidden_size=2048, num_attention_heads=16, num_key_value_heads=4,
                           max_position_embeddings=4096,
                           rope_parameters={"rope_type": "default", "rope_theta": 5.0e6})
    emb = SmolLM3RotaryEmbedding(cfg)
    c, s = emb(torch.zeros(1, dtype=torch.float16), torch.arange(4096).unsqueeze(0))
    cos, sin = oracle.rope_tables(4096, 128, 5.0e6)
    assert max_abs(c[0, :, :64].numpy(), cos) <= 1e-3
    assert max_abs(s[0, :, :64].numpy(), sin) <= 1e-3
    # and HF's second half is the first half repeated (rotate-half convention)
    np.testing.assert_array_equal(c[0, :, :64].numpy(), c[0, :, 64:].numpy())


def test_oracle_rope_matches_golden():
    meta, g = golden()
    S, H, KVH, d = meta["seq_len"], meta["num_heads"], meta["num_kv_heads"], meta["head_dim"]
    cos, sin = oracle.rope_tables(4096, d, meta["rope_theta"])
    q, k = g["q"].copy(), g["k"].copy()
    assert oracle.rope_and_store_kv(q, k, None, None, None, cos, sin, S, H, KVH, d, H * d, KVH * d, 0, True) == 0
    # test_rope.cpp:82-85 tolerance, and at most one fp16 step of the HF fp16 path
    assert tensor_close_mismatches(q, g["q_rope"], 2e-2, 2e-2) == 0
    assert tensor_close_mismatches(k, g["k_rope"], 2e-2, 2e-2) == 0
    assert max_abs(q, g["q_rope"]) <= 4e-3 and max_abs(k, g["k_rope"]) <= 4e-3


def test_oracle_prefill_matches_golden():
    meta, g = golden()
    S, H, KVH, d = meta["seq_len"], meta["num_heads"], meta["num_kv_heads"], meta["head_dim"]
    o16, o32 = oracle.causal_attention(g["q_rope"], g["k_rope"], g["v"], S, H, KVH, d)
    assert tensor_close_mismatches(o16, g["attn"], 2e-2, 2e-2) == 0  # test_causal_attention.cpp:73
    assert_attention_close(g["attn"], o32)


def test_oracle_decode_rows_match_golden_prefill_rows():
    """test_causal_attention.cpp:80-150 on the oracle: decode at kv_len p+1 == prefill row p."""
    meta, g = golden()
    S, H, KVH, d = meta["seq_len"], meta["num_heads"], meta["num_kv_heads"], meta["head_dim"]
    for p in range(S):
        q = np.ascontiguousarray(g["q_rope"][p])
        o16, o32 = oracle.decode_attention(q, g["k_rope"], g["v"], p + 1, H, KVH, d)
        assert tensor_close_mismatches(o16.reshape(-1), g["attn"][p], 2e-2, 2e-2) == 0
        po, pm, pl = oracle.decode_partials(q, g["k_rope"], g["v"], p + 1, H, KVH, d, 0, 12)
        m16, m32 = oracle.merge_partials(po, pm, pl)
        assert max_abs(m32, o32) <= 2e-3


def _kat_inputs(head_dim, kv_heads, length, padded, heads=4):
    """tests/test_causal_attention.cpp:165-175 generators."""
    q_dim, kv_dim = heads * head_dim, kv_heads * head_dim
    stride = kv_dim + (17 if padded else 0)
    q = (2.0 * np.sin((np.arange(q_dim) + 1).astype(np.float32) * np.float32(0.37))).astype(np.float16)
    k = np.full((length + 2) * stride, 123.0, np.float16)
    v = k.copy()
    t = np.arange(length)[:, None]
    i = np.arange(kv_dim)[None, :]
    idx = t * stride + i
    k[idx] = (3.0 * np.cos((t * kv_dim + i + 1).astype(np.float32) * np.float32(0.13))).astype(np.float16)
    v[idx] = np.sin((t * kv_dim + i + 3).astype(np.float32) * np.float32(0.19)).astype(np.float16)
    return q, k, v, stride


def _kat_expected(q, k, v, heads, kv_heads, head_dim, length, stride):
    """The double-precision loop of tests/test_causal_attention.cpp:176-196, in numpy."""
    out = np.zeros(heads * head_dim, np.float16)
    for h in range(heads):
        kh = h // (heads // kv_heads)
        qh = q[h * head_dim:(h + 1) * head_dim].astype(np.float64)
        K = np.stack([k[t * stride + kh * head_dim: t * stride + (kh + 1) * head_dim] for t in range(length)]).astype(np.float64)
        V = np.stack([v[t * stride + kh * head_dim: t * stride + (kh + 1) * head_dim] for t in range(length)]).astype(np.float64)
        sc = K @ qh / math.sqrt(head_dim)
        w = np.exp(sc - sc.max())
        out[h * head_dim:(h + 1) * head_dim] = ((w @ V) / w.sum()).astype(np.float32).astype(np.float16)
    return out


KAT_LENGTHS = [1, 12, 13, 37, 257, 256, 513, 769]


@pytest.mark.parametrize("head_dim", [32, 128])
@pytest.mark.parametrize("kv_heads", [1, 2, 4])
@pytest.mark.parametrize("padded", [False, True])
def test_oracle_flash_decode_known_answer(head_dim, kv_heads, padded):
    heads = 4
    for length in KAT_LENGTHS:
        q, k, v, stride = _kat_inputs(head_dim, kv_heads, length, padded)
        exp = _kat_expected(q, k, v, heads, kv_heads, head_dim, length, stride)
        got16, _ = oracle.decode_attention(q, k, v, length, heads, kv_heads, head_dim, stride)
        assert tensor_close_mismatches(got16.reshape(-1), exp, 2e-3, 2e-3) == 0
        for chunk in (12, 256):
            po, pm, pl = oracle.decode_partials(q, k, v, length, heads, kv_heads, head_dim, stride, chunk)
            m16, _ = oracle.merge_partials(po, pm, pl)
            assert tensor_close_mismatches(m16.reshape(-1), exp, 2e-3, 2e-3) == 0


def test_oracle_unscaled_merge_is_caught():
    """Merging chunk outputs without the e^(m_c - M) rescale must fail the check
    (the property the known-answer generators are built for, :171-172)."""
    q, k, v, stride = _kat_inputs(128, 2, 37, False)
    exp = _kat_expected(q, k, v, 4, 2, 128, 37, stride)
    po, pm, pl = oracle.decode_partials(q, k, v, 37, 4, 2, 128, stride, 12)
    bad = (po.sum(axis=1) / pl.sum(axis=1)[:, None]).astype(np.float16).reshape(-1)
    assert tensor_close_mismatches(bad, exp, 2e-3, 2e-3) > 0


@pytest.mark.parametrize("interleaved", [False, True])
@pytest.mark.parametrize("rotate", [False, True])
@pytest.mark.parametrize("start_pos", [0, 2])
def test_oracle_rope_store_invariants(interleaved, rotate, start_pos):
    """tests/test_rope.cpp:92-195 on the oracle with the golden inputs."""
    meta, g = golden()
    S, H, KVH, d = meta["seq_len"], meta["num_heads"], meta["num_kv_heads"], meta["head_dim"]
    q_dim, kv_dim = H * d, KVH * d
    cos, sin = oracle.rope_tables(4096, d, meta["rope_theta"])
    count = S - start_pos
    max_seq = S + 2
    if interleaved:
        total = q_dim + 2 * kv_dim
        src = np.zeros((count, total), np.float16)
        src[:, :q_dim] = g["q"][start_pos:]
        src[:, q_dim:q_dim + kv_dim] = g["k"][start_pos:]
        src[:, q_dim + kv_dim:] = g["v"][start_pos:]
        qv, kvv, vv = src[:, :q_dim], src[:, q_dim:q_dim + kv_dim], src[:, q_dim + kv_dim:]
        flat = src.reshape(-1)
        qs = ks = total
        qb, kb, vb = flat[0:], flat[q_dim:], flat[q_dim + kv_dim:]
    else:
        flat = np.concatenate([g["q"][start_pos:].ravel(), g["k"][start_pos:].ravel(), g["v"][start_pos:].ravel()])
        qs, ks = q_dim, kv_dim
        qb, kb, vb = flat[0:], flat[count * q_dim:], flat[count * q_dim + count * kv_dim:]
    original = flat.copy()
    cache = np.full((2, 2, max_seq, kv_dim), -123.0, np.float16)  # 2 layers x (K, V)
    kc, vc = cache[1, 0], cache[1, 1]
    # oracle takes contiguous buffers: operate on the flat source through offsets
    buf = flat
    off_k = kb.__array_interface__["data"][0] - buf.__array_interface__["data"][0]
    off_v = vb.__array_interface__["data"][0] - buf.__array_interface__["data"][0]
    L = oracle.lib()
    base = buf.ctypes.data
    cos16, sin16 = np.ascontiguousarray(cos.view(np.uint16)), np.ascontiguousarray(sin.view(np.uint16))
    rc = L.or_rope_and_store_kv(base, base + off_k, base + off_v, kc.ctypes.data, vc.ctypes.data,
                                cos16.ctypes.data, sin16.ctypes.data, count, H, KVH, d, qs, ks, start_pos,
                                1 if rotate else 0)
    assert rc == 0
    exp_k = np.full((max_seq, kv_dim), -123.0, np.float16)
    exp_v = exp_k.copy()
    exp_k[start_pos:S] = (g["k_rope"] if rotate else g["k"])[start_pos:]
    exp_v[start_pos:S] = g["v"][start_pos:]
    assert tensor_close_mismatches(kc, exp_k, 2e-2 if rotate else 0, 2e-2 if rotate else 0) == 0
    np.testing.assert_array_equal(vc.view(np.uint16), exp_v.view(np.uint16))
    np.testing.assert_array_equal(cache[0].view(np.uint16), np.full_like(cache[0], -123.0).view(np.uint16))
    # K/V sources untouched; Q rotated in place or untouched
    if interleaved:
        s2 = buf.reshape(count, -1)
        o2 = original.reshape(count, -1)
        np.testing.assert_array_equal(s2[:, q_dim:].view(np.uint16), o2[:, q_dim:].view(np.uint16))
        qout = s2[:, :q_dim]
    else:
        np.testing.assert_array_equal(buf[count * q_dim:].view(np.uint16), original[count * q_dim:].view(np.uint16))
        qout = buf[:count * q_dim].reshape(count, q_dim)
    ref_q = (g["q_rope"] if rotate else g["q"])[start_pos:]
    assert tensor_close_mismatches(qout, ref_q, 2e-2 if rotate else 0, 2e-2 if rotate else 0) == 0


def test_oracle_prefill_start_pos_and_rows():
    """Row sampling and start_pos offsets agree with the full evaluation."""
    S, H, KVH, d = 70, 4, 2, 32
    q = seeded_f16((S + 5, H * d), 1)
    k = seeded_f16((S + 5, KVH * d), 2)
    v = seeded_f16((S + 5, KVH * d), 3)
    full16, full32 = oracle.causal_attention(q, k, v, S + 5, H, KVH, d)
    rows = [0, 3, 40, 69]
    _, part32 = oracle.causal_attention(q[5:], k, v, S, H, KVH, d, start_pos=5, rows=rows)
    np.testing.assert_allclose(part32, full32[[r + 5 for r in rows]], rtol=0, atol=1e-6)
    assert rel_l2(full16, full32) < 1e-3


def test_torch_reference_path_matches_golden():
    """The CPU-baseline restatement of python/reference.py:62-92 (HF RoPE,
    repeat_interleave, causal SDPA) reproduces the fixtures the reference's
    own generator wrote, in FP16 as the reference runs it and in FP32."""
    torch = pytest.importorskip("torch")
    pytest.importorskip("transformers")
    from oracle import torch_ref
    meta, g = golden()
    S, H, KVH, d = meta["seq_len"], meta["num_heads"], meta["num_kv_heads"], meta["head_dim"]
    q, k, v = (torch.from_numpy(g[n].copy()) for n in ("q", "k", "v"))
    # FP16 as the fixtures were made: within 2e-3; FP32 differs from the FP16
    # fixtures by their own rounding (values up to ~3, fp16 step 2e-3): 1e-2
    for dt, tol in ((torch.float16, 2e-3), (torch.float32, 1e-2)):
        out = torch_ref.prefill(q, k, v, H, KVH, d, meta["rope_theta"], dtype=dt).float().numpy()
        assert tensor_close_mismatches(out, g["attn"], 2e-2, 2e-2) == 0
        assert max_abs(out, g["attn"]) <= tol


def test_torch_reference_decode_matches_oracle():
    """Its one-token form (append + attention over every cached row) against
    the C oracle's double-precision decode."""
    torch = pytest.importorskip("torch")
    pytest.importorskip("transformers")
    from oracle import torch_ref
    H, KVH, d, past = 16, 4, 128, 300
    total = H * d + 2 * KVH * d
    cache_k = seeded_f16((past + 1, KVH * d), 41, std=0.5)
    cache_v = seeded_f16((past + 1, KVH * d), 42, std=0.5)
    new = seeded_f16(total, 43)
    q, kn, vn = new[:H * d].copy(), new[H * d:H * d + KVH * d].copy(), new[H * d + KVH * d:].copy()
    kc, vc = torch.from_numpy(cache_k.astype(np.float32)), torch.from_numpy(cache_v.astype(np.float32))
    got = torch_ref.decode(torch.from_numpy(q), torch.from_numpy(kn), torch.from_numpy(vn), kc, vc, past, H, KVH, d)
    cos, sin = oracle.rope_tables(past + 1, d, 5.0e6)
    ck, cv = cache_k.copy(), cache_v.copy()
    oracle.rope_and_store_kv(q, kn, vn, ck, cv, cos, sin, 1, H, KVH, d, H * d, KVH * d, past, True)
    _, o32 = oracle.decode_attention(q, ck, cv, past + 1, H, KVH, d)
    assert_attention_close(got.numpy(), o32.reshape(-1))


def test_oracle_matches_sharp_golden():
    """The 160-token fixture with a peaked softmax (logit std ~13): RoPE within
    one fp16 step of the reference's FP16 path, attention within the
    reference tolerance and the BASELINE bar."""
    meta, g = golden("sharp")
    S, H, KVH, d = meta["seq_len"], meta["num_heads"], meta["num_kv_heads"], meta["head_dim"]
    cos, sin = oracle.rope_tables(4096, d, meta["rope_theta"])
    q, k = g["q"].copy(), g["k"].copy()
    assert oracle.rope_and_store_kv(q, k, None, None, None, cos, sin, S, H, KVH, d, H * d, KVH * d, 0, True) == 0
    assert tensor_close_mismatches(q, g["q_rope"], 2e-2, 2e-2) == 0
    assert tensor_close_mismatches(k, g["k_rope"], 2e-2, 2e-2) == 0
    o16, o32 = oracle.causal_attention(g["q_rope"], g["k_rope"], g["v"], S, H, KVH, d)
    assert tensor_close_mismatches(o16, g["attn"], 2e-2, 2e-2) == 0
    assert_attention_close(g["attn"], o32)


def test_torch_reference_path_matches_sharp_golden():
    torch = pytest.importorskip("torch")
    pytest.importorskip("transformers")
    from oracle import torch_ref
    meta, g = golden("sharp")
    S, H, KVH, d = meta["seq_len"], meta["num_heads"], meta["num_kv_heads"], meta["head_dim"]
    q, k, v = (torch.from_numpy(g[n].copy()) for n in ("q", "k", "v"))
    out = torch_ref.prefill(q, k, v, H, KVH, d, meta["rope_theta"], dtype=torch.float16).float().numpy()
    assert tensor_close_mismatches(out, g["attn"], 2e-2, 2e-2) == 0
