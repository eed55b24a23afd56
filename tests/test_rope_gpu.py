"""RoPE + KV-cache append on the GPU vs the CPU oracle (bit-exact) and the
golden vectors (the reference's tolerance). Restates tests/test_rope.cpp."""
import numpy as np
import pytest

import b200attn
import oracle
from _gpu import Graph, bits, dev, host
from _util import golden, seeded_f16, tensor_close_mismatches

pytestmark = pytest.mark.gpu

SENTINEL = np.float16(-123.0)


def _tables(max_seq, d, theta):
    cos, sin = b200attn.rope_tables_host(max_seq, d, theta)
    return cos, sin


def test_launch_rope_in_place_matches_golden_and_oracle(cuda):
    """tests/test_rope.cpp:30-90 plus tests/test_qkv_gemm.cpp:87-117 (interleaved rows)."""
    meta, g = golden()
    S, H, KVH, d = meta["seq_len"], meta["num_heads"], meta["num_kv_heads"], meta["head_dim"]
    cos, sin = _tables(4096, d, meta["rope_theta"])
    dcos, dsin = dev(cos), dev(sin)
    for interleaved in (False, True):
        if interleaved:
            total = H * d + 2 * KVH * d
            qkv = np.concatenate([g["q"], g["k"], g["v"]], axis=1)
            buf = dev(qkv)
            b200attn.launch_rope(buf, buf[:, H * d:], dcos, dsin, S, H, KVH, d, total, total)
            out = host(buf)
            q_out, k_out, v_out = out[:, :H * d], out[:, H * d:H * d + KVH * d], out[:, H * d + KVH * d:]
            np.testing.assert_array_equal(bits(v_out), bits(g["v"]))
        else:
            dq, dk = dev(g["q"]), dev(g["k"])
            b200attn.launch_rope(dq, dk, dcos, dsin, S, H, KVH, d, H * d, KVH * d)
            q_out, k_out = host(dq), host(dk)
        torch_sync()
        assert tensor_close_mismatches(q_out, g["q_rope"], 2e-2, 2e-2) == 0
        assert tensor_close_mismatches(k_out, g["k_rope"], 2e-2, 2e-2) == 0
        oq, ok = g["q"].copy(), g["k"].copy()
        oracle.rope_and_store_kv(oq, ok, None, None, None, cos, sin, S, H, KVH, d, H * d, KVH * d, 0, True)
        np.testing.assert_array_equal(bits(q_out), bits(oq))
        np.testing.assert_array_equal(bits(k_out), bits(ok))


def torch_sync():
    import torch
    torch.cuda.synchronize()


@pytest.mark.parametrize("interleaved", [False, True])
@pytest.mark.parametrize("rotate", [False, True])
@pytest.mark.parametrize("start_pos", [0, 2])
def test_rope_and_store_kv_prefill(cuda, interleaved, rotate, start_pos):
    """tests/test_rope.cpp:92-195: sentinels, bit-exact V and NoPE K, untouched
    layer 0, untouched sources, Q rotated in place; here also bit-exact vs the oracle."""
    meta, g = golden()
    S, H, KVH, d = meta["seq_len"], meta["num_heads"], meta["num_kv_heads"], meta["head_dim"]
    q_dim, kv_dim = H * d, KVH * d
    cos, sin = _tables(4096, d, meta["rope_theta"])
    count = S - start_pos
    if interleaved:
        total = q_dim + 2 * kv_dim
        src = np.concatenate([g["q"][start_pos:], g["k"][start_pos:], g["v"][start_pos:]], axis=1).reshape(-1)
        q_off, k_off, v_off, qs, ks = 0, q_dim, q_dim + kv_dim, total, total
    else:
        src = np.concatenate([g["q"][start_pos:].ravel(), g["k"][start_pos:].ravel(), g["v"][start_pos:].ravel()])
        q_off, k_off, v_off, qs, ks = 0, count * q_dim, count * q_dim + count * kv_dim, q_dim, kv_dim
    cache = b200attn.KVCache(2, S + 2, KVH, d, device=cuda)
    cache.buffer.fill_(float(SENTINEL))
    dsrc = dev(src)
    b200attn.launch_rope_and_store_kv(dsrc[q_off:], dsrc[k_off:], dsrc[v_off:], cache.get_k_cache(1),
                                      cache.get_v_cache(1), dev(cos), dev(sin), count, H, KVH, d, qs, ks,
                                      start_pos, rotate)
    torch_sync()
    out_src = host(dsrc)
    kc, vc = host(cache.get_k_cache(1)), host(cache.get_v_cache(1))
    # oracle on the same inputs
    osrc = src.copy()
    ocache = np.full((2, S + 2, kv_dim), SENTINEL, np.float16)
    L = oracle.lib()
    base = osrc.ctypes.data
    c16, s16 = np.ascontiguousarray(cos.view(np.uint16)), np.ascontiguousarray(sin.view(np.uint16))
    assert L.or_rope_and_store_kv(base + 2 * q_off, base + 2 * k_off, base + 2 * v_off, ocache[0].ctypes.data,
                                  ocache[1].ctypes.data, c16.ctypes.data, s16.ctypes.data, count, H, KVH, d, qs,
                                  ks, start_pos, 1 if rotate else 0) == 0
    np.testing.assert_array_equal(bits(kc), bits(ocache[0]))
    np.testing.assert_array_equal(bits(vc), bits(ocache[1]))
    np.testing.assert_array_equal(bits(out_src), bits(osrc))
    # the reference's own checks against the golden fixtures
    exp_k = np.full((S + 2, kv_dim), SENTINEL, np.float16)
    exp_v = exp_k.copy()
    exp_k[start_pos:S] = (g["k_rope"] if rotate else g["k"])[start_pos:]
    exp_v[start_pos:S] = g["v"][start_pos:]
    assert tensor_close_mismatches(kc, exp_k, 2e-2 if rotate else 0, 2e-2 if rotate else 0) == 0
    np.testing.assert_array_equal(bits(vc), bits(exp_v))
    np.testing.assert_array_equal(bits(kc[:start_pos]), bits(exp_k[:start_pos]))
    np.testing.assert_array_equal(bits(kc[S:]), bits(exp_k[S:]))
    for t in (cache.get_k_cache(0), cache.get_v_cache(0)):
        assert np.all(bits(host(t)) == bits(np.array([SENTINEL]))[0])
    q_rows = (out_src[q_off:].reshape(count, -1)[:, :q_dim] if interleaved
              else out_src[:count * q_dim].reshape(count, q_dim))
    ref_q = (g["q_rope"] if rotate else g["q"])[start_pos:]
    assert tensor_close_mismatches(q_rows, ref_q, 2e-2 if rotate else 0, 2e-2 if rotate else 0) == 0
    np.testing.assert_array_equal(bits(out_src[k_off:]) if not interleaved else
                                  bits(out_src.reshape(count, -1)[:, q_dim:]),
                                  bits(src[k_off:]) if not interleaved else bits(src.reshape(count, -1)[:, q_dim:]))


@pytest.mark.parametrize("shape", [
    # (seq, H, KVH, d, q_stride_pad, k_stride_pad, start_pos)   vector path / scalar path
    (1, 16, 4, 128, 0, 0, 65599),
    (7, 16, 4, 128, 1024, 1024, 4093),
    (300, 16, 4, 128, 0, 0, 0),
    (33, 8, 2, 64, 0, 0, 17),
    (5, 4, 4, 32, 0, 0, 3),
    (9, 4, 2, 32, 1, 3, 11),       # odd strides -> scalar kernel
    (6, 6, 3, 20, 0, 0, 2),        # half_dim 10 -> scalar kernel
])
@pytest.mark.parametrize("rotate", [True, False])
def test_rope_store_random_shapes_bit_exact(cuda, shape, rotate):
    seq, H, KVH, d, qpad, kpad, start = shape
    q_dim, kv_dim = H * d, KVH * d
    qs, ks = q_dim + qpad, kv_dim + kpad
    max_seq = start + seq + 3
    cos, sin = _tables(max_seq, d, 5.0e6)
    q = seeded_f16(seq * qs, 10 + seq)
    k = seeded_f16(seq * ks, 20 + seq)
    v = seeded_f16(seq * ks, 30 + seq)
    kc = np.full((max_seq, kv_dim), SENTINEL, np.float16)
    vc = kc.copy()
    dq, dk, dv, dkc, dvc = dev(q), dev(k), dev(v), dev(kc), dev(vc)
    b200attn.launch_rope_and_store_kv(dq, dk, dv, dkc, dvc, dev(cos), dev(sin), seq, H, KVH, d, qs, ks, start, rotate)
    torch_sync()
    oq, ok, okc, ovc = q.copy(), k.copy(), kc.copy(), vc.copy()
    assert oracle.rope_and_store_kv(oq, ok, v, okc, ovc, cos, sin, seq, H, KVH, d, qs, ks, start, rotate) == 0
    np.testing.assert_array_equal(bits(host(dq)), bits(oq))
    np.testing.assert_array_equal(bits(host(dk)), bits(k))  # source never modified with a cache
    np.testing.assert_array_equal(bits(host(dkc)), bits(okc))
    np.testing.assert_array_equal(bits(host(dvc)), bits(ovc))


def test_position_coded_slots_exact(cuda):
    """Each position's table row differs, so a wrong row or slot index is a gross error."""
    seq, H, KVH, d, start = 64, 16, 4, 128, 30000
    max_seq = start + seq
    cos, sin = _tables(max_seq, d, 5.0e6)
    q = seeded_f16((seq, H * d), 5)
    k = seeded_f16((seq, KVH * d), 6)
    v = np.arange(seq * KVH * d, dtype=np.float32).reshape(seq, -1).astype(np.float16)
    kc = np.zeros((max_seq, KVH * d), np.float16)
    dkc, dvc = dev(kc), dev(kc)
    b200attn.launch_rope_and_store_kv(dev(q), dev(k), dev(v), dkc, dvc, dev(cos), dev(sin), seq, H, KVH, d, 0, 0,
                                      start, True)
    torch_sync()
    vc = host(dvc)
    np.testing.assert_array_equal(bits(vc[start:]), bits(v))
    assert not np.any(bits(vc[:start]))
    oq, ok, okc, ovc = q.copy(), k.copy(), kc.copy(), kc.copy()
    oracle.rope_and_store_kv(oq, ok, v, okc, ovc, cos, sin, seq, H, KVH, d, 0, 0, start, True)
    np.testing.assert_array_equal(bits(host(dkc)), bits(okc))


def test_rope_graph_node_update(cuda):
    """Capture the append at start_pos 5, patch to 9 with update_rope_and_store_kv_node
    (rope.hip.cpp:208-241), replay: identical to a direct launch at 9."""
    import torch
    H, KVH, d, max_seq = 16, 4, 128, 32
    cos, sin = _tables(max_seq, d, 5.0e6)
    dcos, dsin = dev(cos), dev(sin)
    qkv = seeded_f16((1, H * d + 2 * KVH * d), 77)
    total = qkv.shape[1]
    for rotate in (True, False):
        buf = dev(qkv)
        kc = torch.zeros((max_seq, KVH * d), dtype=torch.float16, device=cuda)
        vc = torch.zeros_like(kc)
        gph = Graph()
        with gph:
            b200attn.launch_rope_and_store_kv(buf, buf[:, H * d:], buf[:, H * d + KVH * d:], kc, vc, dcos, dsin, 1,
                                              H, KVH, d, total, total, 5, rotate, stream=gph.stream)
            n = gph.last_node()
        b200attn.update_rope_and_store_kv_node(gph.exec_handle, n, 9, rotate)
        gph.launch()
        got_q, got_k, got_v = host(buf), host(kc), host(vc)
        gph.close()
        buf2 = dev(qkv)
        kc2 = torch.zeros_like(kc)
        vc2 = torch.zeros_like(kc)
        b200attn.launch_rope_and_store_kv(buf2, buf2[:, H * d:], buf2[:, H * d + KVH * d:], kc2, vc2, dcos, dsin, 1,
                                          H, KVH, d, total, total, 9, rotate)
        torch_sync()
        np.testing.assert_array_equal(bits(got_q), bits(host(buf2)))
        np.testing.assert_array_equal(bits(got_k), bits(host(kc2)))
        np.testing.assert_array_equal(bits(got_v), bits(host(vc2)))
        assert not np.any(bits(got_k[5])) and np.any(bits(got_k[9]))
