"""Ragged batched decode (one new token for each of B sequences of different
lengths; benchmark config 5) on the GPU vs the CPU oracle, per sequence.
The oracle is the reference's single-sequence algebra
(src/kernels/rope.hip.cpp:61-134, src/kernels/causal_attention.hip.cpp:493-838)
applied to each sequence in turn."""
import numpy as np
import pytest

import b200attn
import oracle
from _gpu import bits, dev, host
from _util import assert_attention_close, seeded_f16

pytestmark = pytest.mark.gpu
D = 128
THETA = 5.0e6


def _sync():
    import torch
    torch.cuda.synchronize()


def _workspace(B, H, KVH, max_len):
    import torch
    n = b200attn.decode_ragged_workspace_bytes(B, H, KVH, max_len)
    return torch.zeros(n, dtype=torch.uint8, device="cuda"), n


def _ragged(q, kc, vc, lens, H, KVH, max_len, bias=0, ws=None, cache_seq_stride=0):
    """q [B][H*D] (numpy or device), kc/vc device caches [B][max_len][KVH*D]."""
    import torch
    B = len(lens)
    dq = q if isinstance(q, torch.Tensor) else dev(q)
    dl = torch.tensor(np.asarray(lens, np.int32) - bias, dtype=torch.int32, device="cuda")
    out = torch.full((B, H * D), -7.0, dtype=torch.float16, device="cuda")
    if ws is None:
        ws = _workspace(B, H, KVH, max_len)
    b200attn.launch_causal_attention_decode_ragged(dq, 0, kc, vc, cache_seq_stride, dl, bias, max_len, out, 0, B, H,
                                                   KVH, D, ws[0], ws[1])
    _sync()
    return host(out)


def _check(got, q, kh, vh, lens, H, KVH):
    for b, n in enumerate(lens):
        if n == 0:
            assert np.all(got[b] == 0)
            continue
        _, o32 = oracle.decode_attention(q[b], kh[b], vh[b], n, H, KVH, D)
        assert_attention_close(got[b], o32.reshape(-1))


@pytest.mark.parametrize("kvh,heads", [(4, 16), (1, 8), (2, 16), (8, 32)])
def test_ragged_lengths_vs_oracle(cuda, kvh, heads):
    """Lengths at every tile / unit edge, including 0 and 1, one launch."""
    lens = [0, 1, 2, 15, 16, 17, 255, 256, 257, 287, 288, 289, 383, 384, 385, 1000, 3001]
    max_len = 3072 + 64
    lens = [min(n, max_len) for n in lens]
    B = len(lens)
    kh = seeded_f16((B, max_len, kvh * D), 11 + kvh)
    vh = seeded_f16((B, max_len, kvh * D), 12 + kvh)
    q = seeded_f16((B, heads * D), 13 + kvh)
    got = _ragged(q, dev(kh), dev(vh), lens, heads, kvh, max_len)
    _check(got, q, kh, vh, lens, heads, kvh)
    assert b200attn.lib().b2_device_error_word() == 0


def test_ragged_config5_shape(cuda):
    """benchmark config 5: 64 sequences, lengths U[512, 16384] from
    numpy default_rng(seed).integers(512, 16385, 64), 16/4 heads, one layer."""
    import torch
    H, KVH, max_len, B = 16, 4, 16384, 64
    lens = [int(x) for x in np.random.default_rng(5).integers(512, 16385, B)]
    kc = torch.empty((B, max_len, KVH * D), dtype=torch.float16, device=cuda)
    vc = torch.empty_like(kc)
    kh = np.empty((B, max_len, KVH * D), np.float16)
    vh = np.empty_like(kh)
    for b in range(B):
        n = lens[b]
        kh[b, :n] = seeded_f16((n, KVH * D), 1000 + b)
        vh[b, :n] = seeded_f16((n, KVH * D), 2000 + b)
        kh[b, n:] = np.float16(3e4)   # rows past a sequence's length are never read
        vh[b, n:] = np.float16(-3e4)
    kc.copy_(torch.from_numpy(kh))
    vc.copy_(torch.from_numpy(vh))
    q = seeded_f16((B, H * D), 77)
    got = _ragged(q, kc, vc, lens, H, KVH, max_len)
    _check(got, q, kh, vh, lens, H, KVH)


def test_ragged_matches_single_sequence_decode(cuda):
    """Each sequence's output equals the single-sequence decode of that sequence."""
    import torch
    H, KVH, max_len = 16, 4, 4096
    lens = [4096, 1, 700, 2049]
    B = len(lens)
    kh = seeded_f16((B, max_len, KVH * D), 31)
    vh = seeded_f16((B, max_len, KVH * D), 32)
    q = seeded_f16((B, H * D), 33)
    kc, vc = dev(kh), dev(vh)
    got = _ragged(q, kc, vc, lens, H, KVH, max_len)
    for b, n in enumerate(lens):
        wsf = torch.empty(b200attn.decode_workspace_floats(H, D, n), dtype=torch.float32, device=cuda)
        c = H * ((n + 255) // 256)
        one = torch.empty(H * D, dtype=torch.float16, device=cuda)
        b200attn.launch_causal_attention_decode(dev(q[b]), kc[b], vc[b], one, wsf[:c * D], wsf[c * D:c * (D + 1)],
                                                wsf[c * (D + 1):], 1, n, n - 1, H, KVH, D, 0, 0)
        _sync()
        assert np.max(np.abs(host(one).astype(np.float32) - got[b].astype(np.float32))) <= 2e-3


def test_ragged_workspace_reuse_and_bias(cuda):
    """One workspace across calls whose unit counts differ (the claim counter is
    reset every call); device lengths with a bias, and clamping at max_kv_len."""
    H, KVH, max_len = 16, 4, 2048
    B = 6
    kh = seeded_f16((B, max_len, KVH * D), 41)
    vh = seeded_f16((B, max_len, KVH * D), 42)
    kc, vc = dev(kh), dev(vh)
    ws = _workspace(B, H, KVH, max_len)
    rng = np.random.default_rng(3)
    for it in range(6):
        lens = [int(x) for x in rng.integers(0, max_len + 1, B)]
        q = seeded_f16((B, H * D), 50 + it)
        got = _ragged(q, kc, vc, lens, H, KVH, max_len, bias=1 if it % 2 else 0, ws=ws)
        _check(got, q, kh, vh, lens, H, KVH)
    # lengths past max_kv_len are clamped
    q = seeded_f16((B, H * D), 99)
    got = _ragged(q, kc, vc, [max_len + 500] * B, H, KVH, max_len, ws=ws)
    _check(got, q, kh, vh, [max_len] * B, H, KVH)
    assert b200attn.lib().b2_device_error_word() == 0


def test_ragged_rope_append_then_decode(cuda):
    """Config-5 step for one layer: RoPE + append of each sequence's new token at
    its own position (bit-exact vs the oracle), then the ragged decode over
    len + 1 tokens."""
    import torch
    H, KVH, max_len = 16, 4, 1024
    lens = [0, 5, 255, 256, 1000]   # tokens already cached; the new one goes to row len
    B = len(lens)
    total = H * D + 2 * KVH * D
    cos, sin = b200attn.rope_tables_host(max_len, D, THETA)
    kh = seeded_f16((B, max_len, KVH * D), 61)
    vh = seeded_f16((B, max_len, KVH * D), 62)
    qkv = seeded_f16((B, total), 63)
    kc, vc = dev(kh), dev(vh)
    dqkv = dev(qkv)
    pos = torch.tensor(lens, dtype=torch.int32, device=cuda)
    b200attn.launch_rope_and_store_kv_ragged(dqkv, dqkv[:, H * D:], dqkv[:, H * D + KVH * D:], kc, vc,
                                             max_len * KVH * D, dev(cos), dev(sin), B, H, KVH, D, total, total, pos,
                                             max_len, True)
    _sync()
    ek, ev = kh.copy(), vh.copy()
    eq = qkv.copy()
    for b, p in enumerate(lens):
        oq, ok, ov = eq[b, :H * D].copy(), eq[b, H * D:H * D + KVH * D].copy(), eq[b, H * D + KVH * D:].copy()
        oracle.rope_and_store_kv(oq, ok, ov, ek[b], ev[b], cos, sin, 1, H, KVH, D, H * D, KVH * D, p, True)
        eq[b, :H * D] = oq
    np.testing.assert_array_equal(bits(host(kc)), bits(ek))
    np.testing.assert_array_equal(bits(host(vc)), bits(ev))
    np.testing.assert_array_equal(bits(host(dqkv)[:, :H * D]), bits(eq[:, :H * D]))
    got = _ragged(dqkv[:, :H * D].contiguous(), kc, vc, [n + 1 for n in lens], H, KVH, max_len)
    _check(got, np.ascontiguousarray(eq[:, :H * D]), ek, ev, [n + 1 for n in lens], H, KVH)


def test_ragged_rope_nope_and_out_of_range(cuda):
    """NoPE layers copy K/V verbatim; a position outside the cache is skipped."""
    import torch
    H, KVH, max_len = 16, 4, 64
    B = 3
    total = H * D + 2 * KVH * D
    cos, sin = b200attn.rope_tables_host(max_len, D, THETA)
    kh = seeded_f16((B, max_len, KVH * D), 71)
    vh = seeded_f16((B, max_len, KVH * D), 72)
    qkv = seeded_f16((B, total), 73)
    kc, vc = dev(kh), dev(vh)
    dqkv = dev(qkv)
    pos = torch.tensor([3, max_len, 63], dtype=torch.int32, device=cuda)
    b200attn.launch_rope_and_store_kv_ragged(dqkv, dqkv[:, H * D:], dqkv[:, H * D + KVH * D:], kc, vc,
                                             max_len * KVH * D, dev(cos), dev(sin), B, H, KVH, D, total, total, pos,
                                             max_len, False)
    _sync()
    ek, ev = kh.copy(), vh.copy()
    ek[0, 3], ev[0, 3] = qkv[0, H * D:H * D + KVH * D], qkv[0, H * D + KVH * D:]
    ek[2, 63], ev[2, 63] = qkv[2, H * D:H * D + KVH * D], qkv[2, H * D + KVH * D:]
    np.testing.assert_array_equal(bits(host(kc)), bits(ek))
    np.testing.assert_array_equal(bits(host(vc)), bits(ev))
    np.testing.assert_array_equal(bits(host(dqkv)), bits(qkv))   # NoPE leaves Q untouched


def _fused_ragged(qkv_d, kc, vc, cache_seq_stride, cos_d, sin_d, rope_rows, rotate, pos, max_len, B, H, KVH,
                  ws=None, append=True):
    import torch
    total = H * D + 2 * KVH * D
    out = torch.full((B, H * D), -7.0, dtype=torch.float16, device="cuda")
    if ws is None:
        ws = _workspace(B, H, KVH, max_len)
    b200attn.launch_decode_step_ragged_fused(qkv_d, total, qkv_d[:, H * D:] if append else None,
                                             qkv_d[:, H * D + KVH * D:] if append else None, total, kc, vc,
                                             cache_seq_stride, cos_d if rotate else None, sin_d if rotate else None,
                                             rope_rows, rotate, pos, max_len, out, 0, B, H, KVH, D, ws[0], ws[1])
    _sync()
    return host(out)


def _oracle_ragged_step(qkv, kh, vh, pos, cos, sin, rotate, H, KVH, max_len):
    """Per sequence: RoPE + append at row p (the reference's launch_rope_and_store_kv,
    rope.hip.cpp:138-196), then decode over rows [0, p]."""
    B = len(pos)
    ek, ev = kh.copy(), vh.copy()
    outs = []
    qd, kd = H * D, KVH * D
    for b, p in enumerate(pos):
        oq, ok, ov = qkv[b, :qd].copy(), qkv[b, qd:qd + kd].copy(), qkv[b, qd + kd:].copy()
        if 0 <= p < max_len:
            oracle.rope_and_store_kv(oq, ok, ov, ek[b], ev[b], cos, sin, 1, H, KVH, D, qd, kd, p, rotate)
        n = min(p + 1, max_len) if p >= 0 else 0
        if n == 0:
            outs.append(None)
            continue
        _, o32 = oracle.decode_attention(oq, ek[b], ev[b], n, H, KVH, D)
        outs.append(o32.reshape(-1))
    return ek, ev, outs


@pytest.mark.parametrize("rotate", [True, False])
@pytest.mark.parametrize("H,KVH", [(16, 4), (4, 1), (8, 2)])
def test_ragged_fused_step_vs_oracle(cuda, rotate, H, KVH):
    """One call per layer: RoPE of each sequence's new token, its K/V append and
    the ragged decode; caches bit-exact vs the oracle, outputs within tolerance,
    the QKV rows untouched. Positions at 0, tile and unit edges, and the last
    row; one and two KV heads (a tensor-parallel rank's share) included."""
    import torch
    max_len = 2048
    pos = [0, 1, 15, 16, 255, 256, 287, 288, 767, 768, 1000, max_len - 1]
    B = len(pos)
    total = H * D + 2 * KVH * D
    cos, sin = b200attn.rope_tables_host(max_len, D, THETA)
    kh = seeded_f16((B, max_len, KVH * D), 81)
    vh = seeded_f16((B, max_len, KVH * D), 82)
    qkv = seeded_f16((B, total), 83)
    kc, vc, dqkv = dev(kh), dev(vh), dev(qkv)
    dpos = torch.tensor(pos, dtype=torch.int32, device=cuda)
    got = _fused_ragged(dqkv, kc, vc, max_len * KVH * D, dev(cos), dev(sin), max_len, rotate, dpos, max_len, B, H, KVH)
    ek, ev, outs = _oracle_ragged_step(qkv, kh, vh, pos, cos, sin, rotate, H, KVH, max_len)
    np.testing.assert_array_equal(bits(host(kc)), bits(ek))
    np.testing.assert_array_equal(bits(host(vc)), bits(ev))
    np.testing.assert_array_equal(bits(host(dqkv)), bits(qkv))  # Q / K / V rows are read, not written
    for b, o32 in enumerate(outs):
        assert_attention_close(got[b], o32)
    assert b200attn.lib().b2_device_error_word() == 0


def test_ragged_fused_step_equals_two_launches(cuda):
    """Same inputs through launch_rope_and_store_kv_ragged + the ragged decode:
    identical caches and bit-identical outputs (same rounding of the rotated Q,
    same units and merge), config-5-like lengths, one workspace for both."""
    import torch
    H, KVH, max_len, B = 16, 4, 4096, 24
    pos = [int(x) for x in np.random.default_rng(9).integers(0, max_len, B)]
    total = H * D + 2 * KVH * D
    cos, sin = b200attn.rope_tables_host(max_len, D, THETA)
    kh = seeded_f16((B, max_len, KVH * D), 91)
    vh = seeded_f16((B, max_len, KVH * D), 92)
    qkv = seeded_f16((B, total), 93)
    ws = _workspace(B, H, KVH, max_len)
    dpos = torch.tensor(pos, dtype=torch.int32, device=cuda)
    kc, vc = dev(kh), dev(vh)
    got = _fused_ragged(dev(qkv), kc, vc, max_len * KVH * D, dev(cos), dev(sin), max_len, True, dpos, max_len, B, H,
                        KVH, ws=ws)
    kc2, vc2, dq2 = dev(kh), dev(vh), dev(qkv)
    b200attn.launch_rope_and_store_kv_ragged(dq2, dq2[:, H * D:], dq2[:, H * D + KVH * D:], kc2, vc2,
                                             max_len * KVH * D, dev(cos), dev(sin), B, H, KVH, D, total, total, dpos,
                                             max_len, True)
    out2 = torch.empty((B, H * D), dtype=torch.float16, device=cuda)
    b200attn.launch_causal_attention_decode_ragged(dq2, total, kc2, vc2, max_len * KVH * D, dpos, 1, max_len, out2,
                                                   0, B, H, KVH, D, ws[0], ws[1])
    _sync()
    np.testing.assert_array_equal(bits(host(kc)), bits(host(kc2)))
    np.testing.assert_array_equal(bits(host(vc)), bits(host(vc2)))
    np.testing.assert_array_equal(bits(got), bits(host(out2)))


def test_ragged_fused_step_bad_and_empty_positions(cuda):
    """A position outside the RoPE table appends nothing, leaves Q unrotated and
    sets bit 1 of the device error word; a negative position gives a zero output;
    without K/V rows nothing is appended."""
    import torch
    H, KVH, max_len = 16, 4, 512
    rope_rows = 300
    pos = [10, 400, -1, 299]
    B = len(pos)
    total = H * D + 2 * KVH * D
    cos, sin = b200attn.rope_tables_host(rope_rows, D, THETA)
    kh = seeded_f16((B, max_len, KVH * D), 101)
    vh = seeded_f16((B, max_len, KVH * D), 102)
    qkv = seeded_f16((B, total), 103)
    kc, vc = dev(kh), dev(vh)
    dpos = torch.tensor(pos, dtype=torch.int32, device=cuda)
    assert b200attn.lib().b2_device_error_word() == 0
    got = _fused_ragged(dev(qkv), kc, vc, max_len * KVH * D, dev(cos), dev(sin), rope_rows, True, dpos, max_len, B,
                        H, KVH)
    assert b200attn.lib().b2_device_error_word() & 2
    assert b200attn.lib().b2_clear_device_error_word() == 0
    ek, ev = kh.copy(), vh.copy()
    qd, kd = H * D, KVH * D
    for b in (0, 3):  # in-table positions are appended as usual
        oq, ok, ov = qkv[b, :qd].copy(), qkv[b, qd:qd + kd].copy(), qkv[b, qd + kd:].copy()
        oracle.rope_and_store_kv(oq, ok, ov, ek[b], ev[b], cos, sin, 1, H, KVH, D, qd, kd, pos[b], True)
        _, o32 = oracle.decode_attention(oq, ek[b], ev[b], pos[b] + 1, H, KVH, D)
        assert_attention_close(got[b], o32.reshape(-1))
    np.testing.assert_array_equal(bits(host(kc)), bits(ek))  # nothing appended at 400 or -1
    np.testing.assert_array_equal(bits(host(vc)), bits(ev))
    # position 400: unrotated Q over the 401 stored rows
    _, o32 = oracle.decode_attention(qkv[1, :qd].copy(), kh[1], vh[1], 401, H, KVH, D)
    assert_attention_close(got[1], o32.reshape(-1))
    assert np.all(got[2] == 0)
    # no K/V rows: nothing appended, attention over the stored rows
    kc3, vc3 = dev(kh), dev(vh)
    got3 = _fused_ragged(dev(qkv), kc3, vc3, max_len * KVH * D, dev(cos), dev(sin), rope_rows, True,
                         torch.tensor([10, 20, 30, 40], dtype=torch.int32, device=cuda), max_len, B, H, KVH,
                         append=False)
    np.testing.assert_array_equal(bits(host(kc3)), bits(kh))
    for b, p in enumerate([10, 20, 30, 40]):
        oq = qkv[b, :qd].copy()
        oracle.rope_and_store_kv(oq, qkv[b, qd:qd + kd].copy(), None, None, None, cos, sin, 1, H, KVH, D, qd, kd, p,
                                 True)
        _, o32 = oracle.decode_attention(oq, kh[b], vh[b], p + 1, H, KVH, D)
        assert_attention_close(got3[b], o32.reshape(-1))
    assert b200attn.lib().b2_device_error_word() == 0  # every position of this call is in the table
