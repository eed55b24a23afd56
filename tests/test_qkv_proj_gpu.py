"""QKV projection, the path's producer (src/kernels/qkv_gemm.hip.cpp:7-115),
and its fused form with the engine's next step, launch_rope_and_store_kv
(include/model_inference.hpp:266-281), in the GEMM epilogue.

The plain GEMM / GEMV against a float64 host product of the same FP16 inputs
(max-abs 1e-2, relative L2 2e-3, the attention outputs' bar). The fused kernel
against the two launches it replaces, bit for bit: the Q/K/V rows and both
caches, with sentinel rows around the written cache rows. And the fused path
end to end against the CPU oracle: host product rounded to FP16, then the
oracle's RoPE/append and causal attention."""
import numpy as np
import pytest

import b200attn
from _gpu import dev, host
from _util import assert_attention_close, seeded_f16

pytestmark = pytest.mark.gpu


def _ref(x, w):
    return (x.astype(np.float64) @ w.astype(np.float64).T).astype(np.float32)


@pytest.mark.parametrize("S,N,K", [
    (254, 3072, 2048),   # config-1 prompt, SmolLM3 fused QKV (Q 2048 | K 512 | V 512)
    (300, 3072, 2048),   # ragged last M tile
    (2048, 3072, 2048),  # 96 output tiles
    (5, 96, 40),         # SIMT shape
])
def test_qkv_gemm(cuda, S, N, K):
    x = seeded_f16((S, K), 41 + S)
    w = seeded_f16((N, K), 42 + N, std=0.02)
    out = dev(np.full((S, N), np.nan, np.float16))
    b200attn.launch_qkv_gemm(dev(x), out, dev(w), S, K, N)
    import torch
    torch.cuda.synchronize()
    assert b200attn.lib().b2_device_error_word() == 0
    assert_attention_close(host(out), _ref(x, w))


@pytest.mark.parametrize("N,K", [(3072, 2048), (320, 512), (64, 40)])
def test_qkv_decode(cuda, N, K):
    x = seeded_f16((1, K), 51 + K)
    w = seeded_f16((N, K), 52 + N, std=0.02)
    out = dev(np.full((1, N), np.nan, np.float16))
    b200attn.launch_qkv_decode(dev(x), out, dev(w), K, N)
    import torch
    torch.cuda.synchronize()
    assert_attention_close(host(out), _ref(x, w))


def _run_both(S, hidden, H, KVH, d, start, rotate, seed, max_seq=None):
    """(fused qkv, k cache, v cache), (two-launch qkv, k cache, v cache) on the
    same inputs; caches start as a NaN sentinel."""
    import torch
    max_seq = max_seq or start + S + 3
    total = (H + 2 * KVH) * d
    x = seeded_f16((S, hidden), seed)
    w = seeded_f16((total, hidden), seed + 1, std=0.03)
    cos, sin = b200attn.rope_tables_host(max_seq, d, 5.0e6)
    dx, dw, dcos, dsin = dev(x), dev(w), dev(cos), dev(sin)
    res = []
    for fused in (True, False):
        qkv = dev(np.full((S, total), np.nan, np.float16))
        kc = dev(np.full((max_seq, KVH * d), np.nan, np.float16))
        vc = dev(np.full((max_seq, KVH * d), np.nan, np.float16))
        if fused:
            b200attn.launch_qkv_gemm_rope_store_kv(dx, qkv, dw, kc, vc, dcos, dsin, S, hidden, H, KVH, d, start,
                                                   rotate)
        else:
            b200attn.launch_qkv_gemm(dx, qkv, dw, S, hidden, total)
            b200attn.launch_rope_and_store_kv(qkv, qkv[:, H * d:], qkv[:, (H + KVH) * d:], kc, vc, dcos, dsin, S, H,
                                              KVH, d, total, total, start, rotate)
        torch.cuda.synchronize()
        res.append((host(qkv), host(kc), host(vc)))
    assert b200attn.lib().b2_device_error_word() == 0
    return (x, w, cos, sin), res[0], res[1]


def _bits(a):
    return np.ascontiguousarray(a).view(np.uint16)


@pytest.mark.parametrize("S,hidden,H,KVH,d,start,rotate", [
    (300, 2048, 16, 4, 128, 0, True),     # SmolLM3 layer, ragged last tile
    (300, 2048, 16, 4, 128, 0, False),    # NoPE layer (every 4th)
    (254, 2048, 16, 4, 128, 37, True),    # continued prompt: cache rows 37..290
    (1, 2048, 16, 4, 128, 600, True),     # one token: the GEMV and the RoPE kernel
    (100, 2048, 16, 4, 128, 9, True),     # one 128-row tile: the single-CTA kernel (longer prompts run CTA pairs)
    (2048, 2048, 16, 4, 128, 0, True),    # 16 M tiles x 12 N tiles: both TMEM accumulators
    (8192, 2048, 16, 4, 128, 0, True),    # one config-3 sequence: 768 tiles, 5-6 per persistent CTA
    (130, 512, 8, 4, 64, 5, True),        # head_dim 64: four heads a tile
    (130, 512, 4, 1, 256, 5, True),       # head_dim 256: half a head pair a tile
    (67, 320, 6, 2, 64, 3, True),         # kv_dim 128: two launches (not a 256 multiple)
    (40, 96, 4, 2, 32, 0, True),          # head_dim 32: two launches
])
def test_fused_matches_two_launches_bitwise(cuda, S, hidden, H, KVH, d, start, rotate):
    _, (fq, fk, fv), (uq, uk, uv) = _run_both(S, hidden, H, KVH, d, start, rotate, 700 + S + d)
    np.testing.assert_array_equal(_bits(fq), _bits(uq))
    np.testing.assert_array_equal(_bits(fk), _bits(uk))
    np.testing.assert_array_equal(_bits(fv), _bits(uv))
    # rows outside start..start+S-1 keep the sentinel
    for c in (fk, fv):
        assert np.isnan(c[:start]).all() and np.isnan(c[start + S:]).all()
        assert not np.isnan(c[start:start + S]).any()


def test_fused_against_the_oracle(cuda):
    """Host product rounded to FP16, the oracle's RoPE/append on it, then the
    oracle's causal attention over the caches against the CUDA prefill over
    the fused kernel's caches."""
    import torch
    import oracle
    S, hidden, H, KVH, d, start = 300, 2048, 16, 4, 128, 0
    (x, w, cos, sin), (fq, fk, fv), _ = _run_both(S, hidden, H, KVH, d, start, True, 811)
    qd, kd = H * d, KVH * d
    ref = _ref(x, w).astype(np.float16)
    q = np.ascontiguousarray(ref[:, :qd])
    k = np.ascontiguousarray(ref[:, qd:qd + kd])
    v = np.ascontiguousarray(ref[:, qd + kd:])
    kc = np.zeros((S + 3, kd), np.float16)
    vc = np.zeros((S + 3, kd), np.float16)
    oracle.rope_and_store_kv(q, k, v, kc, vc, cos, sin, S, H, KVH, d, qd, kd, start, True)
    # the rows: rotated Q, K and V as projected
    assert_attention_close(fq[:, :qd], q.astype(np.float32))
    assert_attention_close(fq[:, qd:], ref[:, qd:].astype(np.float32))
    assert_attention_close(fk[:S], kc[:S].astype(np.float32))
    np.testing.assert_array_equal(_bits(fv[:S]), _bits(fq[:, qd + kd:]))
    # attention over the fused kernel's output
    attn = torch.empty((S, qd), dtype=torch.float16, device=cuda)
    dq, dk, dv = dev(fq), dev(fk), dev(fv)
    b200attn.launch_causal_attention_prefill(dq, dk, dv, attn, S, H, KVH, d, fq.shape[1], kd)
    torch.cuda.synchronize()
    _, o32 = oracle.causal_attention(q, kc, vc, S, H, KVH, d)
    assert_attention_close(host(attn), o32)


def test_fused_rejects_bad_arguments(cuda):
    import torch
    S, hidden, H, KVH, d = 4, 256, 2, 1, 128
    total = (H + 2 * KVH) * d
    x = torch.zeros((S, hidden), dtype=torch.float16, device=cuda)
    w = torch.zeros((total, hidden), dtype=torch.float16, device=cuda)
    qkv = torch.zeros((S, total), dtype=torch.float16, device=cuda)
    kc = torch.zeros((8, KVH * d), dtype=torch.float16, device=cuda)
    with pytest.raises(b200attn.B2Error):
        b200attn.launch_qkv_gemm_rope_store_kv(x, qkv, w, kc, kc, None, None, S, hidden, H, KVH, d, 0, True)
    with pytest.raises(b200attn.B2Error):
        b200attn.launch_qkv_gemm_rope_store_kv(x, qkv, w, None, kc, None, None, S, hidden, H, KVH, d, 0, False)
    # seq_len 0 is a no-op
    assert b200attn.lib().b2_launch_qkv_gemm_rope_store_kv(x.data_ptr(), qkv.data_ptr(), w.data_ptr(),
                                                           kc.data_ptr(), kc.data_ptr(), None, None, 0, hidden, H,
                                                           KVH, d, 0, False, None) == 1
