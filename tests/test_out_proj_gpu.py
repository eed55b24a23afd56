"""Attention output projection (the path's consumer,
src/kernels/attention_out_projection.hip.cpp:8-72): out = in @ W^T + beta * out
on the GPU against a float64 host product of the same FP16 inputs, at the
acceptance bar the attention outputs use (max-abs 1e-2, relative L2 2e-3)."""
import numpy as np
import pytest

import b200attn
from _gpu import dev, host
from _util import assert_attention_close, seeded_f16

pytestmark = pytest.mark.gpu


def _ref(x, w, res, beta):
    out = x.astype(np.float64) @ w.astype(np.float64).T
    if beta != 0.0:
        out += beta * res.astype(np.float64)
    return out.astype(np.float32)


@pytest.mark.parametrize("S,N,K,beta", [
    (254, 2048, 2048, 1.0),     # config-1 prompt, SmolLM3 o_proj, fused residual
    (254, 2048, 2048, 0.0),     # the reference's unit-test form (beta 0 never reads out)
    (300, 2048, 2048, 1.0),     # ragged last M tile
    (2, 256, 64, 0.5),          # smallest tcgen05 shape
    (128, 2048, 2048, 1.0),     # one 128-row tile: the single-CTA kernel (longer prompts run CTA pairs)
    (8192, 2048, 2048, 1.0),    # 512 output tiles: several per persistent CTA, both TMEM accumulators
    (37, 96, 40, 1.0),          # SIMT kernel shapes (hidden not a multiple of 256, K of 64)
    (5, 512, 200, 0.0),
])
def test_out_projection_prefill(cuda, S, N, K, beta):
    x = seeded_f16((S, K), 11 + S)
    w = seeded_f16((N, K), 12 + N, std=0.02)
    res = seeded_f16((S, N), 13 + K)
    out = dev(res if beta != 0.0 else np.full((S, N), np.nan, np.float16))
    b200attn.launch_attention_out_projection(dev(x), out, dev(w), S, N, K // 16 if K % 16 == 0 else 1,
                                             16 if K % 16 == 0 else K, beta)
    import torch
    torch.cuda.synchronize()
    assert b200attn.lib().b2_device_error_word() == 0
    assert_attention_close(host(out), _ref(x, w, res, beta))


@pytest.mark.parametrize("N,K,beta", [(2048, 2048, 1.0), (2048, 2048, 0.0), (300, 512, 1.0), (64, 40, 1.0)])
def test_out_projection_decode(cuda, N, K, beta):
    x = seeded_f16((1, K), 21 + K)
    w = seeded_f16((N, K), 22 + N, std=0.02)
    res = seeded_f16((1, N), 23)
    out = dev(res if beta != 0.0 else np.full((1, N), np.nan, np.float16))
    b200attn.launch_attention_out_projection_decode(dev(x), out, dev(w), N, K // 8 if K % 8 == 0 else 1,
                                                    8 if K % 8 == 0 else K, beta)
    import torch
    torch.cuda.synchronize()
    assert_attention_close(host(out), _ref(x, w, res, beta))


def test_out_projection_consumes_prefill_output(cuda):
    """The path end to end: RoPE/append, causal prefill into packed rows, then
    the o_proj GEMM with the residual added in place (engine order,
    include/model_inference.hpp:272-300)."""
    import torch
    import oracle
    S, H, KVH, d, hidden = 300, 16, 4, 128, 2048
    qkv = seeded_f16((S, H * d + 2 * KVH * d), 31)
    w = seeded_f16((hidden, H * d), 32, std=0.02)
    resid = seeded_f16((S, hidden), 33)
    cos, sin = b200attn.rope_tables_host(S, d, 5.0e6)
    dq = dev(qkv)
    cache = b200attn.KVCache(1, S, KVH, d, device=cuda)
    b200attn.launch_rope_and_store_kv(dq, dq[:, H * d:], dq[:, H * d + KVH * d:], cache.get_k_cache(0),
                                      cache.get_v_cache(0), dev(cos), dev(sin), S, H, KVH, d, qkv.shape[1],
                                      qkv.shape[1], 0, True)
    attn = torch.empty((S, H * d), dtype=torch.float16, device=cuda)
    b200attn.launch_causal_attention_prefill(dq, cache.get_k_cache(0), cache.get_v_cache(0), attn, S, H, KVH, d,
                                             qkv.shape[1], KVH * d)
    x = dev(resid)
    b200attn.launch_attention_out_projection(attn, x, dev(w), S, hidden, H, d, 1.0)
    torch.cuda.synchronize()
    q = np.ascontiguousarray(qkv[:, :H * d])
    k = np.ascontiguousarray(qkv[:, H * d:H * d + KVH * d])
    v = np.ascontiguousarray(qkv[:, H * d + KVH * d:])
    kc, vc = np.zeros((S, KVH * d), np.float16), np.zeros((S, KVH * d), np.float16)
    oracle.rope_and_store_kv(q, k, v, kc, vc, cos, sin, S, H, KVH, d, H * d, KVH * d, 0, True)
    o16, _ = oracle.causal_attention(q, kc, vc, S, H, KVH, d)
    assert_attention_close(host(x), _ref(o16, w, resid, 1.0))
