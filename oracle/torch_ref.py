"""The reference's Python attention path on CPU torch -- TEST / BASELINE ONLY.

Restates python/reference.py:62-92 (the path the reference runs to make its
layer-0 fixtures): rotary cos/sin of the full head dim (HF rotary embedding:
inv_freq = theta^(-2i/d), emb = cat(freqs, freqs)), HF
``apply_rotary_pos_emb`` on Q and K ([1, heads, seq, d]), GQA by
``repeat_interleave`` of the KV heads, then
``F.scaled_dot_product_attention(is_causal=True)`` and the output reshaped to
[seq, heads * d]. The checkpoint's rotary module is replaced by its formula
(the checkpoint is absent). The reference runs it in FP16
(python/reference.py:137-141); FP32 is the second variant timed.

Only bench.py's CPU-baseline legs use this module, as a timed baseline; the
product path never imports it.

Decode (one new token at position p over a cache of p + 1 rows) is the same
sequence with one query row; SDPA's ``is_causal`` mask is aligned to the
top-left corner, so a single query row takes no mask (it attends every cached
row, which is what the causal mask means for the last row).
"""
from __future__ import annotations

import time

import numpy as np


def _rope(positions, head_dim: int, theta: float, dtype):
    import torch
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
    freqs = torch.outer(torch.as_tensor(positions, dtype=torch.float32), inv)
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos()[None].to(dtype), emb.sin()[None].to(dtype)


def prefill(q, k, v, num_heads: int, num_kv_heads: int, head_dim: int, theta: float = 5.0e6, rotate: bool = True,
            dtype=None):
    """q [S, H*d], k/v [S, KVH*d] torch tensors (CPU); returns [S, H*d]."""
    import torch
    import torch.nn.functional as F
    from transformers.models.llama.modeling_llama import apply_rotary_pos_emb
    dtype = dtype or q.dtype
    S = q.shape[0]
    qr = q.to(dtype).view(1, S, num_heads, head_dim).transpose(1, 2)
    kr = k.to(dtype).view(1, S, num_kv_heads, head_dim).transpose(1, 2)
    if rotate:
        cos, sin = _rope(torch.arange(S), head_dim, theta, dtype)
        qr, kr = apply_rotary_pos_emb(qr, kr, cos, sin)
    vr = v.to(dtype).view(1, S, num_kv_heads, head_dim).transpose(1, 2)
    g = num_heads // num_kv_heads
    o = F.scaled_dot_product_attention(qr, kr.repeat_interleave(g, dim=1), vr.repeat_interleave(g, dim=1),
                                       is_causal=True)
    return o.transpose(1, 2).contiguous().reshape(S, -1)


def decode(q, k_new, v_new, k_cache, v_cache, pos: int, num_heads: int, num_kv_heads: int, head_dim: int,
           theta: float = 5.0e6, rotate: bool = True):
    """One new token at position pos: RoPE of q and k_new, append of k/v_new
    into the [max, KVH*d] caches at row pos, attention over rows 0..pos.
    Tensors in the dtype the path runs in; returns [H*d]."""
    import torch
    import torch.nn.functional as F
    from transformers.models.llama.modeling_llama import apply_rotary_pos_emb
    dtype = k_cache.dtype
    qr = q.to(dtype).view(1, 1, num_heads, head_dim).transpose(1, 2)
    kr = k_new.to(dtype).view(1, 1, num_kv_heads, head_dim).transpose(1, 2)
    if rotate:
        cos, sin = _rope([pos], head_dim, theta, dtype)
        qr, kr = apply_rotary_pos_emb(qr, kr, cos, sin)
    k_cache[pos] = kr.transpose(1, 2).reshape(-1)
    v_cache[pos] = v_new.to(dtype)
    n = pos + 1
    kc = k_cache[:n].view(1, n, num_kv_heads, head_dim).transpose(1, 2)
    vc = v_cache[:n].view(1, n, num_kv_heads, head_dim).transpose(1, 2)
    g = num_heads // num_kv_heads
    o = F.scaled_dot_product_attention(qr, kc.repeat_interleave(g, dim=1), vc.repeat_interleave(g, dim=1))
    return o.reshape(-1)


def seeded(shape, seed: int, std: float = 1.0):
    import torch
    rng = np.random.default_rng(seed)
    return torch.from_numpy((rng.standard_normal(shape, dtype=np.float32) * std).astype(np.float16))


def time_calls(fn, budget_s: float, min_reps: int = 1, max_reps: int = 1000, warm: int = 1):
    """Call fn() `warm` times untimed (imports, first-call set-up), then until
    budget_s has passed (at least min_reps times); returns (seconds per call,
    reps)."""
    for _ in range(warm):
        fn()
    reps, t0 = 0, time.perf_counter()
    while True:
        fn()
        reps += 1
        el = time.perf_counter() - t0
        if reps >= max_reps or (reps >= min_reps and el >= budget_s):
            return el / reps, reps
