"""KVCache and RopeCache: the reference's host structs on CUDA memory.

``KVCache`` keeps include/kv_cache.hpp's layout exactly: one buffer of
2 * num_layers * max_seq_len * kv_dim halves; layer l's K at
base + l * 2 * max_seq_len * kv_dim and its V max_seq_len * kv_dim later
(kv_cache.hpp:21-34, :80-82); row t is token t, [t][kv_head][head_dim].
``create_rope_cache`` builds include/rope_cache.hpp:79-105's FP16 cos/sin
tables on the host (b2_fill_rope_tables, FP32 host math) and uploads them.
Device memory comes from torch (plumbing only).
"""
from __future__ import annotations

import numpy as np

from ._lib import check, lib


class KVCache:
    def __init__(self, num_layers: int, max_seq_len: int, num_kv_heads: int, head_dim: int,
                 device="cuda", buffer=None):
        import torch
        self.num_layers = num_layers
        self.max_seq_len = max_seq_len
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.kv_dim = num_kv_heads * head_dim
        shape = (num_layers, 2, max_seq_len, self.kv_dim)
        if buffer is None:
            buffer = torch.empty(shape, dtype=torch.float16, device=device)
        assert tuple(buffer.shape) == shape and buffer.dtype == torch.float16 and buffer.is_contiguous()
        self.buffer = buffer
        self._cached_len = 0

    def layer_stride(self) -> int:
        return 2 * self.max_seq_len * self.kv_dim

    def get_k_cache(self, layer: int):
        """[max_seq_len, kv_dim] view at base + layer * layer_stride (kv_cache.hpp:21-26)."""
        return self.buffer[layer, 0]

    def get_v_cache(self, layer: int):
        """View at base + layer * layer_stride + max_seq_len * kv_dim (kv_cache.hpp:29-34)."""
        return self.buffer[layer, 1]

    def get_cached_len(self) -> int:
        return self._cached_len

    def set_cached_len(self, cached_len: int) -> None:
        if cached_len > self.max_seq_len:  # kv_cache.hpp:40-45
            raise IndexError(f"KV cache capacity exceeded: requested {cached_len} tokens, "
                             f"capacity {self.max_seq_len}")
        self._cached_len = cached_len

    def reset_cache(self) -> None:
        self._cached_len = 0


def rope_tables_host(max_seq_len: int, head_dim: int, rope_theta: float):
    """FP16 cos/sin [max_seq_len, head_dim/2] as numpy float16 (rope_cache.hpp:49-76)."""
    half = head_dim // 2
    cos = np.zeros((max_seq_len, half), np.uint16)
    sin = np.zeros((max_seq_len, half), np.uint16)
    check(lib().b2_fill_rope_tables(max_seq_len, head_dim, float(rope_theta),
                                    cos.ctypes.data, sin.ctypes.data), "fill_rope_tables")
    return cos.view(np.float16), sin.view(np.float16)


class RopeCache:
    def __init__(self, d_cos, d_sin):
        self.d_cos = d_cos
        self.d_sin = d_sin


def create_rope_cache(max_seq_len: int, head_dim: int, rope_theta: float, device="cuda") -> RopeCache:
    import torch
    cos, sin = rope_tables_host(max_seq_len, head_dim, rope_theta)
    return RopeCache(torch.from_numpy(cos).to(device), torch.from_numpy(sin).to(device))
