"""b200attn -- B200-native (sm_100a) GQA attention hot path of the SmolLM3-3B engine.

Python mirror of the reference's kernel API (include/kernels/kernels.hpp) and
host structs (KVCache, RopeCache) over the C-ABI library libb200attn.so.
"""
from ._lib import B2Error, LIB_PATH, lib
from .caches import KVCache, RopeCache, create_rope_cache, rope_tables_host
from .kernels import *  # noqa: F401,F403
from .kernels import __all__ as _k_all

__all__ = ["B2Error", "LIB_PATH", "lib", "KVCache", "RopeCache", "create_rope_cache",
           "rope_tables_host", *_k_all]


def __getattr__(name):
    if name == "KV_CHUNK":
        return int(lib().b2_kv_chunk())
    raise AttributeError(name)
