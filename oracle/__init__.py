"""CPU oracle for the GQA attention hot path -- TEST INFRASTRUCTURE ONLY.

Plain-C restatement (``oracle.c``) of the reference engine's RoPE table,
RoPE + KV-cache append, causal GQA attention and flash-decode split/merge
algebra, wrapped here with ctypes/numpy. Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import
this package, and only as the checker or the timed CPU baseline; the product
path (``llm-inference_b200/b200attn``) never touches it.

Parity pins for this oracle (see tests/test_oracle.py):
* golden vectors produced by the reference's own fixture generator
  (python/reference.py:40-96) on a seeded random-init SmolLM3 layer,
  committed under tests/golden/;
* the self-contained known-answer test of
  tests/test_causal_attention.cpp:152-228 (double softmax, 2e-3);
* the invariants of tests/test_rope.cpp:92-195.
"""
from __future__ import annotations

import ctypes
import hashlib
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "liboracle.so")
_SRC = [os.path.join(_HERE, "oracle.c")]
_lock = threading.Lock()
_lib = None

# -ffp-contract=off: the rotation is two rounded fp32 products and one rounded
# sum, the same sequence the CUDA kernel issues, so results compare bit-exact.
CFLAGS = ["-O3", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off", "-std=c11"]


def _source_hash() -> str:
    h = hashlib.sha256()
    for p in _SRC + [os.path.join(_HERE, "oracle.h")]:
        with open(p, "rb") as f:
            h.update(f.read())
    h.update(" ".join(CFLAGS).encode())
    return h.hexdigest()


def build(force: bool = False) -> str:
    """Compile oracle.c into liboracle.so next to it (gcc, a second or two)
    when the library is missing or was built from other sources or flags
    (content hash kept in liboracle.so.sha256)."""
    want = _source_hash()
    stamp = _SO + ".sha256"
    have = open(stamp).read().strip() if os.path.exists(stamp) else None
    if force or not os.path.exists(_SO) or have != want:
        tmp = _SO + f".tmp{os.getpid()}"
        subprocess.check_call(["gcc", *CFLAGS, *_SRC, "-o", tmp, "-lm"])
        os.replace(tmp, _SO)
        with open(stamp + f".tmp{os.getpid()}", "w") as f:
            f.write(want + "\n")
        os.replace(stamp + f".tmp{os.getpid()}", stamp)
    return _SO


def lib() -> ctypes.CDLL:
    global _lib
    with _lock:
        if _lib is None:
            build()
            L = ctypes.CDLL(_SO)
            P, S, F, I = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_float, ctypes.c_int
            L.or_float_to_half.restype = ctypes.c_uint16
            L.or_float_to_half.argtypes = [F]
            L.or_half_to_float.restype = F
            L.or_half_to_float.argtypes = [ctypes.c_uint16]
            L.or_inverse_frequencies.argtypes = [S, F, P]
            L.or_fill_rope_tables.argtypes = [S, S, F, P, P]
            L.or_rope_and_store_kv.restype = I
            L.or_rope_and_store_kv.argtypes = [P, P, P, P, P, P, P, S, S, S, S, S, S, S, I]
            L.or_causal_attention_rows.argtypes = [P, P, P, S, S, S, S, S, S, S, P, S, P, P, S, I]
            L.or_decode_partials.argtypes = [P, P, P, S, S, S, S, S, S, P, P, P, I]
            L.or_merge_partials.argtypes = [P, P, P, S, S, S, P, P]
            L.or_decode_attention.argtypes = [P, P, P, S, S, S, S, S, P, P, I]
            _lib = L
    return _lib


def _p(a):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def _u16(a):
    a = np.asarray(a)
    if a.dtype == np.float16:
        a = a.view(np.uint16)
    assert a.dtype == np.uint16, a.dtype
    return np.ascontiguousarray(a)


def inverse_frequencies(head_dim: int, theta: float) -> np.ndarray:
    out = np.zeros(head_dim // 2, np.float32)
    lib().or_inverse_frequencies(head_dim, theta, _p(out))
    return out


def rope_tables(max_seq_len: int, head_dim: int, theta: float):
    """FP16 cos/sin tables [max_seq_len, head_dim/2] (rope_cache.hpp:63-76)."""
    cos = np.zeros((max_seq_len, head_dim // 2), np.uint16)
    sin = np.zeros_like(cos)
    lib().or_fill_rope_tables(max_seq_len, head_dim, theta, _p(cos), _p(sin))
    return cos.view(np.float16), sin.view(np.float16)


def rope_and_store_kv(q, k, v, k_cache, v_cache, cos, sin, seq_len, num_heads,
                      num_kv_heads, head_dim, q_stride, k_stride, start_pos,
                      apply_rotation) -> int:
    """In-place on the given (contiguous, fp16 or uint16) numpy buffers."""
    arrs = [q, k, v, k_cache, v_cache]
    for a in arrs:
        if a is not None:
            assert a.flags["C_CONTIGUOUS"] and a.dtype in (np.float16, np.uint16)
    cos, sin = _u16(cos), _u16(sin)
    return lib().or_rope_and_store_kv(
        _p(q), _p(k), _p(v), _p(k_cache), _p(v_cache), _p(cos), _p(sin),
        seq_len, num_heads, num_kv_heads, head_dim, q_stride, k_stride, start_pos,
        1 if apply_rotation else 0)


def causal_attention(q, k, v, seq_len, num_heads, num_kv_heads, head_dim,
                     q_stride=0, kv_stride=0, start_pos=0, rows=None, threads=0):
    """Exact causal GQA attention; returns (fp16 [n_rows, H*d], fp32 same)."""
    q, k, v = _u16(q), _u16(k), _u16(v)
    n = seq_len if rows is None else len(rows)
    rows_arr = None if rows is None else np.ascontiguousarray(np.asarray(rows, np.int64))
    out16 = np.zeros((n, num_heads * head_dim), np.uint16)
    out32 = np.zeros((n, num_heads * head_dim), np.float32)
    lib().or_causal_attention_rows(
        _p(q), _p(k), _p(v), seq_len, start_pos, num_heads, num_kv_heads, head_dim,
        q_stride, kv_stride, _p(rows_arr), 0 if rows is None else len(rows),
        _p(out16), _p(out32), num_heads * head_dim, threads)
    return out16.view(np.float16), out32


def decode_partials(q, k, v, kv_len, num_heads, num_kv_heads, head_dim, kv_stride,
                    chunk, threads=0):
    q, k, v = _u16(q), _u16(k), _u16(v)
    chunks = (kv_len + chunk - 1) // chunk
    o = np.zeros((num_heads, chunks, head_dim), np.float32)
    m = np.zeros((num_heads, chunks), np.float32)
    l = np.zeros((num_heads, chunks), np.float32)
    lib().or_decode_partials(_p(q), _p(k), _p(v), kv_len, num_heads, num_kv_heads,
                             head_dim, kv_stride, chunk, _p(o), _p(m), _p(l), threads)
    return o, m, l


def merge_partials(o, m, l):
    o = np.ascontiguousarray(o, np.float32)
    m = np.ascontiguousarray(m, np.float32)
    l = np.ascontiguousarray(l, np.float32)
    H, C, d = o.shape
    out16 = np.zeros((H, d), np.uint16)
    out32 = np.zeros((H, d), np.float32)
    lib().or_merge_partials(_p(o), _p(m), _p(l), H, C, d, _p(out16), _p(out32))
    return out16.view(np.float16), out32


def decode_attention(q, k, v, kv_len, num_heads, num_kv_heads, head_dim,
                     kv_stride=0, threads=0):
    """Double-precision single-token attention (test_causal_attention.cpp:176-196)."""
    q, k, v = _u16(q), _u16(k), _u16(v)
    out16 = np.zeros((num_heads, head_dim), np.uint16)
    out32 = np.zeros((num_heads, head_dim), np.float32)
    lib().or_decode_attention(_p(q), _p(k), _p(v), kv_len, num_heads, num_kv_heads,
                              head_dim, kv_stride, _p(out16), _p(out32), threads)
    return out16.view(np.float16), out32


def float_to_half_bits(x: float) -> int:
    return int(lib().or_float_to_half(float(x)))
