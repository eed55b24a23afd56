"""Loader for libb200attn.so, the C-ABI CUDA library (include/b200attn.h).

There is no CPU fallback: if the library is missing or cannot be loaded,
every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libb200attn.so")

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None

P = ctypes.c_void_p
S = ctypes.c_size_t
I = ctypes.c_int
F = ctypes.c_float
B = ctypes.c_bool
U64 = ctypes.c_uint64
PP = ctypes.POINTER(ctypes.c_void_p)

# name -> (restype, argtypes); mirrors include/b200attn.h
SIGNATURES: dict[str, tuple] = {
    "b2_kv_chunk": (I, []),
    "b2_decode_workspace_floats": (S, [S, S, S]),
    "b2_status_string": (ctypes.c_char_p, [I]),
    "b2_last_cuda_error": (I, []),
    "b2_kernel_launch_count": (U64, []),
    "b2_device_error_word": (ctypes.c_uint, []),
    "b2_clear_device_error_word": (I, []),
    "b2_fill_rope_tables": (I, [S, S, F, P, P]),
    "b2_launch_rope": (I, [P, P, P, P, S, S, S, S, S, S, S, P]),
    "b2_launch_rope_and_store_kv": (I, [P, P, P, P, P, P, P, S, S, S, S, S, S, S, B, P]),
    "b2_update_rope_and_store_kv_node": (I, [P, P, S, B]),
    "b2_launch_causal_attention_prefill": (I, [P, P, P, P, S, S, S, S, S, S, P]),
    "b2_launch_causal_attention_prefill_batched": (I, [P, P, P, P, S, S, S, S, S, S, S, S, S, S, S, P]),
    "b2_launch_causal_attention_decode": (I, [P, P, P, P, P, P, P, S, S, S, S, S, S, S, S, P, PP, PP]),
    "b2_launch_causal_attention_decode_vectorized": (I, [P, P, P, P, P, P, P, S, S, S, S, S, S, S, S, P, PP, PP]),
    "b2_update_causal_attention_decode_node": (I, [P, P, S]),
    "b2_update_merge_attention_decode_node": (I, [P, P, S]),
    "b2_launch_merge_attention_decode_tiled": (I, [P, P, P, P, S, S, S, P]),
    "b2_launch_rope_and_store_kv_devpos": (I, [P, P, P, P, P, P, P, S, S, S, S, S, S, P, S, B, P]),
    "b2_launch_causal_attention_decode_devlen": (I, [P, P, P, P, P, P, P, P, ctypes.c_int32, S, S, S, S, S, P]),
    "b2_advance_position": (I, [P, ctypes.c_int32, P]),
    "b2_launch_decode_rank_partial_devlen": (I, [P, P, P, P, P, P, P, ctypes.c_int32, S, S, S, S, S, P, P, P, P]),
    "b2_launch_merge_partials_strided": (I, [P, P, P, P, S, S, S, S, S, S, S, P]),
    "b2_launch_causal_attention_decode_noalloc": (I, [P, P, P, P, S, S, S, S, S, S, P]),
    "b2_decode_step_workspace_bytes": (S, [S, S]),
    "b2_decode_exchange_bytes": (S, [S, S]),
    "b2_launch_decode_step_fused_exchange": (
        I, [P, P, P, P, P, P, P, S, B, P, P, ctypes.c_int32, S, P, P, S, S, S, P, S, S, S, P]),
    "b2_ipc_alloc": (I, [S, PP, P]),
    "b2_ipc_open": (I, [P, PP]),
    "b2_ipc_close": (I, [P]),
    "b2_ipc_free": (I, [P]),
    "b2_launch_rope_and_store_kv_ragged": (I, [P, P, P, P, P, S, P, P, S, S, S, S, S, S, P, S, B, P]),
    "b2_decode_ragged_workspace_bytes": (S, [S, S, S, S]),
    "b2_launch_causal_attention_decode_ragged": (
        I, [P, S, P, P, S, P, ctypes.c_int32, S, P, S, S, S, S, S, P, S, P]),
    "b2_launch_decode_step_fused": (I, [P, P, P, P, P, P, P, S, B, P, P, ctypes.c_int32, S, P, P, S, S, S, S, P]),
    "b2_launch_decode_step_ragged_fused": (
        I, [P, S, P, P, S, P, P, S, P, P, S, B, P, S, P, S, S, S, S, S, P, S, P]),
    "b2_launch_attention_out_projection": (I, [P, P, P, S, S, S, S, ctypes.c_float, P]),
    "b2_launch_attention_out_projection_decode": (I, [P, P, P, S, S, S, ctypes.c_float, P]),
    "b2_launch_qkv_gemm": (I, [P, P, P, S, S, S, P]),
    "b2_launch_qkv_decode": (I, [P, P, P, S, S, P]),
    "b2_launch_qkv_gemm_rope_store_kv": (I, [P, P, P, P, P, P, P, S, S, S, S, S, S, B, P]),
    "b2_launch_decode_step_fused_rank_partial": (
        I, [P, P, P, P, P, P, P, S, B, P, P, ctypes.c_int32, S, P, P, P, P, S, S, S, S, P]),
}


class B2Error(RuntimeError):
    def __init__(self, status: int, where: str):
        self.status = status
        msg = lib().b2_status_string(status).decode()
        extra = ""
        if status == -4:  # B2_ERR_CUDA
            extra = f" (cudaError {lib().b2_last_cuda_error()})"
        super().__init__(f"{where}: {msg}{extra} [status {status}]")


def lib() -> ctypes.CDLL:
    """The loaded library; raises if it has not been built."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python llm-inference_b200/build.py` "
                    "(there is no CPU fallback for the attention path)")
            L = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def check(status: int, where: str) -> int:
    if status < 0:
        raise B2Error(status, where)
    return status
