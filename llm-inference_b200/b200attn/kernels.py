"""The reference's attention launchers (include/kernels/kernels.hpp), in Python.

Same names, argument order, meaning and defaults as the C++ declarations; each
forwards to the matching ``b2_*`` C-ABI symbol of libb200attn.so. Buffers are
device pointers given as ``torch.Tensor`` (its ``data_ptr()``) or ``int``;
streams are ``torch.cuda.Stream``, a raw ``int`` handle, or ``None`` for the
legacy default stream (the reference's ``nullptr`` default).

Errors: the reference launchers return ``void`` and silently skip empty or
invalid GQA configurations; these functions do the same (return normally).
Every other failure raises ``B2Error`` where the reference would have exited
the process through HIP_CHECK (include/gpu_utils.hpp:7-14).
"""
from __future__ import annotations

import ctypes

from ._lib import B2Error, check, lib

__all__ = [
    "B2Error", "launch_rope", "launch_rope_and_store_kv", "update_rope_and_store_kv_node",
    "launch_causal_attention_prefill", "launch_causal_attention_decode",
    "launch_causal_attention_decode_vectorized", "update_causal_attention_decode_node",
    "update_merge_attention_decode_node", "launch_merge_attention_decode_tiled",
    "decode_workspace_floats", "kernel_launch_count", "launch_rope_and_store_kv_devpos",
    "launch_causal_attention_decode_devlen", "advance_position", "launch_decode_rank_partial_devlen",
    "launch_merge_partials_strided", "launch_causal_attention_prefill_batched",
    "decode_step_workspace_bytes", "launch_decode_step_fused", "launch_decode_step_fused_rank_partial",
    "launch_rope_and_store_kv_ragged", "decode_ragged_workspace_bytes", "launch_causal_attention_decode_ragged",
    "decode_exchange_bytes", "launch_decode_step_fused_exchange", "ExchangeBuffers",
    "launch_decode_step_ragged_fused", "launch_attention_out_projection", "launch_attention_out_projection_decode",
    "launch_qkv_gemm", "launch_qkv_decode", "launch_qkv_gemm_rope_store_kv",
]


def _ptr(x):
    if x is None:
        return None
    if isinstance(x, int):
        return x
    dp = getattr(x, "data_ptr", None)
    if dp is None:
        raise TypeError(f"expected a device tensor or int pointer, got {type(x)}")
    if getattr(x, "is_cuda", True) is False:
        raise ValueError("b200attn launchers take device buffers; got a host tensor")
    return dp()


def _stream(s):
    if s is None:
        return None
    if isinstance(s, int):
        return s
    return s.cuda_stream


def _kv_chunk() -> int:
    return int(lib().b2_kv_chunk())


def __getattr__(name):
    if name == "KV_CHUNK":
        return _kv_chunk()
    raise AttributeError(name)


def decode_workspace_floats(num_heads: int, head_dim: int, max_kv_len: int) -> int:
    """include/model_inference.hpp:192-198 sizing: H * ceil(max/KV_CHUNK) * (d+2)."""
    return int(lib().b2_decode_workspace_floats(num_heads, head_dim, max_kv_len))


def kernel_launch_count() -> int:
    return int(lib().b2_kernel_launch_count())


def launch_rope(d_q, d_k, d_cos, d_sin, seq_len, num_heads, num_kv_heads, head_dim,
                q_stride, k_stride, start_pos=0, stream=None):
    """kernels.hpp:47-60 -- RoPE on Q and K in place."""
    check(lib().b2_launch_rope(_ptr(d_q), _ptr(d_k), _ptr(d_cos), _ptr(d_sin), seq_len, num_heads,
                               num_kv_heads, head_dim, q_stride, k_stride, start_pos, _stream(stream)),
          "launch_rope")


def launch_rope_and_store_kv(d_q, d_k, d_v, d_k_cache, d_v_cache, d_cos, d_sin, seq_len, num_heads,
                             num_kv_heads, head_dim, q_stride, k_stride, start_pos, apply_rotation,
                             stream=None):
    """kernels.hpp:62-80 -- RoPE Q in place, rotated K + V (or verbatim K/V) into the cache."""
    check(lib().b2_launch_rope_and_store_kv(
        _ptr(d_q), _ptr(d_k), _ptr(d_v), _ptr(d_k_cache), _ptr(d_v_cache), _ptr(d_cos), _ptr(d_sin),
        seq_len, num_heads, num_kv_heads, head_dim, q_stride, k_stride, start_pos, bool(apply_rotation),
        _stream(stream)), "launch_rope_and_store_kv")


def update_rope_and_store_kv_node(graph_exec, node, start_pos, apply_rotation):
    """kernels.hpp:81-86."""
    check(lib().b2_update_rope_and_store_kv_node(int(graph_exec), int(node), start_pos, bool(apply_rotation)),
          "update_rope_and_store_kv_node")


def launch_causal_attention_prefill(d_q, d_k, d_v, d_out, seq_len, num_heads, num_kv_heads, head_dim,
                                    q_stride=0, kv_stride=0, stream=None):
    """kernels.hpp:88-99 (plus the stream the reference lacks)."""
    check(lib().b2_launch_causal_attention_prefill(
        _ptr(d_q), _ptr(d_k), _ptr(d_v), _ptr(d_out), seq_len, num_heads, num_kv_heads, head_dim,
        q_stride, kv_stride, _stream(stream)), "launch_causal_attention_prefill")


def _decode(fn, name, d_q, d_k_cache, d_v_cache, d_out, d_partial_out, d_partial_max,
            d_partial_weight_sum, query_len, kv_cache_len, start_pos, num_heads, num_kv_heads,
            head_dim, q_stride, kv_stride, stream, capture_nodes):
    an = ctypes.c_void_p()
    mn = ctypes.c_void_p()
    check(fn(_ptr(d_q), _ptr(d_k_cache), _ptr(d_v_cache), _ptr(d_out), _ptr(d_partial_out),
             _ptr(d_partial_max), _ptr(d_partial_weight_sum), query_len, kv_cache_len, start_pos,
             num_heads, num_kv_heads, head_dim, q_stride, kv_stride, _stream(stream),
             ctypes.byref(an) if capture_nodes else None,
             ctypes.byref(mn) if capture_nodes else None), name)
    if capture_nodes:
        return an.value, mn.value
    return None


def launch_causal_attention_decode(d_q, d_k_cache, d_v_cache, d_out, d_partial_out, d_partial_max,
                                   d_partial_weight_sum, query_len, kv_cache_len, start_pos, num_heads,
                                   num_kv_heads, head_dim, q_stride, kv_stride, stream=None,
                                   capture_nodes=False):
    """kernels.hpp:104-125. With capture_nodes=True (stream capturing) returns the
    (attention_node, merge_node) handles the reference writes through its out-pointers."""
    return _decode(lib().b2_launch_causal_attention_decode, "launch_causal_attention_decode", d_q,
                   d_k_cache, d_v_cache, d_out, d_partial_out, d_partial_max, d_partial_weight_sum,
                   query_len, kv_cache_len, start_pos, num_heads, num_kv_heads, head_dim, q_stride,
                   kv_stride, stream, capture_nodes)


def launch_causal_attention_decode_vectorized(d_q, d_k_cache, d_v_cache, d_out, d_partial_out,
                                              d_partial_max, d_partial_weight_sum, query_len,
                                              kv_cache_len, start_pos, num_heads, num_kv_heads,
                                              head_dim, q_stride=0, kv_stride=0, stream=None,
                                              capture_nodes=False):
    """kernels.hpp:127-146."""
    return _decode(lib().b2_launch_causal_attention_decode_vectorized,
                   "launch_causal_attention_decode_vectorized", d_q, d_k_cache, d_v_cache, d_out,
                   d_partial_out, d_partial_max, d_partial_weight_sum, query_len, kv_cache_len,
                   start_pos, num_heads, num_kv_heads, head_dim, q_stride, kv_stride, stream,
                   capture_nodes)


def update_causal_attention_decode_node(graph_exec, node, kv_cache_len):
    """kernels.hpp:190-194."""
    check(lib().b2_update_causal_attention_decode_node(int(graph_exec), int(node), kv_cache_len),
          "update_causal_attention_decode_node")


def update_merge_attention_decode_node(graph_exec, node, kv_cache_len):
    """kernels.hpp:148-152."""
    check(lib().b2_update_merge_attention_decode_node(int(graph_exec), int(node), kv_cache_len),
          "update_merge_attention_decode_node")


def launch_merge_attention_decode_tiled(d_partial_output, d_partial_max, d_partial_weight_sum, d_out,
                                        num_heads, num_kv_chunks, head_dim, stream=None):
    """kernels.hpp:157-166 (declared, never defined, in the reference)."""
    check(lib().b2_launch_merge_attention_decode_tiled(
        _ptr(d_partial_output), _ptr(d_partial_max), _ptr(d_partial_weight_sum), _ptr(d_out),
        num_heads, num_kv_chunks, head_dim, _stream(stream)), "launch_merge_attention_decode_tiled")


# ---- graph-static decode step (device-resident positions) -------------------

def launch_rope_and_store_kv_devpos(d_q, d_k, d_v, d_k_cache, d_v_cache, d_cos, d_sin, seq_len, num_heads,
                                    num_kv_heads, head_dim, q_stride, k_stride, d_start_pos, max_seq_len,
                                    apply_rotation, stream=None):
    """launch_rope_and_store_kv with start_pos read from d_start_pos[0] (int32) at launch."""
    check(lib().b2_launch_rope_and_store_kv_devpos(
        _ptr(d_q), _ptr(d_k), _ptr(d_v), _ptr(d_k_cache), _ptr(d_v_cache), _ptr(d_cos), _ptr(d_sin),
        seq_len, num_heads, num_kv_heads, head_dim, q_stride, k_stride, _ptr(d_start_pos), max_seq_len,
        bool(apply_rotation), _stream(stream)), "launch_rope_and_store_kv_devpos")


def launch_causal_attention_decode_devlen(d_q, d_k_cache, d_v_cache, d_out, d_partial_out, d_partial_max,
                                          d_partial_weight_sum, d_kv_len, kv_len_bias, max_kv_len, num_heads,
                                          num_kv_heads, head_dim, kv_stride=0, stream=None):
    """Decode with kv_len = d_kv_len[0] + kv_len_bias (clamped to max_kv_len) read at launch."""
    check(lib().b2_launch_causal_attention_decode_devlen(
        _ptr(d_q), _ptr(d_k_cache), _ptr(d_v_cache), _ptr(d_out), _ptr(d_partial_out), _ptr(d_partial_max),
        _ptr(d_partial_weight_sum), _ptr(d_kv_len), int(kv_len_bias), max_kv_len, num_heads, num_kv_heads,
        head_dim, kv_stride, _stream(stream)), "launch_causal_attention_decode_devlen")


def advance_position(d_pos, delta=1, stream=None):
    check(lib().b2_advance_position(_ptr(d_pos), int(delta), _stream(stream)), "advance_position")


# ---- Fused decode step ----------------------------------------------------------

def decode_step_workspace_bytes(num_heads, num_kv_heads=4):
    """Bytes of the (zero-filled once) workspace of launch_decode_step_fused."""
    return int(lib().b2_decode_step_workspace_bytes(num_heads, num_kv_heads))


def launch_decode_step_fused(d_q, d_k_new, d_v_new, d_k_cache, d_v_cache, d_cos, d_sin, rope_rows, apply_rotation,
                             d_pos, d_kv_len, kv_len_bias, max_kv_len, d_out, d_workspace, workspace_bytes,
                             num_heads, num_kv_heads, head_dim, stream=None):
    """One layer's decode step in one kernel: RoPE of the new token, its K/V
    append at row kv_len - 1, split attention and merge (rope.hip.cpp:138-196 +
    causal_attention.hip.cpp:840-921). d_k_new None appends nothing."""
    check(lib().b2_launch_decode_step_fused(
        _ptr(d_q), _ptr(d_k_new), _ptr(d_v_new), _ptr(d_k_cache), _ptr(d_v_cache), _ptr(d_cos), _ptr(d_sin),
        rope_rows, bool(apply_rotation), _ptr(d_pos), _ptr(d_kv_len), int(kv_len_bias), max_kv_len, _ptr(d_out),
        _ptr(d_workspace), workspace_bytes, num_heads, num_kv_heads, head_dim, _stream(stream)),
        "launch_decode_step_fused")


def launch_decode_step_fused_rank_partial(d_q, d_k_new, d_v_new, d_k_cache, d_v_cache, d_cos, d_sin, rope_rows,
                                          apply_rotation, d_pos, d_kv_len, kv_len_bias, max_kv_len, d_rank_o,
                                          d_rank_m, d_rank_l, d_workspace, workspace_bytes, num_heads,
                                          num_kv_heads, head_dim, stream=None):
    """launch_decode_step_fused writing this rank's (o, m, l) partial instead of fp16 output."""
    check(lib().b2_launch_decode_step_fused_rank_partial(
        _ptr(d_q), _ptr(d_k_new), _ptr(d_v_new), _ptr(d_k_cache), _ptr(d_v_cache), _ptr(d_cos), _ptr(d_sin),
        rope_rows, bool(apply_rotation), _ptr(d_pos), _ptr(d_kv_len), int(kv_len_bias), max_kv_len,
        _ptr(d_rank_o), _ptr(d_rank_m), _ptr(d_rank_l), _ptr(d_workspace), workspace_bytes, num_heads,
        num_kv_heads, head_dim, _stream(stream)), "launch_decode_step_fused_rank_partial")


# ---- Fused decode step across GPUs ---------------------------------------------

def decode_exchange_bytes(world, num_heads):
    return int(lib().b2_decode_exchange_bytes(world, num_heads))


def launch_decode_step_fused_exchange(d_q, d_k_new, d_v_new, d_k_cache, d_v_cache, d_cos, d_sin, rope_rows,
                                      apply_rotation, d_pos, d_kv_len, kv_len_bias, max_kv_len, d_out, d_workspace,
                                      workspace_bytes, world, rank, exchange_buffers, num_heads, num_kv_heads,
                                      head_dim, stream=None):
    """launch_decode_step_fused over this rank's KV range with the cross-rank
    merge done inside the kernel over peer memory; d_out is the full result."""
    import ctypes
    arr = (ctypes.c_void_p * len(exchange_buffers))(*[int(p) for p in exchange_buffers])
    check(lib().b2_launch_decode_step_fused_exchange(
        _ptr(d_q), _ptr(d_k_new), _ptr(d_v_new), _ptr(d_k_cache), _ptr(d_v_cache), _ptr(d_cos), _ptr(d_sin),
        rope_rows, bool(apply_rotation), _ptr(d_pos), _ptr(d_kv_len), int(kv_len_bias), max_kv_len, _ptr(d_out),
        _ptr(d_workspace), workspace_bytes, world, rank, arr, num_heads, num_kv_heads, head_dim, _stream(stream)),
        "launch_decode_step_fused_exchange")


class ExchangeBuffers:
    """This rank's exchange buffer (CUDA IPC) plus every peer's, mapped here.
    `all_gather` gathers a list of python objects from every rank (e.g.
    torch.distributed.all_gather_object wrapped by the caller)."""

    def __init__(self, world, rank, num_heads, all_gather):
        import ctypes
        self.world, self.rank = world, rank
        self.bytes = decode_exchange_bytes(world, num_heads)
        own = ctypes.c_void_p()
        handle = (ctypes.c_char * 64)()
        check(lib().b2_ipc_alloc(self.bytes, ctypes.byref(own), handle), "ipc_alloc")
        self.own = own.value
        handles = all_gather(bytes(handle))
        self.ptrs, self._opened = [], []
        for r, h in enumerate(handles):
            if r == rank:
                self.ptrs.append(self.own)
                continue
            p = ctypes.c_void_p()
            hb = (ctypes.c_char * 64).from_buffer_copy(h)
            check(lib().b2_ipc_open(hb, ctypes.byref(p)), "ipc_open")
            self.ptrs.append(p.value)
            self._opened.append(p.value)

    def close(self):
        for p in self._opened:
            lib().b2_ipc_close(p)
        self._opened = []
        if self.own:
            lib().b2_ipc_free(self.own)
            self.own = None


# ---- Ragged batched decode ----------------------------------------------------

def launch_rope_and_store_kv_ragged(d_q, d_k, d_v, d_k_cache, d_v_cache, cache_seq_stride, d_cos, d_sin, num_seqs,
                                    num_heads, num_kv_heads, head_dim, q_stride, k_stride, d_pos, max_seq_len,
                                    apply_rotation, stream=None):
    """One new token per sequence: token b rotated at d_pos[b] and appended to row
    d_pos[b] of sequence b's cache (cache_seq_stride elements per sequence)."""
    check(lib().b2_launch_rope_and_store_kv_ragged(
        _ptr(d_q), _ptr(d_k), _ptr(d_v), _ptr(d_k_cache), _ptr(d_v_cache), cache_seq_stride, _ptr(d_cos),
        _ptr(d_sin), num_seqs, num_heads, num_kv_heads, head_dim, q_stride, k_stride, _ptr(d_pos), max_seq_len,
        bool(apply_rotation), _stream(stream)), "launch_rope_and_store_kv_ragged")


def decode_ragged_workspace_bytes(num_seqs, num_heads, num_kv_heads, max_kv_len):
    """Bytes of the (zero-filled once) workspace of launch_causal_attention_decode_ragged."""
    return int(lib().b2_decode_ragged_workspace_bytes(num_seqs, num_heads, num_kv_heads, max_kv_len))


def launch_causal_attention_decode_ragged(d_q, q_seq_stride, d_k_cache, d_v_cache, cache_seq_stride, d_kv_len,
                                          kv_len_bias, max_kv_len, d_out, out_seq_stride, num_seqs, num_heads,
                                          num_kv_heads, head_dim, d_workspace, workspace_bytes, stream=None):
    """Decode one token for each of num_seqs sequences of lengths d_kv_len[b] + bias."""
    check(lib().b2_launch_causal_attention_decode_ragged(
        _ptr(d_q), q_seq_stride, _ptr(d_k_cache), _ptr(d_v_cache), cache_seq_stride, _ptr(d_kv_len),
        int(kv_len_bias), max_kv_len, _ptr(d_out), out_seq_stride, num_seqs, num_heads, num_kv_heads, head_dim,
        _ptr(d_workspace), workspace_bytes, _stream(stream)), "launch_causal_attention_decode_ragged")


def launch_decode_step_ragged_fused(d_q, q_seq_stride, d_k_new, d_v_new, kv_new_stride, d_k_cache, d_v_cache,
                                    cache_seq_stride, d_cos, d_sin, rope_rows, apply_rotation, d_pos, max_kv_len,
                                    d_out, out_seq_stride, num_seqs, num_heads, num_kv_heads, head_dim, d_workspace,
                                    workspace_bytes, stream=None):
    """The ragged decode step in one call: each sequence's new K/V row appended
    at row d_pos[b] (K rotated), Q rotated in the kernel, attention over rows
    [0, d_pos[b]] -- launch_rope_and_store_kv_ragged + the ragged decode."""
    check(lib().b2_launch_decode_step_ragged_fused(
        _ptr(d_q), q_seq_stride, _ptr(d_k_new), _ptr(d_v_new), kv_new_stride, _ptr(d_k_cache), _ptr(d_v_cache),
        cache_seq_stride, _ptr(d_cos), _ptr(d_sin), rope_rows, bool(apply_rotation), _ptr(d_pos), max_kv_len,
        _ptr(d_out), out_seq_stride, num_seqs, num_heads, num_kv_heads, head_dim, _ptr(d_workspace),
        workspace_bytes, _stream(stream)), "launch_decode_step_ragged_fused")


# ---- KV-split decode across ranks --------------------------------------------

def launch_decode_rank_partial_devlen(d_q, d_k_cache, d_v_cache, d_partial_out, d_partial_max,
                                      d_partial_weight_sum, d_kv_len, kv_len_bias, max_kv_len, num_heads,
                                      num_kv_heads, head_dim, kv_stride, d_rank_o, d_rank_m, d_rank_l,
                                      stream=None):
    """Reduce this rank's KV range to one (o, m, l) partial per head (fp32)."""
    check(lib().b2_launch_decode_rank_partial_devlen(
        _ptr(d_q), _ptr(d_k_cache), _ptr(d_v_cache), _ptr(d_partial_out), _ptr(d_partial_max),
        _ptr(d_partial_weight_sum), _ptr(d_kv_len), int(kv_len_bias), max_kv_len, num_heads, num_kv_heads,
        head_dim, kv_stride, _ptr(d_rank_o), _ptr(d_rank_m), _ptr(d_rank_l), _stream(stream)),
        "launch_decode_rank_partial_devlen")


def launch_merge_partials_strided(d_o, d_m, d_l, d_out, num_heads, num_chunks, head_dim, o_chunk_stride,
                                  o_head_stride, ml_chunk_stride, ml_head_stride, stream=None):
    """Merge partials with arbitrary (float) strides into d_out [H][d] fp16."""
    check(lib().b2_launch_merge_partials_strided(
        _ptr(d_o), _ptr(d_m), _ptr(d_l), _ptr(d_out), num_heads, num_chunks, head_dim, o_chunk_stride,
        o_head_stride, ml_chunk_stride, ml_head_stride, _stream(stream)), "launch_merge_partials_strided")


def launch_causal_attention_prefill_batched(d_q, d_k, d_v, d_out, batch, seq_len, num_heads, num_kv_heads,
                                            head_dim, q_stride=0, kv_stride=0, q_batch_stride=0,
                                            kv_batch_stride=0, out_batch_stride=0, stream=None, out_stride=0):
    """`batch` independent causal prefills (sequence b at the given batch strides);
    out_stride: output row stride (0 = packed)."""
    check(lib().b2_launch_causal_attention_prefill_batched(
        _ptr(d_q), _ptr(d_k), _ptr(d_v), _ptr(d_out), batch, seq_len, num_heads, num_kv_heads, head_dim,
        q_stride, kv_stride, out_stride, q_batch_stride, kv_batch_stride, out_batch_stride, _stream(stream)),
        "launch_causal_attention_prefill_batched")


def launch_attention_out_projection(d_in, d_out, d_o_proj_weights, seq_len, hidden_size, num_heads, head_dim,
                                    beta=0.0, stream=None):
    """kernels.hpp:168-177 (plus a stream): out = in @ W^T + beta * out."""
    check(lib().b2_launch_attention_out_projection(
        _ptr(d_in), _ptr(d_out), _ptr(d_o_proj_weights), seq_len, hidden_size, num_heads, head_dim, float(beta),
        _stream(stream)), "launch_attention_out_projection")


def launch_attention_out_projection_decode(d_in, d_out, d_o_proj_weights, hidden_size, num_heads, head_dim, beta,
                                           stream=None):
    """kernels.hpp:179-188: one token, out = W @ in + beta * out."""
    check(lib().b2_launch_attention_out_projection_decode(
        _ptr(d_in), _ptr(d_out), _ptr(d_o_proj_weights), hidden_size, num_heads, head_dim, float(beta),
        _stream(stream)), "launch_attention_out_projection_decode")


def launch_qkv_gemm(d_input_norm, d_qkv_out, d_qkv_weights, seq_len, hidden_size, total_qkv_dim, stream=None):
    """kernels.hpp:29-36 (plus a stream): qkv = input @ W_qkv^T."""
    check(lib().b2_launch_qkv_gemm(_ptr(d_input_norm), _ptr(d_qkv_out), _ptr(d_qkv_weights), seq_len, hidden_size,
                                   total_qkv_dim, _stream(stream)), "launch_qkv_gemm")


def launch_qkv_decode(d_input_norm, d_qkv_out, d_qkv_weights, hidden_size, total_qkv_dim, stream=None):
    """kernels.hpp:38-44: one token, qkv = W_qkv @ input."""
    check(lib().b2_launch_qkv_decode(_ptr(d_input_norm), _ptr(d_qkv_out), _ptr(d_qkv_weights), hidden_size,
                                     total_qkv_dim, _stream(stream)), "launch_qkv_decode")


def launch_qkv_gemm_rope_store_kv(d_input_norm, d_qkv_out, d_qkv_weights, d_k_cache, d_v_cache, d_cos, d_sin,
                                  seq_len, hidden_size, num_heads, num_kv_heads, head_dim, start_pos=0,
                                  apply_rotary=True, stream=None):
    """launch_qkv_gemm then launch_rope_and_store_kv on its rows
    (include/model_inference.hpp:266-281) as one kernel, bit-identical to the
    two calls."""
    check(lib().b2_launch_qkv_gemm_rope_store_kv(
        _ptr(d_input_norm), _ptr(d_qkv_out), _ptr(d_qkv_weights), _ptr(d_k_cache), _ptr(d_v_cache), _ptr(d_cos),
        _ptr(d_sin), seq_len, hidden_size, num_heads, num_kv_heads, head_dim, start_pos, bool(apply_rotary),
        _stream(stream)), "launch_qkv_gemm_rope_store_kv")
