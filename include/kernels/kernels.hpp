// Drop-in replacement for the attention part of the reference's
// include/kernels/kernels.hpp (MarcVivas/llm-inference): the same function
// names, parameter order, types (with HIP->CUDA aliases) and default
// arguments, forwarding to the b200attn C ABI (include/b200attn.h).
//
// Error behaviour matches the reference: the cases its launchers silently
// skip (seq_len == 0, kv_len == 0, num_kv_heads == 0, num_heads % num_kv_heads)
// stay silent; anything else that fails throws std::runtime_error where the
// reference would have exited through HIP_CHECK.
//
// Of the reference header's non-attention launchers only the attention output
// projection, the path's consumer, is here; embedding, RMSNorm, the other
// GEMMs, SwiGLU and argmax are not part of this library.
#pragma once

#include <cstddef>
#include <cstdint>

#include "b200attn.h"
#include "b200attn/gpu_utils.hpp"
#include "b200attn/hip_compat.hpp"

// Tokens per flash-decode chunk (reference: 12). Workspaces are sized from it
// (include/model_inference.hpp:192-198).
#define KV_CHUNK 256

namespace b200attn::detail {
inline b2_stream_t s(hipStream_t stream) { return reinterpret_cast<b2_stream_t>(stream); }
}  // namespace b200attn::detail

// kernels.hpp:47-60
inline void launch_rope(__half* d_q, __half* d_k, const __half* d_cos, const __half* d_sin, size_t seq_len,
                        size_t num_heads, size_t num_kv_heads, size_t head_dim, size_t q_stride, size_t k_stride,
                        size_t start_pos = 0) {
    b200attn::check(b2_launch_rope(d_q, d_k, d_cos, d_sin, seq_len, num_heads, num_kv_heads, head_dim, q_stride,
                                   k_stride, start_pos, nullptr),
                    "launch_rope");
}

// kernels.hpp:62-80
inline void launch_rope_and_store_kv(__half* d_q, __half* d_k, __half* d_v, __half* d_k_cache, __half* d_v_cache,
                                     const __half* d_cos, const __half* d_sin, size_t seq_len, size_t num_heads,
                                     size_t num_kv_heads, size_t head_dim, size_t q_stride, size_t k_stride,
                                     size_t start_pos, bool apply_rotation, hipStream_t stream = nullptr) {
    b200attn::check(b2_launch_rope_and_store_kv(d_q, d_k, d_v, d_k_cache, d_v_cache, d_cos, d_sin, seq_len,
                                                num_heads, num_kv_heads, head_dim, q_stride, k_stride, start_pos,
                                                apply_rotation, b200attn::detail::s(stream)),
                    "launch_rope_and_store_kv");
}

// kernels.hpp:81-86
inline void update_rope_and_store_kv_node(hipGraphExec_t graph_exec, hipGraphNode_t node, size_t start_pos,
                                          bool apply_rotation) {
    b200attn::check(b2_update_rope_and_store_kv_node(reinterpret_cast<b2_graph_exec_t>(graph_exec),
                                                     reinterpret_cast<b2_graph_node_t>(node), start_pos,
                                                     apply_rotation),
                    "update_rope_and_store_kv_node");
}

// kernels.hpp:88-99 (the stream parameter is an addition; default = the
// reference's implicit default stream)
inline void launch_causal_attention_prefill(const __half* d_q, const __half* d_k, const __half* d_v, __half* d_out,
                                            size_t seq_len, size_t num_heads, size_t num_kv_heads, size_t head_dim,
                                            size_t q_stride = 0, size_t kv_stride = 0,
                                            hipStream_t stream = nullptr) {
    b200attn::check(b2_launch_causal_attention_prefill(d_q, d_k, d_v, d_out, seq_len, num_heads, num_kv_heads,
                                                       head_dim, q_stride, kv_stride, b200attn::detail::s(stream)),
                    "launch_causal_attention_prefill");
}

// kernels.hpp:104-125
inline void launch_causal_attention_decode(const __half* d_q, const __half* d_k_cache, const __half* d_v_cache,
                                           __half* d_out, float* d_partial_out, float* d_partial_max,
                                           float* d_partial_weight_sum, size_t query_len, size_t kv_cache_len,
                                           size_t start_pos, size_t num_heads, size_t num_kv_heads, size_t head_dim,
                                           size_t q_stride, size_t kv_stride, hipStream_t stream = nullptr,
                                           hipGraphNode_t* attention_node = nullptr,
                                           hipGraphNode_t* merge_node = nullptr) {
    b200attn::check(b2_launch_causal_attention_decode(
                        d_q, d_k_cache, d_v_cache, d_out, d_partial_out, d_partial_max, d_partial_weight_sum,
                        query_len, kv_cache_len, start_pos, num_heads, num_kv_heads, head_dim, q_stride, kv_stride,
                        b200attn::detail::s(stream), reinterpret_cast<b2_graph_node_t*>(attention_node),
                        reinterpret_cast<b2_graph_node_t*>(merge_node)),
                    "launch_causal_attention_decode");
}

// kernels.hpp:127-146
inline void launch_causal_attention_decode_vectorized(
    const __half* d_q, const __half* d_k_cache, const __half* d_v_cache, __half* d_out, float* d_partial_out,
    float* d_partial_max, float* d_partial_weight_sum, size_t query_len, size_t kv_cache_len, size_t start_pos,
    size_t num_heads, size_t num_kv_heads, size_t head_dim, size_t q_stride = 0, size_t kv_stride = 0,
    hipStream_t stream = nullptr, hipGraphNode_t* attention_node = nullptr, hipGraphNode_t* merge_node = nullptr) {
    b200attn::check(b2_launch_causal_attention_decode_vectorized(
                        d_q, d_k_cache, d_v_cache, d_out, d_partial_out, d_partial_max, d_partial_weight_sum,
                        query_len, kv_cache_len, start_pos, num_heads, num_kv_heads, head_dim, q_stride, kv_stride,
                        b200attn::detail::s(stream), reinterpret_cast<b2_graph_node_t*>(attention_node),
                        reinterpret_cast<b2_graph_node_t*>(merge_node)),
                    "launch_causal_attention_decode_vectorized");
}

// kernels.hpp:148-152
inline void update_merge_attention_decode_node(hipGraphExec_t graph_exec, hipGraphNode_t node, size_t kv_cache_len) {
    b200attn::check(b2_update_merge_attention_decode_node(reinterpret_cast<b2_graph_exec_t>(graph_exec),
                                                          reinterpret_cast<b2_graph_node_t>(node), kv_cache_len),
                    "update_merge_attention_decode_node");
}

// kernels.hpp:157-166 (declared but never defined in the reference)
inline void launch_merge_attention_decode_tiled(const float* d_partial_output, const float* d_partial_max,
                                                const float* d_partial_weight_sum, __half* d_out, size_t num_heads,
                                                size_t num_kv_chunks, size_t head_dim,
                                                hipStream_t stream = nullptr) {
    b200attn::check(b2_launch_merge_attention_decode_tiled(d_partial_output, d_partial_max, d_partial_weight_sum,
                                                           d_out, num_heads, num_kv_chunks, head_dim,
                                                           b200attn::detail::s(stream)),
                    "launch_merge_attention_decode_tiled");
}

// kernels.hpp:190-194
inline void update_causal_attention_decode_node(hipGraphExec_t graph_exec, hipGraphNode_t node,
                                                size_t kv_cache_len) {
    b200attn::check(b2_update_causal_attention_decode_node(reinterpret_cast<b2_graph_exec_t>(graph_exec),
                                                           reinterpret_cast<b2_graph_node_t>(node), kv_cache_len),
                    "update_causal_attention_decode_node");
}


// kernels.hpp:29-36 (plus a stream; the reference's rocBLAS call uses the
// handle's)
inline void launch_qkv_gemm(const __half* d_input_norm, __half* d_qkv_out, const __half* d_qkv_weights,
                            size_t seq_len, size_t hidden_size, size_t total_qkv_dim, hipStream_t stream = nullptr) {
    b200attn::check(b2_launch_qkv_gemm(d_input_norm, d_qkv_out, d_qkv_weights, seq_len, hidden_size, total_qkv_dim,
                                       b200attn::detail::s(stream)),
                    "launch_qkv_gemm");
}

// kernels.hpp:38-44
inline void launch_qkv_decode(const __half* d_input_norm, __half* d_qkv_out, const __half* d_qkv_weights,
                              size_t hidden_size, size_t total_qkv_dim, hipStream_t stream = nullptr) {
    b200attn::check(b2_launch_qkv_decode(d_input_norm, d_qkv_out, d_qkv_weights, hidden_size, total_qkv_dim,
                                         b200attn::detail::s(stream)),
                    "launch_qkv_decode");
}

// launch_qkv_gemm + launch_rope_and_store_kv (model_inference.hpp:266-281) in
// one kernel; no counterpart in the reference's header.
inline void launch_qkv_gemm_rope_store_kv(const __half* d_input_norm, __half* d_qkv_out, const __half* d_qkv_weights,
                                          __half* d_k_cache, __half* d_v_cache, const __half* d_cos,
                                          const __half* d_sin, size_t seq_len, size_t hidden_size, size_t num_heads,
                                          size_t num_kv_heads, size_t head_dim, size_t start_pos = 0,
                                          bool apply_rotary = true, hipStream_t stream = nullptr) {
    b200attn::check(b2_launch_qkv_gemm_rope_store_kv(d_input_norm, d_qkv_out, d_qkv_weights, d_k_cache, d_v_cache,
                                                     d_cos, d_sin, seq_len, hidden_size, num_heads, num_kv_heads,
                                                     head_dim, start_pos, apply_rotary, b200attn::detail::s(stream)),
                    "launch_qkv_gemm_rope_store_kv");
}
// kernels.hpp:168-177 (the stream parameter is an addition)
inline void launch_attention_out_projection(const __half* d_in, __half* d_out, const __half* d_o_proj_weights,
                                            size_t seq_len, size_t hidden_size, size_t num_heads, size_t head_dim,
                                            float beta = 0.f, hipStream_t stream = nullptr) {
    b200attn::check(b2_launch_attention_out_projection(d_in, d_out, d_o_proj_weights, seq_len, hidden_size,
                                                       num_heads, head_dim, beta, b200attn::detail::s(stream)),
                    "launch_attention_out_projection");
}

// kernels.hpp:179-188
inline void launch_attention_out_projection_decode(const __half* d_in, __half* d_out,
                                                   const __half* d_o_proj_weights, size_t hidden_size,
                                                   size_t num_heads, size_t head_dim, float beta,
                                                   hipStream_t stream = nullptr) {
    b200attn::check(b2_launch_attention_out_projection_decode(d_in, d_out, d_o_proj_weights, hidden_size,
                                                              num_heads, head_dim, beta,
                                                              b200attn::detail::s(stream)),
                    "launch_attention_out_projection_decode");
}
