/*
 * b200attn -- C ABI of the B200 (sm_100a) GQA attention hot path.
 *
 * Drop-in for the attention entry points of MarcVivas/llm-inference's
 * include/kernels/kernels.hpp. Every reference launcher has one extern "C"
 * symbol here with the same parameter order and meaning; the differences are
 * only those a C ABI needs:
 *   - __half* becomes void* (IEEE binary16 payload, row-major),
 *   - hipStream_t / hipGraphExec_t / hipGraphNode_t become the CUDA handles
 *     below (the same types as cudaStream_t / cudaGraphExec_t /
 *     cudaGraphNode_t, declared here without the CUDA headers),
 *   - every call returns an int status instead of void (B2_OK or
 *     B2_NOTHING_TO_DO on success, a negative B2_ERR_* otherwise); nothing
 *     exits the process or throws across this boundary,
 *   - prefill takes the stream the reference launcher lacks.
 * include/kernels/kernels.hpp in this repository re-declares the reference's
 * C++ names and default arguments on top of these symbols.
 *
 * Ownership: the caller owns every buffer (Q/K/V activations, the KV cache,
 * the RoPE tables, outputs, the decode partial workspace). No call allocates
 * device memory, synchronises, or reads device memory from the host, so every
 * launcher can be captured into a CUDA graph.
 */
#ifndef B200ATTN_H
#define B200ATTN_H

#include <stddef.h>
#include <stdint.h>
#ifndef __cplusplus
#include <stdbool.h>
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Same underlying types as cudaStream_t, cudaGraphExec_t, cudaGraphNode_t. */
typedef struct CUstream_st* b2_stream_t;
typedef struct CUgraphExec_st* b2_graph_exec_t;
typedef struct CUgraphNode_st* b2_graph_node_t;

/* Status codes. */
#define B2_OK 0
#define B2_NOTHING_TO_DO 1       /* a case the reference launcher silently skips */
#define B2_ERR_INVALID_ARG (-1)  /* null buffer, bad GQA config the kernel cannot run */
#define B2_ERR_UNSUPPORTED (-2)  /* shape outside what the kernels implement */
#define B2_ERR_ALIGNMENT (-3)    /* pointer/stride alignment a TMA path needs */
#define B2_ERR_CUDA (-4)         /* a CUDA runtime call failed; see b2_last_cuda_error */
#define B2_ERR_WORKSPACE (-5)    /* workspace smaller than the call needs */
#define B2_ERR_GRAPH (-6)        /* capture query / node patch failed */

/* Tokens per flash-decode chunk; the reference's KV_CHUNK macro
 * (include/kernels/kernels.hpp:103, 12 there). Partial workspaces are sized
 * [num_heads][ceil(kv_len / b2_kv_chunk())]. */
int b2_kv_chunk(void);

/* Floats of decode workspace the reference engine allocates for a cache of
 * max_kv_len tokens: num_heads * ceil(max_kv_len / KV_CHUNK) * (head_dim + 2)
 * (include/model_inference.hpp:192-198). */
size_t b2_decode_workspace_floats(size_t num_heads, size_t head_dim, size_t max_kv_len);

const char* b2_status_string(int status);
int b2_last_cuda_error(void);            /* cudaError_t of the last B2_ERR_CUDA */
uint64_t b2_kernel_launch_count(void);   /* kernels this library has launched */
/* OR of the device-side error bits on the current device: bit 0 = a bounded
 * wait inside a kernel (TMA copy / pipeline barrier) ran out of time and the
 * kernel stopped early; bit 1 = a fused decode step got a RoPE position
 * outside its table. 0 when every kernel completed normally. */
unsigned int b2_device_error_word(void);
/* Reset those bits to 0 on the current device (host-synchronous copy). */
int b2_clear_device_error_word(void);

/* Host-side RoPE tables, include/rope_cache.hpp:49-76 (compute_inverse_frequencies,
 * fill_host_tables): cos/sin[pos][i] = fp16(cos/sin(float(pos) * inv_freq[i])),
 * inv_freq[i] = 1 / theta^(2i/head_dim), FP32 host math. Tables are
 * [max_seq_len][head_dim/2] binary16. Pure host code; no device call. */
int b2_fill_rope_tables(size_t max_seq_len, size_t head_dim, float rope_theta,
                        uint16_t* host_cos, uint16_t* host_sin);

/* include/kernels/kernels.hpp:47-60 launch_rope (src/kernels/rope.hip.cpp:198-205):
 * rotate-half RoPE on Q and K in place at positions start_pos + t. */
int b2_launch_rope(void* d_q, void* d_k, const void* d_cos, const void* d_sin,
                   size_t seq_len, size_t num_heads, size_t num_kv_heads,
                   size_t head_dim, size_t q_stride, size_t k_stride,
                   size_t start_pos, b2_stream_t stream);

/* include/kernels/kernels.hpp:62-80 launch_rope_and_store_kv
 * (src/kernels/rope.hip.cpp:138-196): with apply_rotation, Q is rotated in
 * place and rotated K plus unchanged V are written to cache rows
 * start_pos + t (row stride num_kv_heads * head_dim); without it K and V are
 * copied verbatim (NoPE layers) and Q is untouched. K/V sources are never
 * modified when a cache is given. d_k_cache == NULL with apply_rotation
 * rotates K in place (the launch_rope path). Strides are elements between
 * tokens; V uses k_stride; 0 means packed. */
int b2_launch_rope_and_store_kv(void* d_q, void* d_k, const void* d_v,
                                void* d_k_cache, void* d_v_cache,
                                const void* d_cos, const void* d_sin,
                                size_t seq_len, size_t num_heads, size_t num_kv_heads,
                                size_t head_dim, size_t q_stride, size_t k_stride,
                                size_t start_pos, bool apply_rotation,
                                b2_stream_t stream);

/* include/kernels/kernels.hpp:81-86 update_rope_and_store_kv_node
 * (src/kernels/rope.hip.cpp:208-241): re-point a captured RoPE/append node of
 * graph_exec at a new start_pos. apply_rotation must match the capture. */
int b2_update_rope_and_store_kv_node(b2_graph_exec_t graph_exec, b2_graph_node_t node,
                                     size_t start_pos, bool apply_rotation);

/* include/kernels/kernels.hpp:88-99 launch_causal_attention_prefill
 * (src/kernels/causal_attention.hip.cpp:376-451): out[t][h*d + c] (packed,
 * stride num_heads*head_dim) = softmax_{j<=t}(q_t . k_j / sqrt(d)) V for
 * kv head h / (num_heads / num_kv_heads). start_pos = 0, kv_len = seq_len.
 * Head_dim 128 with 16-byte aligned rows runs the tcgen05/TMA kernel; other
 * shapes run a SIMT kernel. */
int b2_launch_causal_attention_prefill(const void* d_q, const void* d_k, const void* d_v,
                                       void* d_out, size_t seq_len, size_t num_heads,
                                       size_t num_kv_heads, size_t head_dim,
                                       size_t q_stride, size_t kv_stride,
                                       b2_stream_t stream);

/* Batched form of b2_launch_causal_attention_prefill (no reference
 * counterpart; the reference engine is batch 1): `batch` independent
 * sequences of seq_len tokens, sequence b's Q / K / V / out rows starting
 * q_batch_stride / kv_batch_stride / out_batch_stride elements after
 * sequence b-1's (e.g. per-sequence KV caches of one allocation). out_stride
 * is the output row stride (0 = packed num_heads * head_dim), so a block of
 * heads can be written into a wider output. */
int b2_launch_causal_attention_prefill_batched(const void* d_q, const void* d_k, const void* d_v,
                                               void* d_out, size_t batch, size_t seq_len,
                                               size_t num_heads, size_t num_kv_heads, size_t head_dim,
                                               size_t q_stride, size_t kv_stride, size_t out_stride,
                                               size_t q_batch_stride, size_t kv_batch_stride,
                                               size_t out_batch_stride, b2_stream_t stream);

/* include/kernels/kernels.hpp:104-125 launch_causal_attention_decode
 * (src/kernels/causal_attention.hip.cpp:840-921): one query token over
 * kv_cache_len cached tokens, split into KV_CHUNK-token chunks whose (o, m, l)
 * partials go to d_partial_out [H][chunks][d], d_partial_max [H][chunks],
 * d_partial_weight_sum [H][chunks], then merged into d_out [H][d] fp16.
 * Q is one packed [num_heads][head_dim] vector at d_q (q_stride and
 * start_pos are accepted and unused, as in the reference). When
 * attention_node / merge_node are non-null the stream must be capturing and
 * they receive the two captured kernel nodes. */
int b2_launch_causal_attention_decode(const void* d_q, const void* d_k_cache,
                                      const void* d_v_cache, void* d_out,
                                      float* d_partial_out, float* d_partial_max,
                                      float* d_partial_weight_sum,
                                      size_t query_len, size_t kv_cache_len,
                                      size_t start_pos, size_t num_heads,
                                      size_t num_kv_heads, size_t head_dim,
                                      size_t q_stride, size_t kv_stride,
                                      b2_stream_t stream,
                                      b2_graph_node_t* attention_node,
                                      b2_graph_node_t* merge_node);

/* include/kernels/kernels.hpp:127-146 launch_causal_attention_decode_vectorized
 * (src/kernels/causal_attention.hip.cpp:923-972). Same contract as
 * b2_launch_causal_attention_decode (both run the same kernels here). */
int b2_launch_causal_attention_decode_vectorized(const void* d_q, const void* d_k_cache,
                                                 const void* d_v_cache, void* d_out,
                                                 float* d_partial_out, float* d_partial_max,
                                                 float* d_partial_weight_sum,
                                                 size_t query_len, size_t kv_cache_len,
                                                 size_t start_pos, size_t num_heads,
                                                 size_t num_kv_heads, size_t head_dim,
                                                 size_t q_stride, size_t kv_stride,
                                                 b2_stream_t stream,
                                                 b2_graph_node_t* attention_node,
                                                 b2_graph_node_t* merge_node);

/* include/kernels/kernels.hpp:190-194 update_causal_attention_decode_node
 * (src/kernels/causal_attention.hip.cpp:975-1001): patch kv_cache_len (and
 * the chunk count / grid) of a captured split-KV node. */
int b2_update_causal_attention_decode_node(b2_graph_exec_t graph_exec, b2_graph_node_t node,
                                           size_t kv_cache_len);

/* include/kernels/kernels.hpp:148-152 update_merge_attention_decode_node
 * (src/kernels/causal_attention.hip.cpp:1003-1026): patch the chunk count of a
 * captured merge node. */
int b2_update_merge_attention_decode_node(b2_graph_exec_t graph_exec, b2_graph_node_t node,
                                          size_t kv_cache_len);

/* include/kernels/kernels.hpp:157-166 launch_merge_attention_decode_tiled
 * (declared there, defined nowhere): merge caller-provided partials
 * [H][chunks][d] / [H][chunks] / [H][chunks] into d_out [H][d] fp16, warps
 * across chunks and lanes across output dimensions. */
int b2_launch_merge_attention_decode_tiled(const float* d_partial_output,
                                           const float* d_partial_max,
                                           const float* d_partial_weight_sum,
                                           void* d_out, size_t num_heads,
                                           size_t num_kv_chunks, size_t head_dim,
                                           b2_stream_t stream);

/* ---- Graph-static decode step (no per-step node patching) ----------------
 * The reference captures its decode step into a HIP graph once and patches
 * 3 kernel nodes per layer before every token
 * (include/model_inference.hpp:96-123). These variants read the position
 * from device memory instead, so one captured graph serves every step; the
 * caller advances the device position (b2_advance_position) inside the graph
 * or between launches. Results equal the host-length launchers. */

/* b2_launch_rope_and_store_kv with start_pos = d_start_pos[0] read at launch.
 * Tokens whose position start_pos + t >= max_seq_len are skipped (no table
 * read, no cache write); a negative position skips the launch's work. */
int b2_launch_rope_and_store_kv_devpos(void* d_q, void* d_k, const void* d_v,
                                       void* d_k_cache, void* d_v_cache,
                                       const void* d_cos, const void* d_sin,
                                       size_t seq_len, size_t num_heads, size_t num_kv_heads,
                                       size_t head_dim, size_t q_stride, size_t k_stride,
                                       const int32_t* d_start_pos, size_t max_seq_len,
                                       bool apply_rotation, b2_stream_t stream);

/* b2_launch_causal_attention_decode with kv_len = clamp(d_kv_len[0] +
 * kv_len_bias, 0, max_kv_len) read at launch (bias 1 turns a start_pos into
 * the decode length, include/model_inference.hpp:382). The partial workspace
 * is laid out for max_kv_len: [H][ceil(max_kv_len/KV_CHUNK)][d] etc., i.e.
 * b2_decode_workspace_floats(H, d, max_kv_len) floats in the reference's
 * three arrays. kv_len 0 writes a zero output. */
int b2_launch_causal_attention_decode_devlen(const void* d_q, const void* d_k_cache,
                                             const void* d_v_cache, void* d_out,
                                             float* d_partial_out, float* d_partial_max,
                                             float* d_partial_weight_sum,
                                             const int32_t* d_kv_len, int32_t kv_len_bias,
                                             size_t max_kv_len, size_t num_heads,
                                             size_t num_kv_heads, size_t head_dim,
                                             size_t kv_stride, b2_stream_t stream);

/* ---- KV-split decode across GPUs (one rank per GPU) ----------------------
 * Each rank attends over its own contiguous range of the cache and reduces
 * it to one partial per head; the partials of all ranks are exchanged (e.g.
 * an NCCL all-gather) and merged with b2_launch_merge_partials_strided. The
 * algebra is the reference's chunk merge (src/kernels/causal_attention.hip.cpp
 * :719-819) applied once more, with ranks as chunks. */

/* b2_launch_causal_attention_decode_devlen over this rank's range, whose
 * merge writes the rank partial instead of an fp16 output:
 * d_rank_o[h*head_dim + e] = sum_c e^(m_c - M) o_c[e] (fp32, unnormalised),
 * d_rank_m[h] = M = max_c m_c (natural-log units), d_rank_l[h] =
 * sum_c e^(m_c - M) l_c. An empty range gives M = -inf, L = 0, o = 0. */
int b2_launch_decode_rank_partial_devlen(const void* d_q, const void* d_k_cache,
                                         const void* d_v_cache, float* d_partial_out,
                                         float* d_partial_max, float* d_partial_weight_sum,
                                         const int32_t* d_kv_len, int32_t kv_len_bias,
                                         size_t max_kv_len, size_t num_heads,
                                         size_t num_kv_heads, size_t head_dim, size_t kv_stride,
                                         float* d_rank_o, float* d_rank_m, float* d_rank_l,
                                         b2_stream_t stream);

/* Merge num_chunks partials per head with arbitrary strides (in floats):
 * o of (chunk c, head h) at d_o + c*o_chunk_stride + h*o_head_stride, m and l
 * at d_m / d_l + c*ml_chunk_stride + h*ml_head_stride. Writes d_out [H][d]
 * fp16. With strides (d, chunks*d, 1, chunks) this is the reference merge. */
int b2_launch_merge_partials_strided(const float* d_o, const float* d_m, const float* d_l,
                                     void* d_out, size_t num_heads, size_t num_chunks,
                                     size_t head_dim, size_t o_chunk_stride,
                                     size_t o_head_stride, size_t ml_chunk_stride,
                                     size_t ml_head_stride, b2_stream_t stream);

/* d_pos[0] += delta on the stream (one thread), for device-resident positions. */
int b2_advance_position(int32_t* d_pos, int32_t delta, b2_stream_t stream);

/* ---- Fused decode step (one kernel per layer) -----------------------------
 * No single counterpart in the reference: it replaces, for one decode token
 * of one layer, the reference's launch_rope_and_store_kv
 * (src/kernels/rope.hip.cpp:138-196) followed by
 * launch_causal_attention_decode and its merge
 * (src/kernels/causal_attention.hip.cpp:840-921), i.e. the three nodes per
 * layer of include/model_inference.hpp:96-123, with one graph-static call:
 * one split-attention kernel that also does the RoPE and the append, whose
 * CTAs take 16-token tiles from a shared counter until none are left and
 * whose first min(splits, num_heads) CTAs then merge the split partials of
 * one head each.
 *  - kv_len = clamp(d_kv_len[0] + kv_len_bias, 0, max_kv_len), read at launch.
 *  - Q (d_q, [num_heads][128], before RoPE) is rotated in registers at
 *    position d_pos[0] when apply_rotation; d_q is read, never written.
 *  - With d_k_new != NULL the new token's K (rotated when apply_rotation) and
 *    V ([num_kv_heads][128] each) are written to cache row kv_len - 1 of
 *    d_k_cache / d_v_cache (packed rows of num_kv_heads * 128) before that
 *    row is attended. d_k_new == NULL appends nothing (e.g. a rank that does
 *    not own the newest row).
 *  - A position outside [0, rope_rows) with apply_rotation appends nothing,
 *    leaves Q unrotated and sets bit 1 of b2_device_error_word.
 *  - Output: d_out [num_heads][128] fp16 = the attention of the rotated Q over
 *    rows [0, kv_len), equal to the reference's launch sequence within
 *    floating-point reassociation; kv_len 0 writes zeros.
 *  - head_dim 128, num_kv_heads in {1,2,4,8}, num_heads / num_kv_heads <= 8;
 *    16-byte aligned pointers. Other shapes return B2_ERR_UNSUPPORTED.
 *  - d_workspace holds b2_decode_step_workspace_bytes(num_heads, num_kv_heads)
 *    bytes (split partials and three counter words) and must be ZERO-FILLED
 *    once before its first use; each call leaves the words consistent for the
 *    next (after a device error bit 0, zero it again). One workspace
 *    serves any number of calls ordered on one stream (e.g. every layer of a
 *    captured step); calls that can overlap on the GPU need separate
 *    workspaces. */
size_t b2_decode_step_workspace_bytes(size_t num_heads, size_t num_kv_heads);
int b2_launch_decode_step_fused(const void* d_q, const void* d_k_new, const void* d_v_new,
                                void* d_k_cache, void* d_v_cache,
                                const void* d_cos, const void* d_sin, size_t rope_rows,
                                bool apply_rotation, const int32_t* d_pos,
                                const int32_t* d_kv_len, int32_t kv_len_bias, size_t max_kv_len,
                                void* d_out, void* d_workspace, size_t workspace_bytes,
                                size_t num_heads, size_t num_kv_heads, size_t head_dim,
                                b2_stream_t stream);

/* b2_launch_decode_step_fused over this rank's range of the cache, writing the
 * rank partial of b2_launch_decode_rank_partial_devlen (d_rank_o unnormalised
 * fp32 [H][128], d_rank_m natural-log max, d_rank_l weight sum) instead of an
 * fp16 output, for a KV-split decode across GPUs. */
int b2_launch_decode_step_fused_rank_partial(const void* d_q, const void* d_k_new, const void* d_v_new,
                                             void* d_k_cache, void* d_v_cache,
                                             const void* d_cos, const void* d_sin, size_t rope_rows,
                                             bool apply_rotation, const int32_t* d_pos,
                                             const int32_t* d_kv_len, int32_t kv_len_bias,
                                             size_t max_kv_len, float* d_rank_o, float* d_rank_m,
                                             float* d_rank_l, void* d_workspace, size_t workspace_bytes,
                                             size_t num_heads, size_t num_kv_heads, size_t head_dim,
                                             b2_stream_t stream);

/* ---- Fused decode step across GPUs (exchange inside the kernel) -----------
 * b2_launch_decode_step_fused over this rank's KV range (as the _rank_partial
 * form) whose merging CTAs publish each head's rank partial straight into
 * every rank's exchange buffer (peer stores over NVLink, release flags),
 * wait (bounded, 2 s) for every rank's partial of that head and write the
 * merged fp16 output: d_out holds the full attention on every rank. The
 * cross-rank merge is the reference's chunk merge with ranks as chunks
 * (src/kernels/causal_attention.hip.cpp:719-819).
 *  - exchange_buffers: HOST array of `world` (2..8) device pointers, every
 *    rank's exchange buffer mapped into this process ([rank] = its own, from
 *    b2_ipc_alloc; the others from b2_ipc_open of their handles), each
 *    b2_decode_exchange_bytes(world, num_heads) bytes, zero at allocation.
 *  - Every rank must make the same sequence of calls (one exchange per call),
 *    each rank on its own GPU; a rank that stops makes the others time out
 *    (device error bit 0) instead of hanging. */
size_t b2_decode_exchange_bytes(size_t world, size_t num_heads);
int b2_launch_decode_step_fused_exchange(const void* d_q, const void* d_k_new, const void* d_v_new,
                                         void* d_k_cache, void* d_v_cache,
                                         const void* d_cos, const void* d_sin, size_t rope_rows,
                                         bool apply_rotation, const int32_t* d_pos,
                                         const int32_t* d_kv_len, int32_t kv_len_bias,
                                         size_t max_kv_len, void* d_out, void* d_workspace,
                                         size_t workspace_bytes, size_t world, size_t rank,
                                         void* const* exchange_buffers, size_t num_heads,
                                         size_t num_kv_heads, size_t head_dim, b2_stream_t stream);

/* CUDA IPC helpers for exchange buffers: allocate `bytes` zero-filled device
 * memory and export its 64-byte handle; map a peer's handle into this
 * process; unmap; free. */
int b2_ipc_alloc(size_t bytes, void** d_ptr, void* handle_out);
int b2_ipc_open(const void* handle, void** d_ptr);
int b2_ipc_close(void* d_ptr);
int b2_ipc_free(void* d_ptr);

/* ---- Ragged batched decode (continuous batching) ---------------------------
 * No counterpart in the reference, whose engine decodes one sequence per
 * call (src/kernels/causal_attention.hip.cpp:840-921); these apply the same
 * split-KV attention and chunk merge (:493-595, :719-819) to B sequences of
 * different lengths in one launch pair.
 *
 * b2_launch_rope_and_store_kv_ragged: b2_launch_rope_and_store_kv_devpos for
 * one new token per sequence: token b (Q / K / V rows b, strides q_stride /
 * k_stride, 0 = packed) is rotated at position d_pos[b] and its K/V written
 * to row d_pos[b] of sequence b's cache, which starts cache_seq_stride
 * elements after sequence b-1's (>= max_seq_len * num_kv_heads * head_dim).
 * Tokens whose position is outside [0, max_seq_len) are skipped. */
int b2_launch_rope_and_store_kv_ragged(void* d_q, void* d_k, const void* d_v,
                                       void* d_k_cache, void* d_v_cache, size_t cache_seq_stride,
                                       const void* d_cos, const void* d_sin, size_t num_seqs,
                                       size_t num_heads, size_t num_kv_heads, size_t head_dim,
                                       size_t q_stride, size_t k_stride, const int32_t* d_pos,
                                       size_t max_seq_len, bool apply_rotation, b2_stream_t stream);

/* One query token per sequence: out[b] ([num_heads][128] fp16 at
 * d_out + b * out_seq_stride) = attention of Q row b (d_q + b * q_seq_stride)
 * over rows [0, len_b) of sequence b's cache (d_k_cache / d_v_cache +
 * b * cache_seq_stride, packed rows of num_kv_heads * 128), len_b =
 * clamp(d_kv_len[b] + kv_len_bias, 0, max_kv_len), read at launch (graph
 * static). Strides in elements; 0 = packed (cache: max_kv_len rows). A
 * sequence of length 0 gets a zero output. head_dim 128, num_kv_heads in
 * {1,2,4,8}, num_heads / num_kv_heads <= 8, num_seqs <= 1024; 16-byte
 * aligned buffers and row strides.
 * d_workspace: b2_decode_ragged_workspace_bytes(num_seqs, num_heads,
 * num_kv_heads, max_kv_len) bytes, ZERO-FILLED once before first use (each
 * call leaves its counter at zero again); one workspace per stream. */
size_t b2_decode_ragged_workspace_bytes(size_t num_seqs, size_t num_heads, size_t num_kv_heads,
                                        size_t max_kv_len);
int b2_launch_causal_attention_decode_ragged(const void* d_q, size_t q_seq_stride,
                                             const void* d_k_cache, const void* d_v_cache,
                                             size_t cache_seq_stride, const int32_t* d_kv_len,
                                             int32_t kv_len_bias, size_t max_kv_len, void* d_out,
                                             size_t out_seq_stride, size_t num_seqs, size_t num_heads,
                                             size_t num_kv_heads, size_t head_dim, void* d_workspace,
                                             size_t workspace_bytes, b2_stream_t stream);

/* The ragged decode step in one call (the two launches above, fused): for
 * each sequence b, with p = d_pos[b] (its new token's position and cache row):
 *  - the new K row (d_k_new + b * kv_new_stride, [num_kv_heads][128]) rotated
 *    at p when apply_rotation, and the V row, are written to row p of
 *    sequence b's cache before that row is attended (d_k_new == NULL appends
 *    nothing);
 *  - Q row b (d_q + b * q_seq_stride, read, never written) is rotated at p
 *    when apply_rotation;
 *  - out[b] = attention of the rotated Q over rows [0, min(p + 1, max_kv_len)).
 * A position outside [0, rope_rows) with apply_rotation appends nothing,
 * leaves Q unrotated and sets bit 1 of b2_device_error_word; p < 0 gives a
 * zero output. kv_new_stride 0 = packed (num_kv_heads * 128). Results equal
 * b2_launch_rope_and_store_kv_ragged followed by
 * b2_launch_causal_attention_decode_ragged (kv_len d_pos, bias 1); same
 * shapes, alignment and workspace as the decode. */
int b2_launch_decode_step_ragged_fused(const void* d_q, size_t q_seq_stride, const void* d_k_new,
                                       const void* d_v_new, size_t kv_new_stride, void* d_k_cache,
                                       void* d_v_cache, size_t cache_seq_stride, const void* d_cos,
                                       const void* d_sin, size_t rope_rows, bool apply_rotation,
                                       const int32_t* d_pos, size_t max_kv_len, void* d_out,
                                       size_t out_seq_stride, size_t num_seqs, size_t num_heads,
                                       size_t num_kv_heads, size_t head_dim, void* d_workspace,
                                       size_t workspace_bytes, b2_stream_t stream);

/* ---- Attention output projection (the path's consumer) ---------------------
 * include/kernels/kernels.hpp:168-177 launch_attention_out_projection
 * (src/kernels/attention_out_projection.hip.cpp:8-58): out[t][n] =
 * sum_k in[t][k] * w[n][k] + beta * out[t][n] for t < seq_len, n <
 * hidden_size, k < num_heads * head_dim; in is the packed attention output
 * [seq][num_heads * head_dim], w the o_proj weights [hidden][num_heads *
 * head_dim] (PyTorch [out, in]), out [seq][hidden] holds the residual on
 * entry (beta = 1: the fused residual add) and is not read when beta = 0.
 * FP16 in and out, FP32 accumulation. hidden a multiple of 256, K a multiple
 * of 64 and 16-byte aligned rows run the tcgen05 GEMM; other shapes a SIMT
 * kernel. seq_len, hidden or K of 0: B2_NOTHING_TO_DO. Adds a stream. */
int b2_launch_attention_out_projection(const void* d_in, void* d_out, const void* d_o_proj_weights,
                                       size_t seq_len, size_t hidden_size, size_t num_heads,
                                       size_t head_dim, float beta, b2_stream_t stream);

/* include/kernels/kernels.hpp:179-188 launch_attention_out_projection_decode
 * (attention_out_projection.hip.cpp:60-71, launch_matrix_vector_mul): the same
 * for one token, a bandwidth-bound GEMV (K a multiple of 256 up to 4096 and
 * aligned rows; otherwise the SIMT kernel). The GEMV reads the weights before
 * waiting for the kernel it follows on the stream (programmatic dependent
 * launch), so the weights must not be written by that kernel. */
int b2_launch_attention_out_projection_decode(const void* d_in, void* d_out, const void* d_o_proj_weights,
                                              size_t hidden_size, size_t num_heads, size_t head_dim,
                                              float beta, b2_stream_t stream);

/* include/kernels/kernels.hpp:29-36 launch_qkv_gemm
 * (src/kernels/qkv_gemm.hip.cpp:7-100): qkv[t][n] = sum_k in[t][k] * w[n][k]
 * for t < seq_len, n < total_qkv_dim, k < hidden_size; in the normed hidden
 * states [seq][hidden], w the fused projection [total_qkv_dim][hidden] (Q, K,
 * V weights stacked, PyTorch [out, in]), qkv [seq][total_qkv_dim] = the
 * [t][Q | K | V] rows. FP16 in and out, FP32 accumulation; the same kernels
 * and shape rules as b2_launch_attention_out_projection with beta 0. Adds a
 * stream (the reference uses the rocBLAS handle's). */
int b2_launch_qkv_gemm(const void* d_input_norm, void* d_qkv_out, const void* d_qkv_weights,
                       size_t seq_len, size_t hidden_size, size_t total_qkv_dim, b2_stream_t stream);

/* include/kernels/kernels.hpp:38-44 launch_qkv_decode
 * (src/kernels/qkv_gemm.hip.cpp:102-115): the same for one token, the GEMV of
 * b2_launch_attention_out_projection_decode (weights read before the
 * dependency wait). */
int b2_launch_qkv_decode(const void* d_input_norm, void* d_qkv_out, const void* d_qkv_weights,
                         size_t hidden_size, size_t total_qkv_dim, b2_stream_t stream);

/* launch_qkv_gemm followed by launch_rope_and_store_kv on its output, the
 * engine's two steps (include/model_inference.hpp:266-281, q/k/v strides
 * total_qkv_dim = (num_heads + 2 * num_kv_heads) * head_dim), in one kernel:
 * the RoPE and the cache append run in the GEMM epilogue on the FP16-rounded
 * products. Afterwards qkv holds rotated Q and K, V as projected (exactly
 * the state the two calls leave), and the caches hold rotated K and V at rows
 * start_pos..start_pos + seq_len - 1; every value is bit-identical to the two
 * calls'. apply_rotary false: a NoPE layer (Q untouched, K stored as is).
 * Fused when seq_len > 1, head_dim is 64, 128 or 256, num_heads * head_dim
 * and num_kv_heads * head_dim are multiples of 256, hidden_size a multiple of
 * 64 and every pointer 16-byte aligned; other shapes (one token among them:
 * the GEMV) run the two launches.
 * seq_len 0: B2_NOTHING_TO_DO. */
int b2_launch_qkv_gemm_rope_store_kv(const void* d_input_norm, void* d_qkv_out, const void* d_qkv_weights,
                                     void* d_k_cache, void* d_v_cache, const void* d_cos, const void* d_sin,
                                     size_t seq_len, size_t hidden_size, size_t num_heads,
                                     size_t num_kv_heads, size_t head_dim, size_t start_pos,
                                     bool apply_rotary, b2_stream_t stream);

/* ---- Decode without a caller workspace ------------------------------------
 * No counterpart in the reference (whose decode launchers always take the
 * three partial arrays). For callers that cannot provide scratch memory: a
 * plugin host that passes only inputs and outputs, a serving process whose
 * memory pool owns all of HBM, a latency-critical thread that must not call
 * cudaMalloc. Same contract and result as b2_launch_causal_attention_decode,
 * but the split partials live in a fixed device array inside the library, of
 * B2_NOALLOC_SCRATCH_BYTES per GPU, held by every GPU that loads the library
 * until the process exits.
 *  - A call is accepted when the reference-sized workspace of the call,
 *    b2_decode_workspace_floats(num_heads, head_dim, kv_cache_len) floats,
 *    fits in the array (num_heads 16, head_dim 128: up to 129,024 cached
 *    tokens); larger calls return B2_ERR_WORKSPACE and launch nothing.
 *  - The call allocates nothing: no cudaMalloc, no cudaFree, no allocating
 *    library routine. The first call on each device looks up the array's
 *    device address (cudaGetSymbolAddress) with that device current; make
 *    that first call before any stream capture. The address is kept per
 *    device together with the id of the context it was read in; after a
 *    context reset (cudaDeviceReset, primary context released) the next
 *    call looks it up again, so it too belongs outside a capture.
 *  - All calls share the one array, which keeps the last call's contents.
 *    Nothing in it needs to start at zero: each call writes every partial
 *    it reads. Calls whose kernels can overlap on the GPU (different streams
 *    without ordering between them) race on the array and give wrong
 *    results; order them on one stream. */
#define B2_NOALLOC_SCRATCH_BYTES (4u * 1024u * 1024u)
int b2_launch_causal_attention_decode_noalloc(const void* d_q, const void* d_k_cache,
                                              const void* d_v_cache, void* d_out,
                                              size_t query_len, size_t kv_cache_len,
                                              size_t num_heads, size_t num_kv_heads,
                                              size_t head_dim, size_t kv_stride,
                                              b2_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* B200ATTN_H */
