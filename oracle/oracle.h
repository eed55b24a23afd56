/*
 * CPU oracle for the GQA attention hot path -- TEST INFRASTRUCTURE ONLY.
 *
 * This is a plain-C restatement of the reference engine's algorithm
 * (MarcVivas/llm-inference, HIP/C++), used as the checker in tests/, in
 * __graft_entry__.smoke() and as bench.py's timed CPU baseline. It is never
 * the product path: the product is the CUDA library under llm-inference_b200/.
 *
 * FP16 values travel as raw IEEE binary16 bit patterns (uint16_t).
 * Every function names the reference file:line it restates.
 */
#ifndef B2_ORACLE_H
#define B2_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* binary16 <-> binary32 conversions (round to nearest even), the same
 * semantics as __half2float / __float2half in the reference kernels. */
float or_half_to_float(uint16_t h);
uint16_t or_float_to_half(float f);
void or_halves_to_floats(const uint16_t* src, float* dst, size_t n);
void or_floats_to_halves(const float* src, uint16_t* dst, size_t n);

/* include/rope_cache.hpp:49-60 compute_inverse_frequencies */
void or_inverse_frequencies(size_t head_dim, float rope_theta, float* inv_freq);

/* include/rope_cache.hpp:63-76 fill_host_tables: [max_seq_len][head_dim/2] */
void or_fill_rope_tables(size_t max_seq_len, size_t head_dim, float rope_theta,
                         uint16_t* cos_table, uint16_t* sin_table);

/* src/kernels/rope.hip.cpp:61-134 (rope_and_store_kv) and :9-42
 * (copy_to_kv_cache), dispatched as launch_rope_and_store_kv does (:138-196).
 * k_cache == NULL with apply_rotation rotates K in place (launch_rope).
 * Returns 0, or -1 for an argument the reference cannot execute. */
int or_rope_and_store_kv(uint16_t* q, uint16_t* k, const uint16_t* v,
                         uint16_t* k_cache, uint16_t* v_cache,
                         const uint16_t* cos_table, const uint16_t* sin_table,
                         size_t seq_len, size_t num_heads, size_t num_kv_heads,
                         size_t head_dim, size_t q_stride, size_t k_stride,
                         size_t start_pos, int apply_rotation);

/* Causal GQA attention in double precision: the math that
 * src/kernels/causal_attention.hip.cpp:148-372 computes (scale 1/sqrt(d),
 * key > start_pos + query masked), evaluated exactly rather than in tile
 * order. Query token i sits at absolute position start_pos + i and attends
 * keys [0, start_pos + i]. Only the query rows listed in `rows` (or all rows
 * when rows == NULL) are produced; output row r is written at
 * out[r * out_stride + h * head_dim + c] in fp16 (out16) and/or fp32 (out32).
 * Strides are in elements; 0 means packed. */
void or_causal_attention_rows(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                              size_t seq_len, size_t start_pos,
                              size_t num_heads, size_t num_kv_heads, size_t head_dim,
                              size_t q_stride, size_t kv_stride,
                              const int64_t* rows, size_t num_rows,
                              uint16_t* out16, float* out32, size_t out_stride,
                              int num_threads);

/* Flash-decode split stage, src/kernels/causal_attention.hip.cpp:619-716:
 * per (head, chunk of `chunk` tokens) in fp32, m = max s, l = sum e^(s-m),
 * o = sum e^(s-m) v. Layout [num_heads][num_chunks][head_dim] and
 * [num_heads][num_chunks]. Q is one packed [num_heads][head_dim] vector. */
void or_decode_partials(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                        size_t kv_len, size_t num_heads, size_t num_kv_heads,
                        size_t head_dim, size_t kv_stride, size_t chunk,
                        float* partial_o, float* partial_m, float* partial_l,
                        int num_threads);

/* Flash-decode merge, src/kernels/causal_attention.hip.cpp:719-838:
 * M = max m_c, L = sum e^(m_c-M) l_c, out = sum e^(m_c-M) o_c / L. */
void or_merge_partials(const float* partial_o, const float* partial_m,
                       const float* partial_l, size_t num_heads,
                       size_t num_chunks, size_t head_dim,
                       uint16_t* out16, float* out32);

/* Double-precision single-token attention over kv_len cached tokens, the
 * independent CPU softmax of tests/test_causal_attention.cpp:176-196. */
void or_decode_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                         size_t kv_len, size_t num_heads, size_t num_kv_heads,
                         size_t head_dim, size_t kv_stride,
                         uint16_t* out16, float* out32, int num_threads);

#ifdef __cplusplus
}
#endif
#endif
