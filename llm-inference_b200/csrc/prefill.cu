// Prefill entry points: validation and dispatch
// (src/kernels/causal_attention.hip.cpp:376-451 launch_causal_attention_prefill).
#include <math.h>

#include "b2_common.cuh"
#include "prefill.h"

namespace b2 {

static int prefill_common(const void* d_q, const void* d_k, const void* d_v, void* d_out, size_t batch,
                          size_t seq_len, size_t num_heads, size_t num_kv_heads, size_t head_dim, size_t q_stride,
                          size_t kv_stride, size_t out_stride, size_t q_batch_stride, size_t kv_batch_stride,
                          size_t out_batch_stride, cudaStream_t stream) {
    // causal_attention.hip.cpp:392-399: silent no-ops.
    if (batch == 0 || seq_len == 0 || num_kv_heads == 0) return B2_NOTHING_TO_DO;
    if (num_heads % num_kv_heads != 0) return B2_NOTHING_TO_DO;
    if (head_dim == 0) return B2_NOTHING_TO_DO;
    if (!d_q || !d_k || !d_v || !d_out) return B2_ERR_INVALID_ARG;
    if (seq_len > 0x7fffffffull || num_heads > 65535 || batch > 65535 || head_dim > 4096) return B2_ERR_UNSUPPORTED;
    PrefillArgs a{};
    a.q = static_cast<const __half*>(d_q);
    a.k = static_cast<const __half*>(d_k);
    a.v = static_cast<const __half*>(d_v);
    a.out = static_cast<__half*>(d_out);
    a.q_stride = q_stride ? q_stride : num_heads * head_dim;
    a.kv_stride = kv_stride ? kv_stride : num_kv_heads * head_dim;
    a.out_stride = out_stride ? out_stride : num_heads * head_dim;  // packed as the reference (:370)
    if (a.out_stride < num_heads * head_dim) return B2_ERR_INVALID_ARG;
    a.q_batch_stride = q_batch_stride;
    a.kv_batch_stride = kv_batch_stride;
    a.out_batch_stride = out_batch_stride;
    a.seq_len = static_cast<uint32_t>(seq_len);
    a.start_pos = 0;
    a.num_heads = static_cast<uint32_t>(num_heads);
    a.num_kv_heads = static_cast<uint32_t>(num_kv_heads);
    a.head_dim = static_cast<uint32_t>(head_dim);
    a.group = static_cast<uint32_t>(num_heads / num_kv_heads);
    a.scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(head_dim));
    const int st = launch_prefill_sm100(a, static_cast<uint32_t>(batch), stream);
    if (st != B2_ERR_UNSUPPORTED) return st;
    return launch_prefill_simt(a, static_cast<uint32_t>(batch), stream);
}

}  // namespace b2

extern "C" int b2_launch_causal_attention_prefill(const void* d_q, const void* d_k, const void* d_v, void* d_out,
                                                  size_t seq_len, size_t num_heads, size_t num_kv_heads,
                                                  size_t head_dim, size_t q_stride, size_t kv_stride,
                                                  b2_stream_t stream) {
    return b2::prefill_common(d_q, d_k, d_v, d_out, 1, seq_len, num_heads, num_kv_heads, head_dim, q_stride,
                              kv_stride, 0, 0, 0, 0, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int b2_launch_causal_attention_prefill_batched(const void* d_q, const void* d_k, const void* d_v,
                                                          void* d_out, size_t batch, size_t seq_len,
                                                          size_t num_heads, size_t num_kv_heads, size_t head_dim,
                                                          size_t q_stride, size_t kv_stride, size_t out_stride,
                                                          size_t q_batch_stride, size_t kv_batch_stride,
                                                          size_t out_batch_stride, b2_stream_t stream) {
    if (batch > 1 && (q_batch_stride == 0 || kv_batch_stride == 0 || out_batch_stride == 0))
        return B2_ERR_INVALID_ARG;
    return b2::prefill_common(d_q, d_k, d_v, d_out, batch, seq_len, num_heads, num_kv_heads, head_dim, q_stride,
                              kv_stride, out_stride, q_batch_stride, kv_batch_stride, out_batch_stride,
                              reinterpret_cast<cudaStream_t>(stream));
}
