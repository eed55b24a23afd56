// Causal GQA prefill: arguments shared by the tcgen05 and SIMT kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace b2 {

struct PrefillArgs {
    const __half* q;
    const __half* k;
    const __half* v;
    __half* out;
    uint64_t q_stride;    // elements between query tokens
    uint64_t kv_stride;   // elements between key/value tokens
    uint64_t out_stride;  // elements between output tokens
    uint64_t q_batch_stride;    // elements between sequences (batched entry)
    uint64_t kv_batch_stride;
    uint64_t out_batch_stride;
    uint32_t seq_len;     // query tokens
    uint32_t start_pos;   // absolute position of query 0; keys [0, start_pos + i]
    uint32_t num_heads;
    uint32_t num_kv_heads;
    uint32_t head_dim;
    uint32_t group;       // num_heads / num_kv_heads
    float scale_log2;     // log2(e) / sqrt(head_dim)
};

// tcgen05 + TMA kernel (head_dim 128, 16-byte aligned rows). Returns
// B2_ERR_UNSUPPORTED for shapes it does not take, without launching.
int launch_prefill_sm100(const PrefillArgs& a, uint32_t batch, cudaStream_t stream);
// SIMT kernel for everything else.
int launch_prefill_simt(const PrefillArgs& a, uint32_t batch, cudaStream_t stream);

}  // namespace b2
