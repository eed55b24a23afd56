// Causal GQA prefill, SIMT kernel for shapes the tcgen05 kernel does not take
// (head_dim != 128, rows that are not 16-byte aligned). Restates the math of
// src/kernels/causal_attention.hip.cpp:271-374 (scale 1/sqrt(d), keys
// j <= start_pos + i, online softmax, packed fp16 output) with one warp per
// (query row, head): lanes split head_dim, keys are visited in order with a
// running (max, sum) and a rescaled accumulator. Keys above the diagonal are
// never visited (the reference masks them with -inf instead).
#include <math.h>

#include "b2_common.cuh"
#include "prefill.h"

namespace b2 {
namespace {

constexpr int kMaxPerLane = 8;  // head_dim <= 256

__global__ void __launch_bounds__(128) prefill_simt_kernel(const PrefillArgs a) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t i = blockIdx.x * 4 + warp;
    const uint32_t h = blockIdx.y;
    const uint32_t b = blockIdx.z;
    if (i >= a.seq_len) return;
    const uint32_t kvh = h / a.group;
    const uint32_t d = a.head_dim;
    const __half* q = a.q + b * a.q_batch_stride + static_cast<uint64_t>(i) * a.q_stride + static_cast<uint64_t>(h) * d;
    const __half* kb = a.k + b * a.kv_batch_stride + static_cast<uint64_t>(kvh) * d;
    const __half* vb = a.v + b * a.kv_batch_stride + static_cast<uint64_t>(kvh) * d;
    float qv[kMaxPerLane], acc[kMaxPerLane];
#pragma unroll
    for (int r = 0; r < kMaxPerLane; ++r) {
        const uint32_t e = lane + 32 * r;
        qv[r] = e < d ? __half2float(q[e]) * a.scale_log2 : 0.f;
        acc[r] = 0.f;
    }
    float m = -INFINITY, l = 0.f;
    const uint32_t last = a.start_pos + i;  // inclusive
    for (uint32_t j = 0; j <= last; ++j) {
        const __half* kr = kb + static_cast<uint64_t>(j) * a.kv_stride;
        float dot = 0.f;
#pragma unroll
        for (int r = 0; r < kMaxPerLane; ++r) {
            const uint32_t e = lane + 32 * r;
            if (e < d) dot = fmaf(qv[r], __half2float(kr[e]), dot);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
        const float mn = fmaxf(m, dot);
        const float al = exp2f(m - mn);
        const float p = exp2f(dot - mn);
        l = fmaf(l, al, p);
        m = mn;
        const __half* vr = vb + static_cast<uint64_t>(j) * a.kv_stride;
#pragma unroll
        for (int r = 0; r < kMaxPerLane; ++r) {
            const uint32_t e = lane + 32 * r;
            if (e < d) acc[r] = fmaf(acc[r], al, p * __half2float(vr[e]));
        }
    }
    __half* out = a.out + b * a.out_batch_stride + static_cast<uint64_t>(i) * a.out_stride + static_cast<uint64_t>(h) * d;
    const float inv = 1.f / l;
#pragma unroll
    for (int r = 0; r < kMaxPerLane; ++r) {
        const uint32_t e = lane + 32 * r;
        if (e < d) out[e] = __float2half_rn(acc[r] * inv);
    }
}

}  // namespace

int launch_prefill_simt(const PrefillArgs& a, uint32_t batch, cudaStream_t stream) {
    if (a.head_dim > 32 * kMaxPerLane) return B2_ERR_UNSUPPORTED;
    const dim3 grid((a.seq_len + 3) / 4, a.num_heads, batch);
    prefill_simt_kernel<<<grid, 128, 0, stream>>>(a);
    return launch_status();
}

}  // namespace b2
