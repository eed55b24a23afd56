// RopeCache for the CUDA build (include/rope_cache.hpp): FP16 cos/sin tables
// [max_seq_len][head_dim/2], computed on the host in FP32 by
// b2_fill_rope_tables and uploaded once.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

#include "b200attn/gpu_utils.hpp"

namespace b200attn {

struct RopeCache {
    __half* d_cos = nullptr;
    __half* d_sin = nullptr;

    RopeCache() = default;
    ~RopeCache() { release(); }
    RopeCache(const RopeCache&) = delete;
    RopeCache& operator=(const RopeCache&) = delete;
    RopeCache(RopeCache&& o) noexcept : d_cos(o.d_cos), d_sin(o.d_sin) { o.d_cos = o.d_sin = nullptr; }
    RopeCache& operator=(RopeCache&& o) noexcept {
        if (this != &o) {
            release();
            d_cos = o.d_cos;
            d_sin = o.d_sin;
            o.d_cos = o.d_sin = nullptr;
        }
        return *this;
    }

  private:
    void release() noexcept {
        if (d_cos) (void)cudaFree(d_cos);
        if (d_sin) (void)cudaFree(d_sin);
        d_cos = d_sin = nullptr;
    }
};

// include/rope_cache.hpp:79-105 create_rope_cache.
inline RopeCache create_rope_cache(size_t max_seq_len, size_t head_dim, float rope_theta) {
    RopeCache cache;
    const size_t total = max_seq_len * (head_dim / 2);
    std::vector<uint16_t> host_cos(total), host_sin(total);
    check(b2_fill_rope_tables(max_seq_len, head_dim, rope_theta, host_cos.data(), host_sin.data()),
          "create_rope_cache");
    B2_CUDA_CHECK(cudaMalloc(&cache.d_cos, total * sizeof(__half)));
    B2_CUDA_CHECK(cudaMalloc(&cache.d_sin, total * sizeof(__half)));
    B2_CUDA_CHECK(cudaMemcpy(cache.d_cos, host_cos.data(), total * sizeof(__half), cudaMemcpyHostToDevice));
    B2_CUDA_CHECK(cudaMemcpy(cache.d_sin, host_sin.data(), total * sizeof(__half), cudaMemcpyHostToDevice));
    return cache;
}

}  // namespace b200attn
