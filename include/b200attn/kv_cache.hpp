// KVCache for the CUDA build: include/kv_cache.hpp's layout unchanged.
// One allocation of 2 * num_layers * max_seq_len * kv_dim halves; layer l's K
// at base + l * 2 * max_seq_len * kv_dim, its V max_seq_len * kv_dim later;
// row t = token t, [t][kv_head][head_dim].
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <stdexcept>
#include <string>

#include "b200attn/gpu_utils.hpp"

namespace b200attn {

struct KVCacheShape {
    size_t num_layers;
    size_t max_seq_len;
    size_t num_kv_heads;
    size_t head_dim;
};

class KVCache {
    __half* d_kv_buffer = nullptr;
    KVCacheShape shape;
    size_t current_cache_len = 0;

  public:
    explicit KVCache(const KVCacheShape& s) : shape(s) {
        B2_CUDA_CHECK(cudaMalloc(&d_kv_buffer, compute_total_bytes()));
    }
    ~KVCache() {
        if (d_kv_buffer) (void)cudaFree(d_kv_buffer);
    }
    KVCache(const KVCache&) = delete;
    KVCache& operator=(const KVCache&) = delete;
    KVCache(KVCache&& o) noexcept
        : d_kv_buffer(o.d_kv_buffer), shape(o.shape), current_cache_len(o.current_cache_len) {
        o.d_kv_buffer = nullptr;
        o.current_cache_len = 0;
    }
    KVCache& operator=(KVCache&&) = delete;

    [[nodiscard]] __half* get_k_cache(size_t layer_idx) noexcept { return d_kv_buffer + layer_idx * layer_stride(); }
    [[nodiscard]] const __half* get_k_cache(size_t layer_idx) const noexcept {
        return d_kv_buffer + layer_idx * layer_stride();
    }
    [[nodiscard]] __half* get_v_cache(size_t layer_idx) noexcept {
        return d_kv_buffer + layer_idx * layer_stride() + shape.max_seq_len * kv_dim();
    }
    [[nodiscard]] const __half* get_v_cache(size_t layer_idx) const noexcept {
        return d_kv_buffer + layer_idx * layer_stride() + shape.max_seq_len * kv_dim();
    }
    size_t get_cached_len() const noexcept { return current_cache_len; }
    void set_cached_len(size_t cached_len) {
        if (cached_len > shape.max_seq_len)
            throw std::out_of_range("KV cache capacity exceeded: requested " + std::to_string(cached_len) +
                                    " tokens, capacity " + std::to_string(shape.max_seq_len));
        current_cache_len = cached_len;
    }
    void reset_cache() { current_cache_len = 0; }

    size_t kv_dim() const noexcept { return shape.num_kv_heads * shape.head_dim; }
    size_t layer_stride() const noexcept { return 2 * kv_dim() * shape.max_seq_len; }

  private:
    size_t compute_total_bytes() const { return 2 * kv_dim() * shape.max_seq_len * sizeof(__half) * shape.num_layers; }
};

}  // namespace b200attn
