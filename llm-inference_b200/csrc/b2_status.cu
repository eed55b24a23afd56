// Status strings, error bookkeeping, launch counter, graph-node helpers and
// the host-side RoPE table (include/rope_cache.hpp:49-76).
#include <atomic>
#include <cmath>
#include <vector>

#include "b2_common.cuh"

namespace b2 {

static std::atomic<int> g_last_cuda_error{0};
static std::atomic<uint64_t> g_launches{0};

void note_cuda_error(cudaError_t e) { g_last_cuda_error.store(static_cast<int>(e)); }
void count_launch(uint64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

int last_captured_node(cudaStream_t stream, cudaGraphNode_t* node) {
    cudaStreamCaptureStatus status = cudaStreamCaptureStatusNone;
    const cudaGraphNode_t* deps = nullptr;
    size_t count = 0;
    const cudaError_t e = cudaStreamGetCaptureInfo(stream, &status, nullptr, nullptr, &deps, &count);
    if (e != cudaSuccess) {
        note_cuda_error(e);
        return B2_ERR_CUDA;
    }
    if (status != cudaStreamCaptureStatusActive || count != 1) return B2_ERR_GRAPH;
    *node = deps[0];
    return B2_OK;
}

int node_kernel_params(cudaGraphNode_t node, const void* const* expected, int n_expected,
                       cudaKernelNodeParams* params) {
    if (node == nullptr) return B2_ERR_INVALID_ARG;
    const cudaError_t e = cudaGraphKernelNodeGetParams(node, params);
    if (e != cudaSuccess) {
        note_cuda_error(e);
        return B2_ERR_CUDA;
    }
    for (int i = 0; i < n_expected; ++i)
        if (params->func == expected[i]) return B2_OK;
    return B2_ERR_GRAPH;
}

}  // namespace b2

extern "C" {

int b2_kv_chunk(void) { return 256; }

size_t b2_decode_workspace_floats(size_t num_heads, size_t head_dim, size_t max_kv_len) {
    const size_t chunk = static_cast<size_t>(b2_kv_chunk());
    const size_t chunks = (max_kv_len + chunk - 1) / chunk;
    return num_heads * chunks * (head_dim + 2);
}

const char* b2_status_string(int status) {
    switch (status) {
        case B2_OK: return "ok";
        case B2_NOTHING_TO_DO: return "nothing to do (skipped as the reference does)";
        case B2_ERR_INVALID_ARG: return "invalid argument";
        case B2_ERR_UNSUPPORTED: return "unsupported shape";
        case B2_ERR_ALIGNMENT: return "misaligned pointer or stride";
        case B2_ERR_CUDA: return "CUDA runtime error";
        case B2_ERR_WORKSPACE: return "workspace too small";
        case B2_ERR_GRAPH: return "graph capture / node error";
        default: return "unknown status";
    }
}

int b2_last_cuda_error(void) { return b2::g_last_cuda_error.load(); }

uint64_t b2_kernel_launch_count(void) { return b2::g_launches.load(); }

unsigned int b2_device_error_word(void) {
    return b2::device_error_decode() | b2::device_error_prefill() | b2::device_error_ragged() |
           b2::device_error_proj();
}

int b2_clear_device_error_word(void) {
    int st = b2::clear_device_error_decode();
    if (st == B2_OK) st = b2::clear_device_error_prefill();
    if (st == B2_OK) st = b2::clear_device_error_ragged();
    return st != B2_OK ? st : b2::clear_device_error_proj();
}

int b2_fill_rope_tables(size_t max_seq_len, size_t head_dim, float rope_theta,
                        uint16_t* host_cos, uint16_t* host_sin) {
    if (head_dim == 0 || (head_dim & 1) || host_cos == nullptr || host_sin == nullptr)
        return B2_ERR_INVALID_ARG;
    const size_t half_dim = head_dim / 2;
    std::vector<float> inv_freq(half_dim);
    for (size_t i = 0; i < half_dim; ++i) {
        const float exponent = static_cast<float>(2 * i) / static_cast<float>(head_dim);
        inv_freq[i] = 1.0f / std::pow(rope_theta, exponent);
    }
    for (size_t pos = 0; pos < max_seq_len; ++pos) {
        for (size_t i = 0; i < half_dim; ++i) {
            const float angle = static_cast<float>(pos) * inv_freq[i];
            const __half c = __float2half_rn(std::cos(angle));
            const __half s = __float2half_rn(std::sin(angle));
            host_cos[pos * half_dim + i] = *reinterpret_cast<const uint16_t*>(&c);
            host_sin[pos * half_dim + i] = *reinterpret_cast<const uint16_t*>(&s);
        }
    }
    return B2_OK;
}

}  // extern "C"
