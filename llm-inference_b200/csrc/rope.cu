// RoPE + FP16 KV-cache append for sm_100a.
//
// Restates src/kernels/rope.hip.cpp of the reference:
//   rope_and_store_kv (:61-134)  rotate-half Q in place, rotated K + verbatim
//                                V into cache row start_pos + t
//   copy_to_kv_cache  (:9-42)    NoPE layers: K and V copied verbatim
//   launch_*          (:138-205) dispatch, seq_len == 0 -> no-op
//   update_rope_and_store_kv_node (:208-241)
//
// Memory-bound. The reference gives every (token, head) a 64-thread block of
// 2-byte accesses. Here a thread owns eight rotation pairs of one head: it
// reads 2 x 16 B of the head plus 2 x 16 B of the cos/sin row and writes
// 2 x 16 B, so every access is a full 16-byte vector and a warp covers four
// 256-byte head rows. Work items are flattened over (token, slot, lane) with
// slot = Q head | K head | V head, and a grid-stride loop sized to the SM
// count. Rows that are not 16-byte aligned (odd strides) take a scalar
// kernel with the same arithmetic.
//
// Arithmetic is the reference's fp32 x0*c - x1*s / x1*c + x0*s with every
// product and sum rounded separately (__fmul_rn/__fsub_rn: no FMA
// contraction), then round-to-nearest fp16, so results are bit-identical to
// the CPU oracle evaluated the same way.
#include <algorithm>

#include "b2_common.cuh"
#include "b2_ptx.cuh"

namespace b2 {
namespace {

struct RopeArgs {
    __half* q;
    __half* k;
    const __half* v;
    __half* k_cache;
    __half* v_cache;
    const __half* cos;
    const __half* sin;
    uint64_t q_stride;  // elements between tokens
    uint64_t k_stride;  // elements between tokens (K and V)
    uint64_t total_items;
    uint32_t num_heads;
    uint32_t num_kv_heads;
    uint32_t head_dim;
    uint32_t half_dim;
    uint32_t kv_dim;
    uint32_t lanes;      // work lanes per head row
    uint32_t slots;      // head slots per token
    uint32_t start_pos;  // patched by b2_update_rope_and_store_kv_node
    // Graph-static variant: when set, start_pos is read from device memory at
    // launch and tokens at positions >= max_seq_len are skipped.
    const int32_t* start_pos_dev;
    uint32_t max_seq_len;
    // Ragged batch: token t is sequence t's new token, at position
    // pos_per_token[t], appended to the cache that starts cache_seq_stride
    // elements after sequence t-1's.
    const int32_t* pos_per_token;
    uint64_t cache_seq_stride;
};

__device__ __forceinline__ bool resolve_start(const RopeArgs& a, uint32_t& start) {
    if (a.pos_per_token != nullptr) {
        start = 0;
        return true;
    }
    if (a.start_pos_dev == nullptr) {
        start = a.start_pos;
        return true;
    }
    const int32_t s = __ldg(a.start_pos_dev);
    if (s < 0) return false;
    start = static_cast<uint32_t>(s);
    return true;
}

// Position of token t and the element offset of its cache row; false = skip
// the token (graph-static position past the cache, or a ragged position
// outside [0, max_seq_len)).
__device__ __forceinline__ bool token_row(const RopeArgs& a, uint32_t start, uint64_t t, uint64_t& pos,
                                          uint64_t& crow) {
    if (a.pos_per_token != nullptr) {
        const int32_t p = __ldg(a.pos_per_token + t);
        if (p < 0 || static_cast<uint32_t>(p) >= a.max_seq_len) return false;
        pos = static_cast<uint64_t>(p);
        crow = t * a.cache_seq_stride + pos * a.kv_dim;
        return true;
    }
    pos = static_cast<uint64_t>(start) + t;
    if (a.start_pos_dev && pos >= a.max_seq_len) return false;
    crow = pos * a.kv_dim;
    return true;
}

__device__ __forceinline__ void rot2(float x0, float x1, float c, float s, float& o0, float& o1) {
    o0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    o1 = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, s));
}

// Vectorised rotate (+ store) kernel: lanes = half_dim / 8.
__global__ void __launch_bounds__(256) rope_store_vec8_kernel(const RopeArgs a) {
    pdl_wait_primary();
    pdl_launch_dependents();
    uint32_t start;
    if (!resolve_start(a, start)) return;
    const uint64_t per_token = static_cast<uint64_t>(a.slots) * a.lanes;
    for (uint64_t id = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; id < a.total_items;
         id += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint64_t t = id / per_token;
        const uint32_t r = static_cast<uint32_t>(id - t * per_token);
        const uint32_t slot = r / a.lanes;
        const uint32_t e = (r - slot * a.lanes) * 8;
        uint64_t pos, crow;
        if (!token_row(a, start, t, pos, crow)) continue;
        if (slot < a.num_heads + a.num_kv_heads) {
            __half* src;
            __half* dst;
            if (slot < a.num_heads) {
                src = a.q + t * a.q_stride + static_cast<uint64_t>(slot) * a.head_dim;
                dst = src;
            } else {
                const uint32_t j = slot - a.num_heads;
                src = a.k + t * a.k_stride + static_cast<uint64_t>(j) * a.head_dim;
                dst = a.k_cache ? a.k_cache + crow + static_cast<uint64_t>(j) * a.head_dim : src;
            }
            uint4 lo = *reinterpret_cast<const uint4*>(src + e);
            uint4 hi = *reinterpret_cast<const uint4*>(src + a.half_dim + e);
            const uint4 cv = __ldg(reinterpret_cast<const uint4*>(a.cos + pos * a.half_dim + e));
            const uint4 sv = __ldg(reinterpret_cast<const uint4*>(a.sin + pos * a.half_dim + e));
            rot8_pairs(lo, hi, cv, sv);
            *reinterpret_cast<uint4*>(dst + e) = lo;
            *reinterpret_cast<uint4*>(dst + a.half_dim + e) = hi;
        } else {
            const uint32_t j = slot - a.num_heads - a.num_kv_heads;
            const __half* src = a.v + t * a.k_stride + static_cast<uint64_t>(j) * a.head_dim;
            __half* dst = a.v_cache + crow + static_cast<uint64_t>(j) * a.head_dim;
            const uint4 lo = *reinterpret_cast<const uint4*>(src + e);
            const uint4 hi = *reinterpret_cast<const uint4*>(src + a.half_dim + e);
            *reinterpret_cast<uint4*>(dst + e) = lo;
            *reinterpret_cast<uint4*>(dst + a.half_dim + e) = hi;
        }
    }
}

// Scalar rotate (+ store) kernel: lanes = half_dim, any stride / alignment.
__global__ void __launch_bounds__(256) rope_store_scalar_kernel(const RopeArgs a) {
    pdl_wait_primary();
    pdl_launch_dependents();
    uint32_t start;
    if (!resolve_start(a, start)) return;
    const uint64_t per_token = static_cast<uint64_t>(a.slots) * a.lanes;
    for (uint64_t id = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; id < a.total_items;
         id += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint64_t t = id / per_token;
        const uint32_t r = static_cast<uint32_t>(id - t * per_token);
        const uint32_t slot = r / a.lanes;
        const uint32_t i = r - slot * a.lanes;
        uint64_t pos, crow;
        if (!token_row(a, start, t, pos, crow)) continue;
        if (slot < a.num_heads + a.num_kv_heads) {
            __half* src;
            __half* dst;
            if (slot < a.num_heads) {
                src = a.q + t * a.q_stride + static_cast<uint64_t>(slot) * a.head_dim;
                dst = src;
            } else {
                const uint32_t j = slot - a.num_heads;
                src = a.k + t * a.k_stride + static_cast<uint64_t>(j) * a.head_dim;
                dst = a.k_cache ? a.k_cache + crow + static_cast<uint64_t>(j) * a.head_dim : src;
            }
            const float x0 = __half2float(src[i]);
            const float x1 = __half2float(src[i + a.half_dim]);
            const float c = __half2float(a.cos[pos * a.half_dim + i]);
            const float s = __half2float(a.sin[pos * a.half_dim + i]);
            float o0, o1;
            rot2(x0, x1, c, s, o0, o1);
            dst[i] = __float2half_rn(o0);
            dst[i + a.half_dim] = __float2half_rn(o1);
        } else {
            const uint32_t j = slot - a.num_heads - a.num_kv_heads;
            const __half* src = a.v + t * a.k_stride + static_cast<uint64_t>(j) * a.head_dim;
            __half* dst = a.v_cache + crow + static_cast<uint64_t>(j) * a.head_dim;
            dst[i] = src[i];
            dst[i + a.half_dim] = src[i + a.half_dim];
        }
    }
}

// NoPE append: K and V rows copied verbatim. lanes = kv_dim / 8 (vec8) or
// kv_dim (scalar); slots = 2 (K, V).
__global__ void __launch_bounds__(256) kv_copy_vec8_kernel(const RopeArgs a) {
    pdl_wait_primary();
    pdl_launch_dependents();
    uint32_t start;
    if (!resolve_start(a, start)) return;
    const uint64_t per_token = 2ull * a.lanes;
    for (uint64_t id = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; id < a.total_items;
         id += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint64_t t = id / per_token;
        const uint32_t r = static_cast<uint32_t>(id - t * per_token);
        const bool is_v = r >= a.lanes;
        const uint32_t e = (is_v ? r - a.lanes : r) * 8;
        const __half* src = (is_v ? a.v : a.k) + t * a.k_stride + e;
        uint64_t pos, crow;
        if (!token_row(a, start, t, pos, crow)) continue;
        __half* dst = (is_v ? a.v_cache : a.k_cache) + crow + e;
        *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
    }
}

__global__ void __launch_bounds__(256) kv_copy_scalar_kernel(const RopeArgs a) {
    pdl_wait_primary();
    pdl_launch_dependents();
    uint32_t start;
    if (!resolve_start(a, start)) return;
    const uint64_t per_token = 2ull * a.lanes;
    for (uint64_t id = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; id < a.total_items;
         id += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint64_t t = id / per_token;
        const uint32_t r = static_cast<uint32_t>(id - t * per_token);
        const bool is_v = r >= a.lanes;
        const uint32_t e = is_v ? r - a.lanes : r;
        const __half* src = (is_v ? a.v : a.k) + t * a.k_stride + e;
        uint64_t pos, crow;
        if (!token_row(a, start, t, pos, crow)) continue;
        __half* dst = (is_v ? a.v_cache : a.k_cache) + crow + e;
        *dst = *src;
    }
}

int sm_count() {
    static int count = [] {
        int dev = 0, n = 148;
        if (cudaGetDevice(&dev) == cudaSuccess)
            cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        return n > 0 ? n : 148;
    }();
    return count;
}

const void* const kRopeKernels[] = {
    reinterpret_cast<const void*>(rope_store_vec8_kernel),
    reinterpret_cast<const void*>(rope_store_scalar_kernel),
};
const void* const kCopyKernels[] = {
    reinterpret_cast<const void*>(kv_copy_vec8_kernel),
    reinterpret_cast<const void*>(kv_copy_scalar_kernel),
};

}  // namespace
}  // namespace b2

using namespace b2;

namespace b2 {
namespace {

int launch_rope_impl(void* d_q, void* d_k, const void* d_v, void* d_k_cache, void* d_v_cache, const void* d_cos,
                     const void* d_sin, size_t seq_len, size_t num_heads, size_t num_kv_heads, size_t head_dim,
                     size_t q_stride, size_t k_stride, size_t start_pos, const int32_t* start_pos_dev,
                     size_t max_seq_len, bool apply_rotation, b2_stream_t stream_handle,
                     const int32_t* pos_per_token = nullptr, size_t cache_seq_stride = 0) {
    if (seq_len == 0) return B2_NOTHING_TO_DO;  // rope.hip.cpp:156
    if (head_dim == 0 || (head_dim & 1) || d_k == nullptr) return B2_ERR_INVALID_ARG;
    if (num_kv_heads == 0 && num_heads == 0) return B2_NOTHING_TO_DO;
    const size_t kv_dim = num_kv_heads * head_dim;
    if (q_stride == 0) q_stride = num_heads * head_dim;
    if (k_stride == 0) k_stride = kv_dim;
    if (start_pos + seq_len > 0xffffffffull || head_dim > 0xffffu * 2 || num_heads > 0xffffu ||
        num_kv_heads > 0xffffu)
        return B2_ERR_UNSUPPORTED;
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_handle);
    const bool store = d_k_cache != nullptr;
    if (store && (d_v_cache == nullptr || d_v == nullptr)) return B2_ERR_INVALID_ARG;

    RopeArgs a{};
    a.q = static_cast<__half*>(d_q);
    a.k = static_cast<__half*>(d_k);
    a.v = static_cast<const __half*>(d_v);
    a.k_cache = static_cast<__half*>(d_k_cache);
    a.v_cache = static_cast<__half*>(d_v_cache);
    a.cos = static_cast<const __half*>(d_cos);
    a.sin = static_cast<const __half*>(d_sin);
    a.q_stride = q_stride;
    a.k_stride = k_stride;
    a.num_heads = static_cast<uint32_t>(num_heads);
    a.num_kv_heads = static_cast<uint32_t>(num_kv_heads);
    a.head_dim = static_cast<uint32_t>(head_dim);
    a.half_dim = static_cast<uint32_t>(head_dim / 2);
    a.kv_dim = static_cast<uint32_t>(kv_dim);
    a.start_pos = static_cast<uint32_t>(start_pos);
    a.start_pos_dev = start_pos_dev;
    a.max_seq_len = static_cast<uint32_t>(max_seq_len > 0xffffffffull ? 0xffffffffull : max_seq_len);
    a.pos_per_token = pos_per_token;
    a.cache_seq_stride = cache_seq_stride;

    const bool rows16 = (k_stride % 8 == 0) && (cache_seq_stride % 8 == 0) && aligned16(d_k) &&
                        (!store || (aligned16(d_v) && aligned16(d_k_cache) && aligned16(d_v_cache)));
    if (apply_rotation) {
        if (d_cos == nullptr || d_sin == nullptr || (num_heads && d_q == nullptr)) return B2_ERR_INVALID_ARG;
        const bool vec = (a.half_dim % 8 == 0) && rows16 && (num_heads == 0 || (q_stride % 8 == 0 && aligned16(d_q))) &&
                         aligned16(d_cos) && aligned16(d_sin);
        a.lanes = vec ? a.half_dim / 8 : a.half_dim;
        a.slots = a.num_heads + a.num_kv_heads + (store ? a.num_kv_heads : 0);
        a.total_items = static_cast<uint64_t>(seq_len) * a.slots * a.lanes;
        const int blocks = static_cast<int>(std::min<uint64_t>((a.total_items + 255) / 256, 16ull * sm_count()));
        if (vec)
            return launch_pdl(rope_store_vec8_kernel, dim3(blocks), dim3(256), 0, stream, a);
        else
            return launch_pdl(rope_store_scalar_kernel, dim3(blocks), dim3(256), 0, stream, a);
    }
    // NoPE: copy_to_kv_cache (rope.hip.cpp:181-195). A cache is required.
    if (!store) return B2_ERR_INVALID_ARG;
    const bool vec = (kv_dim % 8 == 0) && rows16;
    a.lanes = vec ? a.kv_dim / 8 : a.kv_dim;
    a.slots = 2;
    a.total_items = static_cast<uint64_t>(seq_len) * 2 * a.lanes;
    const int blocks = static_cast<int>(std::min<uint64_t>((a.total_items + 255) / 256, 16ull * sm_count()));
    if (vec)
        return launch_pdl(kv_copy_vec8_kernel, dim3(blocks), dim3(256), 0, stream, a);
    else
        return launch_pdl(kv_copy_scalar_kernel, dim3(blocks), dim3(256), 0, stream, a);
}

}  // namespace
}  // namespace b2

extern "C" int b2_launch_rope_and_store_kv(void* d_q, void* d_k, const void* d_v, void* d_k_cache,
                                           void* d_v_cache, const void* d_cos, const void* d_sin,
                                           size_t seq_len, size_t num_heads, size_t num_kv_heads,
                                           size_t head_dim, size_t q_stride, size_t k_stride,
                                           size_t start_pos, bool apply_rotation,
                                           b2_stream_t stream_handle) {
    return launch_rope_impl(d_q, d_k, d_v, d_k_cache, d_v_cache, d_cos, d_sin, seq_len, num_heads, num_kv_heads,
                            head_dim, q_stride, k_stride, start_pos, nullptr, 0, apply_rotation, stream_handle);
}

extern "C" int b2_launch_rope_and_store_kv_devpos(void* d_q, void* d_k, const void* d_v, void* d_k_cache,
                                                  void* d_v_cache, const void* d_cos, const void* d_sin,
                                                  size_t seq_len, size_t num_heads, size_t num_kv_heads,
                                                  size_t head_dim, size_t q_stride, size_t k_stride,
                                                  const int32_t* d_start_pos, size_t max_seq_len,
                                                  bool apply_rotation, b2_stream_t stream_handle) {
    if (d_start_pos == nullptr || max_seq_len == 0) return B2_ERR_INVALID_ARG;
    return launch_rope_impl(d_q, d_k, d_v, d_k_cache, d_v_cache, d_cos, d_sin, seq_len, num_heads, num_kv_heads,
                            head_dim, q_stride, k_stride, 0, d_start_pos, max_seq_len, apply_rotation,
                            stream_handle);
}

extern "C" int b2_launch_rope_and_store_kv_ragged(void* d_q, void* d_k, const void* d_v, void* d_k_cache,
                                                  void* d_v_cache, size_t cache_seq_stride, const void* d_cos,
                                                  const void* d_sin, size_t num_seqs, size_t num_heads,
                                                  size_t num_kv_heads, size_t head_dim, size_t q_stride,
                                                  size_t k_stride, const int32_t* d_pos, size_t max_seq_len,
                                                  bool apply_rotation, b2_stream_t stream_handle) {
    if (d_pos == nullptr || max_seq_len == 0) return B2_ERR_INVALID_ARG;
    if (d_k_cache != nullptr && num_seqs > 1 && cache_seq_stride < max_seq_len * num_kv_heads * head_dim)
        return B2_ERR_INVALID_ARG;  // the sequences' caches would overlap
    return launch_rope_impl(d_q, d_k, d_v, d_k_cache, d_v_cache, d_cos, d_sin, num_seqs, num_heads, num_kv_heads,
                            head_dim, q_stride, k_stride, 0, nullptr, max_seq_len, apply_rotation, stream_handle,
                            d_pos, cache_seq_stride);
}

extern "C" int b2_launch_rope(void* d_q, void* d_k, const void* d_cos, const void* d_sin, size_t seq_len,
                              size_t num_heads, size_t num_kv_heads, size_t head_dim, size_t q_stride,
                              size_t k_stride, size_t start_pos, b2_stream_t stream) {
    return b2_launch_rope_and_store_kv(d_q, d_k, nullptr, nullptr, nullptr, d_cos, d_sin, seq_len, num_heads,
                                       num_kv_heads, head_dim, q_stride, k_stride, start_pos, true, stream);
}

extern "C" int b2_update_rope_and_store_kv_node(b2_graph_exec_t graph_exec, b2_graph_node_t node_handle,
                                                size_t start_pos, bool apply_rotation) {
    if (graph_exec == nullptr) return B2_ERR_INVALID_ARG;
    if (start_pos > 0xffffffffull) return B2_ERR_UNSUPPORTED;
    cudaGraphNode_t node = reinterpret_cast<cudaGraphNode_t>(node_handle);
    cudaKernelNodeParams params{};
    const int st = apply_rotation ? node_kernel_params(node, kRopeKernels, 2, &params)
                                  : node_kernel_params(node, kCopyKernels, 2, &params);
    if (st != B2_OK) return st;
    RopeArgs a = *static_cast<const RopeArgs*>(params.kernelParams[0]);
    a.start_pos = static_cast<uint32_t>(start_pos);
    void* args[1] = {&a};
    params.kernelParams = args;
    params.extra = nullptr;
    return cuda_status(cudaGraphExecKernelNodeSetParams(reinterpret_cast<cudaGraphExec_t>(graph_exec), node, &params));
}
