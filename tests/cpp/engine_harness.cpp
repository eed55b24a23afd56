// A C++ host for the attention path -- TEST INFRASTRUCTURE.
//
// Drives libb200attn.so only through the drop-in header the reference engine
// includes (include/kernels/kernels.hpp, with include/b200attn/kv_cache.hpp and
// rope_cache.hpp standing in for include/kv_cache.hpp and rope_cache.hpp), the
// way the reference drives its own kernels:
//
//   engine <inputs.bin> <outputs.bin>
//       The per-layer call sequence of include/model_inference.hpp: prefill
//       (:272-292) -- launch_rope_and_store_kv in place on [Q|K|V] rows of
//       stride 3072, then launch_causal_attention_prefill from the cache,
//       NoPE on every 4th layer -- and decode (:96-123, :358-388): the first
//       token's layers captured into one CUDA graph with last_captured_node
//       and the attention / merge nodes, later tokens replayed after
//       update_rope_and_store_kv_node, update_causal_attention_decode_node and
//       update_merge_attention_decode_node. Inputs and outputs are raw files
//       the pytest driver writes and checks against the CPU oracle.
//   known-answer
//       tests/test_causal_attention.cpp:152-228 restated: deterministic sin /
//       cos inputs, double-precision CPU softmax, guard elements, tolerance
//       2e-3, over head_dim {32, 128} x KV heads {1, 2, 4} x lengths around
//       KV_CHUNK x packed / padded rows.
//   golden <dir>
//       tests/test_causal_attention.cpp:15-78 and :80-150 on the committed
//       layer-0 fixtures: prefill from a cache with populated spare rows, and
//       decode at every position (packed and interleaved Q) against the
//       fixture's prefill rows, with output guards, tolerance 2e-2.
//   qkv <inputs.bin> <outputs.bin>
//       The engine's QKV step (include/model_inference.hpp:266-281):
//       launch_qkv_gemm into [Q|K|V] rows, then launch_rope_and_store_kv on
//       them into the cache, next to launch_qkv_gemm_rope_store_kv doing both
//       in one kernel on separate buffers; the two results must agree bit for
//       bit (rows and cache rows), and the fused one is written out for the
//       pytest driver to check against the CPU oracle.
//   weights <weights.bin> <chunk_bytes>
//       include/b200attn/weights.hpp on a file the reference's exporter
//       wrote: header, tokenizer JSON, pipelined upload (small chunks to run
//       the two staging buffers many times), then every carved tensor copied
//       back; prints one JSON line per tensor (name, elements, float64 sum
//       and sum of squares, first values) for the pytest driver to check.
//
// Exit status 0 when every check passed; failures are printed.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <format>
#include <fstream>
#include <span>
#include <stdexcept>
#include <string>
#include <vector>

#include "b200attn/kv_cache.hpp"
#include "b200attn/rope_cache.hpp"
#include "b200attn/weights.hpp"
#include "kernels/kernels.hpp"

using b200attn::KVCache;
using b200attn::last_captured_node;

namespace {

int g_failures = 0;

void fail(const std::string& what) {
    ++g_failures;
    if (g_failures <= 20) std::fputs(("FAIL " + what + "\n").c_str(), stderr);
}

// tests/test_utils.hpp:30-62: |a - e| <= atol + rtol |e| for every element.
size_t count_mismatches(std::span<const __half> actual, std::span<const __half> expected, float atol, float rtol,
                        float* max_diff = nullptr) {
    size_t bad = 0;
    float worst = 0.f;
    for (size_t i = 0; i < actual.size(); ++i) {
        const float a = __half2float(actual[i]), e = __half2float(expected[i]);
        const float d = std::fabs(a - e);
        worst = std::max(worst, d);
        if (!(d <= atol + rtol * std::fabs(e))) ++bad;
    }
    if (max_diff) *max_diff = worst;
    return bad;
}

bool all_finite(std::span<const __half> x) {
    return std::all_of(x.begin(), x.end(), [](__half h) { return std::isfinite(__half2float(h)); });
}

template <class T>
std::vector<T> read_file(const std::string& path) {
    std::ifstream f(path, std::ios::binary | std::ios::ate);
    if (!f) throw std::runtime_error("cannot open " + path);
    const auto bytes = static_cast<size_t>(f.tellg());
    std::vector<T> v(bytes / sizeof(T));
    f.seekg(0);
    f.read(reinterpret_cast<char*>(v.data()), static_cast<std::streamsize>(v.size() * sizeof(T)));
    return v;
}

template <class T>
T* device_copy(const std::vector<T>& h) {
    T* d = nullptr;
    B2_CUDA_CHECK(cudaMalloc(&d, h.size() * sizeof(T)));
    B2_CUDA_CHECK(cudaMemcpy(d, h.data(), h.size() * sizeof(T), cudaMemcpyHostToDevice));
    return d;
}

// ------------------------------------------------------------------ engine
struct DecodeLayerNodes {
    cudaGraphNode_t store_kv = nullptr;
    cudaGraphNode_t attention = nullptr;
    cudaGraphNode_t merge = nullptr;
};

int run_engine(const std::string& in_path, const std::string& out_path) {
    const auto in = read_file<uint16_t>(in_path);
    if (in.size() < 32) throw std::runtime_error("short input file");
    uint64_t hdr[8];
    std::memcpy(hdr, in.data(), sizeof(hdr));
    if (hdr[0] != 0x62323030656e67ull) throw std::runtime_error("bad input magic");
    const size_t L = hdr[1], S = hdr[2], T = hdr[3], H = hdr[4], KVH = hdr[5], d = hdr[6], max_seq = hdr[7];
    const size_t q_dim = H * d, kv_dim = KVH * d, total = q_dim + 2 * kv_dim;
    if (S + T > max_seq) throw std::runtime_error("prompt + decode tokens exceed max_seq");
    const __half* prompt = reinterpret_cast<const __half*>(in.data() + 32);  // [L][S][total]
    const __half* news = prompt + L * S * total;                              // [T][L][total]
    if (in.size() != 32 + L * S * total + T * L * total) throw std::runtime_error("input size mismatch");

    KVCache kv_cache({L, max_seq, KVH, d});
    const b200attn::RopeCache rope = b200attn::create_rope_cache(max_seq, d, 5.0e6f);
    __half *d_scratch_a = nullptr, *d_scratch_b = nullptr, *d_rows = nullptr, *d_dec_out = nullptr;
    B2_CUDA_CHECK(cudaMalloc(&d_scratch_a, max_seq * total * sizeof(__half)));
    B2_CUDA_CHECK(cudaMalloc(&d_scratch_b, max_seq * q_dim * sizeof(__half)));
    B2_CUDA_CHECK(cudaMalloc(&d_rows, L * total * sizeof(__half)));
    B2_CUDA_CHECK(cudaMalloc(&d_dec_out, L * q_dim * sizeof(__half)));
    // decode partials sized as include/model_inference.hpp:192-198 does
    const size_t chunk_capacity = (max_seq + KV_CHUNK - 1) / KV_CHUNK;
    const size_t partial_count = H * chunk_capacity;
    float *d_partial_output = nullptr, *d_partial_max = nullptr, *d_partial_weight_sum = nullptr;
    B2_CUDA_CHECK(cudaMalloc(&d_partial_output, partial_count * d * sizeof(float)));
    B2_CUDA_CHECK(cudaMalloc(&d_partial_max, partial_count * sizeof(float)));
    B2_CUDA_CHECK(cudaMalloc(&d_partial_weight_sum, partial_count * sizeof(float)));

    std::vector<__half> prefill_out(L * S * q_dim), decode_out(T * L * q_dim);

    // ---- prefill, layer by layer, on the default stream
    for (size_t layer = 0; layer < L; ++layer) {
        B2_CUDA_CHECK(cudaMemcpy(d_scratch_a, prompt + layer * S * total, S * total * sizeof(__half),
                                 cudaMemcpyHostToDevice));
        const bool apply_rotation = (layer + 1) % 4 != 0;
        launch_rope_and_store_kv(d_scratch_a, d_scratch_a + q_dim, d_scratch_a + q_dim + kv_dim,
                                 kv_cache.get_k_cache(layer), kv_cache.get_v_cache(layer), rope.d_cos, rope.d_sin, S,
                                 H, KVH, d, total, total, 0, apply_rotation);
        launch_causal_attention_prefill(d_scratch_a, kv_cache.get_k_cache(layer), kv_cache.get_v_cache(layer),
                                        d_scratch_b, S, H, KVH, d, total, kv_dim);
        B2_CUDA_CHECK(cudaGetLastError());
        B2_CUDA_CHECK(cudaMemcpy(prefill_out.data() + layer * S * q_dim, d_scratch_b, S * q_dim * sizeof(__half),
                                 cudaMemcpyDeviceToHost));
    }
    kv_cache.set_cached_len(S);

    // ---- decode: capture once, then patch the changing nodes per token
    cudaStream_t stream = nullptr;
    B2_CUDA_CHECK(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t graph_exec = nullptr;
    std::vector<DecodeLayerNodes> decode_nodes(L);
    auto enqueue_decode = [&](size_t start_pos) {
        for (size_t layer = 0; layer < L; ++layer) {
            __half* row = d_rows + layer * total;
            const bool apply_rotation = (layer + 1) % 4 != 0;
            launch_rope_and_store_kv(row, row + q_dim, row + q_dim + kv_dim, kv_cache.get_k_cache(layer),
                                     kv_cache.get_v_cache(layer), rope.d_cos, rope.d_sin, 1, H, KVH, d, total, total,
                                     start_pos, apply_rotation, stream);
            decode_nodes[layer].store_kv = last_captured_node(stream);
            launch_causal_attention_decode_vectorized(
                row, kv_cache.get_k_cache(layer), kv_cache.get_v_cache(layer), d_dec_out + layer * q_dim,
                d_partial_output, d_partial_max, d_partial_weight_sum, 1, start_pos + 1, start_pos, H, KVH, d, total,
                kv_dim, stream, &decode_nodes[layer].attention, &decode_nodes[layer].merge);
        }
    };
    for (size_t t = 0; t < T; ++t) {
        const size_t start_pos = kv_cache.get_cached_len();
        B2_CUDA_CHECK(cudaMemcpyAsync(d_rows, news + t * L * total, L * total * sizeof(__half),
                                      cudaMemcpyHostToDevice, stream));
        if (!graph_exec) {
            B2_CUDA_CHECK(cudaStreamBeginCapture(stream, cudaStreamCaptureModeGlobal));
            enqueue_decode(start_pos);
            B2_CUDA_CHECK(cudaStreamEndCapture(stream, &graph));
            B2_CUDA_CHECK(cudaGraphInstantiate(&graph_exec, graph, 0));
        } else {
            for (size_t layer = 0; layer < L; ++layer) {
                const auto& nodes = decode_nodes[layer];
                const bool apply_rotation = (layer + 1) % 4 != 0;
                const size_t kv_len = start_pos + 1;
                update_rope_and_store_kv_node(graph_exec, nodes.store_kv, start_pos, apply_rotation);
                update_causal_attention_decode_node(graph_exec, nodes.attention, kv_len);
                update_merge_attention_decode_node(graph_exec, nodes.merge, kv_len);
            }
        }
        B2_CUDA_CHECK(cudaGraphLaunch(graph_exec, stream));
        B2_CUDA_CHECK(cudaMemcpyAsync(decode_out.data() + t * L * q_dim, d_dec_out, L * q_dim * sizeof(__half),
                                      cudaMemcpyDeviceToHost, stream));
        B2_CUDA_CHECK(cudaStreamSynchronize(stream));
        kv_cache.set_cached_len(start_pos + 1);
    }
    if (b2_device_error_word() != 0) fail("device error word set");

    // ---- outputs: prefill [L][S][q_dim], decode [T][L][q_dim], then the
    // caches' first S + T rows, [L][K|V][S + T][kv_dim]
    std::vector<__half> caches(L * 2 * (S + T) * kv_dim);
    for (size_t layer = 0; layer < L; ++layer) {
        B2_CUDA_CHECK(cudaMemcpy(caches.data() + (layer * 2) * (S + T) * kv_dim, kv_cache.get_k_cache(layer),
                                 (S + T) * kv_dim * sizeof(__half), cudaMemcpyDeviceToHost));
        B2_CUDA_CHECK(cudaMemcpy(caches.data() + (layer * 2 + 1) * (S + T) * kv_dim, kv_cache.get_v_cache(layer),
                                 (S + T) * kv_dim * sizeof(__half), cudaMemcpyDeviceToHost));
    }
    std::ofstream out(out_path, std::ios::binary);
    out.write(reinterpret_cast<const char*>(prefill_out.data()), prefill_out.size() * sizeof(__half));
    out.write(reinterpret_cast<const char*>(decode_out.data()), decode_out.size() * sizeof(__half));
    out.write(reinterpret_cast<const char*>(caches.data()), caches.size() * sizeof(__half));
    if (!out) throw std::runtime_error("cannot write " + out_path);

    B2_CUDA_CHECK(cudaGraphExecDestroy(graph_exec));
    B2_CUDA_CHECK(cudaGraphDestroy(graph));
    B2_CUDA_CHECK(cudaStreamDestroy(stream));
    for (void* p : {static_cast<void*>(d_scratch_a), static_cast<void*>(d_scratch_b), static_cast<void*>(d_rows),
                    static_cast<void*>(d_dec_out), static_cast<void*>(d_partial_output),
                    static_cast<void*>(d_partial_max), static_cast<void*>(d_partial_weight_sum)})
        B2_CUDA_CHECK(cudaFree(p));
    std::fputs(std::format("engine: {} layers, prompt {} tokens, {} decode tokens, {} failures\n", L, S, T,
                           g_failures)
                   .c_str(),
               stdout);
    return g_failures == 0 ? 0 : 1;
}

// ------------------------------------------------------------ known answer
int run_known_answer() {
    const size_t lengths[] = {1, KV_CHUNK, KV_CHUNK + 1, 3 * KV_CHUNK + 1, 257};
    size_t cases = 0;
    for (size_t head_dim : {size_t(32), size_t(128)}) {
        for (size_t kv_heads : {size_t(1), size_t(2), size_t(4)}) {
            const size_t heads = 4, q_dim = heads * head_dim, kv_dim = kv_heads * head_dim;
            for (size_t len : lengths) {
                for (bool padded : {false, true}) {
                    const size_t stride = kv_dim + (padded ? 17 : 0);
                    std::vector<__half> q(q_dim), k((len + 2) * stride, __float2half(123.f));
                    auto v = k;
                    for (size_t i = 0; i < q.size(); ++i) q[i] = __float2half(2.f * std::sin(float(i + 1) * .37f));
                    for (size_t t = 0; t < len; ++t)
                        for (size_t i = 0; i < kv_dim; ++i) {
                            k[t * stride + i] = __float2half(3.f * std::cos(float(t * kv_dim + i + 1) * .13f));
                            v[t * stride + i] = __float2half(std::sin(float(t * kv_dim + i + 3) * .19f));
                        }
                    // double-precision softmax over every cached row
                    std::vector<__half> expected(q_dim);
                    for (size_t h = 0; h < heads; ++h) {
                        const size_t kh = h / (heads / kv_heads);
                        std::vector<double> score(len);
                        double top = -INFINITY, den = 0.;
                        for (size_t t = 0; t < len; ++t) {
                            double dot = 0.;
                            for (size_t c = 0; c < head_dim; ++c)
                                dot += double(__half2float(q[h * head_dim + c])) *
                                       __half2float(k[t * stride + kh * head_dim + c]);
                            score[t] = dot / std::sqrt(double(head_dim));
                            top = std::max(top, score[t]);
                        }
                        for (auto& s : score) {
                            s = std::exp(s - top);
                            den += s;
                        }
                        for (size_t c = 0; c < head_dim; ++c) {
                            double num = 0.;
                            for (size_t t = 0; t < len; ++t) num += score[t] * __half2float(v[t * stride + kh * head_dim + c]);
                            expected[h * head_dim + c] = __float2half(float(num / den));
                        }
                    }
                    const size_t states = heads * ((len + KV_CHUNK - 1) / KV_CHUNK);
                    __half *dq = device_copy(q), *dk = device_copy(k), *dv = device_copy(v), *dout = nullptr;
                    float *partial = nullptr, *maximum = nullptr, *sum = nullptr;
                    std::vector<__half> actual(q_dim + 2, __float2half(-123.f));
                    dout = device_copy(actual);
                    B2_CUDA_CHECK(cudaMalloc(&partial, states * head_dim * sizeof(float)));
                    B2_CUDA_CHECK(cudaMalloc(&maximum, states * sizeof(float)));
                    B2_CUDA_CHECK(cudaMalloc(&sum, states * sizeof(float)));
                    launch_causal_attention_decode(dq, dk, dv, dout + 1, partial, maximum, sum, 1, len, len - 1, heads,
                                                   kv_heads, head_dim, 0, padded ? stride : 0);
                    B2_CUDA_CHECK(cudaGetLastError());
                    B2_CUDA_CHECK(cudaDeviceSynchronize());
                    B2_CUDA_CHECK(cudaMemcpy(actual.data(), dout, actual.size() * sizeof(__half),
                                             cudaMemcpyDeviceToHost));
                    const std::string tag =
                        std::format("known-answer d={} kvh={} len={} padded={}", head_dim, kv_heads, len, padded);
                    if (__half2float(actual.front()) != -123.f || __half2float(actual.back()) != -123.f)
                        fail(tag + ": output guard overwritten");
                    const auto result = std::span<const __half>(actual).subspan(1, q_dim);
                    float worst = 0.f;
                    if (!all_finite(result)) fail(tag + ": non-finite output");
                    if (const size_t bad = count_mismatches(result, expected, 2e-3f, 2e-3f, &worst))
                        fail(tag + std::format(": {} mismatches, max diff {}", bad, worst));
                    for (void* p : {static_cast<void*>(dq), static_cast<void*>(dk), static_cast<void*>(dv),
                                    static_cast<void*>(dout), static_cast<void*>(partial),
                                    static_cast<void*>(maximum), static_cast<void*>(sum)})
                        B2_CUDA_CHECK(cudaFree(p));
                    ++cases;
                }
            }
        }
    }
    std::fputs(std::format("known-answer: {} cases, {} failures\n", cases, g_failures).c_str(), stdout);
    return g_failures == 0 ? 0 : 1;
}

// ------------------------------------------------------------------ golden
int run_golden(const std::string& dir) {
    // the fixtures' geometry (tests/golden/meta.json): 16 / 4 heads, 128
    const size_t H = 16, KVH = 4, d = 128, q_dim = H * d, kv_dim = KVH * d;
    const auto q = read_file<__half>(dir + "/layer0_q_rope.bin");
    const auto k = read_file<__half>(dir + "/layer0_k_rope.bin");
    const auto v = read_file<__half>(dir + "/layer0_v_proj_out.bin");
    const auto expected = read_file<__half>(dir + "/layer0_attn_out.bin");
    const size_t S = q.size() / q_dim;
    if (S < 5 || k.size() != S * kv_dim || v.size() != k.size() || expected.size() != q.size())
        throw std::runtime_error("fixture sizes do not match 16 / 4 heads of 128");

    // :15-78 prefill from a cache whose spare rows hold 123
    {
        KVCache cache({1, S + 2, KVH, d});
        std::vector<__half> ck((S + 2) * kv_dim, __float2half(123.f)), cv = ck;
        std::copy(k.begin(), k.end(), ck.begin());
        std::copy(v.begin(), v.end(), cv.begin());
        B2_CUDA_CHECK(cudaMemcpy(cache.get_k_cache(0), ck.data(), ck.size() * sizeof(__half), cudaMemcpyHostToDevice));
        B2_CUDA_CHECK(cudaMemcpy(cache.get_v_cache(0), cv.data(), cv.size() * sizeof(__half), cudaMemcpyHostToDevice));
        __half* dq = device_copy(q);
        __half* dout = nullptr;
        B2_CUDA_CHECK(cudaMalloc(&dout, expected.size() * sizeof(__half)));
        launch_causal_attention_prefill(dq, cache.get_k_cache(0), cache.get_v_cache(0), dout, S, H, KVH, d, q_dim,
                                        kv_dim);
        B2_CUDA_CHECK(cudaGetLastError());
        B2_CUDA_CHECK(cudaDeviceSynchronize());
        std::vector<__half> actual(expected.size());
        B2_CUDA_CHECK(cudaMemcpy(actual.data(), dout, actual.size() * sizeof(__half), cudaMemcpyDeviceToHost));
        float worst = 0.f;
        if (const size_t bad = count_mismatches(actual, expected, 2e-2f, 2e-2f, &worst))
            fail(std::format("golden prefill: {} mismatches, max diff {}", bad, worst));
        B2_CUDA_CHECK(cudaFree(dq));
        B2_CUDA_CHECK(cudaFree(dout));

        // :80-150 decode at every position vs the prefill rows
        for (bool interleaved : {false, true}) {
            for (size_t position = 0; position < S; ++position) {
                const size_t stride = interleaved ? q_dim + 2 * kv_dim : q_dim;
                std::vector<__half> input(stride, __float2half(-123.f));
                std::copy_n(q.data() + position * q_dim, q_dim, input.data());
                const size_t states = H * ((position + 1 + KV_CHUNK - 1) / KV_CHUNK);
                __half* d_q = device_copy(input);
                std::vector<__half> output(3 * q_dim, __float2half(-123.f));
                const auto guards = output;
                __half* d_output = device_copy(output);
                float *d_partial = nullptr, *d_max = nullptr, *d_sum = nullptr;
                B2_CUDA_CHECK(cudaMalloc(&d_partial, states * d * sizeof(float)));
                B2_CUDA_CHECK(cudaMalloc(&d_max, states * sizeof(float)));
                B2_CUDA_CHECK(cudaMalloc(&d_sum, states * sizeof(float)));
                launch_causal_attention_decode(d_q, cache.get_k_cache(0), cache.get_v_cache(0), d_output + q_dim,
                                               d_partial, d_max, d_sum, 1, position + 1, position, H, KVH, d,
                                               interleaved ? stride : 0, 0);
                B2_CUDA_CHECK(cudaGetLastError());
                B2_CUDA_CHECK(cudaDeviceSynchronize());
                B2_CUDA_CHECK(cudaMemcpy(output.data(), d_output, output.size() * sizeof(__half),
                                         cudaMemcpyDeviceToHost));
                const auto actual_row = std::span<const __half>(output).subspan(q_dim, q_dim);
                const std::string tag = std::format("golden decode position {} interleaved {}", position, interleaved);
                if (!all_finite(actual_row)) fail(tag + ": non-finite output");
                if (const size_t bad = count_mismatches(
                        actual_row, std::span<const __half>(expected).subspan(position * q_dim, q_dim), 2e-2f, 2e-2f))
                    fail(tag + std::format(": {} mismatches", bad));
                if (std::memcmp(output.data(), guards.data(), q_dim * sizeof(__half)) != 0 ||
                    std::memcmp(output.data() + 2 * q_dim, guards.data() + 2 * q_dim, q_dim * sizeof(__half)) != 0)
                    fail(tag + ": output guards overwritten");
                for (void* p : {static_cast<void*>(d_q), static_cast<void*>(d_output), static_cast<void*>(d_partial),
                                static_cast<void*>(d_max), static_cast<void*>(d_sum)})
                    B2_CUDA_CHECK(cudaFree(p));
            }
        }
    }
    std::fputs(std::format("golden: {} tokens, prefill + {} decode positions x 2 layouts, {} failures\n", S, S,
                           g_failures)
                   .c_str(),
               stdout);
    return g_failures == 0 ? 0 : 1;
}

// --------------------------------------------------------------------- qkv
int run_qkv(const std::string& in_path, const std::string& out_path) {
    const auto in = read_file<uint16_t>(in_path);
    if (in.size() < 40) throw std::runtime_error("short input file");
    uint64_t hdr[10];
    std::memcpy(hdr, in.data(), sizeof(hdr));
    if (hdr[0] != 0x62323030716b76ull) throw std::runtime_error("bad input magic");
    const size_t S = hdr[1], hidden = hdr[2], H = hdr[3], KVH = hdr[4], d = hdr[5], start = hdr[6],
                 max_seq = hdr[8];
    const bool rotate = hdr[7] != 0;
    const size_t q_dim = H * d, kv_dim = KVH * d, total = q_dim + 2 * kv_dim;
    const __half* x_h = reinterpret_cast<const __half*>(in.data() + sizeof(hdr) / 2);
    const __half* w_h = x_h + S * hidden;
    if (in.size() != sizeof(hdr) / 2 + S * hidden + total * hidden) throw std::runtime_error("input size");
    const b200attn::RopeCache rope = b200attn::create_rope_cache(max_seq, d, 5.0e6f);
    __half *d_x = nullptr, *d_w = nullptr;
    B2_CUDA_CHECK(cudaMalloc(&d_x, S * hidden * sizeof(__half)));
    B2_CUDA_CHECK(cudaMalloc(&d_w, total * hidden * sizeof(__half)));
    B2_CUDA_CHECK(cudaMemcpy(d_x, x_h, S * hidden * sizeof(__half), cudaMemcpyHostToDevice));
    B2_CUDA_CHECK(cudaMemcpy(d_w, w_h, total * hidden * sizeof(__half), cudaMemcpyHostToDevice));
    // two sets of rows and caches; caches start as a 0x7e00 (NaN) sentinel
    struct Out {
        __half* rows = nullptr;
        KVCache* cache = nullptr;
    } two, one;
    for (Out* o : {&two, &one}) {
        B2_CUDA_CHECK(cudaMalloc(&o->rows, S * total * sizeof(__half)));
        o->cache = new KVCache({1, max_seq, KVH, d});
        B2_CUDA_CHECK(cudaMemset(o->cache->get_k_cache(0), 0x7e, max_seq * kv_dim * sizeof(__half)));
        B2_CUDA_CHECK(cudaMemset(o->cache->get_v_cache(0), 0x7e, max_seq * kv_dim * sizeof(__half)));
    }
    // the engine's two calls (d_scratch_b -> d_scratch_a, then RoPE/append in place)
    launch_qkv_gemm(d_x, two.rows, d_w, S, hidden, total);
    launch_rope_and_store_kv(two.rows, two.rows + q_dim, two.rows + q_dim + kv_dim, two.cache->get_k_cache(0),
                             two.cache->get_v_cache(0), rope.d_cos, rope.d_sin, S, H, KVH, d, total, total, start,
                             rotate);
    // the same in one kernel
    launch_qkv_gemm_rope_store_kv(d_x, one.rows, d_w, one.cache->get_k_cache(0), one.cache->get_v_cache(0),
                                  rope.d_cos, rope.d_sin, S, hidden, H, KVH, d, start, rotate);
    B2_CUDA_CHECK(cudaDeviceSynchronize());
    auto host = [](const __half* dptr, size_t n) {
        std::vector<uint16_t> h(n);
        B2_CUDA_CHECK(cudaMemcpy(h.data(), dptr, n * sizeof(__half), cudaMemcpyDeviceToHost));
        return h;
    };
    const auto r2 = host(two.rows, S * total), r1 = host(one.rows, S * total);
    const auto k2 = host(two.cache->get_k_cache(0), max_seq * kv_dim), k1 = host(one.cache->get_k_cache(0), max_seq * kv_dim);
    const auto v2 = host(two.cache->get_v_cache(0), max_seq * kv_dim), v1 = host(one.cache->get_v_cache(0), max_seq * kv_dim);
    if (r1 != r2) fail("qkv rows: fused differs from launch_qkv_gemm + launch_rope_and_store_kv");
    if (k1 != k2) fail("k cache: fused differs from the two calls");
    if (v1 != v2) fail("v cache: fused differs from the two calls");
    for (size_t t = 0; t < max_seq; ++t) {
        const bool written = t >= start && t < start + S;
        for (size_t c = 0; c < kv_dim; ++c)
            if ((k1[t * kv_dim + c] == 0x7e7e) == written) {
                fail(std::format("k cache row {} {}", t, written ? "not written" : "written"));
                t = max_seq;
                break;
            }
    }
    std::ofstream f(out_path, std::ios::binary);
    f.write(reinterpret_cast<const char*>(r1.data()), static_cast<std::streamsize>(r1.size() * 2));
    f.write(reinterpret_cast<const char*>(k1.data() + start * kv_dim), static_cast<std::streamsize>(S * kv_dim * 2));
    f.write(reinterpret_cast<const char*>(v1.data() + start * kv_dim), static_cast<std::streamsize>(S * kv_dim * 2));
    for (Out* o : {&two, &one}) {
        B2_CUDA_CHECK(cudaFree(o->rows));
        delete o->cache;
    }
    B2_CUDA_CHECK(cudaFree(d_x));
    B2_CUDA_CHECK(cudaFree(d_w));
    std::fputs(std::format("qkv: {} tokens, hidden {}, {}/{} heads x {}, start {}, rotate {}: {} failures\n", S,
                           hidden, H, KVH, d, start, rotate ? 1 : 0, g_failures)
                   .c_str(),
               stdout);
    return g_failures == 0 ? 0 : 1;
}

// ----------------------------------------------------------------- weights
int run_weights(const std::string& path, size_t chunk) {
    b200attn::LoadedModel m = b200attn::load_weights_file(path, nullptr, chunk);
    const auto& c = m.config;
    std::fputs(std::format("{{\"header\": [{}, {}, {}, {}, {}, {}, {}, {}, {}, {}], \"tokenizer_bytes\": {}}}\n",
                           c.vocab_size, c.hidden_size, c.num_layers, c.num_heads, c.num_kv_heads, c.head_dim,
                           c.intermediate_size, c.max_seq_len, c.rms_norm_eps, c.rope_theta,
                           m.tokenizer_json.size())
                   .c_str(),
               stdout);
    std::fputs(("tokenizer " + m.tokenizer_json + "\n").c_str(), stdout);
    const size_t h = c.hidden_size, q = size_t(c.num_heads) * c.head_dim, kv = size_t(c.num_kv_heads) * c.head_dim,
                 inter = c.intermediate_size;
    auto report = [](const std::string& name, const __half* dptr, size_t n) {
        std::vector<__half> hbuf(n);
        B2_CUDA_CHECK(cudaMemcpy(hbuf.data(), dptr, n * sizeof(__half), cudaMemcpyDeviceToHost));
        double sum = 0., sumsq = 0.;
        for (const __half x : hbuf) {
            const double v = __half2float(x);
            sum += v;
            sumsq += v * v;
        }
        auto at = [&hbuf](size_t i) { return static_cast<double>(__half2float(hbuf[i])); };
        std::fputs(std::format("{{\"name\": \"{}\", \"n\": {}, \"sum\": {:.17g}, \"sumsq\": {:.17g}, \"first\": "
                               "[{:.17g}, {:.17g}, {:.17g}, {:.17g}]}}\n",
                               name, n, sum, sumsq, at(0), at(1), at(2), at(3))
                       .c_str(),
                   stdout);
    };
    const auto& w = m.weights;
    report("embedding_tokens", w.embedding_tokens, size_t(c.vocab_size) * h);
    for (size_t i = 0; i < w.transformer_blocks.size(); ++i) {
        const auto& b = w.transformer_blocks[i];
        const std::string p = std::format("layers.{}.", i);
        report(p + "input_normalization", b.input_normalization, h);
        report(p + "q_proj", b.q_proj, q * h);
        report(p + "k_proj", b.k_proj, kv * h);
        report(p + "v_proj", b.v_proj, kv * h);
        report(p + "o_proj", b.o_proj, h * q);
        report(p + "post_attn_norm", b.post_attn_norm, h);
        report(p + "gate_proj", b.gate_proj, inter * h);
        report(p + "up_proj", b.up_proj, inter * h);
        report(p + "down_proj", b.down_proj, h * inter);
    }
    report("final_norm", w.final_norm, h);
    report("lm_head", w.lm_head, size_t(c.vocab_size) * h);
    return 0;
}

}  // namespace

int main(int argc, char** argv) {
    try {
        const std::string mode = argc > 1 ? argv[1] : "";
        if (mode == "engine" && argc == 4) return run_engine(argv[2], argv[3]);
        if (mode == "known-answer" && argc == 2) return run_known_answer();
        if (mode == "golden" && argc == 3) return run_golden(argv[2]);
        if (mode == "weights" && argc == 4) return run_weights(argv[2], std::stoull(argv[3]));
        if (mode == "qkv" && argc == 4) return run_qkv(argv[2], argv[3]);
        std::fputs("usage: engine_harness engine <in> <out> | known-answer | golden <dir> | weights <file> <chunk> | "
                   "qkv <in> <out>\n",
                   stderr);
        return 2;
    } catch (const std::exception& e) {
        std::fputs((std::string("error: ") + e.what() + "\n").c_str(), stderr);
        return 3;
    }
}
