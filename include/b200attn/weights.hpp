// weights.bin loader for the CUDA build: the file format that the reference's
// python/export_weights.py:20-135 writes and include/model.hpp:17-92 +
// include/device_weights.hpp:56-108 read, unchanged:
//
//   [ModelConfig, 44 bytes: "QWEN", 8 x uint32, 2 x float32]
//   [uint32 tokenizer JSON length][tokenizer JSON bytes]
//   [zero padding to a 64-byte file offset]
//   [FP16 tensors, row-major, in network order: embed_tokens [vocab][hidden];
//    per layer: input_layernorm [hidden], q_proj [q_dim][hidden],
//    k_proj [kv_dim][hidden], v_proj [kv_dim][hidden], o_proj [hidden][q_dim],
//    post_attention_layernorm [hidden], gate_proj [inter][hidden],
//    up_proj [inter][hidden], down_proj [hidden][inter];
//    final norm [hidden]; lm_head [vocab][hidden]]
//
// Everything after the padding goes to the GPU as one allocation, and the
// per-tensor pointers are carved from it in that order (the reference's
// DeviceWeights). The upload streams the file through two pinned staging
// buffers with cudaMemcpyAsync, so reading the next chunk overlaps the copy of
// the previous one (the reference copies from the pageable mmap in one call).
//
// Differences from the reference, on purpose: the payload size is checked
// against the size the header implies (the reference trusts it, so a file
// with the optional q_norm / k_norm tensors that export_weights.py may write
// would be silently misread); errors throw std::runtime_error; the tokenizer
// JSON is returned as bytes (tokenizer construction is outside this library).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "b200attn/gpu_utils.hpp"

namespace b200attn {

#pragma pack(push, 1)
// include/model_config.hpp:9-55: the 44-byte header, field for field.
struct ModelConfig {
    char magic[4];
    uint32_t vocab_size;
    uint32_t hidden_size;
    uint32_t num_layers;
    uint32_t num_heads;
    uint32_t num_kv_heads;
    uint32_t head_dim;
    uint32_t intermediate_size;
    uint32_t max_seq_len;
    float rms_norm_eps;
    float rope_theta;
};
#pragma pack(pop)
static_assert(sizeof(ModelConfig) == 44, "weights.bin header is 44 bytes");

// include/device_weights.hpp:9-35: one transformer block's tensors.
struct TransformerBlock {
    const __half* input_normalization = nullptr;  // [hidden]
    const __half* q_proj = nullptr;               // [num_heads * head_dim][hidden]
    const __half* k_proj = nullptr;               // [num_kv_heads * head_dim][hidden]
    const __half* v_proj = nullptr;               // [num_kv_heads * head_dim][hidden]
    const __half* o_proj = nullptr;               // [hidden][num_heads * head_dim]
    const __half* post_attn_norm = nullptr;       // [hidden]
    const __half* gate_proj = nullptr;            // [intermediate][hidden]
    const __half* up_proj = nullptr;              // [intermediate][hidden]
    const __half* down_proj = nullptr;            // [hidden][intermediate]
};

// Parse and check the header (include/model_config.hpp:31-43).
inline ModelConfig parse_model_config(const void* bytes, size_t size) {
    if (size < sizeof(ModelConfig)) throw std::runtime_error("weights.bin: shorter than its 44-byte header");
    ModelConfig c;
    std::memcpy(&c, bytes, sizeof(c));
    if (std::memcmp(c.magic, "QWEN", 4) != 0) throw std::runtime_error("weights.bin: magic is not 'QWEN'");
    return c;
}

// Elements of every tensor in file order, as the loader claims them.
inline size_t weight_elements(const ModelConfig& c) {
    const size_t h = c.hidden_size, q = size_t(c.num_heads) * c.head_dim, kv = size_t(c.num_kv_heads) * c.head_dim,
                 inter = c.intermediate_size, vocab = c.vocab_size;
    const size_t per_layer = h + q * h + 2 * kv * h + h * q + h + 2 * inter * h + h * inter;
    return vocab * h + c.num_layers * per_layer + h + vocab * h;
}

// Byte offset of the weights: after the header, the tokenizer length word and
// the tokenizer JSON, rounded up to 64 (include/model.hpp:72-76).
inline size_t weights_offset(uint32_t tokenizer_bytes) {
    const size_t raw = sizeof(ModelConfig) + sizeof(uint32_t) + tokenizer_bytes;
    return (raw + 63) & ~size_t(63);
}

class DeviceWeights {
  public:
    const __half* embedding_tokens = nullptr;  // [vocab][hidden]
    std::vector<TransformerBlock> transformer_blocks;
    const __half* final_norm = nullptr;        // [hidden]
    const __half* lm_head = nullptr;           // [vocab][hidden]

    DeviceWeights() = default;
    DeviceWeights(const DeviceWeights&) = delete;
    DeviceWeights& operator=(const DeviceWeights&) = delete;
    DeviceWeights(DeviceWeights&& o) noexcept { *this = std::move(o); }
    DeviceWeights& operator=(DeviceWeights&& o) noexcept {
        if (this != &o) {
            release();
            embedding_tokens = o.embedding_tokens;
            transformer_blocks = std::move(o.transformer_blocks);
            final_norm = o.final_norm;
            lm_head = o.lm_head;
            buffer_ = o.buffer_;
            bytes_ = o.bytes_;
            o.buffer_ = nullptr;
            o.bytes_ = 0;
        }
        return *this;
    }
    ~DeviceWeights() { release(); }

    __half* raw_device_buffer() const noexcept { return buffer_; }
    size_t total_bytes() const noexcept { return bytes_; }

    // Allocate the device buffer for `c` and carve the tensor pointers
    // (include/device_weights.hpp:74-108 order).
    void allocate(const ModelConfig& c) {
        release();
        bytes_ = weight_elements(c) * sizeof(__half);
        B2_CUDA_CHECK(cudaMalloc(&buffer_, bytes_));
        const __half* cursor = buffer_;
        auto claim = [&cursor](size_t n) {
            const __half* p = cursor;
            cursor += n;
            return p;
        };
        const size_t h = c.hidden_size, q = size_t(c.num_heads) * c.head_dim,
                     kv = size_t(c.num_kv_heads) * c.head_dim, inter = c.intermediate_size;
        embedding_tokens = claim(size_t(c.vocab_size) * h);
        transformer_blocks.assign(c.num_layers, TransformerBlock{});
        for (auto& b : transformer_blocks) {
            b.input_normalization = claim(h);
            b.q_proj = claim(h * q);
            b.k_proj = claim(h * kv);
            b.v_proj = claim(h * kv);
            b.o_proj = claim(q * h);
            b.post_attn_norm = claim(h);
            b.gate_proj = claim(h * inter);
            b.up_proj = claim(h * inter);
            b.down_proj = claim(inter * h);
        }
        final_norm = claim(h);
        lm_head = claim(size_t(c.vocab_size) * h);
    }

  private:
    void release() noexcept {
        if (buffer_) (void)cudaFree(buffer_);
        buffer_ = nullptr;
        bytes_ = 0;
    }
    __half* buffer_ = nullptr;
    size_t bytes_ = 0;
};

struct LoadedModel {
    ModelConfig config{};
    std::string tokenizer_json;
    DeviceWeights weights;
};

// Read weights.bin: check the header and the payload size, keep the tokenizer
// JSON, and upload the weights to the current device through two pinned
// staging buffers (chunk_bytes each) on `stream`.
inline LoadedModel load_weights_file(const std::string& path, cudaStream_t stream = nullptr,
                                     size_t chunk_bytes = size_t(64) << 20) {
    std::unique_ptr<FILE, int (*)(FILE*)> f(std::fopen(path.c_str(), "rb"), &std::fclose);
    if (!f) throw std::runtime_error("weights.bin: cannot open " + path);
    LoadedModel m;
    unsigned char head[sizeof(ModelConfig) + sizeof(uint32_t)];
    if (std::fread(head, 1, sizeof(head), f.get()) != sizeof(head))
        throw std::runtime_error("weights.bin: missing the header or the tokenizer length field");
    m.config = parse_model_config(head, sizeof(head));
    uint32_t tok_len = 0;
    std::memcpy(&tok_len, head + sizeof(ModelConfig), sizeof(tok_len));
    m.tokenizer_json.resize(tok_len);
    if (tok_len && std::fread(m.tokenizer_json.data(), 1, tok_len, f.get()) != tok_len)
        throw std::runtime_error("weights.bin: tokenizer payload truncated");
    const size_t offset = weights_offset(tok_len);
    if (std::fseek(f.get(), 0, SEEK_END) != 0) throw std::runtime_error("weights.bin: cannot seek");
    const long end = std::ftell(f.get());
    const size_t need = weight_elements(m.config) * sizeof(__half);
    if (end < 0 || size_t(end) < offset || size_t(end) - offset != need)
        throw std::runtime_error("weights.bin: payload is " +
                                 std::to_string(end < 0 || size_t(end) < offset ? 0 : size_t(end) - offset) +
                                 " bytes, the header implies " + std::to_string(need) +
                                 " (a file with q_norm / k_norm tensors is not this layout)");
    if (std::fseek(f.get(), long(offset), SEEK_SET) != 0) throw std::runtime_error("weights.bin: cannot seek");
    m.weights.allocate(m.config);

    void* stage[2] = {nullptr, nullptr};
    cudaEvent_t done[2] = {nullptr, nullptr};
    B2_CUDA_CHECK(cudaMallocHost(&stage[0], chunk_bytes));
    B2_CUDA_CHECK(cudaMallocHost(&stage[1], chunk_bytes));
    B2_CUDA_CHECK(cudaEventCreateWithFlags(&done[0], cudaEventDisableTiming));
    B2_CUDA_CHECK(cudaEventCreateWithFlags(&done[1], cudaEventDisableTiming));
    auto* dst = reinterpret_cast<unsigned char*>(m.weights.raw_device_buffer());
    size_t copied = 0;
    bool ok = true;
    for (int i = 0; copied < need; ++i) {
        const int k = i & 1;
        if (i >= 2) B2_CUDA_CHECK(cudaEventSynchronize(done[k]));  // this staging buffer is free again
        const size_t n = std::min(chunk_bytes, need - copied);
        if (std::fread(stage[k], 1, n, f.get()) != n) {
            ok = false;
            break;
        }
        B2_CUDA_CHECK(cudaMemcpyAsync(dst + copied, stage[k], n, cudaMemcpyHostToDevice, stream));
        B2_CUDA_CHECK(cudaEventRecord(done[k], stream));
        copied += n;
    }
    B2_CUDA_CHECK(cudaStreamSynchronize(stream));
    for (int k = 0; k < 2; ++k) {
        B2_CUDA_CHECK(cudaEventDestroy(done[k]));
        B2_CUDA_CHECK(cudaFreeHost(stage[k]));
    }
    if (!ok) throw std::runtime_error("weights.bin: short read of the weights");
    return m;
}

}  // namespace b200attn
