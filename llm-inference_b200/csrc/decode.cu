// Split-KV flash-decode for sm_100a: split stage + merge.
//
// Restates src/kernels/causal_attention.hip.cpp of the reference:
//   causal_attention_decode{,_vectorized} (:493-595, :619-716)  per (head,
//       chunk) partial (o, m, l) over one query token
//   merge_attention_decode (:719-838)  M = max m_c, L = sum e^(m_c-M) l_c,
//       out = sum e^(m_c-M) o_c / L
//   launchers (:840-972), graph-node patchers (:975-1026)
// Partial workspace layout is the reference's: o [H][chunks][d] fp32,
// m and l [H][chunks] fp32, m in natural-log units of q.k/sqrt(d).
//
// Fast split kernel (head_dim 128, 16-byte aligned rows, group <= 8): one CTA
// per (KV head, KV_CHUNK-token chunk), 4 warps x 64 tokens. Every K/V row of
// the chunk is read exactly once for all query heads of its GQA group (the
// reference grid (head, chunk) re-reads each KV byte once per query head).
// Scores and P.V run on the tensor cores with mma.sync m16n8k16 (f16 in,
// f32 accumulate) with tokens as the M dimension:
//   S^T[16 tok x 8 heads] = K[16 tok x 128] . Q^T            (8 MMAs)
//   O^T[128 x 8 heads]   += V^T[128 x 16 tok] . P^T[16 tok x 8] (8 MMAs)
// The contraction order over head_dim is permuted so that each lane's A/B
// fragments are whole 16-byte loads of K, V and Q (16 B per lane, 64-128
// contiguous bytes per row per instruction); the same permutation is applied
// to Q, and the P.V output rows are mapped back when stored. The online
// softmax runs on the S fragments in the log2 domain with shuffles.
// Other shapes run a SIMT split kernel with the same partial format.
#include <math.h>

#include "b2_common.cuh"

namespace b2 {
namespace {

constexpr int kChunk = 256;  // KV_CHUNK
constexpr int kDecWarps = 4;
constexpr int kTokPerWarp = kChunk / kDecWarps;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

struct DecodeArgs {
    const __half* q;
    const __half* k;
    const __half* v;
    float* po;
    float* pm;
    float* pl;
    uint64_t kv_stride;   // elements between cached tokens
    uint32_t kv_len;      // patched by b2_update_causal_attention_decode_node
    uint32_t num_chunks;  // patched, = ceil(kv_len / KV_CHUNK)
    uint32_t num_heads;
    uint32_t num_kv_heads;
    uint32_t head_dim;
    uint32_t group;
    float scale_log2;     // log2(e) / sqrt(head_dim)
    float scale;          // 1 / sqrt(head_dim)
};

struct MergeArgs {
    const float* po;
    const float* pm;
    const float* pl;
    __half* out;
    uint32_t num_heads;
    uint32_t head_dim;
    uint32_t num_chunks;  // patched by b2_update_merge_attention_decode_node
};

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 ld_stream(const __half* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ uint32_t word(const uint4& v, int i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// ---------------------------------------------------------------------------
// Fast split kernel. grid = (num_kv_heads, num_chunks), block = 128.
__global__ void __launch_bounds__(128) decode_split_mma_kernel(const DecodeArgs a) {
    __shared__ float sm_m[kDecWarps][8];
    __shared__ float sm_l[kDecWarps][8];
    __shared__ float sm_o[kDecWarps][8][128];

    const uint32_t kvh = blockIdx.x;
    const uint32_t chunk = blockIdx.y;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2;
    const int t = lane & 3;
    const uint32_t group = a.group;

    const uint32_t c0 = chunk * kChunk;
    const uint32_t c1 = min(c0 + kChunk, a.kv_len);
    const uint32_t w0 = c0 + warp * kTokPerWarp;
    const uint32_t w1 = min(w0 + kTokPerWarp, c1);

    // Q fragments (B of the score MMA): head g of the group, 4 x 16 B.
    uint32_t qf[8][2];
    if (static_cast<uint32_t>(g) < group) {
        const __half* qrow = a.q + static_cast<uint64_t>(kvh * group + g) * 128;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint4 w = *reinterpret_cast<const uint4*>(qrow + 32 * j + 8 * t);
            qf[2 * j][0] = w.x;
            qf[2 * j][1] = w.y;
            qf[2 * j + 1][0] = w.z;
            qf[2 * j + 1][1] = w.w;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) qf[j][0] = qf[j][1] = 0u;
    }

    float o[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

    const __half* kbase = a.k + static_cast<uint64_t>(kvh) * 128;
    const __half* vbase = a.v + static_cast<uint64_t>(kvh) * 128;
    const uint64_t stride = a.kv_stride;
    const uint4 zero4 = make_uint4(0u, 0u, 0u, 0u);

    for (uint32_t tb = w0; tb < w1; tb += 16) {
        // ---- loads: K rows tb+g, tb+g+8; V rows tb+{2t,2t+1,2t+8,2t+9}
        uint4 ka[4], kb[4], va[4][2];
        const uint32_t ra = tb + g, rb = tb + g + 8;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            ka[j] = ra < w1 ? ld_stream(kbase + ra * stride + 32 * j + 8 * t) : zero4;
            kb[j] = rb < w1 ? ld_stream(kbase + rb * stride + 32 * j + 8 * t) : zero4;
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t r = tb + 2 * t + (i & 1) + (i >> 1) * 8;
#pragma unroll
            for (int b = 0; b < 2; ++b) va[i][b] = r < w1 ? ld_stream(vbase + r * stride + 64 * b + 8 * g) : zero4;
        }

        // ---- scores
        float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            mma16816(s, ka[j].x, kb[j].x, ka[j].y, kb[j].y, qf[2 * j][0], qf[2 * j][1]);
            mma16816(s, ka[j].z, kb[j].z, ka[j].w, kb[j].w, qf[2 * j + 1][0], qf[2 * j + 1][1]);
        }
        const bool va_ok = ra < w1, vb_ok = rb < w1;
        s[0] = va_ok ? s[0] * a.scale_log2 : -INFINITY;
        s[1] = va_ok ? s[1] * a.scale_log2 : -INFINITY;
        s[2] = vb_ok ? s[2] * a.scale_log2 : -INFINITY;
        s[3] = vb_ok ? s[3] * a.scale_log2 : -INFINITY;

        // ---- online softmax (heads 2t, 2t+1 of this lane)
        float mx0 = fmaxf(s[0], s[2]), mx1 = fmaxf(s[1], s[3]);
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
        }
        const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
        const float al0 = exp2f(m0 - mn0), al1 = exp2f(m1 - mn1);
        const float p0 = exp2f(s[0] - mn0), p1 = exp2f(s[1] - mn1);
        const float p2 = exp2f(s[2] - mn0), p3 = exp2f(s[3] - mn1);
        l0 = fmaf(l0, al0, p0 + p2);
        l1 = fmaf(l1, al1, p1 + p3);
        m0 = mn0;
        m1 = mn1;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            o[i][0] *= al0;
            o[i][1] *= al1;
            o[i][2] *= al0;
            o[i][3] *= al1;
        }

        // ---- P^T fragments: column (head) g, tokens {2t,2t+1} and {2t+8,2t+9}
        const uint32_t X = pack_half2(p0, p1);  // token g,   heads 2t, 2t+1
        const uint32_t Y = pack_half2(p2, p3);  // token g+8, heads 2t, 2t+1
        const int src_a = 8 * t + (g >> 1);
        const int src_b = 8 * t + 4 + (g >> 1);
        const uint32_t Xa = __shfl_sync(0xffffffffu, X, src_a);
        const uint32_t Xb = __shfl_sync(0xffffffffu, X, src_b);
        const uint32_t Ya = __shfl_sync(0xffffffffu, Y, src_a);
        const uint32_t Yb = __shfl_sync(0xffffffffu, Y, src_b);
        const uint32_t sel = (g & 1) ? 0x7632u : 0x5410u;
        const uint32_t pb0 = __byte_perm(Xa, Xb, sel);
        const uint32_t pb1 = __byte_perm(Ya, Yb, sel);

        // ---- O^T += V^T . P^T over 8 row tiles of head_dim
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
            const int b = mt >> 2, q = mt & 3;
            const uint32_t w0a = word(va[0][b], q), w1a = word(va[1][b], q);
            const uint32_t w2a = word(va[2][b], q), w3a = word(va[3][b], q);
            mma16816(o[mt], __byte_perm(w0a, w1a, 0x5410u), __byte_perm(w0a, w1a, 0x7632u),
                     __byte_perm(w2a, w3a, 0x5410u), __byte_perm(w2a, w3a, 0x7632u), pb0, pb1);
        }
    }

    // Per-warp row sums: reduce the per-lane partial sums over the 8 token rows.
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
        l0 += __shfl_xor_sync(0xffffffffu, l0, off);
        l1 += __shfl_xor_sync(0xffffffffu, l1, off);
    }
    if (g == 0) {
        sm_m[warp][2 * t] = m0;
        sm_m[warp][2 * t + 1] = m1;
        sm_l[warp][2 * t] = l0;
        sm_l[warp][2 * t + 1] = l1;
    }
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
        const int d = 64 * (mt >> 2) + 8 * g + 2 * (mt & 3);
        sm_o[warp][2 * t][d] = o[mt][0];
        sm_o[warp][2 * t + 1][d] = o[mt][1];
        sm_o[warp][2 * t][d + 1] = o[mt][2];
        sm_o[warp][2 * t + 1][d + 1] = o[mt][3];
    }
    __syncthreads();

    // Combine the 4 warps: one (m, l, o) per head of the group.
    const uint32_t chunks = a.num_chunks;
    for (uint32_t idx = threadIdx.x; idx < group * 128; idx += blockDim.x) {
        const uint32_t hh = idx >> 7, d = idx & 127;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kDecWarps; ++w) M = fmaxf(M, sm_m[w][hh]);
        float L = 0.f, O = 0.f;
#pragma unroll
        for (int w = 0; w < kDecWarps; ++w) {
            const float sc = exp2f(sm_m[w][hh] - M);
            L = fmaf(sc, sm_l[w][hh], L);
            O = fmaf(sc, sm_o[w][hh][d], O);
        }
        const uint64_t state = static_cast<uint64_t>(kvh * group + hh) * chunks + chunk;
        a.po[state * 128 + d] = O;
        if (d == 0) {
            a.pm[state] = M * kLn2;
            a.pl[state] = L;
        }
    }
}

// ---------------------------------------------------------------------------
// SIMT split kernel for any head_dim / stride / alignment.
// grid = (num_heads, num_chunks), block = 128; partials identical in meaning.
__global__ void __launch_bounds__(128) decode_split_simt_kernel(const DecodeArgs a) {
    __shared__ float scores[kChunk];
    __shared__ float red[4];
    const uint32_t h = blockIdx.x;
    const uint32_t chunk = blockIdx.y;
    const uint32_t kvh = h / a.group;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t c0 = chunk * kChunk;
    const uint32_t c1 = min(c0 + kChunk, a.kv_len);
    const uint32_t n = c1 - c0;
    const __half* qrow = a.q + static_cast<uint64_t>(h) * a.head_dim;

    for (uint32_t i = warp; i < n; i += 4) {
        const __half* krow = a.k + static_cast<uint64_t>(c0 + i) * a.kv_stride + static_cast<uint64_t>(kvh) * a.head_dim;
        float dot = 0.f;
        for (uint32_t e = lane; e < a.head_dim; e += 32) dot = fmaf(__half2float(qrow[e]), __half2float(krow[e]), dot);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
        if (lane == 0) scores[i] = dot * a.scale;
    }
    __syncthreads();
    float mx = -INFINITY;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) mx = fmaxf(mx, scores[i]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    __syncthreads();
    float sum = 0.f;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
        const float p = expf(scores[i] - mx);
        scores[i] = p;
        sum += p;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    if (lane == 0) red[warp] = sum;
    __syncthreads();
    sum = red[0] + red[1] + red[2] + red[3];
    const uint64_t state = static_cast<uint64_t>(h) * a.num_chunks + chunk;
    for (uint32_t e = threadIdx.x; e < a.head_dim; e += blockDim.x) {
        float acc = 0.f;
        for (uint32_t i = 0; i < n; ++i) {
            const __half* vrow = a.v + static_cast<uint64_t>(c0 + i) * a.kv_stride + static_cast<uint64_t>(kvh) * a.head_dim;
            acc = fmaf(scores[i], __half2float(vrow[e]), acc);
        }
        a.po[state * a.head_dim + e] = acc;
    }
    if (threadIdx.x == 0) {
        a.pm[state] = mx;
        a.pl[state] = sum;
    }
}

// ---------------------------------------------------------------------------
// Merge: grid = (num_heads, ceil(head_dim / 64)), block = 256. Warps stride
// over chunks, lanes over two output dimensions each.
__global__ void __launch_bounds__(256) merge_partials_kernel(const MergeArgs a) {
    __shared__ float red[8];
    __shared__ float acc_s[8][64];
    const uint32_t h = blockIdx.x;
    const uint32_t d0 = blockIdx.y * 64;
    const uint32_t chunks = a.num_chunks;
    const uint32_t d = a.head_dim;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float* pm = a.pm + static_cast<uint64_t>(h) * chunks;
    const float* pl = a.pl + static_cast<uint64_t>(h) * chunks;
    const float* po = a.po + static_cast<uint64_t>(h) * chunks * d;

    float mx = -INFINITY;
    for (uint32_t c = threadIdx.x; c < chunks; c += blockDim.x) mx = fmaxf(mx, pm[c]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    mx = red[0];
#pragma unroll
    for (int w = 1; w < 8; ++w) mx = fmaxf(mx, red[w]);
    __syncthreads();

    float den = 0.f;
    for (uint32_t c = threadIdx.x; c < chunks; c += blockDim.x) den = fmaf(expf(pm[c] - mx), pl[c], den);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) den += __shfl_xor_sync(0xffffffffu, den, off);
    if (lane == 0) red[warp] = den;
    __syncthreads();
    den = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) den += red[w];

    const uint32_t e0 = d0 + 2 * lane, e1 = e0 + 1;
    float s0 = 0.f, s1 = 0.f;
    for (uint32_t c = warp; c < chunks; c += 8) {
        const float sc = expf(pm[c] - mx);
        const float* row = po + static_cast<uint64_t>(c) * d;
        if (e0 < d) s0 = fmaf(sc, row[e0], s0);
        if (e1 < d) s1 = fmaf(sc, row[e1], s1);
    }
    acc_s[warp][2 * lane] = s0;
    acc_s[warp][2 * lane + 1] = s1;
    __syncthreads();
    if (threadIdx.x < 64 && d0 + threadIdx.x < d) {
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) s += acc_s[w][threadIdx.x];
        a.out[static_cast<uint64_t>(h) * d + d0 + threadIdx.x] = __float2half_rn(s / den);
    }
}

const void* const kSplitKernels[] = {
    reinterpret_cast<const void*>(decode_split_mma_kernel),
    reinterpret_cast<const void*>(decode_split_simt_kernel),
};
const void* const kMergeKernels[] = {reinterpret_cast<const void*>(merge_partials_kernel)};

int launch_merge(const float* po, const float* pm, const float* pl, __half* out, uint32_t heads, uint32_t chunks,
                 uint32_t head_dim, cudaStream_t stream) {
    MergeArgs m{po, pm, pl, out, heads, head_dim, chunks};
    const dim3 grid(heads, (head_dim + 63) / 64);
    merge_partials_kernel<<<grid, 256, 0, stream>>>(m);
    return launch_status();
}

int launch_decode(const void* d_q, const void* d_k, const void* d_v, void* d_out, float* po, float* pm, float* pl,
                  size_t query_len, size_t kv_len, size_t num_heads, size_t num_kv_heads, size_t head_dim,
                  size_t kv_stride, b2_stream_t stream_handle, b2_graph_node_t* attention_node,
                  b2_graph_node_t* merge_node) {
    // causal_attention.hip.cpp:860-866, :945-946: silent no-ops.
    if (query_len == 0 || kv_len == 0 || num_kv_heads == 0 || head_dim == 0) return B2_NOTHING_TO_DO;
    if (num_heads % num_kv_heads != 0) return B2_NOTHING_TO_DO;
    if (!d_q || !d_k || !d_v || !d_out || !po || !pm || !pl) return B2_ERR_INVALID_ARG;
    const size_t chunks = (kv_len + kChunk - 1) / kChunk;
    if (kv_len > 0xffffffffull - kChunk || chunks > 65535 || num_heads > 65535 || head_dim > 4096)
        return B2_ERR_UNSUPPORTED;
    if (kv_stride == 0) kv_stride = num_kv_heads * head_dim;
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_handle);
    const size_t group = num_heads / num_kv_heads;

    DecodeArgs a{};
    a.q = static_cast<const __half*>(d_q);
    a.k = static_cast<const __half*>(d_k);
    a.v = static_cast<const __half*>(d_v);
    a.po = po;
    a.pm = pm;
    a.pl = pl;
    a.kv_stride = kv_stride;
    a.kv_len = static_cast<uint32_t>(kv_len);
    a.num_chunks = static_cast<uint32_t>(chunks);
    a.num_heads = static_cast<uint32_t>(num_heads);
    a.num_kv_heads = static_cast<uint32_t>(num_kv_heads);
    a.head_dim = static_cast<uint32_t>(head_dim);
    a.group = static_cast<uint32_t>(group);
    a.scale = 1.0f / sqrtf(static_cast<float>(head_dim));
    a.scale_log2 = a.scale * kLog2e;

    const bool fast = head_dim == 128 && group <= 8 && aligned16(d_q) && aligned16(d_k) && aligned16(d_v) &&
                      (kv_stride % 8 == 0);
    if (fast) {
        decode_split_mma_kernel<<<dim3(a.num_kv_heads, a.num_chunks), 128, 0, stream>>>(a);
    } else {
        decode_split_simt_kernel<<<dim3(a.num_heads, a.num_chunks), 128, 0, stream>>>(a);
    }
    int st = launch_status();
    if (st != B2_OK) return st;
    if (attention_node) {
        cudaGraphNode_t n = nullptr;
        if ((st = last_captured_node(stream, &n)) != B2_OK) return st;
        *attention_node = reinterpret_cast<b2_graph_node_t>(n);
    }
    st = launch_merge(po, pm, pl, static_cast<__half*>(d_out), a.num_heads, a.num_chunks, a.head_dim, stream);
    if (st != B2_OK) return st;
    if (merge_node) {
        cudaGraphNode_t n = nullptr;
        if ((st = last_captured_node(stream, &n)) != B2_OK) return st;
        *merge_node = reinterpret_cast<b2_graph_node_t>(n);
    }
    return B2_OK;
}

}  // namespace
}  // namespace b2

using namespace b2;

extern "C" int b2_launch_causal_attention_decode(const void* d_q, const void* d_k_cache, const void* d_v_cache,
                                                 void* d_out, float* d_partial_out, float* d_partial_max,
                                                 float* d_partial_weight_sum, size_t query_len,
                                                 size_t kv_cache_len, size_t start_pos, size_t num_heads,
                                                 size_t num_kv_heads, size_t head_dim, size_t q_stride,
                                                 size_t kv_stride, b2_stream_t stream,
                                                 b2_graph_node_t* attention_node, b2_graph_node_t* merge_node) {
    (void)start_pos;  // decode attends [0, kv_cache_len); the reference ignores it too (:943)
    (void)q_stride;   // the single decode query is one packed [num_heads][head_dim] vector
    return launch_decode(d_q, d_k_cache, d_v_cache, d_out, d_partial_out, d_partial_max, d_partial_weight_sum,
                         query_len, kv_cache_len, num_heads, num_kv_heads, head_dim, kv_stride, stream,
                         attention_node, merge_node);
}

extern "C" int b2_launch_causal_attention_decode_vectorized(
    const void* d_q, const void* d_k_cache, const void* d_v_cache, void* d_out, float* d_partial_out,
    float* d_partial_max, float* d_partial_weight_sum, size_t query_len, size_t kv_cache_len, size_t start_pos,
    size_t num_heads, size_t num_kv_heads, size_t head_dim, size_t q_stride, size_t kv_stride, b2_stream_t stream,
    b2_graph_node_t* attention_node, b2_graph_node_t* merge_node) {
    return b2_launch_causal_attention_decode(d_q, d_k_cache, d_v_cache, d_out, d_partial_out, d_partial_max,
                                             d_partial_weight_sum, query_len, kv_cache_len, start_pos, num_heads,
                                             num_kv_heads, head_dim, q_stride, kv_stride, stream, attention_node,
                                             merge_node);
}

extern "C" int b2_update_causal_attention_decode_node(b2_graph_exec_t graph_exec, b2_graph_node_t node_handle,
                                                      size_t kv_cache_len) {
    if (graph_exec == nullptr || kv_cache_len == 0) return B2_ERR_INVALID_ARG;
    const size_t chunks = (kv_cache_len + kChunk - 1) / kChunk;
    if (chunks > 65535) return B2_ERR_UNSUPPORTED;
    cudaGraphNode_t node = reinterpret_cast<cudaGraphNode_t>(node_handle);
    cudaKernelNodeParams params{};
    const int st = node_kernel_params(node, kSplitKernels, 2, &params);
    if (st != B2_OK) return st;
    DecodeArgs a = *static_cast<const DecodeArgs*>(params.kernelParams[0]);
    a.kv_len = static_cast<uint32_t>(kv_cache_len);
    a.num_chunks = static_cast<uint32_t>(chunks);
    void* args[1] = {&a};
    params.kernelParams = args;
    params.extra = nullptr;
    params.gridDim.y = static_cast<unsigned>(chunks);
    return cuda_status(cudaGraphExecKernelNodeSetParams(reinterpret_cast<cudaGraphExec_t>(graph_exec), node, &params));
}

extern "C" int b2_update_merge_attention_decode_node(b2_graph_exec_t graph_exec, b2_graph_node_t node_handle,
                                                     size_t kv_cache_len) {
    if (graph_exec == nullptr || kv_cache_len == 0) return B2_ERR_INVALID_ARG;
    const size_t chunks = (kv_cache_len + kChunk - 1) / kChunk;
    if (chunks > 65535) return B2_ERR_UNSUPPORTED;
    cudaGraphNode_t node = reinterpret_cast<cudaGraphNode_t>(node_handle);
    cudaKernelNodeParams params{};
    const int st = node_kernel_params(node, kMergeKernels, 1, &params);
    if (st != B2_OK) return st;
    MergeArgs m = *static_cast<const MergeArgs*>(params.kernelParams[0]);
    m.num_chunks = static_cast<uint32_t>(chunks);
    void* args[1] = {&m};
    params.kernelParams = args;
    params.extra = nullptr;
    return cuda_status(cudaGraphExecKernelNodeSetParams(reinterpret_cast<cudaGraphExec_t>(graph_exec), node, &params));
}

extern "C" int b2_launch_merge_attention_decode_tiled(const float* d_partial_output, const float* d_partial_max,
                                                      const float* d_partial_weight_sum, void* d_out,
                                                      size_t num_heads, size_t num_kv_chunks, size_t head_dim,
                                                      b2_stream_t stream) {
    if (num_heads == 0 || num_kv_chunks == 0 || head_dim == 0) return B2_NOTHING_TO_DO;
    if (!d_partial_output || !d_partial_max || !d_partial_weight_sum || !d_out) return B2_ERR_INVALID_ARG;
    if (num_heads > 65535 || num_kv_chunks > 0xffffffffull || head_dim > 4096) return B2_ERR_UNSUPPORTED;
    return launch_merge(d_partial_output, d_partial_max, d_partial_weight_sum, static_cast<__half*>(d_out),
                        static_cast<uint32_t>(num_heads), static_cast<uint32_t>(num_kv_chunks),
                        static_cast<uint32_t>(head_dim), reinterpret_cast<cudaStream_t>(stream));
}
