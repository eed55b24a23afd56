// Split-KV flash-decode for sm_100a: split stage + merge.
//
// Restates src/kernels/causal_attention.hip.cpp of the reference:
//   causal_attention_decode{,_vectorized} (:493-595, :619-716)  partial
//       (o, m, l) per (head, split) over one query token
//   merge_attention_decode (:719-838)  M = max m_s, L = sum e^(m_s-M) l_s,
//       out = sum e^(m_s-M) o_s / L
//   launchers (:840-972), graph-node patchers (:975-1026)
// Partials keep the reference's meaning (o unnormalised fp32, m in natural-log
// units of q.k/sqrt(d), l = sum e^(s-m)) in a compact [H][S][d] / [H][S]
// layout, S = number of splits <= ceil(kv_len / KV_CHUNK), so they always fit
// the workspace the reference sizes from KV_CHUNK.
//
// Split kernels (all with one query token, kv heads x group query heads):
//
// * decode_split_tma_kernel -- head_dim 128, packed cache rows
//   (kv_stride = num_kv_heads * 128), 1/2/4/8 KV heads, group <= 8.
//   Persistent: one CTA per SM, S = min(#SMs, ceil(kv_len / 256)) contiguous
//   token ranges. A producer warp streams 16-token tiles of K and V (all KV
//   heads of a token are one contiguous row) into a ring of shared-memory
//   stages with 1-D TMA bulk copies (cp.async.bulk + mbarrier complete_tx,
//   L2 evict-first); 8 consumer warps (KV head x tile parity) turn each tile
//   into scores and P.V on the tensor cores. Every KV byte is read once for
//   all query heads of its group.
// * decode_split_mma_kernel -- head_dim 128, any 16-byte aligned row stride:
//   one CTA per (KV head, 256-token chunk), 16-byte loads straight into MMA
//   fragments.
// * decode_split_simt_kernel -- everything else (any head_dim, stride,
//   alignment), one CTA per (query head, chunk).
//
// Tensor-core tile math (both MMA kernels), mma.sync m16n8k16 f16->f32 with
// tokens as M:   S^T[16 tok x 8 heads] = K[16 x 128] . Q^T   (8 MMAs)
//                O^T[128 x 8 heads]   += V^T[128 x 16] . P^T   (8 MMAs)
// The contraction order over head_dim is permuted so that every A/B fragment
// is a whole 16-byte load of K, V or Q; P^T is re-distributed with 4
// shuffles; the online softmax runs in the log2 domain on the S fragments.
//
// Merge: one CTA per (head, 64 output dims), launched with programmatic
// dependent launch so its launch overlaps the split kernel's tail.
#include <math.h>

#include <atomic>
#include <mutex>

#include "b2_common.cuh"
#include "b2_ptx.cuh"

namespace b2 {
namespace {

constexpr int kChunk = 256;  // KV_CHUNK
constexpr int kTile = 16;    // tokens per MMA tile
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr uint32_t kNoCap = 0xffffffffu;

// TMA kernel shape
constexpr int kTmaConsumers = 8;
constexpr int kTmaThreads = (kTmaConsumers + 1) * 32;
constexpr uint32_t kTmaSmemBudget = 192 * 1024;

struct DecodeArgs {
    const __half* q;
    const __half* k;
    const __half* v;
    float* po;
    float* pm;
    float* pl;
    uint64_t kv_stride;   // elements between cached tokens
    uint32_t kv_len;      // patched by b2_update_causal_attention_decode_node
    uint32_t splits_cap;  // splits = min(splits_cap, ceil(kv_len / KV_CHUNK))
    uint32_t num_heads;
    uint32_t num_kv_heads;
    uint32_t head_dim;
    uint32_t group;
    float scale_log2;     // log2(e) / sqrt(head_dim)
    float scale;          // 1 / sqrt(head_dim)
    // Graph-static variant: kv_len = clamp(*kv_len_dev + kv_len_bias, 0,
    // max_kv_len), read at launch.
    const int32_t* kv_len_dev;
    int32_t kv_len_bias;
    uint32_t max_kv_len;
    uint32_t stages;      // TMA kernel: ring depth
};

struct MergeArgs {
    const float* po;
    const float* pm;
    const float* pl;
    __half* out;
    uint32_t num_heads;
    uint32_t head_dim;
    uint32_t kv_len;      // patched by b2_update_merge_attention_decode_node
    uint32_t splits_cap;
    const int32_t* kv_len_dev;
    int32_t kv_len_bias;
    uint32_t max_kv_len;
    // Explicit partial addressing (strided merge); when `strided` is 0 the
    // compact [H][S][d] / [H][S] layout is used.
    uint32_t strided;
    uint32_t strided_chunks;
    uint64_t o_head, o_chunk, ml_head, ml_chunk;
    // Rank-partial output instead of out: o = sum e^(m_s-M) o_s (fp32),
    // M (natural log units) and L = sum e^(m_s-M) l_s per head.
    float* rank_o;
    float* rank_m;
    float* rank_l;
};

struct Extent {
    uint32_t kv_len;
    uint32_t splits;
};

template <class A>
__device__ __forceinline__ Extent decode_extent(const A& a) {
    uint32_t len = a.kv_len;
    if (a.kv_len_dev != nullptr) {
        int64_t n = static_cast<int64_t>(__ldg(a.kv_len_dev)) + a.kv_len_bias;
        n = n < 0 ? 0 : (n > a.max_kv_len ? a.max_kv_len : n);
        len = static_cast<uint32_t>(n);
    }
    const uint32_t chunks = (len + kChunk - 1) / kChunk;
    return {len, min(chunks, a.splits_cap)};
}

// Token range [begin, end) of split s when kv_len tokens are cut into
// `splits` ranges of a 16-token multiple.
__device__ __forceinline__ void split_range(uint32_t kv_len, uint32_t splits, uint32_t s, uint32_t& begin,
                                            uint32_t& end) {
    uint32_t per = (kv_len + splits - 1) / splits;
    per = (per + kTile - 1) / kTile * kTile;
    begin = min(s * per, kv_len);
    end = min(begin + per, kv_len);
}

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

// Online-softmax state of one warp: heads 2t, 2t+1 of the group (lane = 4g+t),
// O^T fragments for 8 row tiles of head_dim.
struct WarpState {
    float o[8][4];
    float m0, m1, l0, l1;
};

__device__ __forceinline__ void state_init(WarpState& st) {
#pragma unroll
    for (int i = 0; i < 8; ++i) st.o[i][0] = st.o[i][1] = st.o[i][2] = st.o[i][3] = 0.f;
    st.m0 = st.m1 = -INFINITY;
    st.l0 = st.l1 = 0.f;
}

// Q fragments (B of the score MMA) for the heads of one GQA group.
__device__ __forceinline__ void load_q_frags(const __half* q, uint32_t kvh, uint32_t group, int g, int t,
                                             uint32_t (&qf)[8][2]) {
    if (static_cast<uint32_t>(g) < group) {
        const __half* qrow = q + static_cast<uint64_t>(kvh * group + g) * 128;
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
}

// One 16-token tile. ka/kb: K rows g and g+8 (4 x 16 B at 32j + 8t); va:
// V rows 2t, 2t+1, 2t+8, 2t+9 (2 x 16 B at 64b + 8g); rows at or past
// `valid` must be zero in ka/kb/va and are masked out of the softmax.
__device__ __forceinline__ void tile_update(WarpState& st, const uint4 (&ka)[4], const uint4 (&kb)[4],
                                            const uint4 (&va)[4][2], const uint32_t (&qf)[8][2], int g, int t,
                                            uint32_t valid, float scale_log2) {
    float s[4] = {0.f, 0.f, 0.f, 0.f};
    float s2[4] = {0.f, 0.f, 0.f, 0.f};  // two accumulation chains halve the MMA latency
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        if (j & 1) {
            mma16816(s2, ka[j].x, kb[j].x, ka[j].y, kb[j].y, qf[2 * j][0], qf[2 * j][1]);
            mma16816(s2, ka[j].z, kb[j].z, ka[j].w, kb[j].w, qf[2 * j + 1][0], qf[2 * j + 1][1]);
        } else {
            mma16816(s, ka[j].x, kb[j].x, ka[j].y, kb[j].y, qf[2 * j][0], qf[2 * j][1]);
            mma16816(s, ka[j].z, kb[j].z, ka[j].w, kb[j].w, qf[2 * j + 1][0], qf[2 * j + 1][1]);
        }
    }
    const bool ok_a = static_cast<uint32_t>(g) < valid, ok_b = static_cast<uint32_t>(g + 8) < valid;
    s[0] = ok_a ? (s[0] + s2[0]) * scale_log2 : -INFINITY;
    s[1] = ok_a ? (s[1] + s2[1]) * scale_log2 : -INFINITY;
    s[2] = ok_b ? (s[2] + s2[2]) * scale_log2 : -INFINITY;
    s[3] = ok_b ? (s[3] + s2[3]) * scale_log2 : -INFINITY;

    float mx0 = fmaxf(s[0], s[2]), mx1 = fmaxf(s[1], s[3]);
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
    }
    const float mn0 = fmaxf(st.m0, mx0), mn1 = fmaxf(st.m1, mx1);
    const float al0 = exp2f(st.m0 - mn0), al1 = exp2f(st.m1 - mn1);
    const float p0 = exp2f(s[0] - mn0), p1 = exp2f(s[1] - mn1);
    const float p2 = exp2f(s[2] - mn0), p3 = exp2f(s[3] - mn1);
    st.l0 = fmaf(st.l0, al0, p0 + p2);
    st.l1 = fmaf(st.l1, al1, p1 + p3);
    st.m0 = mn0;
    st.m1 = mn1;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        st.o[i][0] *= al0;
        st.o[i][1] *= al1;
        st.o[i][2] *= al0;
        st.o[i][3] *= al1;
    }

    // P^T fragments: column (head) g, tokens {2t,2t+1} and {2t+8,2t+9}.
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

#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
        const int b = mt >> 2, q = mt & 3;
        const uint32_t w0 = word(va[0][b], q), w1 = word(va[1][b], q);
        const uint32_t w2 = word(va[2][b], q), w3 = word(va[3][b], q);
        mma16816(st.o[mt], __byte_perm(w0, w1, 0x5410u), __byte_perm(w0, w1, 0x7632u),
                 __byte_perm(w2, w3, 0x5410u), __byte_perm(w2, w3, 0x7632u), pb0, pb1);
    }
}

// Reduce the per-lane row sums over the 8 token rows (lanes with equal t).
__device__ __forceinline__ void state_finish(WarpState& st) {
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
        st.l0 += __shfl_xor_sync(0xffffffffu, st.l0, off);
        st.l1 += __shfl_xor_sync(0xffffffffu, st.l1, off);
    }
}

// Store one warp's state into slot `slot`: m/l [slot][8 heads], o [slot][8][128].
__device__ __forceinline__ void state_to_smem(const WarpState& st, int slot, float* sm_m, float* sm_l, float* sm_o,
                                              int g, int t) {
    if (g == 0) {
        sm_m[slot * 8 + 2 * t] = st.m0;
        sm_m[slot * 8 + 2 * t + 1] = st.m1;
        sm_l[slot * 8 + 2 * t] = st.l0;
        sm_l[slot * 8 + 2 * t + 1] = st.l1;
    }
    float* o = sm_o + slot * 8 * 128;
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
        const int d = 64 * (mt >> 2) + 8 * g + 2 * (mt & 3);
        o[(2 * t) * 128 + d] = st.o[mt][0];
        o[(2 * t + 1) * 128 + d] = st.o[mt][1];
        o[(2 * t) * 128 + d + 1] = st.o[mt][2];
        o[(2 * t + 1) * 128 + d + 1] = st.o[mt][3];
    }
}

// Combine `nslots` warp states of one KV head (slots first, first+stride, ...)
// into the partial of (head kvh*group + hh, split), idx = hh*128 + d.
__device__ __forceinline__ void combine_write(const float* sm_m, const float* sm_l, const float* sm_o, int first,
                                              int stride, int nslots, uint32_t kvh, uint32_t group, uint32_t split,
                                              uint32_t splits, float* po, float* pm, float* pl, uint32_t idx) {
    const uint32_t hh = idx >> 7, d = idx & 127;
    float M = -INFINITY;
    for (int w = 0; w < nslots; ++w) M = fmaxf(M, sm_m[(first + w * stride) * 8 + hh]);
    float L = 0.f, O = 0.f;
    for (int w = 0; w < nslots; ++w) {
        const int sl = first + w * stride;
        const float m = sm_m[sl * 8 + hh];
        const float sc = (m == -INFINITY) ? 0.f : exp2f(m - M);
        L = fmaf(sc, sm_l[sl * 8 + hh], L);
        O = fmaf(sc, sm_o[(sl * 8 + hh) * 128 + d], O);
    }
    const uint64_t state = static_cast<uint64_t>(kvh * group + hh) * splits + split;
    po[state * 128 + d] = O;
    if (d == 0) {
        pm[state] = M == -INFINITY ? -INFINITY : M * kLn2;
        pl[state] = L;
    }
}

// ---------------------------------------------------------------------------
// Persistent TMA split kernel. grid = min(#SMs, chunks), block = 9 warps.
__global__ void __launch_bounds__(kTmaThreads, 1) decode_split_tma_kernel(const DecodeArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const Extent ext = decode_extent(a);
    const uint32_t split = blockIdx.x;
    pdl_launch_dependents();
    if (split >= ext.splits) return;
    uint32_t begin, end;
    split_range(ext.kv_len, ext.splits, split, begin, end);

    const uint32_t KVH = a.num_kv_heads;
    const uint32_t row_bytes = KVH * 256;            // one token, all KV heads
    const uint32_t tile_bytes = kTile * row_bytes;   // per K (and per V)
    const uint32_t stages = a.stages;
    uint8_t* ring = smem;                            // [stages][K tile | V tile]
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + stages * 2 * tile_bytes);
    uint64_t* empty = full + stages;
    const uint32_t ntiles = (end - begin + kTile - 1) / kTile;
    const uint32_t npar = kTmaConsumers / KVH;       // consumer warps per KV head

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], KVH);
        }
        fence_mbarrier_init();
    }
    __syncthreads();

    bool ok = true;
    WarpState st;
    state_init(st);
    if (warp == kTmaConsumers) {
        // ---- producer
        if (lane == 0) {
            const uint64_t policy = l2_evict_first_policy();
            const uint8_t* kg = reinterpret_cast<const uint8_t*>(a.k);
            const uint8_t* vg = reinterpret_cast<const uint8_t*>(a.v);
            uint32_t issued = 0;
            for (uint32_t i = 0; i < ntiles; ++i) {
                const uint32_t s = i % stages, round = i / stages;
                if (round > 0 && !(ok = mbar_wait(&empty[s], (round - 1) & 1))) break;
                const uint32_t t0 = begin + i * kTile;
                const uint32_t rows = min(static_cast<uint32_t>(kTile), end - t0);
                const uint32_t bytes = rows * row_bytes;
                uint8_t* st = ring + s * 2 * tile_bytes;
                mbar_arrive_expect_tx(&full[s], 2 * bytes);
                bulk_g2s(st, kg + static_cast<uint64_t>(t0) * row_bytes, bytes, &full[s], policy);
                bulk_g2s(st + tile_bytes, vg + static_cast<uint64_t>(t0) * row_bytes, bytes, &full[s], policy);
                issued = i + 1;
            }
            // Never leave the CTA with copies in flight into its shared memory:
            // the last `stages` issued tiles are awaited (immediate when the
            // consumers already drained them).
            const uint32_t first = issued > stages ? issued - stages : 0;
            for (uint32_t i = first; i < issued; ++i) (void)mbar_wait(&full[i % stages], (i / stages) & 1);
        }
    } else {
        // ---- consumers: warp = KV head (warp % KVH) x tile parity (warp / KVH)
        const uint32_t kvh = warp % KVH, par = warp / KVH;
        const int g = lane >> 2, t = lane & 3;
        uint32_t qf[8][2];
        load_q_frags(a.q, kvh, a.group, g, t, qf);
        const uint4 zero4 = make_uint4(0u, 0u, 0u, 0u);
        for (uint32_t i = par; i < ntiles; i += npar) {
            const uint32_t s = i % stages, round = i / stages;
            if (!mbar_wait(&full[s], round & 1)) {
                ok = false;
                break;
            }
            const uint8_t* kt = ring + s * 2 * tile_bytes + kvh * 256;
            const uint8_t* vt = kt + tile_bytes;
            const uint32_t valid = min(static_cast<uint32_t>(kTile), end - (begin + i * kTile));
            uint4 ka[4], kb[4], va[4][2];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                ka[j] = static_cast<uint32_t>(g) < valid
                            ? *reinterpret_cast<const uint4*>(kt + g * row_bytes + (32 * j + 8 * t) * 2)
                            : zero4;
                kb[j] = static_cast<uint32_t>(g + 8) < valid
                            ? *reinterpret_cast<const uint4*>(kt + (g + 8) * row_bytes + (32 * j + 8 * t) * 2)
                            : zero4;
            }
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const uint32_t row = 2 * t + (r & 1) + (r >> 1) * 8;
#pragma unroll
                for (int b = 0; b < 2; ++b)
                    va[r][b] = row < valid
                                   ? *reinterpret_cast<const uint4*>(vt + row * row_bytes + (64 * b + 8 * g) * 2)
                                   : zero4;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            tile_update(st, ka, kb, va, qf, g, t, valid, a.scale_log2);
        }
        state_finish(st);
    }
    // All ring reads and copies are done: reuse the ring for the combine.
    __syncthreads();
    float* sm_m = reinterpret_cast<float*>(ring);
    float* sm_l = sm_m + kTmaConsumers * 8;
    float* sm_o = sm_l + kTmaConsumers * 8;
    if (warp < kTmaConsumers) state_to_smem(st, warp, sm_m, sm_l, sm_o, lane >> 2, lane & 3);
    __syncthreads();
    // Slots of KV head h are h, h + KVH, ...: combine and write the partials.
    for (uint32_t idx = threadIdx.x; idx < KVH * a.group * 128; idx += kTmaThreads) {
        const uint32_t h = idx / (a.group * 128);
        combine_write(sm_m, sm_l, sm_o, static_cast<int>(h), static_cast<int>(KVH), static_cast<int>(npar), h,
                      a.group, split, ext.splits, a.po, a.pm, a.pl, idx - h * a.group * 128);
    }
    if (!ok) atomicOr(&g_device_error, kErrWaitTimeout);
}

// ---------------------------------------------------------------------------
// Register-path split kernel. grid = (num_kv_heads, chunks), block = 128.
__global__ void __launch_bounds__(128) decode_split_mma_kernel(const DecodeArgs a) {
    __shared__ float sm_m[4 * 8];
    __shared__ float sm_l[4 * 8];
    __shared__ float sm_o[4 * 8 * 128];
    const uint32_t kvh = blockIdx.x;
    const uint32_t chunk = blockIdx.y;
    const Extent ext = decode_extent(a);
    pdl_launch_dependents();
    if (chunk >= ext.splits) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const uint32_t c0 = chunk * kChunk;
    const uint32_t c1 = min(c0 + kChunk, ext.kv_len);
    const uint32_t w0 = c0 + warp * (kChunk / 4);
    const uint32_t w1 = min(w0 + kChunk / 4, c1);

    uint32_t qf[8][2];
    load_q_frags(a.q, kvh, a.group, g, t, qf);
    WarpState st;
    state_init(st);
    const __half* kbase = a.k + static_cast<uint64_t>(kvh) * 128;
    const __half* vbase = a.v + static_cast<uint64_t>(kvh) * 128;
    const uint64_t stride = a.kv_stride;
    const uint4 zero4 = make_uint4(0u, 0u, 0u, 0u);
    for (uint32_t tb = w0; tb < w1; tb += kTile) {
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
        tile_update(st, ka, kb, va, qf, g, t, w1 - tb, a.scale_log2);
    }
    state_finish(st);
    state_to_smem(st, warp, sm_m, sm_l, sm_o, g, t);
    __syncthreads();
    for (uint32_t idx = threadIdx.x; idx < a.group * 128; idx += blockDim.x)
        combine_write(sm_m, sm_l, sm_o, 0, 1, 4, kvh, a.group, chunk, ext.splits, a.po, a.pm, a.pl, idx);
}

// ---------------------------------------------------------------------------
// SIMT split kernel for any head_dim / stride / alignment.
// grid = (num_heads, chunks), block = 128.
__global__ void __launch_bounds__(128) decode_split_simt_kernel(const DecodeArgs a) {
    __shared__ float scores[kChunk];
    __shared__ float red[4];
    const uint32_t h = blockIdx.x;
    const uint32_t chunk = blockIdx.y;
    const Extent ext = decode_extent(a);
    pdl_launch_dependents();
    if (chunk >= ext.splits) return;
    const uint32_t kvh = h / a.group;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t c0 = chunk * kChunk;
    const uint32_t c1 = min(c0 + kChunk, ext.kv_len);
    const uint32_t n = c1 - c0;
    const __half* qrow = a.q + static_cast<uint64_t>(h) * a.head_dim;

    for (uint32_t i = warp; i < n; i += 4) {
        const __half* krow =
            a.k + static_cast<uint64_t>(c0 + i) * a.kv_stride + static_cast<uint64_t>(kvh) * a.head_dim;
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
    const uint64_t state = static_cast<uint64_t>(h) * ext.splits + chunk;
    for (uint32_t e = threadIdx.x; e < a.head_dim; e += blockDim.x) {
        float acc = 0.f;
        for (uint32_t i = 0; i < n; ++i) {
            const __half* vrow =
                a.v + static_cast<uint64_t>(c0 + i) * a.kv_stride + static_cast<uint64_t>(kvh) * a.head_dim;
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
// over splits (four in flight per warp), lanes over two output dimensions.
__global__ void __launch_bounds__(256) merge_partials_kernel(const MergeArgs a) {
    __shared__ float red[8];
    __shared__ float acc_s[8][64];
    pdl_wait_primary();
    const uint32_t h = blockIdx.x;
    const uint32_t d0 = blockIdx.y * 64;
    const uint32_t d = a.head_dim;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint32_t n;
    uint64_t o_head, o_chunk, ml_head, ml_chunk;
    if (a.strided) {
        n = a.strided_chunks;
        o_head = a.o_head, o_chunk = a.o_chunk, ml_head = a.ml_head, ml_chunk = a.ml_chunk;
    } else {
        n = decode_extent(a).splits;
        o_head = static_cast<uint64_t>(n) * d, o_chunk = d, ml_head = n, ml_chunk = 1;
    }
    if (n == 0) {  // graph-static launch with an empty range: defined output
        for (uint32_t e = d0 + threadIdx.x; e < min(d0 + 64, d); e += blockDim.x) {
            if (a.rank_o)
                a.rank_o[static_cast<uint64_t>(h) * d + e] = 0.f;
            else
                a.out[static_cast<uint64_t>(h) * d + e] = __float2half_rn(0.f);
        }
        if (a.rank_o && blockIdx.y == 0 && threadIdx.x == 0) {
            a.rank_m[h] = -INFINITY;
            a.rank_l[h] = 0.f;
        }
        return;
    }
    const float* pm = a.pm + h * ml_head;
    const float* pl = a.pl + h * ml_head;
    const float* po = a.po + h * o_head;

    float mx = -INFINITY;
    for (uint32_t c = threadIdx.x; c < n; c += blockDim.x) mx = fmaxf(mx, pm[c * ml_chunk]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    mx = red[0];
#pragma unroll
    for (int w = 1; w < 8; ++w) mx = fmaxf(mx, red[w]);
    __syncthreads();

    float den = 0.f;
    for (uint32_t c = threadIdx.x; c < n; c += blockDim.x) {
        const float m = pm[c * ml_chunk];
        if (m != -INFINITY) den = fmaf(expf(m - mx), pl[c * ml_chunk], den);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) den += __shfl_xor_sync(0xffffffffu, den, off);
    if (lane == 0) red[warp] = den;
    __syncthreads();
    den = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) den += red[w];

    const uint32_t e0 = d0 + 2 * lane, e1 = e0 + 1;
    float s0 = 0.f, s1 = 0.f;
    uint32_t c = warp;
    for (; c + 24 < n; c += 32) {  // four independent splits per iteration
        float sc[4], x0[4], x1[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const uint32_t cc = c + 8 * u;
            const float m = pm[cc * ml_chunk];
            sc[u] = m == -INFINITY ? 0.f : expf(m - mx);
            const float* row = po + cc * o_chunk;
            x0[u] = e0 < d ? row[e0] : 0.f;
            x1[u] = e1 < d ? row[e1] : 0.f;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            s0 = fmaf(sc[u], x0[u], s0);
            s1 = fmaf(sc[u], x1[u], s1);
        }
    }
    for (; c < n; c += 8) {
        const float m = pm[c * ml_chunk];
        const float sc = m == -INFINITY ? 0.f : expf(m - mx);
        const float* row = po + c * o_chunk;
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
        if (a.rank_o)
            a.rank_o[static_cast<uint64_t>(h) * d + d0 + threadIdx.x] = s;
        else
            a.out[static_cast<uint64_t>(h) * d + d0 + threadIdx.x] = __float2half_rn(s / den);
    }
    if (a.rank_o && blockIdx.y == 0 && threadIdx.x == 0) {
        a.rank_m[h] = mx;
        a.rank_l[h] = den;
    }
}

__global__ void advance_position_kernel(int32_t* pos, int32_t delta) { *pos += delta; }

const void* const kSplitKernels[] = {
    reinterpret_cast<const void*>(decode_split_tma_kernel),
    reinterpret_cast<const void*>(decode_split_mma_kernel),
    reinterpret_cast<const void*>(decode_split_simt_kernel),
};
const void* const kMergeKernels[] = {reinterpret_cast<const void*>(merge_partials_kernel)};

// ---------------------------------------------------------------------------
// Host side

int device_sms() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
    return n;
}

// cudaFuncSetAttribute for the TMA kernel's dynamic shared memory, once per device.
int ensure_tma_smem() {
    static std::atomic<uint64_t> done_mask{0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return B2_ERR_CUDA;
    const uint64_t bit = 1ull << (dev & 63);
    if (done_mask.load() & bit) return B2_OK;
    const int st = cuda_status(cudaFuncSetAttribute(decode_split_tma_kernel,
                                                    cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                    static_cast<int>(kTmaSmemBudget + 1024)));
    if (st == B2_OK) done_mask.fetch_or(bit);
    return st;
}

int launch_merge_kernel(const MergeArgs& m, cudaStream_t stream) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(m.num_heads, (m.head_dim + 63) / 64);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, merge_partials_kernel, m);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        note_cuda_error(e);
        return B2_ERR_CUDA;
    }
    return launch_status();
}

MergeArgs merge_args_from(const DecodeArgs& a, __half* out, float* rank_o, float* rank_m, float* rank_l) {
    MergeArgs m{};
    m.po = a.po;
    m.pm = a.pm;
    m.pl = a.pl;
    m.out = out;
    m.num_heads = a.num_heads;
    m.head_dim = a.head_dim;
    m.kv_len = a.kv_len;
    m.splits_cap = a.splits_cap;
    m.kv_len_dev = a.kv_len_dev;
    m.kv_len_bias = a.kv_len_bias;
    m.max_kv_len = a.max_kv_len;
    m.rank_o = rank_o;
    m.rank_m = rank_m;
    m.rank_l = rank_l;
    return m;
}

// kv_len_dev == nullptr: host length kv_len (the reference's launchers).
// kv_len_dev != nullptr: graph-static launch sized for max_kv_len.
int launch_decode(const void* d_q, const void* d_k, const void* d_v, void* d_out, float* po, float* pm, float* pl,
                  size_t query_len, size_t kv_len, const int32_t* kv_len_dev, int32_t kv_len_bias,
                  size_t max_kv_len, size_t num_heads, size_t num_kv_heads, size_t head_dim, size_t kv_stride,
                  b2_stream_t stream_handle, b2_graph_node_t* attention_node, b2_graph_node_t* merge_node,
                  float* rank_o = nullptr, float* rank_m = nullptr, float* rank_l = nullptr) {
    // causal_attention.hip.cpp:860-866, :945-946: silent no-ops.
    const size_t extent = kv_len_dev ? max_kv_len : kv_len;
    if (query_len == 0 || extent == 0 || num_kv_heads == 0 || head_dim == 0) return B2_NOTHING_TO_DO;
    if (num_heads % num_kv_heads != 0) return B2_NOTHING_TO_DO;
    if (!d_q || !d_k || !d_v || (!d_out && !rank_o) || !po || !pm || !pl) return B2_ERR_INVALID_ARG;
    const size_t chunks = (extent + kChunk - 1) / kChunk;
    if (extent > 0x7fffffffull - kChunk || chunks > 65535 || num_heads > 65535 || head_dim > 4096)
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
    a.kv_len = static_cast<uint32_t>(extent);
    a.splits_cap = kNoCap;
    a.num_heads = static_cast<uint32_t>(num_heads);
    a.num_kv_heads = static_cast<uint32_t>(num_kv_heads);
    a.head_dim = static_cast<uint32_t>(head_dim);
    a.group = static_cast<uint32_t>(group);
    a.scale = 1.0f / sqrtf(static_cast<float>(head_dim));
    a.scale_log2 = a.scale * kLog2e;
    a.kv_len_dev = kv_len_dev;
    a.kv_len_bias = kv_len_bias;
    a.max_kv_len = static_cast<uint32_t>(max_kv_len);

    const bool mma_ok = head_dim == 128 && group <= 8 && aligned16(d_q) && aligned16(d_k) && aligned16(d_v) &&
                        (kv_stride % 8 == 0);
    const bool tma_ok = mma_ok && kv_stride == num_kv_heads * head_dim &&
                        (num_kv_heads == 1 || num_kv_heads == 2 || num_kv_heads == 4 || num_kv_heads == 8);
    int st;
    if (tma_ok) {
        if ((st = ensure_tma_smem()) != B2_OK) return st;
        const uint32_t stage_bytes = 2u * kTile * static_cast<uint32_t>(num_kv_heads) * 256u;
        a.stages = min(8u, kTmaSmemBudget / stage_bytes);
        a.splits_cap = static_cast<uint32_t>(device_sms());
        const uint32_t grid = static_cast<uint32_t>(chunks < a.splits_cap ? chunks : a.splits_cap);
        const size_t smem = a.stages * stage_bytes + 2 * a.stages * sizeof(uint64_t);
        decode_split_tma_kernel<<<grid, kTmaThreads, smem, stream>>>(a);
    } else if (mma_ok) {
        decode_split_mma_kernel<<<dim3(a.num_kv_heads, static_cast<uint32_t>(chunks)), 128, 0, stream>>>(a);
    } else {
        decode_split_simt_kernel<<<dim3(a.num_heads, static_cast<uint32_t>(chunks)), 128, 0, stream>>>(a);
    }
    st = launch_status();
    if (st != B2_OK) return st;
    if (attention_node) {
        cudaGraphNode_t n = nullptr;
        if ((st = last_captured_node(stream, &n)) != B2_OK) return st;
        *attention_node = reinterpret_cast<b2_graph_node_t>(n);
    }
    st = launch_merge_kernel(merge_args_from(a, static_cast<__half*>(d_out), rank_o, rank_m, rank_l), stream);
    if (st != B2_OK) return st;
    if (merge_node) {
        cudaGraphNode_t n = nullptr;
        if ((st = last_captured_node(stream, &n)) != B2_OK) return st;
        *merge_node = reinterpret_cast<b2_graph_node_t>(n);
    }
    return B2_OK;
}

}  // namespace

unsigned int device_error_decode() {
    unsigned int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v)) != cudaSuccess) return 0;
    return v;
}

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
                         query_len, kv_cache_len, nullptr, 0, 0, num_heads, num_kv_heads, head_dim, kv_stride, stream,
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
    if (chunks > 65535 || kv_cache_len > 0x7fffffffull - kChunk) return B2_ERR_UNSUPPORTED;
    cudaGraphNode_t node = reinterpret_cast<cudaGraphNode_t>(node_handle);
    cudaKernelNodeParams params{};
    const int st = node_kernel_params(node, kSplitKernels, 3, &params);
    if (st != B2_OK) return st;
    DecodeArgs a = *static_cast<const DecodeArgs*>(params.kernelParams[0]);
    if (a.kv_len_dev != nullptr) return B2_ERR_GRAPH;  // graph-static nodes need no patching
    a.kv_len = static_cast<uint32_t>(kv_cache_len);
    void* args[1] = {&a};
    params.kernelParams = args;
    params.extra = nullptr;
    if (params.func == kSplitKernels[0])
        params.gridDim.x = static_cast<unsigned>(chunks < a.splits_cap ? chunks : a.splits_cap);
    else
        params.gridDim.y = static_cast<unsigned>(chunks);
    return cuda_status(cudaGraphExecKernelNodeSetParams(reinterpret_cast<cudaGraphExec_t>(graph_exec), node, &params));
}

extern "C" int b2_update_merge_attention_decode_node(b2_graph_exec_t graph_exec, b2_graph_node_t node_handle,
                                                     size_t kv_cache_len) {
    if (graph_exec == nullptr || kv_cache_len == 0) return B2_ERR_INVALID_ARG;
    const size_t chunks = (kv_cache_len + kChunk - 1) / kChunk;
    if (chunks > 65535 || kv_cache_len > 0x7fffffffull - kChunk) return B2_ERR_UNSUPPORTED;
    cudaGraphNode_t node = reinterpret_cast<cudaGraphNode_t>(node_handle);
    cudaKernelNodeParams params{};
    const int st = node_kernel_params(node, kMergeKernels, 1, &params);
    if (st != B2_OK) return st;
    MergeArgs m = *static_cast<const MergeArgs*>(params.kernelParams[0]);
    if (m.kv_len_dev != nullptr || m.strided) return B2_ERR_GRAPH;
    m.kv_len = static_cast<uint32_t>(kv_cache_len);
    void* args[1] = {&m};
    params.kernelParams = args;
    params.extra = nullptr;
    return cuda_status(cudaGraphExecKernelNodeSetParams(reinterpret_cast<cudaGraphExec_t>(graph_exec), node, &params));
}

extern "C" int b2_launch_merge_partials_strided(const float* d_o, const float* d_m, const float* d_l, void* d_out,
                                                size_t num_heads, size_t num_chunks, size_t head_dim,
                                                size_t o_chunk_stride, size_t o_head_stride,
                                                size_t ml_chunk_stride, size_t ml_head_stride,
                                                b2_stream_t stream) {
    if (num_heads == 0 || num_chunks == 0 || head_dim == 0) return B2_NOTHING_TO_DO;
    if (!d_o || !d_m || !d_l || !d_out) return B2_ERR_INVALID_ARG;
    if (num_heads > 65535 || num_chunks > 0x7fffffffull || head_dim > 4096) return B2_ERR_UNSUPPORTED;
    MergeArgs m{};
    m.po = d_o;
    m.pm = d_m;
    m.pl = d_l;
    m.out = static_cast<__half*>(d_out);
    m.num_heads = static_cast<uint32_t>(num_heads);
    m.head_dim = static_cast<uint32_t>(head_dim);
    m.strided = 1;
    m.strided_chunks = static_cast<uint32_t>(num_chunks);
    m.o_head = o_head_stride;
    m.o_chunk = o_chunk_stride;
    m.ml_head = ml_head_stride;
    m.ml_chunk = ml_chunk_stride;
    return launch_merge_kernel(m, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int b2_launch_merge_attention_decode_tiled(const float* d_partial_output, const float* d_partial_max,
                                                      const float* d_partial_weight_sum, void* d_out,
                                                      size_t num_heads, size_t num_kv_chunks, size_t head_dim,
                                                      b2_stream_t stream) {
    return b2_launch_merge_partials_strided(d_partial_output, d_partial_max, d_partial_weight_sum, d_out, num_heads,
                                            num_kv_chunks, head_dim, head_dim, num_kv_chunks * head_dim, 1,
                                            num_kv_chunks, stream);
}

extern "C" int b2_launch_causal_attention_decode_devlen(const void* d_q, const void* d_k_cache,
                                                        const void* d_v_cache, void* d_out, float* d_partial_out,
                                                        float* d_partial_max, float* d_partial_weight_sum,
                                                        const int32_t* d_kv_len, int32_t kv_len_bias,
                                                        size_t max_kv_len, size_t num_heads, size_t num_kv_heads,
                                                        size_t head_dim, size_t kv_stride, b2_stream_t stream) {
    if (d_kv_len == nullptr) return B2_ERR_INVALID_ARG;
    return launch_decode(d_q, d_k_cache, d_v_cache, d_out, d_partial_out, d_partial_max, d_partial_weight_sum, 1, 0,
                         d_kv_len, kv_len_bias, max_kv_len, num_heads, num_kv_heads, head_dim, kv_stride, stream,
                         nullptr, nullptr);
}

extern "C" int b2_launch_decode_rank_partial_devlen(const void* d_q, const void* d_k_cache, const void* d_v_cache,
                                                    float* d_partial_out, float* d_partial_max,
                                                    float* d_partial_weight_sum, const int32_t* d_kv_len,
                                                    int32_t kv_len_bias, size_t max_kv_len, size_t num_heads,
                                                    size_t num_kv_heads, size_t head_dim, size_t kv_stride,
                                                    float* d_rank_o, float* d_rank_m, float* d_rank_l,
                                                    b2_stream_t stream) {
    if (d_kv_len == nullptr || !d_rank_o || !d_rank_m || !d_rank_l) return B2_ERR_INVALID_ARG;
    return launch_decode(d_q, d_k_cache, d_v_cache, nullptr, d_partial_out, d_partial_max, d_partial_weight_sum, 1,
                         0, d_kv_len, kv_len_bias, max_kv_len, num_heads, num_kv_heads, head_dim, kv_stride, stream,
                         nullptr, nullptr, d_rank_o, d_rank_m, d_rank_l);
}

extern "C" int b2_advance_position(int32_t* d_pos, int32_t delta, b2_stream_t stream) {
    if (d_pos == nullptr) return B2_ERR_INVALID_ARG;
    advance_position_kernel<<<1, 1, 0, reinterpret_cast<cudaStream_t>(stream)>>>(d_pos, delta);
    return launch_status();
}

// ---------------------------------------------------------------------------
// Flash-decode without a caller workspace.
//
// Some callers cannot hand this library scratch memory: a plugin host that
// passes only its input and output buffers, a serving process whose memory
// pool already owns all of HBM, or a latency-critical thread that must not
// call cudaMalloc (it can synchronise the whole device). For them the split-KV
// partials live in this fixed array instead. Every GPU that loads the library
// holds the array (B2_NOALLOC_SCRATCH_BYTES) until the process exits.
static __device__ __align__(256) float g_b2_noalloc_scratch[B2_NOALLOC_SCRATCH_BYTES / sizeof(float)];

namespace b2 {
namespace {

std::mutex g_noalloc_mutex;
float* g_noalloc_ptr[64] = {};  // device address of the array, per device

// Resolve the array's device address for the current device (once per device).
// The name is a host-side stand-in in host code; the kernels need the address.
int noalloc_scratch(float** out) {
    int dev = 0;
    const cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        note_cuda_error(e);
        return B2_ERR_CUDA;
    }
    if (dev < 0 || dev >= 64) return B2_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (g_noalloc_ptr[dev] == nullptr) {
        void* p = nullptr;
        const cudaError_t s = cudaGetSymbolAddress(&p, g_b2_noalloc_scratch);
        if (s != cudaSuccess || p == nullptr) {
            note_cuda_error(s);
            return B2_ERR_CUDA;
        }
        g_noalloc_ptr[dev] = static_cast<float*>(p);
    }
    *out = g_noalloc_ptr[dev];
    return B2_OK;
}

}  // namespace
}  // namespace b2

extern "C" int b2_launch_causal_attention_decode_noalloc(const void* d_q, const void* d_k_cache,
                                                         const void* d_v_cache, void* d_out, size_t query_len,
                                                         size_t kv_cache_len, size_t num_heads, size_t num_kv_heads,
                                                         size_t head_dim, size_t kv_stride, b2_stream_t stream) {
    if (query_len == 0 || kv_cache_len == 0 || num_kv_heads == 0 || head_dim == 0) return B2_NOTHING_TO_DO;
    if (num_heads % num_kv_heads != 0) return B2_NOTHING_TO_DO;
    if (!d_q || !d_k_cache || !d_v_cache || !d_out) return B2_ERR_INVALID_ARG;
    // The partials take at most the reference-sized workspace for this call.
    const size_t chunks = (kv_cache_len + kChunk - 1) / kChunk;
    const size_t need = b2_decode_workspace_floats(num_heads, head_dim, kv_cache_len);
    if (need > B2_NOALLOC_SCRATCH_BYTES / sizeof(float)) return B2_ERR_WORKSPACE;
    float* scratch = nullptr;
    const int st = noalloc_scratch(&scratch);
    if (st != B2_OK) return st;
    float* po = scratch;
    float* pm = po + num_heads * chunks * head_dim;
    float* pl = pm + num_heads * chunks;
    return launch_decode(d_q, d_k_cache, d_v_cache, d_out, po, pm, pl, query_len, kv_cache_len, nullptr, 0, 0,
                         num_heads, num_kv_heads, head_dim, kv_stride, stream, nullptr, nullptr);
}
