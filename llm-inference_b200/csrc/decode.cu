// Split-KV flash-decode for sm_100a: split stage + merge.
//
// Restates src/kernels/causal_attention.hip.cpp of the reference:
//   causal_attention_decode{,_vectorized} (:493-595, :619-716)  partial
//       (o, m, l) per (head, split) over one query token
//   merge_attention_decode (:719-838)  M = max m_s, L = sum e^(m_s-M) l_s,
//       out = sum e^(m_s-M) o_s / L
//   launchers (:840-972), graph-node patchers (:975-1026)
// Partials keep the reference's meaning (o = sum e^(s-m) v unnormalised fp32,
// l = sum e^(s-m), m in natural-log units of q.k/sqrt(d)) in a compact
// [H][S][d] / [H][S] layout, S = number of splits <= ceil(kv_len / KV_CHUNK),
// so they always fit the workspace the reference sizes from KV_CHUNK. One
// difference: m is the running max of a lazily rescaled online softmax and may
// trail the split's true max by less than 8 log2 units (o and l are relative
// to that m, so the merge algebra is unchanged and exact).
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
#include <string.h>

#include <atomic>
#include <mutex>

#include <cuda.h>

#include "b2_common.cuh"
#include "b2_ptx.cuh"
#include "decode_tile.cuh"
#include "tcgen05.cuh"

namespace b2 {
namespace {

constexpr uint32_t kNoCap = 0xffffffffu;

// TMA kernel shape
constexpr int kTmaConsumers = 12;  // 3 per KV head at 4 KV heads; 13 warps <= 4 per sub-partition
constexpr int kTmaThreads = (kTmaConsumers + 1) * 32;
constexpr uint32_t kTmaSmemBudget = 200 * 1024;

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
    uint32_t split_tokens;  // tokens per split before capping at the SM count (0 = KV_CHUNK)
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
    uint32_t split_tokens;  // as DecodeArgs::split_tokens
};

struct Extent {
    uint32_t kv_len;
    uint32_t splits;
};

template <class A>
__device__ __forceinline__ Extent decode_extent(const A& a) {
    uint32_t len = a.kv_len;
    if (a.kv_len_dev != nullptr) {
        // L2 load: the value may have been written by the kernel this one overlapped
        int64_t n = static_cast<int64_t>(__ldcg(a.kv_len_dev)) + a.kv_len_bias;
        n = n < 0 ? 0 : (n > a.max_kv_len ? a.max_kv_len : n);
        len = static_cast<uint32_t>(n);
    }
    const uint32_t per = a.split_tokens ? a.split_tokens : static_cast<uint32_t>(kChunk);
    const uint32_t chunks = (len + per - 1) / per;
    return {len, min(chunks, a.splits_cap)};
}

// ---------------------------------------------------------------------------
// Fused decode step (graph-static): extra inputs of decode_tma_kernel<true>.
constexpr uint32_t kMaxWorld = 8;       // ranks of one NVLink domain
constexpr uint32_t kExchangePitch = 132;  // exchange words per (slot, rank, head): o[128], m, l
struct StepExt {
    const __half* q_new;     // the new token's Q, not rotated, [H][128]
    const __half* k_new;     // its K (not rotated) [KVH][128]; nullptr = no append on this rank
    const __half* v_new;     // its V [KVH][128]
    __half* k_cache;         // writable views of the cache (the append target)
    __half* v_cache;
    const __half* cos;       // RoPE tables [table_rows][64]
    const __half* sin;
    const int32_t* pos_dev;  // RoPE position of the new token
    uint32_t rotate;         // 1 = RoPE, 0 = NoPE layer
    uint32_t table_rows;
    uint32_t* counters;      // [0] next unclaimed pool tile (0 at launch), [1] CTA arrivals (only
                             // grows), [2] the arrivals count at launch start
    __half* out;             // [H][128] fp16 result, or the rank partial below
    float* rank_o;
    float* rank_m;
    float* rank_l;
    // Cross-GPU exchange (world > 1): every rank's exchange buffer, mapped
    // into this process (peers[rank] is this rank's own); layout in
    // exchange_words(). epoch: this rank's count of exchanges so far.
    uint32_t world;
    uint32_t rank;
    uint32_t* epoch;
    float* peers[kMaxWorld];
};

constexpr uint32_t kStepMaxSplits = 256;      // partial slots in a fused-step workspace

// ---------------------------------------------------------------------------
// Persistent TMA split kernel. grid = min(#SMs, chunks), block = 13 warps: a
// producer warp streams 16-token K and V tiles with tensor-map copies
// (column block by column block, 128-byte swizzled) into a ring of stages;
// 12 consumer warps (KV head x tile parity) run the MMA tile math; the CTA's
// states are combined into one (o, m, l) partial per head.
// Static (reference launchers): CTA `split` owns a contiguous token range.
// kFused (the fused decode step): each CTA streams an even share of ~1/2 of
// the tiles, then claims tiles from a global counter, so all CTAs finish
// together whatever their DRAM share; Q is rotated in registers; consumer
// warp 0 of the last split appends the new token's K/V at row kv_len - 1
// before its producer copies the tile holding that row; splits
// 0 .. min(S, H) - 1 then merge the split partials (step_merge).
// ---- in-kernel merge of the fused step -------------------------------------

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void step_store(const StepExt& x, uint32_t h, uint32_t d, float o, float M, float L) {
    if (x.rank_o) {
        x.rank_o[h * 128 + d] = o;
        if (d == 0) {
            x.rank_m[h] = M;
            x.rank_l[h] = L;
        }
    } else {
        x.out[h * 128 + d] = __float2half_rn(o / L);
    }
}

// Exchange buffer of one rank: [2 slots][world][H][kExchangePitch] 8-byte
// words {value, exchange number}, then this rank's exchange counter. Rank r's
// partial of head h for exchange e sits in slot e & 1, row (r, h): o[0..127],
// m, l. Each value travels with its exchange number in one 8-byte store, so a
// reader polls the words themselves and needs no fence or flag (the writer
// cannot reuse a slot before every rank has read it: exchange e + 2 starts
// only after all ranks finished exchange e + 1, which follows their reads of e).
__host__ __device__ __forceinline__ uint64_t exchange_words(uint32_t world, uint32_t H) {
    return 2ull * world * H * kExchangePitch;
}

__device__ __forceinline__ void st_pair_sys(uint2* p, float v, uint32_t e) {
    asm volatile("st.relaxed.sys.global.v2.b32 [%0], {%1, %2};" ::"l"(p), "r"(__float_as_uint(v)), "r"(e)
                 : "memory");
}
__device__ __forceinline__ uint2 ld_pair_sys(const uint2* p) {
    uint2 v;
    asm volatile("ld.relaxed.sys.global.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p) : "memory");
    return v;
}

// Publish this rank's partial of head h for dims d0 .. d0 + nd - 1 (O of dim
// d0 + i held by thread i; M, L) to every rank, wait (bounded) for every
// rank's words of those dims for exchange e, and write the merged fp16
// output there. Threads 0 .. nd - 1 of the CTA take part (two CTAs may serve
// the two halves of a head: both write the same M and L words); returns
// false on a timeout.
__device__ __noinline__ bool step_exchange_head(const StepExt& x, uint32_t H, uint32_t h, uint32_t e, float O,
                                                float M, float L, uint32_t d0, uint32_t nd) {
    const uint32_t slot = e & 1, world = x.world;
    if (threadIdx.x >= nd) return true;
    const uint32_t d = d0 + threadIdx.x;
    for (uint32_t r = 0; r < world; ++r) {
        uint2* dst = reinterpret_cast<uint2*>(x.peers[r]) +
                     ((static_cast<uint64_t>(slot) * world + x.rank) * H + h) * kExchangePitch;
        st_pair_sys(dst + d, O, e);
        if (threadIdx.x == 0) {
            st_pair_sys(dst + 128, M, e);
            st_pair_sys(dst + 129, L, e);
        }
    }
    // every rank's words of this head, all loads in flight at once; only the
    // words that do not carry exchange e yet are read again
    const uint2* own = reinterpret_cast<const uint2*>(x.peers[x.rank]);
    const uint64_t t0 = global_timer_ns();
    float mv[kMaxWorld], lv[kMaxWorld], ov[kMaxWorld];
    uint2 wo[kMaxWorld], wm[kMaxWorld], wl[kMaxWorld];
#pragma unroll
    for (uint32_t r = 0; r < kMaxWorld; ++r) wo[r] = wm[r] = wl[r] = make_uint2(0u, e + 1u);  // not yet read
    bool ok = true;
    for (;;) {
        bool ready = true;
#pragma unroll
        for (uint32_t r = 0; r < kMaxWorld; ++r) {
            if (r < world) {
                const uint2* src = own + ((static_cast<uint64_t>(slot) * world + r) * H + h) * kExchangePitch;
                if (wo[r].y != e) wo[r] = ld_pair_sys(src + d);
                if (wm[r].y != e) wm[r] = ld_pair_sys(src + 128);
                if (wl[r].y != e) wl[r] = ld_pair_sys(src + 129);
            }
        }
#pragma unroll
        for (uint32_t r = 0; r < kMaxWorld; ++r)
            if (r < world) ready = ready && wo[r].y == e && wm[r].y == e && wl[r].y == e;
        if (ready) break;
        if (global_timer_ns() - t0 > kWaitBudgetNs) {
            ok = false;
            break;
        }
        __nanosleep(20);
    }
    if (!ok) {
        atomicOr(&g_device_error, kErrWaitTimeout);
        return false;
    }
#pragma unroll
    for (uint32_t r = 0; r < kMaxWorld; ++r) {
        ov[r] = __uint_as_float(wo[r].x);
        mv[r] = __uint_as_float(wm[r].x);
        lv[r] = __uint_as_float(wl[r].x);
    }
    float Mx = -INFINITY;
#pragma unroll
    for (uint32_t r = 0; r < kMaxWorld; ++r)
        if (r < world) Mx = fmaxf(Mx, mv[r]);
    float Ox = 0.f, Lx = 0.f;
#pragma unroll
    for (uint32_t r = 0; r < kMaxWorld; ++r) {
        if (r < world) {
            const float sc = mv[r] == -INFINITY ? 0.f : expf(mv[r] - Mx);
            Ox = fmaf(sc, ov[r], Ox);
            Lx = fmaf(sc, lv[r], Lx);
        }
    }
    x.out[h * 128 + d] = __float2half_rn(Lx > 0.f ? Ox / Lx : 0.f);
    return true;
}

__device__ __forceinline__ void step_write_empty(uint32_t H, const StepExt& x, uint32_t tid, uint32_t nthreads) {
    for (uint32_t i = tid; i < H * 128; i += nthreads) {
        if (x.rank_o) {
            x.rank_o[i] = 0.f;
            if ((i & 127) == 0) {
                x.rank_m[i >> 7] = -INFINITY;
                x.rank_l[i >> 7] = 0.f;
            }
        } else {
            x.out[i] = __float2half_rn(0.f);
        }
    }
}

__device__ __forceinline__ void red_add_release_gpu(uint32_t* p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Every CTA has written its partials -- o as [H][2 halves][S][64] (each half
// head's rows contiguous), m (natural log) and l as [H][S] -- and adds one to
// the arrival counter counters[1] with a release reduction; the counter only
// grows, and counters[2] holds its value at the start of the launch (`base`,
// read after the dependency wait). Splits r < R = min(S, 2H) merge the half
// heads r, r + R, ...: once the counter reaches base + S (acquire) the CTA
// copies the half head's S rows of 64 floats into shared memory with one
// bulk copy while its threads reduce the head's S maxima and weight sums,
// then 12 warps sum the weighted rows (two rows per warp step, four dims per
// lane, 24 interleaved row groups) and 64 threads add the group sums. Merging
// split 0 resets the tile counter and records base + S for the next launch
// (no other CTA reads either word again in this launch). The merging CTAs
// wait for CTAs that may start after them, which every launch can schedule:
// there is one CTA per SM and at most as many CTAs as SMs.
// epoch_next: the exchange number of this launch (world > 1).
__device__ __forceinline__ void step_merge(const DecodeArgs& a, const StepExt& x, uint32_t S, uint32_t split,
                                           uint8_t* smem, uint64_t* bar, uint32_t base, uint32_t epoch_next) {
    __shared__ uint32_t ok_s;
    __shared__ float red_s[2][kTmaThreads / 32];
    const uint32_t H = a.num_heads;
    const uint32_t R = min(S, 2 * H);
    // the CTA's partial stores happen before thread 0's release
    __syncthreads();
    const bool merger = split < R;
    if (threadIdx.x == 0) {
        red_add_release_gpu(&x.counters[1], 1u);
        if (merger) {
            uint32_t ok = 1u;
            const uint64_t t0 = global_timer_ns();
            while (ld_acquire_gpu(&x.counters[1]) - base < S) {
                if (global_timer_ns() - t0 > kWaitBudgetNs) {
                    atomicOr(&g_device_error, kErrWaitTimeout);
                    ok = 0u;
                    break;
                }
            }
            if (ok && split == 0) {
                x.counters[0] = 0u;
                x.counters[2] = base + S;
                if (x.world > 1) *x.epoch = epoch_next;
            }
            // the partials were written through the generic proxy; the bulk
            // copies below read them through the async proxy
            fence_proxy_async_global();
            ok_s = ok;
        }
    }
    if (!merger) return;
    __syncthreads();
    if (ok_s == 0u) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int kWarps = kTmaThreads / 32;
    float* rows = reinterpret_cast<float*>(smem);     // [S][64]
    float* wts = rows + static_cast<size_t>(S) * 64;  // [S]
    float* sums = wts + kStepMaxSplits;              // [24][64]
    const uint32_t sub = static_cast<uint32_t>(lane) >> 4, col4 = static_cast<uint32_t>(lane) & 15;
    uint32_t phase = 0;
    for (uint32_t item = split; item < 2 * H; item += R, phase ^= 1u) {
        const uint32_t h = item >> 1, d0 = (item & 1) * 64;
        if (threadIdx.x == 0) {
            mbar_arrive_expect_tx(bar, S * 256u);
            bulk_g2s_plain(rows, a.po + static_cast<uint64_t>(item) * S * 64, S * 256u, bar);
        }
        const uint32_t c = threadIdx.x;
        const float m = c < S ? __ldcg(a.pm + static_cast<uint64_t>(h) * S + c) : -INFINITY;
        const float l = c < S ? __ldcg(a.pl + static_cast<uint64_t>(h) * S + c) : 0.f;
        float v = m;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
        if (lane == 0) red_s[0][warp] = v;
        __syncthreads();
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) M = fmaxf(M, red_s[0][w]);
        const float wt = m == -INFINITY ? 0.f : expf(m - M);
        if (c < S) wts[c] = wt;
        v = wt * l;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
        if (lane == 0) red_s[1][warp] = v;
        // every thread must see the bulk copy land before the rows are read;
        // after a timeout (error word already set) the CTA leaves the loop
        // together instead of summing rows that never arrived or reusing the
        // buffer and barrier under a copy that may still be in flight
        if (!__syncthreads_and(mbar_wait(bar, phase) ? 1 : 0)) return;
        float L = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) L += red_s[1][w];
        if (warp < 12) {
            // row group g = 2 * warp + sub sums rows g, g + 24, ... for dims 4 * col4 .. + 3
            const uint32_t g = 2 * static_cast<uint32_t>(warp) + sub;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
            for (uint32_t cc = g; cc < S; cc += 24) {
                const float wc = wts[cc];
                const float4 r4 = reinterpret_cast<const float4*>(rows + cc * 64)[col4];
                acc.x = fmaf(wc, r4.x, acc.x);
                acc.y = fmaf(wc, r4.y, acc.y);
                acc.z = fmaf(wc, r4.z, acc.z);
                acc.w = fmaf(wc, r4.w, acc.w);
            }
            reinterpret_cast<float4*>(sums + g * 64)[col4] = acc;
        }
        __syncthreads();
        if (threadIdx.x < 64) {
            const uint32_t d = threadIdx.x;
            float O = 0.f;
#pragma unroll
            for (int g = 0; g < 24; ++g) O += sums[g * 64 + d];
            if (x.world <= 1) step_store(x, h, d0 + d, O, M, L);
            else (void)step_exchange_head(x, H, h, epoch_next, O, M, L, d0, 64);
        }
        __syncthreads();  // rows, weights and sums are reused by the next item
    }
}

constexpr uint32_t kAppendBarrier = 1;  // named barrier: appending consumer warp -> producer warp
constexpr uint32_t kPrefetchTiles = 4;  // tiles per CTA warmed in L2 before the dependency wait
constexpr uint32_t kPostPrefetchTiles = 2;  // and the next ones, right after it

// Fused kernel: tiles dealt out evenly to each split before the claimed pool
// (half of them: at 64K a larger pool let the CTAs finish 0.2 us closer).
__device__ __forceinline__ uint32_t fused_share(uint32_t total_tiles, uint32_t splits) {
    return (total_tiles / 2) / splits;
}

__device__ __forceinline__ bool split_index_ok(const Extent& e, uint32_t split) { return split < e.splits; }

// The first tiles a split streams (up to kPrefetchTiles): its own range
// (static) or its even share (fused).
__device__ __forceinline__ void own_tiles(const Extent& e, uint32_t split, bool fused, uint32_t rows,
                                          uint32_t& first, uint32_t& count) {
    if (fused) {
        const uint32_t per = fused_share((e.kv_len + rows - 1) / rows, e.splits);
        first = split * per;
        count = min(per, kPrefetchTiles);
    } else {
        uint32_t b, en;
        split_range(e.kv_len, e.splits, split, b, en);
        first = b / kTile;
        // whole tiles only: a partial last tile could run past the cache
        count = min((en - b) / kTile, kPrefetchTiles);
    }
}

__device__ __forceinline__ uint8_t* stg_of(uint8_t* ring, uint32_t s, uint32_t tile_bytes) {
    return ring + s * 2 * tile_bytes;
}

// Combine of one split's consumer warp states into its partial. The warps of
// KV head h are h, h + KVH, ... (one per tile parity); warps of parity >= 1
// leave their state in shared memory `sm` and the parity-0 warp of each KV
// head folds them into its own registers -- every lane reads the fragment
// positions it holds itself -- and writes the partial from registers: po
// [head][splits][128] (kHalves: [head][2][splits][64], the fused step's
// merge layout), pm (natural-log max) and pl [head][splits]. Every thread of
// the CTA calls it (one barrier when npar > 1).
template <uint32_t KVH, bool kHalves>
__device__ __forceinline__ void combine_split(WarpState& st, uint32_t warp, uint32_t lane, float* sm, uint32_t group,
                                              uint32_t split, uint32_t splits, float* po, float* pm, float* pl) {
    constexpr uint32_t npar = kTmaConsumers / KVH;
    float* sm_m = sm;                        // [slot][8]
    float* sm_l = sm_m + kTmaConsumers * 8;  // [slot][8]
    float* sm_o = sm_l + kTmaConsumers * 8;  // [slot][8][kOStride]
    const int g = static_cast<int>(lane >> 2), t = static_cast<int>(lane & 3);
    if constexpr (npar > 1) {
        if (warp >= KVH && warp < KVH * npar) state_to_smem(st, static_cast<int>(warp), sm_m, sm_l, sm_o, g, t);
        __syncthreads();
    }
    if (warp >= KVH) return;
    float M0 = st.m0, M1 = st.m1;
#pragma unroll
    for (uint32_t j = 1; j < npar; ++j) {
        const uint32_t slot = warp + KVH * j;
        M0 = fmaxf(M0, sm_m[slot * 8 + 2 * t]);
        M1 = fmaxf(M1, sm_m[slot * 8 + 2 * t + 1]);
    }
    if constexpr (npar > 1) {
        const float a0 = st.m0 == -INFINITY ? 0.f : ex2(st.m0 - M0);
        const float a1 = st.m1 == -INFINITY ? 0.f : ex2(st.m1 - M1);
        float L0 = st.l0 * a0, L1 = st.l1 * a1;
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
            st.o[mt][0] *= a0;
            st.o[mt][2] *= a0;
            st.o[mt][1] *= a1;
            st.o[mt][3] *= a1;
        }
#pragma unroll
        for (uint32_t j = 1; j < npar; ++j) {
            const uint32_t slot = warp + KVH * j;
            const float m0 = sm_m[slot * 8 + 2 * t], m1 = sm_m[slot * 8 + 2 * t + 1];
            const float s0 = m0 == -INFINITY ? 0.f : ex2(m0 - M0);
            const float s1 = m1 == -INFINITY ? 0.f : ex2(m1 - M1);
            L0 = fmaf(s0, sm_l[slot * 8 + 2 * t], L0);
            L1 = fmaf(s1, sm_l[slot * 8 + 2 * t + 1], L1);
            const float* o0 = sm_o + (slot * 8 + 2 * t) * kOStride;
            const float* o1 = o0 + kOStride;
#pragma unroll
            for (int mt = 0; mt < 8; ++mt) {
                const int d = 64 * (mt >> 2) + 8 * g + 2 * (mt & 3);
                st.o[mt][0] = fmaf(s0, o0[d], st.o[mt][0]);
                st.o[mt][1] = fmaf(s1, o1[d], st.o[mt][1]);
                st.o[mt][2] = fmaf(s0, o0[d + 1], st.o[mt][2]);
                st.o[mt][3] = fmaf(s1, o1[d + 1], st.o[mt][3]);
            }
        }
        st.m0 = M0;
        st.m1 = M1;
        st.l0 = L0;
        st.l1 = L1;
    }
    store_warp_partial(st, po, pm, pl, static_cast<uint64_t>(splits) * 128, kHalves ? 64 : 128,
                       kHalves ? static_cast<uint64_t>(splits) * 64 : 64, splits, 1, split, warp * group, group, g, t);
}

template <bool kFused, uint32_t KVH>
__global__ void __launch_bounds__(kTmaThreads, 1)
    decode_tma_kernel(const DecodeArgs a, const StepExt x, const __grid_constant__ CUtensorMap map_k,
                      const __grid_constant__ CUtensorMap map_v) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint32_t stage_valid[32];  // kFused: rows of the tile in each stage, 0 = no more tiles
    __shared__ uint64_t merge_bar;        // kFused: bulk copies of the merge
    constexpr uint32_t row_bytes = KVH * 256;          // one token, all KV heads
    // The fused step stages kSub 16-token sub-tiles per KV head when there are
    // fewer than 4 KV heads, so every stage carries 16 KB per operand (a
    // one-head row is 256 B: 16-token stages would spend a stage's fixed cost
    // on 4 KB); consumer warp j = warp / KVH of a head takes sub-tile j % kSub
    // of every npar-th stage.
    constexpr uint32_t kSub = (kFused && KVH < 4) ? 4 / KVH : 1;
    constexpr uint32_t kRows = kTile * kSub;           // tokens per stage
    constexpr uint32_t tile_bytes = kRows * row_bytes; // per K (and per V): [2*KVH blocks][kRows rows][128 B]
    const uint32_t stages = a.stages;
    // 128-byte swizzled TMA boxes want 1024-byte aligned destinations
    uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(ring + stages * 2 * tile_bytes);
    uint64_t* empty = full + stages;
    constexpr uint32_t npar = kTmaConsumers / (KVH * kSub);  // stage parities; divides `stages`
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // While the previous kernel finishes (nothing here depends on its output):
    // barriers, tensor-map prefetch, and this CTA's first tiles pulled into
    // L2. The length read for the prefetch may be stale (it can be the
    // previous kernel's output); a prefetch only warms L2, so any tile below
    // max_kv_len is harmless.
    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], KVH * kSub);
        }
        if (kFused) mbar_init(&merge_bar, 1);
        fence_mbarrier_init();
    }
    if (warp == kTmaConsumers) {
        if (lane == 0) {
            tc::prefetch_tensormap(&map_k);
            tc::prefetch_tensormap(&map_v);
        }
        if (lane < 2 * kPrefetchTiles) {
            const Extent pre = decode_extent(a);
            if (split_index_ok(pre, blockIdx.x)) {
                uint32_t first, count;
                own_tiles(pre, blockIdx.x, kFused, kRows, first, count);
                const uint32_t j = static_cast<uint32_t>(lane) >> 1;
                if (j < count) {
                    const uint64_t off = static_cast<uint64_t>(first + j) * tile_bytes;
                    bulk_prefetch_l2(reinterpret_cast<const uint8_t*>((lane & 1) ? a.v : a.k) + off, tile_bytes);
                }
            }
        }
    }
    __syncthreads();
    pdl_wait_primary();  // Q, the cache and the device length may come from the previous kernel
    pdl_launch_dependents();
    // every load that only depends on the previous kernel goes out at once
    int32_t pos = 0;
    uint32_t base = 0, epoch_next = 0;
    if (kFused) {
        if (x.pos_dev != nullptr) pos = __ldcg(x.pos_dev);
        if (threadIdx.x == 0) base = __ldcg(&x.counters[2]);
        if (x.world > 1) epoch_next = __ldcg(x.epoch) + 1u;
    }
    const Extent ext = decode_extent(a);
    const uint32_t split = blockIdx.x;
    if (kFused && ext.splits == 0) {  // empty cache: defined output
        if (split == 0) {
            if (x.world > 1) {
                // nothing to attend here, but the other ranks wait for this rank's partials
                for (uint32_t h = 0; h < a.num_heads; ++h)
                    (void)step_exchange_head(x, a.num_heads, h, epoch_next, 0.f, -INFINITY, 0.f, 0, 128);
                if (threadIdx.x == 0) *x.epoch = epoch_next;
            } else {
                step_write_empty(a.num_heads, x, threadIdx.x, blockDim.x);
            }
        }
        return;
    }
    if (split >= ext.splits) return;
    uint32_t begin, end;
    split_range(ext.kv_len, ext.splits, split, begin, end);
    const uint32_t ntiles = (end - begin + kTile - 1) / kTile;

    bool rope_ok = true;
    if (kFused) {
        rope_ok = !x.rotate || (pos >= 0 && static_cast<uint32_t>(pos) < x.table_rows);
        if (!rope_ok && split == 0 && threadIdx.x == 0) atomicOr(&g_device_error, kErrBadPosition);
    }

    bool ok = true;
    WarpState st;
    state_init(st);
    if (warp == kTmaConsumers) {
        // ---- producer warp
        const uint64_t policy = l2_evict_first_policy();
        uint32_t i = 0;
        if constexpr (kFused) {
            // Tile order of split s: its even share [s*per, (s+1)*per) of ~1/2
            // of the tiles (the last split puts the last tile, which holds the
            // new row, after its first two, once consumer warp 0 has appended
            // the row), then tiles of the pool [S*per, total - 1), claimed one
            // at a time from the counter with the next two claims in flight
            // (`claimed`, `claimed2`, used in turn: each read sits in its own
            // branch so it waits for its own round trip only), so CTAs that
            // run ahead take more.
            const uint32_t total = (ext.kv_len + kRows - 1) / kRows;
            const uint32_t per = fused_share(total, ext.splits);  // per * S <= total - 1
            const uint32_t pool = per * ext.splits, pool_end = total - 1;
            const bool tail_split = split + 1 == ext.splits;
            uint32_t own = split * per, own_end = own + per;
            // With an own share the first claim goes out after the first copy
            // (its round trip is hidden behind the share); without one, now.
            uint32_t claimed = lane == 0 && pool < pool_end && per == 0 ? atomicAdd(&x.counters[0], 1u) : 0u;
            uint32_t claimed2 = lane == 0 && pool < pool_end && per == 0 ? atomicAdd(&x.counters[0], 1u) : 0u;
            bool toggle = false;
            bool first_claim = per != 0 && pool < pool_end;
            // The tiles after the ones warmed before the wait: HBM starts on
            // them while the first copies come from L2.
            {
                const uint32_t tj = own + kPrefetchTiles + (static_cast<uint32_t>(lane) >> 1);
                if (lane < 2 * kPostPrefetchTiles && tj < own_end)
                    bulk_prefetch_l2(reinterpret_cast<const uint8_t*>((lane & 1) ? a.v : a.k) +
                                         static_cast<uint64_t>(tj) * tile_bytes,
                                     tile_bytes);
            }
            bool tail_pending = tail_split;
            const uint32_t tail_at = min(2u, per);
            uint32_t cur = 0, cur_left = 0;
            for (;; ++i) {
                uint32_t tile;
                if (tail_pending && i == tail_at) {
                    tile = total - 1;
                    tail_pending = false;
                    // consumer warp 0 appends the new row (generic stores + proxy
                    // fence) and arrives here before this tile is copied
                    if (x.k_new != nullptr && rope_ok) named_barrier_sync(kAppendBarrier, 64);
                } else if (own < own_end) {
                    tile = own++;
                } else {
                    if (cur_left == 0) {
                        if (toggle) {
                            cur = pool + __shfl_sync(0xffffffffu, claimed2, 0);
                            cur_left = cur < pool_end ? 1u : 0u;
                            if (lane == 0 && cur_left != 0) claimed2 = atomicAdd(&x.counters[0], 1u);
                        } else {
                            cur = pool + __shfl_sync(0xffffffffu, claimed, 0);
                            cur_left = cur < pool_end ? 1u : 0u;
                            if (lane == 0 && cur_left != 0) claimed = atomicAdd(&x.counters[0], 1u);
                        }
                        toggle = !toggle;
                    }
                    tile = cur_left != 0 ? cur++ : total;
                    if (cur_left != 0) --cur_left;
                }
                const uint32_t s = i % stages, round = i / stages;
                if (tile >= total) {
                    // no tiles left: one empty stage per consumer parity ends its loop
                    for (uint32_t e = 0; e < npar; ++e, ++i) {
                        const uint32_t se = i % stages, re = i / stages;
                        if (lane == 0) {
                            if (re > 0 && !mbar_wait(&empty[se], (re - 1) & 1)) ok = false;
                            stage_valid[se] = 0;
                            mbar_arrive(&full[se]);
                        }
                    }
                    ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
                    break;
                }
                const uint32_t t0 = tile * kRows;
                bool w_ok = true;
                if (lane == 0 && round > 0) w_ok = mbar_wait(&empty[s], (round - 1) & 1);
                if (!__shfl_sync(0xffffffffu, w_ok ? 1 : 0, 0)) {
                    ok = false;
                    break;
                }
                if (lane == 0) {
                    stage_valid[s] = min(kRows, ext.kv_len - t0);
                    mbar_arrive_expect_tx(&full[s], 2 * tile_bytes);
                    tc::tma_load_3d_hint(stg_of(ring, s, tile_bytes), &map_k, 0, static_cast<int32_t>(t0), 0,
                                         &full[s], policy);
                    tc::tma_load_3d_hint(stg_of(ring, s, tile_bytes) + tile_bytes, &map_v, 0,
                                         static_cast<int32_t>(t0), 0, &full[s], policy);
                }
                if (first_claim) {
                    first_claim = false;
                    if (lane == 0) {
                        claimed = atomicAdd(&x.counters[0], 1u);
                        claimed2 = atomicAdd(&x.counters[0], 1u);
                    }
                }
                __syncwarp();
            }
        } else {
            for (; i < ntiles; ++i) {
                const uint32_t s = i % stages, round = i / stages;
                bool w_ok = true;
                if (lane == 0 && round > 0) w_ok = mbar_wait(&empty[s], (round - 1) & 1);
                if (!__shfl_sync(0xffffffffu, w_ok ? 1 : 0, 0)) {
                    ok = false;
                    break;
                }
                const int32_t t0 = static_cast<int32_t>(begin + i * kTile);
                if (lane == 0) {
                    // whole boxes: rows past the tensor's end arrive zero-filled, rows
                    // past this split's end are masked by the consumers
                    mbar_arrive_expect_tx(&full[s], 2 * tile_bytes);
                    tc::tma_load_3d_hint(stg_of(ring, s, tile_bytes), &map_k, 0, t0, 0, &full[s], policy);
                    tc::tma_load_3d_hint(stg_of(ring, s, tile_bytes) + tile_bytes, &map_v, 0, t0, 0, &full[s],
                                         policy);
                }
                __syncwarp();
            }
        }
        const uint32_t issued = i;
        // Never leave the CTA with copies in flight into its shared memory.
        if (lane == 0) {
            const uint32_t first = issued > stages ? issued - stages : 0;
            for (uint32_t i = first; i < issued; ++i) (void)mbar_wait(&full[i % stages], (i / stages) & 1);
        }
    } else {
        // ---- consumers: warp = KV head (warp % KVH) x sub-tile x stage parity
        const uint32_t kvh = warp % KVH, sub = (warp / KVH) % kSub, par = warp / (KVH * kSub);
        const int g = lane >> 2, t = lane & 3;
        if constexpr (kFused) {
            if (warp == 0 && split + 1 == ext.splits && x.k_new != nullptr && rope_ok) {
                // append the new token at row kv_len - 1; the producer copies
                // that row's tile only after the barrier below
                const uint32_t last_row = ext.kv_len - 1;
                const uint64_t row = static_cast<uint64_t>(last_row) * a.kv_stride;
                for (uint32_t gi = lane; gi < KVH * 8; gi += 32) {
                    const uint32_t h = gi >> 3, e = (gi & 7) * 8;
                    uint4 lo = *reinterpret_cast<const uint4*>(x.k_new + h * 128 + e);
                    uint4 hi = *reinterpret_cast<const uint4*>(x.k_new + h * 128 + 64 + e);
                    if (x.rotate) {
                        const uint64_t ti = static_cast<uint64_t>(pos) * 64 + e;
                        rot8_pairs(lo, hi, *reinterpret_cast<const uint4*>(x.cos + ti),
                                   *reinterpret_cast<const uint4*>(x.sin + ti));
                    }
                    *reinterpret_cast<uint4*>(x.k_cache + row + h * 128 + e) = lo;
                    *reinterpret_cast<uint4*>(x.k_cache + row + h * 128 + 64 + e) = hi;
                    *reinterpret_cast<uint4*>(x.v_cache + row + h * 128 + e) =
                        *reinterpret_cast<const uint4*>(x.v_new + h * 128 + e);
                    *reinterpret_cast<uint4*>(x.v_cache + row + h * 128 + 64 + e) =
                        *reinterpret_cast<const uint4*>(x.v_new + h * 128 + 64 + e);
                }
                // the producer's tensor copies (async proxy) must see these stores
                asm volatile("fence.proxy.async.global;" ::: "memory");
                named_barrier_arrive(kAppendBarrier, 64);
            }
        }
        uint32_t qf[8][2];
        {
            // Q of the new token (rotated in registers by the fused step; pairs
            // (e, e+64) sit in words j and j+2)
            if (static_cast<uint32_t>(g) < a.group) {
                const __half* qrow = (kFused ? x.q_new : a.q) + static_cast<uint64_t>(kvh * a.group + g) * 128;
                uint4 w[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) w[j] = *reinterpret_cast<const uint4*>(qrow + 32 * j + 8 * t);
                if (kFused && x.rotate && rope_ok) {
#pragma unroll
                    for (int j = 0; j < 2; ++j) {
                        const uint64_t ti = static_cast<uint64_t>(pos) * 64 + 32 * j + 8 * t;
                        rot8_pairs(w[j], w[j + 2], *reinterpret_cast<const uint4*>(x.cos + ti),
                                   *reinterpret_cast<const uint4*>(x.sin + ti));
                    }
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    qf[2 * j][0] = w[j].x;
                    qf[2 * j][1] = w[j].y;
                    qf[2 * j + 1][0] = w[j].z;
                    qf[2 * j + 1][1] = w[j].w;
                }
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) qf[j][0] = qf[j][1] = 0u;
            }
        }
        // warps past KVH * npar (8 KV heads: 4 of 12) have no tiles
        for (uint32_t i = par; par < npar; i += npar) {
            if (!kFused && i >= ntiles) break;
            const uint32_t s = i % stages, round = i / stages;
            if (!mbar_wait(&full[s], round & 1)) {
                ok = false;
                break;
            }
            uint32_t valid;
            if constexpr (kFused) {
                const uint32_t rows = stage_valid[s];
                if (rows == 0) break;  // the producer ran out of tiles
                // this warp's sub-tile: rows [16 sub, 16 sub + 16) of the stage
                valid = rows > sub * kTile ? min(static_cast<uint32_t>(kTile), rows - sub * kTile) : 0u;
                if (kSub > 1 && valid == 0) {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&empty[s]);
                    continue;
                }
            } else {
                valid = min(static_cast<uint32_t>(kTile), end - (begin + i * kTile));
            }
            // head kvh's two 64-column blocks of the stage are kRows rows each
            const uint8_t* kt = ring + s * 2 * tile_bytes + kvh * (2 * kRows * 128) + sub * (kTile * 128);
            const uint8_t* vt = kt + tile_bytes;
            float sc[4];
            uint4 va[4][2];
            if (valid == kTile) {
                uint4 ka[4], kb[4];
                load_k_frags_sw<false, kRows * 128>(kt, g, t, valid, ka, kb);
                tile_scores<false>(sc, ka, kb, qf, tile_token(g), valid, a.scale_log2);
                load_v_frags_sw<false, kRows * 128>(vt, g, t, valid, va);
            } else {
                uint4 ka[4], kb[4];
                load_k_frags_sw<true, kRows * 128>(kt, g, t, valid, ka, kb);
                tile_scores<true>(sc, ka, kb, qf, tile_token(g), valid, a.scale_log2);
                load_v_frags_sw<true, kRows * 128>(vt, g, t, valid, va);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);  // the stage can be refilled
            tile_softmax_pv(st, sc, va, g, t);
        }
        state_finish(st);
    }
    // All ring reads and copies are done: reuse the ring for the combine.
    __syncthreads();
    combine_split<KVH, kFused>(st, static_cast<uint32_t>(warp), static_cast<uint32_t>(lane), reinterpret_cast<float*>(ring),
                       a.group, split, ext.splits, a.po, a.pm, a.pl);
    if (!ok) atomicOr(&g_device_error, kErrWaitTimeout);
    if constexpr (kFused) {
        // the merging CTAs read these partials with bulk (async-proxy) copies
        if (warp < static_cast<int>(KVH)) fence_proxy_async_global();
        step_merge(a, x, ext.splits, split, ring, &merge_bar, base, epoch_next);
    }
}

// ---------------------------------------------------------------------------
// Register-path split kernel. grid = (num_kv_heads, chunks), block = 128.
__global__ void __launch_bounds__(128) decode_split_mma_kernel(const DecodeArgs a) {
    __shared__ float sm_m[4 * 8];
    __shared__ float sm_l[4 * 8];
    __shared__ float sm_o[4 * 8 * kOStride];
    const uint32_t kvh = blockIdx.x;
    const uint32_t chunk = blockIdx.y;
    pdl_wait_primary();
    pdl_launch_dependents();
    const Extent ext = decode_extent(a);
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
        float sc[4];
        tile_scores<true>(sc, ka, kb, qf, g, w1 - tb, a.scale_log2);
        tile_softmax_pv(st, sc, va, g, t);
    }
    state_finish(st);
    state_to_smem(st, warp, sm_m, sm_l, sm_o, g, t);
    __syncthreads();
    for (uint32_t idx = threadIdx.x; idx < a.group * 128; idx += blockDim.x)
        combine_write(sm_m, sm_l, sm_o, 0, 1, 4, kvh, a.group, chunk, ext.splits, a.po, a.pm, a.pl, idx);  // 4 warps
}

// ---------------------------------------------------------------------------
// SIMT split kernel for any head_dim / stride / alignment.
// grid = (num_heads, chunks), block = 128.
__global__ void __launch_bounds__(128) decode_split_simt_kernel(const DecodeArgs a) {
    __shared__ float scores[kChunk];
    __shared__ float red[4];
    const uint32_t h = blockIdx.x;
    const uint32_t chunk = blockIdx.y;
    pdl_wait_primary();
    pdl_launch_dependents();
    const Extent ext = decode_extent(a);
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
// Merge: grid = (num_heads, ceil(head_dim / 64)), block = 512. Warp w takes
// splits w, w + 16, ...; a lane owns two output dims. Each batch of kMergeBatch
// splits per warp is loaded in one round (m, l, o all in flight) and folded
// into a running (max, sum, o) with the same rescaling as the split kernels;
// warp 0 then merges the 16 warp states.
constexpr int kMergeWarps = 16;
constexpr int kMergeBatch = 10;

__global__ void __launch_bounds__(kMergeWarps * 32) merge_partials_kernel(const MergeArgs a) {
    __shared__ float red_m[kMergeWarps];
    __shared__ float red_l[kMergeWarps];
    __shared__ float2 acc_s[kMergeWarps][32];
    pdl_wait_primary();
    pdl_launch_dependents();
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
    const uint32_t e0 = d0 + 2 * lane, e1 = e0 + 1;
    if (n == 0) {  // graph-static launch with an empty range: defined output
        if (warp == 0) {
            if (a.rank_o) {
                if (e0 < d) a.rank_o[static_cast<uint64_t>(h) * d + e0] = 0.f;
                if (e1 < d) a.rank_o[static_cast<uint64_t>(h) * d + e1] = 0.f;
                if (blockIdx.y == 0 && lane == 0) {
                    a.rank_m[h] = -INFINITY;
                    a.rank_l[h] = 0.f;
                }
            } else {
                if (e0 < d) a.out[static_cast<uint64_t>(h) * d + e0] = __float2half_rn(0.f);
                if (e1 < d) a.out[static_cast<uint64_t>(h) * d + e1] = __float2half_rn(0.f);
            }
        }
        return;
    }
    const float* pm = a.pm + h * ml_head;
    const float* pl = a.pl + h * ml_head;
    const float* po = a.po + h * o_head;

    float m_run = -INFINITY, l_run = 0.f, ax = 0.f, ay = 0.f;
    for (uint32_t base = warp; base < n; base += kMergeWarps * kMergeBatch) {
        float mv[kMergeBatch], lv[kMergeBatch], ox[kMergeBatch], oy[kMergeBatch];
#pragma unroll
        for (int u = 0; u < kMergeBatch; ++u) {
            const uint32_t c = base + kMergeWarps * u;
            const bool in = c < n;
            mv[u] = in ? pm[c * ml_chunk] : -INFINITY;
            lv[u] = in ? pl[c * ml_chunk] : 0.f;
            const float* row = po + c * o_chunk;
            ox[u] = in && e0 < d ? row[e0] : 0.f;
            oy[u] = in && e1 < d ? row[e1] : 0.f;
        }
        float bm = m_run;
#pragma unroll
        for (int u = 0; u < kMergeBatch; ++u) bm = fmaxf(bm, mv[u]);
        if (bm > m_run) {
            const float sc = m_run == -INFINITY ? 0.f : expf(m_run - bm);
            ax *= sc;
            ay *= sc;
            l_run *= sc;
            m_run = bm;
        }
#pragma unroll
        for (int u = 0; u < kMergeBatch; ++u) {
            if (mv[u] != -INFINITY) {
                const float w = expf(mv[u] - m_run);
                ax = fmaf(w, ox[u], ax);
                ay = fmaf(w, oy[u], ay);
                l_run = fmaf(w, lv[u], l_run);
            }
        }
    }
    if (lane == 0) {
        red_m[warp] = m_run;
        red_l[warp] = l_run;
    }
    acc_s[warp][lane] = make_float2(ax, ay);
    __syncthreads();
    if (warp != 0) return;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kMergeWarps; ++w) M = fmaxf(M, red_m[w]);
    float L = 0.f, sx = 0.f, sy = 0.f;
#pragma unroll
    for (int w = 0; w < kMergeWarps; ++w) {
        const float m = red_m[w];
        const float sc = m == -INFINITY ? 0.f : expf(m - M);
        L = fmaf(sc, red_l[w], L);
        sx = fmaf(sc, acc_s[w][lane].x, sx);
        sy = fmaf(sc, acc_s[w][lane].y, sy);
    }
    if (a.rank_o) {
        if (e0 < d) a.rank_o[static_cast<uint64_t>(h) * d + e0] = sx;
        if (e1 < d) a.rank_o[static_cast<uint64_t>(h) * d + e1] = sy;
        if (blockIdx.y == 0 && lane == 0) {
            a.rank_m[h] = M;
            a.rank_l[h] = L;
        }
    } else {
        const float inv = 1.f / L;
        if (e0 < d) a.out[static_cast<uint64_t>(h) * d + e0] = __float2half_rn(sx * inv);
        if (e1 < d) a.out[static_cast<uint64_t>(h) * d + e1] = __float2half_rn(sy * inv);
    }
}

__global__ void advance_position_kernel(int32_t* pos, int32_t delta) {
    pdl_wait_primary();
    pdl_launch_dependents();
    *pos += delta;
}

const void* const kSplitKernels[] = {
    reinterpret_cast<const void*>(decode_tma_kernel<false, 1>), reinterpret_cast<const void*>(decode_tma_kernel<false, 2>),
    reinterpret_cast<const void*>(decode_tma_kernel<false, 4>), reinterpret_cast<const void*>(decode_tma_kernel<false, 8>),
    reinterpret_cast<const void*>(decode_split_mma_kernel),    reinterpret_cast<const void*>(decode_split_simt_kernel),
};
constexpr int kNumTmaKernels = 4;  // the first entries of kSplitKernels take (DecodeArgs, StepExt)
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
    const void* kernels[] = {
        reinterpret_cast<const void*>(decode_tma_kernel<false, 1>), reinterpret_cast<const void*>(decode_tma_kernel<false, 2>),
        reinterpret_cast<const void*>(decode_tma_kernel<false, 4>), reinterpret_cast<const void*>(decode_tma_kernel<false, 8>),
        reinterpret_cast<const void*>(decode_tma_kernel<true, 1>),  reinterpret_cast<const void*>(decode_tma_kernel<true, 2>),
        reinterpret_cast<const void*>(decode_tma_kernel<true, 4>),  reinterpret_cast<const void*>(decode_tma_kernel<true, 8>),
    };
    int st = B2_OK;
    for (const void* k : kernels) {
        st = cuda_status(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              static_cast<int>(kTmaSmemBudget + 2048)));
        if (st != B2_OK) return st;
    }
    done_mask.fetch_or(bit);
    return st;
}

// Tensor maps of one cache (K or V): rows of num_kv_heads * 256 bytes, boxes
// of kTile rows. A few per thread are kept: the eager launchers re-use them
// layer after layer while the length and base are unchanged.
int cache_tensor_map(CUtensorMap* out, const void* base, uint32_t rows, uint32_t num_kv_heads, uint32_t box_rows) {
    struct Entry {
        const void* base;
        uint32_t rows, kvh, box_rows;
        CUtensorMap map;
    };
    thread_local Entry cache[8] = {};
    thread_local uint32_t next = 0;
    for (const Entry& e : cache)
        if (e.base == base && e.rows == rows && e.kvh == num_kv_heads && e.box_rows == box_rows) {
            *out = e.map;
            return B2_OK;
        }
    Entry& e = cache[next++ & 7];
    if (encode_token_rows_by_column_block(&e.map, base, rows, num_kv_heads * 256u, box_rows) != 0) {
        e.base = nullptr;
        return B2_ERR_CUDA;
    }
    e.base = base;
    e.rows = rows;
    e.kvh = num_kv_heads;
    e.box_rows = box_rows;
    *out = e.map;
    return B2_OK;
}

// Tokens per ring stage of the TMA kernel (its kRows): the fused step stages
// 4 / KVH sixteen-token sub-tiles per head when there are fewer than 4 KV heads.
uint32_t stage_rows(uint32_t num_kv_heads, bool fused) {
    return fused && num_kv_heads < 4 ? kTile * (4u / num_kv_heads) : kTile;
}

// Ring depth: each stage is always consumed by the same warps (a warp waits
// on a stage's next phase only after consuming the current one), so the depth
// is a multiple of the stage parities.
uint32_t tma_stages(uint32_t num_kv_heads, uint32_t rows) {
    const uint32_t stage_bytes = 2u * rows * num_kv_heads * 256u;
    const uint32_t npar = kTmaConsumers / (num_kv_heads * (rows / kTile));
    return (kTmaSmemBudget / stage_bytes) / npar * npar;
}

size_t tma_smem_bytes(uint32_t num_kv_heads, uint32_t stages, uint32_t rows) {
    return static_cast<size_t>(stages) * 2u * rows * num_kv_heads * 256u + 2 * stages * sizeof(uint64_t) +
           1024;  // alignment slack
}

// Launch the TMA kernel over caches a.k / a.v of `map_rows` rows.
template <bool kFused>
int launch_tma_kernel(const DecodeArgs& a, const StepExt& x, uint32_t grid, uint32_t map_rows, cudaStream_t stream) {
    CUtensorMap mk, mv;
    const uint32_t rows = stage_rows(a.num_kv_heads, kFused);
    int st = cache_tensor_map(&mk, a.k, map_rows, a.num_kv_heads, rows);
    if (st == B2_OK) st = cache_tensor_map(&mv, a.v, map_rows, a.num_kv_heads, rows);
    if (st != B2_OK) return st;
    const size_t smem = tma_smem_bytes(a.num_kv_heads, a.stages, rows);
    switch (a.num_kv_heads) {
        case 1:
            return launch_pdl(decode_tma_kernel<kFused, 1>, dim3(grid), dim3(kTmaThreads), smem, stream, a, x, mk, mv);
        case 2:
            return launch_pdl(decode_tma_kernel<kFused, 2>, dim3(grid), dim3(kTmaThreads), smem, stream, a, x, mk, mv);
        case 4:
            return launch_pdl(decode_tma_kernel<kFused, 4>, dim3(grid), dim3(kTmaThreads), smem, stream, a, x, mk, mv);
        case 8:
            return launch_pdl(decode_tma_kernel<kFused, 8>, dim3(grid), dim3(kTmaThreads), smem, stream, a, x, mk, mv);
        default: return B2_ERR_UNSUPPORTED;
    }
}

int launch_merge_kernel(const MergeArgs& m, cudaStream_t stream) {
    return launch_pdl(merge_partials_kernel, dim3(m.num_heads, (m.head_dim + 63) / 64), dim3(kMergeWarps * 32), 0,
                      stream, m);
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
    m.split_tokens = a.split_tokens;
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
        a.stages = tma_stages(a.num_kv_heads, stage_rows(a.num_kv_heads, false));
        if (a.stages == 0) return B2_ERR_UNSUPPORTED;
        a.splits_cap = static_cast<uint32_t>(device_sms());
        const uint32_t grid = static_cast<uint32_t>(chunks < a.splits_cap ? chunks : a.splits_cap);
        st = launch_tma_kernel<false>(a, StepExt{}, grid, a.kv_len, stream);
    } else if (mma_ok) {
        st = launch_pdl(decode_split_mma_kernel, dim3(a.num_kv_heads, static_cast<uint32_t>(chunks)), dim3(128), 0,
                        stream, a);
    } else {
        st = launch_pdl(decode_split_simt_kernel, dim3(a.num_heads, static_cast<uint32_t>(chunks)), dim3(128), 0,
                        stream, a);
    }
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

// Workspace of the fused step: partials for up to kStepMaxSplits splits
// ([H][2 halves][S][64] o, [H][S] m, [H][S] l, floats), then the 3 counter
// words of StepExt::counters.
struct StepWorkspace {
    size_t po, pm, pl, counter, total_bytes;
};

StepWorkspace step_workspace_layout(size_t num_heads, size_t /*num_kv_heads*/) {
    StepWorkspace w{};
    w.po = 0;
    w.pm = w.po + num_heads * kStepMaxSplits * 128;
    w.pl = w.pm + num_heads * kStepMaxSplits;
    w.counter = w.pl + num_heads * kStepMaxSplits;
    w.total_bytes = (w.counter * sizeof(float) + 3 * sizeof(uint32_t) + 255) / 256 * 256;
    return w;
}

int launch_decode_step(const void* d_q, const void* d_k_new, const void* d_v_new, void* d_k_cache, void* d_v_cache,
                       const void* d_cos, const void* d_sin, size_t rope_rows, bool apply_rotation,
                       const int32_t* d_pos, const int32_t* d_kv_len, int32_t kv_len_bias, size_t max_kv_len,
                       void* d_out, float* d_rank_o, float* d_rank_m, float* d_rank_l, void* d_workspace,
                       size_t workspace_bytes, size_t num_heads, size_t num_kv_heads, size_t head_dim,
                       b2_stream_t stream_handle, size_t world = 1, size_t rank_index = 0,
                       void* const* exchange_buffers = nullptr) {
    if (max_kv_len == 0 || num_kv_heads == 0 || head_dim == 0) return B2_NOTHING_TO_DO;
    if (world > 1) {
        if (world > kMaxWorld || rank_index >= world || exchange_buffers == nullptr) return B2_ERR_INVALID_ARG;
        for (size_t r = 0; r < world; ++r)
            if (exchange_buffers[r] == nullptr || !aligned16(exchange_buffers[r])) return B2_ERR_INVALID_ARG;
    }
    if (num_heads % num_kv_heads != 0) return B2_NOTHING_TO_DO;
    const bool rank = d_rank_o != nullptr || d_rank_m != nullptr || d_rank_l != nullptr;
    if (!d_q || !d_k_cache || !d_v_cache || !d_kv_len || !d_workspace) return B2_ERR_INVALID_ARG;
    if (rank ? (!d_rank_o || !d_rank_m || !d_rank_l || d_out) : !d_out) return B2_ERR_INVALID_ARG;
    if (d_k_new && !d_v_new) return B2_ERR_INVALID_ARG;
    if (apply_rotation && (!d_cos || !d_sin || !d_pos || rope_rows == 0)) return B2_ERR_INVALID_ARG;
    const size_t group = num_heads / num_kv_heads;
    if (head_dim != 128 || group > 8 ||
        !(num_kv_heads == 1 || num_kv_heads == 2 || num_kv_heads == 4 || num_kv_heads == 8))
        return B2_ERR_UNSUPPORTED;
    // splits of 64 tokens, capped at the SM count: short per-rank ranges
    // (several GPUs) still spread over every SM
    constexpr uint32_t kStepSplitTokens = 64;
    const size_t chunks = (max_kv_len + kStepSplitTokens - 1) / kStepSplitTokens;
    if (max_kv_len > 0x7fffffffull - kChunk || rope_rows > 0x7fffffffull) return B2_ERR_UNSUPPORTED;
    const void* ptrs[] = {d_q, d_k_new, d_v_new, d_k_cache, d_v_cache, d_cos, d_sin, d_out, d_rank_o, d_workspace};
    for (const void* p : ptrs)
        if (p && !aligned16(p)) return B2_ERR_ALIGNMENT;
    const StepWorkspace w = step_workspace_layout(num_heads, num_kv_heads);
    if (workspace_bytes < w.total_bytes) return B2_ERR_WORKSPACE;
    const uint32_t sms = static_cast<uint32_t>(device_sms());
    if (sms > kStepMaxSplits) return B2_ERR_UNSUPPORTED;
    int st = ensure_tma_smem();
    if (st != B2_OK) return st;

    float* ws = static_cast<float*>(d_workspace);
    DecodeArgs a{};
    a.q = static_cast<const __half*>(d_q);
    a.k = static_cast<const __half*>(d_k_cache);
    a.v = static_cast<const __half*>(d_v_cache);
    a.po = ws + w.po;
    a.pm = ws + w.pm;
    a.pl = ws + w.pl;
    a.kv_stride = num_kv_heads * head_dim;
    a.kv_len = static_cast<uint32_t>(max_kv_len);
    a.splits_cap = sms;
    a.num_heads = static_cast<uint32_t>(num_heads);
    a.num_kv_heads = static_cast<uint32_t>(num_kv_heads);
    a.head_dim = static_cast<uint32_t>(head_dim);
    a.group = static_cast<uint32_t>(group);
    a.scale = 1.0f / sqrtf(static_cast<float>(head_dim));
    a.scale_log2 = a.scale * kLog2e;
    a.kv_len_dev = d_kv_len;
    a.kv_len_bias = kv_len_bias;
    a.max_kv_len = static_cast<uint32_t>(max_kv_len);
    a.split_tokens = kStepSplitTokens;
    a.stages = tma_stages(a.num_kv_heads, stage_rows(a.num_kv_heads, true));
    if (a.stages == 0) return B2_ERR_UNSUPPORTED;

    StepExt x{};
    x.q_new = static_cast<const __half*>(d_q);
    x.k_new = static_cast<const __half*>(d_k_new);
    x.v_new = static_cast<const __half*>(d_v_new);
    x.k_cache = static_cast<__half*>(d_k_cache);
    x.v_cache = static_cast<__half*>(d_v_cache);
    x.cos = static_cast<const __half*>(d_cos);
    x.sin = static_cast<const __half*>(d_sin);
    x.pos_dev = d_pos;
    x.rotate = apply_rotation ? 1u : 0u;
    x.table_rows = static_cast<uint32_t>(rope_rows);
    x.counters = reinterpret_cast<uint32_t*>(ws + w.counter);
    x.out = static_cast<__half*>(d_out);
    x.rank_o = d_rank_o;
    x.rank_m = d_rank_m;
    x.rank_l = d_rank_l;
    x.world = static_cast<uint32_t>(world > 1 ? world : 1);
    x.rank = static_cast<uint32_t>(rank_index);
    if (world > 1) {
        for (size_t r = 0; r < world; ++r) x.peers[r] = static_cast<float*>(exchange_buffers[r]);
        x.epoch = reinterpret_cast<uint32_t*>(reinterpret_cast<uint2*>(x.peers[rank_index]) +
                                              exchange_words(x.world, a.num_heads));
    }
    const uint32_t grid = static_cast<uint32_t>(chunks < sms ? chunks : sms);
    return launch_tma_kernel<true>(a, x, grid, a.max_kv_len, reinterpret_cast<cudaStream_t>(stream_handle));
}

}  // namespace

unsigned int device_error_decode() {
    unsigned int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v)) != cudaSuccess) return 0;
    return v;
}

int clear_device_error_decode() {
    const unsigned int zero = 0;
    return cuda_status(cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero)));
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
    const int st = node_kernel_params(node, kSplitKernels, kNumTmaKernels + 2, &params);
    if (st != B2_OK) return st;
    DecodeArgs a = *static_cast<const DecodeArgs*>(params.kernelParams[0]);
    if (a.kv_len_dev != nullptr) return B2_ERR_GRAPH;  // graph-static nodes need no patching
    a.kv_len = static_cast<uint32_t>(kv_cache_len);
    bool tma = false;
    for (int i = 0; i < kNumTmaKernels; ++i) tma = tma || params.func == kSplitKernels[i];
    StepExt x{};
    CUtensorMap mk{}, mv{};
    if (tma) {
        // the tensor maps cover the cache rows read at the new length
        x = *static_cast<const StepExt*>(params.kernelParams[1]);
        const uint32_t rows = stage_rows(a.num_kv_heads, false);  // the patched nodes are split kernels
        int s2 = cache_tensor_map(&mk, a.k, a.kv_len, a.num_kv_heads, rows);
        if (s2 == B2_OK) s2 = cache_tensor_map(&mv, a.v, a.kv_len, a.num_kv_heads, rows);
        if (s2 != B2_OK) return s2;
    }
    void* args[4] = {&a, &x, &mk, &mv};
    params.kernelParams = args;
    params.extra = nullptr;
    if (tma)
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

extern "C" size_t b2_decode_step_workspace_bytes(size_t num_heads, size_t num_kv_heads) {
    if (num_kv_heads == 0) return 0;
    return b2::step_workspace_layout(num_heads, num_kv_heads).total_bytes;
}

extern "C" int b2_launch_decode_step_fused(const void* d_q, const void* d_k_new, const void* d_v_new,
                                           void* d_k_cache, void* d_v_cache, const void* d_cos, const void* d_sin,
                                           size_t rope_rows, bool apply_rotation, const int32_t* d_pos,
                                           const int32_t* d_kv_len, int32_t kv_len_bias, size_t max_kv_len,
                                           void* d_out, void* d_workspace, size_t workspace_bytes,
                                           size_t num_heads, size_t num_kv_heads, size_t head_dim,
                                           b2_stream_t stream) {
    return b2::launch_decode_step(d_q, d_k_new, d_v_new, d_k_cache, d_v_cache, d_cos, d_sin, rope_rows,
                                  apply_rotation, d_pos, d_kv_len, kv_len_bias, max_kv_len, d_out, nullptr, nullptr,
                                  nullptr, d_workspace, workspace_bytes, num_heads, num_kv_heads, head_dim, stream);
}

extern "C" int b2_launch_decode_step_fused_rank_partial(
    const void* d_q, const void* d_k_new, const void* d_v_new, void* d_k_cache, void* d_v_cache, const void* d_cos,
    const void* d_sin, size_t rope_rows, bool apply_rotation, const int32_t* d_pos, const int32_t* d_kv_len,
    int32_t kv_len_bias, size_t max_kv_len, float* d_rank_o, float* d_rank_m, float* d_rank_l, void* d_workspace,
    size_t workspace_bytes, size_t num_heads, size_t num_kv_heads, size_t head_dim, b2_stream_t stream) {
    if (!d_rank_o || !d_rank_m || !d_rank_l) return B2_ERR_INVALID_ARG;
    return b2::launch_decode_step(d_q, d_k_new, d_v_new, d_k_cache, d_v_cache, d_cos, d_sin, rope_rows,
                                  apply_rotation, d_pos, d_kv_len, kv_len_bias, max_kv_len, nullptr, d_rank_o,
                                  d_rank_m, d_rank_l, d_workspace, workspace_bytes, num_heads, num_kv_heads,
                                  head_dim, stream);
}

extern "C" size_t b2_decode_exchange_bytes(size_t world, size_t num_heads) {
    if (world == 0 || world > b2::kMaxWorld) return 0;
    // exchange words + the exchange counter, rounded to 256 B
    const size_t words = b2::exchange_words(static_cast<uint32_t>(world), static_cast<uint32_t>(num_heads));
    return (words * sizeof(uint2) + sizeof(uint32_t) + 255) / 256 * 256;
}

extern "C" int b2_launch_decode_step_fused_exchange(
    const void* d_q, const void* d_k_new, const void* d_v_new, void* d_k_cache, void* d_v_cache, const void* d_cos,
    const void* d_sin, size_t rope_rows, bool apply_rotation, const int32_t* d_pos, const int32_t* d_kv_len,
    int32_t kv_len_bias, size_t max_kv_len, void* d_out, void* d_workspace, size_t workspace_bytes,
    size_t world, size_t rank, void* const* exchange_buffers, size_t num_heads, size_t num_kv_heads,
    size_t head_dim, b2_stream_t stream) {
    if (world < 2) return B2_ERR_INVALID_ARG;
    return b2::launch_decode_step(d_q, d_k_new, d_v_new, d_k_cache, d_v_cache, d_cos, d_sin, rope_rows,
                                  apply_rotation, d_pos, d_kv_len, kv_len_bias, max_kv_len, d_out, nullptr, nullptr,
                                  nullptr, d_workspace, workspace_bytes, num_heads, num_kv_heads, head_dim, stream,
                                  world, rank, exchange_buffers);
}

extern "C" int b2_ipc_alloc(size_t bytes, void** d_ptr, void* handle_out) {
    if (d_ptr == nullptr || handle_out == nullptr || bytes == 0) return B2_ERR_INVALID_ARG;
    *d_ptr = nullptr;
    void* p = nullptr;
    int st = b2::cuda_status(cudaMalloc(&p, bytes));
    if (st != B2_OK) return st;
    st = b2::cuda_status(cudaMemset(p, 0, bytes));
    cudaIpcMemHandle_t h;
    if (st == B2_OK) st = b2::cuda_status(cudaIpcGetMemHandle(&h, p));
    if (st != B2_OK) {
        cudaFree(p);
        return st;
    }
    memcpy(handle_out, &h, sizeof(h));
    *d_ptr = p;
    return B2_OK;
}

extern "C" int b2_ipc_open(const void* handle, void** d_ptr) {
    if (d_ptr == nullptr || handle == nullptr) return B2_ERR_INVALID_ARG;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    return b2::cuda_status(cudaIpcOpenMemHandle(d_ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

extern "C" int b2_ipc_close(void* d_ptr) {
    if (d_ptr == nullptr) return B2_ERR_INVALID_ARG;
    return b2::cuda_status(cudaIpcCloseMemHandle(d_ptr));
}

extern "C" int b2_ipc_free(void* d_ptr) {
    if (d_ptr == nullptr) return B2_ERR_INVALID_ARG;
    return b2::cuda_status(cudaFree(d_ptr));
}

extern "C" int b2_advance_position(int32_t* d_pos, int32_t delta, b2_stream_t stream) {
    if (d_pos == nullptr) return B2_ERR_INVALID_ARG;
    return launch_pdl(advance_position_kernel, dim3(1), dim3(1), 0, reinterpret_cast<cudaStream_t>(stream), d_pos,
                      delta);
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
// device address of the array per device, with the id of the context it was
// looked up in: a context torn down and recreated (cudaDeviceReset, primary
// context released) loads the module again, possibly at another address
float* g_noalloc_ptr[64] = {};
unsigned long long g_noalloc_ctx[64] = {};

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

// Id of the calling thread's current context (0 when it cannot be read).
unsigned long long current_context_id() {
    static CtxGetCurrentFn get_current = nullptr;
    static CtxGetIdFn get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<CtxGetCurrentFn>(p);
        p = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<CtxGetIdFn>(p);
    });
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (get_current == nullptr || get_id == nullptr || get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
    if (get_id(ctx, &id) != CUDA_SUCCESS) return 0;
    return id;
}

// Resolve the array's device address for the current device, once per device
// and context. The name is a host-side stand-in in host code; the kernels need
// the address.
int noalloc_scratch(float** out) {
    int dev = 0;
    const cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        note_cuda_error(e);
        return B2_ERR_CUDA;
    }
    if (dev < 0 || dev >= 64) return B2_ERR_UNSUPPORTED;
    // 0 until the runtime has made the device's context current on this
    // thread; the symbol lookup below does that, and the id is read again
    const unsigned long long ctx = current_context_id();
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (g_noalloc_ptr[dev] == nullptr || ctx == 0 || g_noalloc_ctx[dev] != ctx) {
        void* p = nullptr;
        const cudaError_t s = cudaGetSymbolAddress(&p, g_b2_noalloc_scratch);
        if (s != cudaSuccess || p == nullptr) {
            note_cuda_error(s);
            return B2_ERR_CUDA;
        }
        g_noalloc_ptr[dev] = static_cast<float*>(p);
        g_noalloc_ctx[dev] = ctx != 0 ? ctx : current_context_id();
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
