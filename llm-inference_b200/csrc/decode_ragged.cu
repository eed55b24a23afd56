// Ragged batched flash-decode for sm_100a: one new query token for each of B
// sequences whose caches hold different numbers of tokens (the continuous-
// batching decode step; benchmark config 5: 64 sequences, 512..16384 tokens).
//
// The reference engine decodes one sequence at a time
// (src/kernels/causal_attention.hip.cpp:840-921 launch_causal_attention_decode);
// the algebra here is the same split-KV attention and chunk merge (:493-595,
// :719-819), applied to all sequences in one persistent launch:
//
//   * Work unit = (sequence, a range of unit_tokens cached tokens). Units are
//     claimed from a global counter by persistent CTAs (one per SM), so the
//     batch's ~Σ len / unit_tokens units spread evenly however the lengths
//     are distributed. unit_tokens is chosen per launch from the batch's
//     device lengths: about 4.5 units per CTA, between 256 and 768 tokens
//     (a multiple of the consumer parities' tiles) -- short batches get small
//     units for balance, long ones large units for fewer partials.
//   * A producer warp streams each unit's 16-token K/V tiles (4-D tensor
//     map: {64 fp16, row, column block, sequence}, 128-byte swizzle) into the
//     stage ring, plus the sequence's Q row into one of two Q slots; the unit
//     is padded with empty stages to a multiple of the consumer parities so
//     every consumer warp sees every unit.
//   * 12 consumer warps (KV head x tile parity; with fewer than 4 KV heads a
//     stage holds several 16-token sub-tiles per head, one per warp) run the
//     same MMA tile math as the single-sequence kernel and, at each unit
//     boundary, write their own (o, m, l) state as a partial: no CTA-wide
//     barrier per unit, so the producer keeps streaming across unit
//     boundaries.
//   * A merge kernel (one CTA per (sequence, head), four groups of 128
//     threads) folds the npar partials of each of the sequence's units and
//     writes the fp16 output.
#include <math.h>

#include <atomic>
#include <mutex>

#include "b2_common.cuh"
#include "b2_ptx.cuh"
#include "decode_tile.cuh"
#include "tcgen05.cuh"

namespace b2 {
namespace {

constexpr int kRgConsumers = 12;
constexpr int kRgThreads = (kRgConsumers + 1) * 32;
constexpr uint32_t kRgMaxSeqs = 1024;
constexpr uint32_t kRgQSlots = 2;
// Dynamic shared memory requested per CTA at most; with the ~8.6 KB of static
// tables (unit prefix sums, lengths) the CTA stays under 227 KB.
constexpr uint32_t kRgSmemLimit = 214 * 1024;
constexpr uint32_t kNoUnit = 0xffffffffu;

// Unit geometry per KV-head count: npar consumer warps per KV head; a unit is
// a multiple of npar tiles, from at least 16 tiles (256 tokens, the KV_CHUNK)
// up to at least 48 tiles: the largest that still gives every CTA about 4.5
// units (balance), since each unit costs npar partials per head (traffic).
constexpr uint32_t kRgHalfUnitsPerCta = 9;
__host__ __device__ constexpr uint32_t rg_npar(uint32_t kvh) { return kRgConsumers / kvh; }
// With fewer than 4 KV heads a stage carries 4 / KVH sixteen-token sub-tiles
// per head (16 KB per operand: a one-head row is 256 B), one per warp of a
// stage parity; units stay multiples of npar tiles = (npar / sub) stages.
__host__ __device__ constexpr uint32_t rg_sub(uint32_t kvh) { return kvh < 4 ? 4 / kvh : 1; }
__host__ __device__ constexpr uint32_t rg_round_tiles(uint32_t kvh, uint32_t tiles) {
    return rg_npar(kvh) * ((tiles + rg_npar(kvh) - 1) / rg_npar(kvh));
}
__host__ __device__ constexpr uint32_t rg_min_unit_tokens(uint32_t kvh) { return rg_round_tiles(kvh, 16) * kTile; }
__host__ __device__ constexpr uint32_t rg_max_unit_tokens(uint32_t kvh) { return rg_round_tiles(kvh, 48) * kTile; }
// The unit size for a batch of `total_tiles` 16-token tiles over `ctas` CTAs.
__host__ __device__ inline uint32_t rg_unit_tokens(uint32_t kvh, uint32_t total_tiles, uint32_t ctas) {
    const uint32_t want = static_cast<uint32_t>(2ull * total_tiles / (static_cast<uint64_t>(ctas) * kRgHalfUnitsPerCta));
    const uint32_t t = rg_round_tiles(kvh, want) * kTile;
    return t < rg_min_unit_tokens(kvh) ? rg_min_unit_tokens(kvh) : (t > rg_max_unit_tokens(kvh) ? rg_max_unit_tokens(kvh) : t);
}

struct RaggedArgs {
    const __half* q;        // sequence b's query row at q + b * q_seq_stride, [H][128]
    uint64_t q_seq_stride;  // elements
    const int32_t* kv_len;  // [B]; length = clamp(kv_len[b] + bias, 0, max_kv_len)
    int32_t kv_len_bias;
    uint32_t max_kv_len;
    __half* out;            // sequence b's output at out + b * out_seq_stride, [H][128]
    uint64_t out_seq_stride;
    float* po;              // [P][H][128] partial o (unnormalised), P = units * npar
    float* pm;              // [P][H] natural-log max
    float* pl;              // [P][H] weight sum
    uint32_t* counter;      // next unclaimed unit; 0 at launch, reset by the merge
    uint32_t* unit_word;    // this launch's unit size in tokens, for the merge
    uint32_t num_seqs;
    uint32_t num_heads;
    uint32_t group;
    uint32_t stages;
    float scale_log2;
    // fused step only: kv_len holds each sequence's new-token position (bias
    // 1); the new K/V rows (b at k_new / v_new + b * kv_new_stride) are
    // appended at that row of the sequence's cache, Q is rotated in registers
    const __half* k_new;    // nullptr: no append
    const __half* v_new;
    uint64_t kv_new_stride;
    __half* k_cache;        // writable views of the cached rows
    __half* v_cache;
    uint64_t cache_seq_stride;
    const __half* cos;      // RoPE tables [table_rows][64]
    const __half* sin;
    uint32_t rotate;
    uint32_t table_rows;
};

__device__ __forceinline__ uint32_t rg_len(const RaggedArgs& a, uint32_t b) {
    int64_t n = static_cast<int64_t>(__ldg(a.kv_len + b)) + a.kv_len_bias;
    n = n < 0 ? 0 : (n > a.max_kv_len ? a.max_kv_len : n);
    return static_cast<uint32_t>(n);
}

// Bytes of one Q slot: the H query rows.
__host__ __device__ constexpr uint32_t rg_qslot_bytes(uint32_t heads, bool) { return heads * 256; }

// kStep: the fused step -- RoPE of each sequence's new token (the producer
// rotates Q into the Q slot, and rotates K and appends it with V before it
// copies the tile holding that row), then the same split attention.
template <uint32_t KVH, bool kStep>
__global__ void __launch_bounds__(kRgThreads, 1)
    decode_ragged_kernel(const RaggedArgs a, const __grid_constant__ CUtensorMap map_k,
                         const __grid_constant__ CUtensorMap map_v) {
    constexpr uint32_t npar = rg_npar(KVH);        // consumer warps per KV head (partials per unit and head)
    constexpr uint32_t kSub = rg_sub(KVH);         // 16-token sub-tiles per head in a stage
    constexpr uint32_t kRows = kTile * kSub;       // tokens per stage
    constexpr uint32_t spar = npar / kSub;         // stage parities
    constexpr uint32_t row_bytes = KVH * 256;
    constexpr uint32_t tile_bytes = kRows * row_bytes;
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint32_t prefix[kRgMaxSeqs + 1];  // units before sequence b
    __shared__ uint32_t lens[kRgMaxSeqs];
    __shared__ uint32_t st_valid[32], st_unit[32], st_local[32];
    __shared__ uint32_t unit_s;
    __shared__ int32_t rawpos[kStep ? kRgMaxSeqs : 1];  // fused step: the new token's position

    pdl_wait_primary();  // lengths, Q and the caches may come from the previous kernel
    pdl_launch_dependents();
    const uint32_t B = a.num_seqs;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp == 0) {
        // the batch's tiles give the unit size, then the units' prefix sums
        uint32_t tiles = 0;
        for (uint32_t b = lane; b < B; b += 32) {
            const uint32_t len = rg_len(a, b);
            lens[b] = len;
            tiles += (len + kTile - 1) / kTile;
            if constexpr (kStep) {
                const int32_t p = __ldg(a.kv_len + b);
                rawpos[b] = p;
                if (a.rotate && !(p >= 0 && static_cast<uint32_t>(p) < a.table_rows) && blockIdx.x == 0)
                    atomicOr(&g_device_error, kErrBadPosition);
            }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) tiles += __shfl_xor_sync(0xffffffffu, tiles, off);
        const uint32_t unit_tokens = rg_unit_tokens(KVH, tiles, gridDim.x);
        if (lane == 0) {
            unit_s = unit_tokens;
            if (blockIdx.x == 0) *a.unit_word = unit_tokens;
        }
        __syncwarp();
        uint32_t carry = 0;
        for (uint32_t base = 0; base < B; base += 32) {
            const uint32_t b = base + lane;
            uint32_t u = 0;
            if (b < B) u = (lens[b] + unit_tokens - 1) / unit_tokens;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const uint32_t n = __shfl_up_sync(0xffffffffu, u, off);
                if (lane >= off) u += n;
            }
            if (b < B) prefix[b + 1] = carry + u;
            carry += __shfl_sync(0xffffffffu, u, 31);
        }
        if (lane == 0) prefix[0] = 0;
    }

    const uint32_t stages = a.stages;
    const uint32_t q_bytes = a.num_heads * 256;
    const uint32_t qslot_bytes = rg_qslot_bytes(a.num_heads, kStep);
    uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* qslots = ring + stages * 2 * tile_bytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(qslots + kRgQSlots * qslot_bytes);
    uint64_t* empty = full + stages;
    uint64_t* qfull = empty + stages;
    uint64_t* qempty = qfull + kRgQSlots;
    if (threadIdx.x == 32) {
        for (uint32_t s = 0; s < stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], KVH * kSub);
        }
        for (uint32_t s = 0; s < kRgQSlots; ++s) {
            mbar_init(&qfull[s], 1);
            mbar_init(&qempty[s], KVH * npar);
        }
        fence_mbarrier_init();
    }
    __syncthreads();
    const uint32_t U = prefix[B];
    const uint32_t unit_tokens = unit_s;

    bool ok = true;
    if (warp == kRgConsumers) {
        // ---- producer
        if (lane == 0) {
            tc::prefetch_tensormap(&map_k);
            tc::prefetch_tensormap(&map_v);
        }
        const uint64_t policy = l2_evict_first_policy();
        uint32_t i = 0, k = 0;
        uint32_t claimed = lane == 0 ? atomicAdd(a.counter, 1u) : 0u;
        for (;;) {
            const uint32_t u = __shfl_sync(0xffffffffu, claimed, 0);
            if (u >= U) break;
            if (lane == 0) claimed = atomicAdd(a.counter, 1u);  // the next claim is in flight meanwhile
            uint32_t lo = 0, hi = B;  // prefix[lo] <= u < prefix[hi]
            while (hi - lo > 1) {
                const uint32_t mid = (lo + hi) >> 1;
                if (prefix[mid] <= u) lo = mid;
                else hi = mid;
            }
            const uint32_t b = lo, len = lens[b];
            const uint32_t t_begin = (u - prefix[b]) * unit_tokens;
            const uint32_t t_end = min(len, t_begin + unit_tokens);
            const uint32_t ntiles = (t_end - t_begin + kRows - 1) / kRows;
            const uint32_t nstages = (ntiles + spar - 1) / spar * spar;
            // fused step: rotate Q (position in the tables), append the new row
            // (its unit is the sequence's last; the position is in the cache)
            int32_t p = 0;
            bool rot = false, app = false;
            if constexpr (kStep) {
                p = rawpos[b];
                const bool in_table = p >= 0 && static_cast<uint32_t>(p) < a.table_rows;
                rot = a.rotate && in_table;
                app = a.k_new != nullptr && (!a.rotate || in_table) && p >= 0 &&
                      static_cast<uint32_t>(p) < a.max_kv_len && t_end == len;
            }
            // the sequence's Q row into Q slot k % 2: one bulk copy, or (fused
            // step with RoPE) rotated by the warp's lanes and stored, 16 bytes
            // of a head's first and second half per piece
            const uint32_t qs = k % kRgQSlots;
            uint8_t* slot = qslots + qs * qslot_bytes;
            bool w_ok = true;
            if (lane == 0 && k >= kRgQSlots) w_ok = mbar_wait(&qempty[qs], ((k / kRgQSlots) - 1) & 1);
            if (!__shfl_sync(0xffffffffu, w_ok ? 1 : 0, 0)) {
                ok = false;
                break;
            }
            const __half* qsrc = a.q + static_cast<uint64_t>(b) * a.q_seq_stride;
            if (rot) {
                for (uint32_t gi = lane; gi < a.num_heads * 8; gi += 32) {
                    const uint32_t hh = gi >> 3, e = (gi & 7) * 8;
                    uint4 lo4 = *reinterpret_cast<const uint4*>(qsrc + hh * 128 + e);
                    uint4 hi4 = *reinterpret_cast<const uint4*>(qsrc + hh * 128 + 64 + e);
                    const uint64_t ti = static_cast<uint64_t>(p) * 64 + e;
                    rot8_pairs(lo4, hi4, *reinterpret_cast<const uint4*>(a.cos + ti),
                               *reinterpret_cast<const uint4*>(a.sin + ti));
                    *reinterpret_cast<uint4*>(slot + (hh * 128 + e) * 2) = lo4;
                    *reinterpret_cast<uint4*>(slot + (hh * 128 + 64 + e) * 2) = hi4;
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&qfull[qs]);
            } else if (lane == 0) {
                // the slot may hold rotated rows stored through the generic proxy
                if constexpr (kStep) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_arrive_expect_tx(&qfull[qs], q_bytes);
                bulk_g2s_plain(slot, qsrc, q_bytes, &qfull[qs]);
            }
            for (uint32_t j = 0; j < nstages; ++j, ++i) {
                const uint32_t s = i % stages, round = i / stages;
                if (lane == 0 && round > 0) w_ok = mbar_wait(&empty[s], (round - 1) & 1);
                if (!__shfl_sync(0xffffffffu, w_ok ? 1 : 0, 0)) {
                    ok = false;
                    break;
                }
                if (kStep && app && j + 1 == ntiles) {
                    // the new token's K (rotated) and V into row p before the tile
                    // that holds it is copied; the warp's stores reach the tensor
                    // copy through the proxy fence of every lane and the warp sync
                    const uint64_t row = static_cast<uint64_t>(b) * a.cache_seq_stride + static_cast<uint64_t>(p) * (KVH * 128);
                    const __half* kn = a.k_new + static_cast<uint64_t>(b) * a.kv_new_stride;
                    const __half* vn = a.v_new + static_cast<uint64_t>(b) * a.kv_new_stride;
                    for (uint32_t gi = lane; gi < KVH * 8; gi += 32) {
                        const uint32_t hh = gi >> 3, e = (gi & 7) * 8;
                        uint4 lo4 = *reinterpret_cast<const uint4*>(kn + hh * 128 + e);
                        uint4 hi4 = *reinterpret_cast<const uint4*>(kn + hh * 128 + 64 + e);
                        if (a.rotate) {
                            const uint64_t ti = static_cast<uint64_t>(p) * 64 + e;
                            rot8_pairs(lo4, hi4, *reinterpret_cast<const uint4*>(a.cos + ti),
                                       *reinterpret_cast<const uint4*>(a.sin + ti));
                        }
                        *reinterpret_cast<uint4*>(a.k_cache + row + hh * 128 + e) = lo4;
                        *reinterpret_cast<uint4*>(a.k_cache + row + hh * 128 + 64 + e) = hi4;
                        *reinterpret_cast<uint4*>(a.v_cache + row + hh * 128 + e) =
                            *reinterpret_cast<const uint4*>(vn + hh * 128 + e);
                        *reinterpret_cast<uint4*>(a.v_cache + row + hh * 128 + 64 + e) =
                            *reinterpret_cast<const uint4*>(vn + hh * 128 + 64 + e);
                    }
                    asm volatile("fence.proxy.async.global;" ::: "memory");
                    __syncwarp();
                }
                if (lane == 0) {
                    const uint32_t t0 = t_begin + j * kRows;
                    st_unit[s] = u;
                    st_local[s] = k;
                    if (j < ntiles) {
                        st_valid[s] = min(kRows, t_end - t0);
                        mbar_arrive_expect_tx(&full[s], 2 * tile_bytes);
                        uint8_t* stg = ring + s * 2 * tile_bytes;
                        tc::tma_load_4d_hint(stg, &map_k, 0, static_cast<int32_t>(t0), 0, static_cast<int32_t>(b),
                                             &full[s], policy);
                        tc::tma_load_4d_hint(stg + tile_bytes, &map_v, 0, static_cast<int32_t>(t0), 0,
                                             static_cast<int32_t>(b), &full[s], policy);
                    } else {
                        st_valid[s] = 0;  // padding: every parity sees the unit
                        mbar_arrive(&full[s]);
                    }
                }
                __syncwarp();
            }
            if (!ok) break;
            ++k;
        }
        if (ok) {
            // one end marker per stage parity
            for (uint32_t e = 0; e < spar; ++e, ++i) {
                const uint32_t s = i % stages, round = i / stages;
                if (lane == 0) {
                    if (round > 0 && !mbar_wait(&empty[s], (round - 1) & 1)) ok = false;
                    st_unit[s] = kNoUnit;
                    st_valid[s] = 0;
                    mbar_arrive(&full[s]);
                }
            }
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        }
        // never leave the CTA with copies in flight into its shared memory
        if (lane == 0) {
            const uint32_t first = i > stages ? i - stages : 0;
            for (uint32_t j = first; j < i; ++j) (void)mbar_wait(&full[j % stages], (j / stages) & 1);
            for (uint32_t j = k > kRgQSlots ? k - kRgQSlots : 0; j < k; ++j)
                (void)mbar_wait(&qfull[j % kRgQSlots], (j / kRgQSlots) & 1);
        }
    } else if (static_cast<uint32_t>(warp) / KVH < npar) {
        // ---- consumers: warp = KV head (warp % KVH) x j (warp / KVH): sub-tile
        // j % kSub of every spar-th stage from stage parity j / kSub
        const uint32_t kvh = warp % KVH, jw = warp / KVH, sub = jw % kSub, par = jw / kSub;
        const int g = lane >> 2, t = lane & 3;
        WarpState st;
        state_init(st);
        uint32_t qf[8][2];
        uint32_t cur_local = kNoUnit, cur_unit = 0;
        for (uint32_t i = par;; i += spar) {
            const uint32_t s = i % stages, round = i / stages;
            if (!mbar_wait(&full[s], round & 1)) {
                ok = false;
                break;
            }
            const uint32_t u = st_unit[s], kl = st_local[s], rows = st_valid[s];
            // this warp's rows of the stage: [16 sub, 16 sub + 16)
            const uint32_t valid = rows > sub * kTile ? min(static_cast<uint32_t>(kTile), rows - sub * kTile) : 0u;
            if (u == kNoUnit || kl != cur_local) {
                if (cur_local != kNoUnit) {
                    state_finish(st);
                    store_warp_partial(st, a.po, a.pm, a.pl, 128, static_cast<uint64_t>(a.num_heads) * 128, 64, 1,
                                       a.num_heads, cur_unit * npar + jw, kvh * a.group, a.group, g, t);
                    state_init(st);
                }
                if (u == kNoUnit) break;
                const uint32_t qs = kl % kRgQSlots;
                if (!mbar_wait(&qfull[qs], (kl / kRgQSlots) & 1)) {
                    ok = false;
                    break;
                }
                if (static_cast<uint32_t>(g) < a.group) {
                    const uint8_t* qrow = qslots + qs * qslot_bytes + (kvh * a.group + g) * 256;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const uint4 w = lds128(qrow + (32 * j + 8 * t) * 2);
                        qf[2 * j][0] = w.x;
                        qf[2 * j][1] = w.y;
                        qf[2 * j + 1][0] = w.z;
                        qf[2 * j + 1][1] = w.w;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 8; ++j) qf[j][0] = qf[j][1] = 0u;
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&qempty[qs]);
                cur_local = kl;
                cur_unit = u;
            }
            if (valid != 0) {
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
                if (lane == 0) mbar_arrive(&empty[s]);
                tile_softmax_pv(st, sc, va, g, t);
            } else {
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
            }
        }
    }
    if (!ok) atomicOr(&g_device_error, kErrWaitTimeout);
}

// One CTA per (sequence, head), 4 groups of 128 threads (thread = output dim):
// group g folds the sequence's partials g, g + 4, ... (online rescale, batches
// of 8 in flight), the four group states meet in shared memory and threads
// 0..127 write the fp16 output. Block (0, 0) resets the claim counter for the
// next launch.
constexpr int kRgMergeBatch = 8;
constexpr int kRgMergeGroups = 4;
constexpr int kRgMergeThreads = 128 * kRgMergeGroups;

__global__ void __launch_bounds__(kRgMergeThreads) merge_ragged_kernel(const RaggedArgs a, uint32_t npar) {
    __shared__ uint32_t part_s[kRgMergeThreads / 32];
    __shared__ float grp_m[kRgMergeGroups], grp_l[kRgMergeGroups];
    __shared__ float grp_o[kRgMergeGroups][128];
    pdl_wait_primary();
    pdl_launch_dependents();
    const uint32_t unit_tokens = __ldcg(a.unit_word);  // written by the decode kernel
    const uint32_t b = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
    const uint32_t d = tid & 127, grp = tid >> 7;
    if (b == 0 && h == 0 && tid == 0) *a.counter = 0u;
    // units of the sequences before b
    uint32_t before = 0;
    for (uint32_t j = tid; j < b; j += kRgMergeThreads) before += (rg_len(a, j) + unit_tokens - 1) / unit_tokens;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) before += __shfl_xor_sync(0xffffffffu, before, off);
    if ((tid & 31) == 0) part_s[tid >> 5] = before;
    __syncthreads();
    before = 0;
#pragma unroll
    for (int w = 0; w < kRgMergeThreads / 32; ++w) before += part_s[w];
    const uint32_t units = (rg_len(a, b) + unit_tokens - 1) / unit_tokens;
    const uint32_t p0 = before * npar, n = units * npar;
    const uint32_t H = a.num_heads;
    float M = -INFINITY, L = 0.f, O = 0.f;
    for (uint32_t base = grp; base < n; base += kRgMergeBatch * kRgMergeGroups) {
        float mv[kRgMergeBatch], lv[kRgMergeBatch], ov[kRgMergeBatch];
#pragma unroll
        for (int u = 0; u < kRgMergeBatch; ++u) {
            const uint32_t c = base + u * kRgMergeGroups;
            const uint64_t p = static_cast<uint64_t>(p0 + c) * H + h;
            mv[u] = c < n ? __ldg(a.pm + p) : -INFINITY;
            lv[u] = c < n ? __ldg(a.pl + p) : 0.f;
            ov[u] = c < n ? __ldg(a.po + p * 128 + d) : 0.f;
        }
        float bm = M;
#pragma unroll
        for (int u = 0; u < kRgMergeBatch; ++u) bm = fmaxf(bm, mv[u]);
        if (bm == -INFINITY) continue;
        const float sc = M == -INFINITY ? 0.f : expf(M - bm);
        O *= sc;
        L *= sc;
        M = bm;
#pragma unroll
        for (int u = 0; u < kRgMergeBatch; ++u) {
            const float w = mv[u] == -INFINITY ? 0.f : expf(mv[u] - M);
            O = fmaf(w, ov[u], O);
            L = fmaf(w, lv[u], L);
        }
    }
    grp_o[grp][d] = O;
    if (d == 0) {
        grp_m[grp] = M;
        grp_l[grp] = L;
    }
    __syncthreads();
    if (grp != 0) return;
    float Mx = -INFINITY;
#pragma unroll
    for (int g = 0; g < kRgMergeGroups; ++g) Mx = fmaxf(Mx, grp_m[g]);
    float Ox = 0.f, Lx = 0.f;
#pragma unroll
    for (int g = 0; g < kRgMergeGroups; ++g) {
        const float sc = grp_m[g] == -INFINITY ? 0.f : expf(grp_m[g] - Mx);
        Ox = fmaf(sc, grp_o[g][d], Ox);
        Lx = fmaf(sc, grp_l[g], Lx);
    }
    a.out[static_cast<uint64_t>(b) * a.out_seq_stride + h * 128 + d] = __float2half_rn(Lx > 0.f ? Ox / Lx : 0.f);
}

bool rg_kvh_ok(size_t kvh) { return kvh == 1 || kvh == 2 || kvh == 4 || kvh == 8; }

int device_sms_rg() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
    return n;
}

struct RgWorkspace {
    size_t po, pm, pl, counter, total_bytes;  // counter: the claim counter, then the unit-size word
};

RgWorkspace rg_layout(size_t num_seqs, size_t num_heads, size_t num_kv_heads, size_t max_kv_len) {
    RgWorkspace w{};
    const uint32_t kvh = static_cast<uint32_t>(num_kv_heads);
    const size_t units = num_seqs * ((max_kv_len + rg_min_unit_tokens(kvh) - 1) / rg_min_unit_tokens(kvh));
    const size_t P = units * rg_npar(kvh);
    w.po = 0;
    w.pm = w.po + P * num_heads * 128;
    w.pl = w.pm + P * num_heads;
    w.counter = w.pl + P * num_heads;
    w.total_bytes = (w.counter * sizeof(float) + 2 * sizeof(uint32_t) + 255) / 256 * 256;
    return w;
}

template <uint32_t KVH, bool kStep>
int launch_ragged_kvh(const RaggedArgs& a, const CUtensorMap& mk, const CUtensorMap& mv, uint32_t grid, size_t smem,
                      cudaStream_t stream) {
    static std::atomic<uint64_t> attr_done{0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return B2_ERR_CUDA;
    const uint64_t bit = 1ull << (dev & 63);
    if (!(attr_done.load() & bit)) {
        const int st = cuda_status(cudaFuncSetAttribute(decode_ragged_kernel<KVH, kStep>,
                                                        cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                        static_cast<int>(kRgSmemLimit)));
        if (st != B2_OK) return st;
        attr_done.fetch_or(bit);
    }
    return launch_pdl(decode_ragged_kernel<KVH, kStep>, dim3(grid), dim3(kRgThreads), smem, stream, a, mk, mv);
}

// Inputs of one ragged launch (the plain decode, or the fused step).
struct RaggedCall {
    const void* q;
    size_t q_seq_stride;
    const void* k_cache;
    const void* v_cache;
    size_t cache_seq_stride;
    const int32_t* kv_len;
    int32_t kv_len_bias;
    size_t max_kv_len;
    void* out;
    size_t out_seq_stride;
    size_t num_seqs, num_heads, num_kv_heads, head_dim;
    void* workspace;
    size_t workspace_bytes;
    // fused step
    bool step;
    const void* k_new;
    const void* v_new;
    size_t kv_new_stride;
    const void* cos;
    const void* sin;
    size_t rope_rows;
    bool rotate;
};

int launch_ragged(RaggedCall c, cudaStream_t stream) {
    if (c.num_seqs == 0 || c.max_kv_len == 0 || c.num_kv_heads == 0 || c.head_dim == 0) return B2_NOTHING_TO_DO;
    if (c.num_heads % c.num_kv_heads != 0) return B2_NOTHING_TO_DO;
    if (!c.q || !c.k_cache || !c.v_cache || !c.kv_len || !c.out || !c.workspace) return B2_ERR_INVALID_ARG;
    const size_t group = c.num_heads / c.num_kv_heads;
    if (c.head_dim != 128 || !rg_kvh_ok(c.num_kv_heads) || group > 8 || c.num_seqs > kRgMaxSeqs ||
        c.max_kv_len > 0x7fffffffull)
        return B2_ERR_UNSUPPORTED;
    const size_t kv_dim = c.num_kv_heads * c.head_dim;
    if (c.q_seq_stride == 0) c.q_seq_stride = c.num_heads * c.head_dim;
    if (c.out_seq_stride == 0) c.out_seq_stride = c.num_heads * c.head_dim;
    if (c.cache_seq_stride == 0) c.cache_seq_stride = c.max_kv_len * kv_dim;
    if (c.q_seq_stride < c.num_heads * c.head_dim || c.out_seq_stride < c.num_heads * c.head_dim)
        return B2_ERR_INVALID_ARG;
    if (c.num_seqs > 1 && c.cache_seq_stride < c.max_kv_len * kv_dim) return B2_ERR_INVALID_ARG;  // caches overlap
    if (!aligned16(c.q) || !aligned16(c.k_cache) || !aligned16(c.v_cache) || !aligned16(c.workspace) ||
        c.q_seq_stride % 8 != 0 || c.cache_seq_stride % 8 != 0)
        return B2_ERR_ALIGNMENT;
    if (c.step) {
        if (c.k_new && !c.v_new) return B2_ERR_INVALID_ARG;
        if (c.rotate && (!c.cos || !c.sin || c.rope_rows == 0)) return B2_ERR_INVALID_ARG;
        if (c.rope_rows > 0x7fffffffull) return B2_ERR_UNSUPPORTED;
        if (c.kv_new_stride == 0) c.kv_new_stride = kv_dim;
        if (c.k_new && c.kv_new_stride < kv_dim) return B2_ERR_INVALID_ARG;
        if ((c.k_new && (!aligned16(c.k_new) || !aligned16(c.v_new) || c.kv_new_stride % 8 != 0)) ||
            (c.rotate && (!aligned16(c.cos) || !aligned16(c.sin))))
            return B2_ERR_ALIGNMENT;
    }
    const RgWorkspace w = rg_layout(c.num_seqs, c.num_heads, c.num_kv_heads, c.max_kv_len);
    if (c.workspace_bytes < w.total_bytes) return B2_ERR_WORKSPACE;
    const uint32_t kvh = static_cast<uint32_t>(c.num_kv_heads);
    const uint32_t npar = rg_npar(kvh);                     // partials per unit and head
    const uint32_t rows = kTile * rg_sub(kvh);             // tokens per stage
    const uint32_t spar = rg_npar(kvh) / rg_sub(kvh);       // stage parities: the ring depth's divisor
    const size_t stage_bytes = 2ull * rows * kvh * 256;
    const size_t fixed = 1024 + kRgQSlots * rg_qslot_bytes(static_cast<uint32_t>(c.num_heads), c.step) + 256;
    uint32_t stages = static_cast<uint32_t>((kRgSmemLimit - fixed) / stage_bytes) / spar * spar;
    if (stages > 32) stages = 32 / spar * spar;
    if (stages == 0) return B2_ERR_UNSUPPORTED;

    float* ws = static_cast<float*>(c.workspace);
    RaggedArgs a{};
    a.q = static_cast<const __half*>(c.q);
    a.q_seq_stride = c.q_seq_stride;
    a.kv_len = c.kv_len;
    a.kv_len_bias = c.kv_len_bias;
    a.max_kv_len = static_cast<uint32_t>(c.max_kv_len);
    a.out = static_cast<__half*>(c.out);
    a.out_seq_stride = c.out_seq_stride;
    a.po = ws + w.po;
    a.pm = ws + w.pm;
    a.pl = ws + w.pl;
    a.counter = reinterpret_cast<uint32_t*>(ws + w.counter);
    a.unit_word = a.counter + 1;
    a.num_seqs = static_cast<uint32_t>(c.num_seqs);
    a.num_heads = static_cast<uint32_t>(c.num_heads);
    a.group = static_cast<uint32_t>(group);
    a.stages = stages;
    a.scale_log2 = kLog2e / sqrtf(static_cast<float>(c.head_dim));
    if (c.step) {
        a.k_new = static_cast<const __half*>(c.k_new);
        a.v_new = static_cast<const __half*>(c.v_new);
        a.kv_new_stride = c.kv_new_stride;
        a.k_cache = static_cast<__half*>(const_cast<void*>(c.k_cache));
        a.v_cache = static_cast<__half*>(const_cast<void*>(c.v_cache));
        a.cache_seq_stride = c.cache_seq_stride;
        a.cos = static_cast<const __half*>(c.cos);
        a.sin = static_cast<const __half*>(c.sin);
        a.rotate = c.rotate ? 1u : 0u;
        a.table_rows = static_cast<uint32_t>(c.rope_rows);
    }

    CUtensorMap mk, mv;
    if (encode_token_rows_by_column_block_seqs(&mk, c.k_cache, c.max_kv_len, kvh * 256, c.num_seqs,
                                               c.cache_seq_stride * 2, rows) != 0 ||
        encode_token_rows_by_column_block_seqs(&mv, c.v_cache, c.max_kv_len, kvh * 256, c.num_seqs,
                                               c.cache_seq_stride * 2, rows) != 0)
        return B2_ERR_CUDA;
    const size_t smem = fixed + stages * stage_bytes + 2 * (stages + kRgQSlots) * sizeof(uint64_t);
    const uint32_t grid = static_cast<uint32_t>(device_sms_rg());
    int st;
    if (c.step) {
        switch (kvh) {
            case 1: st = launch_ragged_kvh<1, true>(a, mk, mv, grid, smem, stream); break;
            case 2: st = launch_ragged_kvh<2, true>(a, mk, mv, grid, smem, stream); break;
            case 4: st = launch_ragged_kvh<4, true>(a, mk, mv, grid, smem, stream); break;
            default: st = launch_ragged_kvh<8, true>(a, mk, mv, grid, smem, stream); break;
        }
    } else {
        switch (kvh) {
            case 1: st = launch_ragged_kvh<1, false>(a, mk, mv, grid, smem, stream); break;
            case 2: st = launch_ragged_kvh<2, false>(a, mk, mv, grid, smem, stream); break;
            case 4: st = launch_ragged_kvh<4, false>(a, mk, mv, grid, smem, stream); break;
            default: st = launch_ragged_kvh<8, false>(a, mk, mv, grid, smem, stream); break;
        }
    }
    if (st != B2_OK) return st;
    return launch_pdl(merge_ragged_kernel, dim3(a.num_seqs, a.num_heads), dim3(kRgMergeThreads), 0, stream, a, npar);
}

}  // namespace

unsigned int device_error_ragged() {
    unsigned int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v)) != cudaSuccess) return 0;
    return v;
}

int clear_device_error_ragged() {
    const unsigned int zero = 0;
    return cuda_status(cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero)));
}

}  // namespace b2

extern "C" size_t b2_decode_ragged_workspace_bytes(size_t num_seqs, size_t num_heads, size_t num_kv_heads,
                                                   size_t max_kv_len) {
    if (!b2::rg_kvh_ok(num_kv_heads)) return 0;
    return b2::rg_layout(num_seqs, num_heads, num_kv_heads, max_kv_len).total_bytes;
}

extern "C" int b2_launch_causal_attention_decode_ragged(const void* d_q, size_t q_seq_stride, const void* d_k_cache,
                                                        const void* d_v_cache, size_t cache_seq_stride,
                                                        const int32_t* d_kv_len, int32_t kv_len_bias,
                                                        size_t max_kv_len, void* d_out, size_t out_seq_stride,
                                                        size_t num_seqs, size_t num_heads, size_t num_kv_heads,
                                                        size_t head_dim, void* d_workspace, size_t workspace_bytes,
                                                        b2_stream_t stream_handle) {
    b2::RaggedCall c{};
    c.q = d_q;
    c.q_seq_stride = q_seq_stride;
    c.k_cache = d_k_cache;
    c.v_cache = d_v_cache;
    c.cache_seq_stride = cache_seq_stride;
    c.kv_len = d_kv_len;
    c.kv_len_bias = kv_len_bias;
    c.max_kv_len = max_kv_len;
    c.out = d_out;
    c.out_seq_stride = out_seq_stride;
    c.num_seqs = num_seqs;
    c.num_heads = num_heads;
    c.num_kv_heads = num_kv_heads;
    c.head_dim = head_dim;
    c.workspace = d_workspace;
    c.workspace_bytes = workspace_bytes;
    return b2::launch_ragged(c, reinterpret_cast<cudaStream_t>(stream_handle));
}

extern "C" int b2_launch_decode_step_ragged_fused(const void* d_q, size_t q_seq_stride, const void* d_k_new,
                                                  const void* d_v_new, size_t kv_new_stride, void* d_k_cache,
                                                  void* d_v_cache, size_t cache_seq_stride, const void* d_cos,
                                                  const void* d_sin, size_t rope_rows, bool apply_rotation,
                                                  const int32_t* d_pos, size_t max_kv_len, void* d_out,
                                                  size_t out_seq_stride, size_t num_seqs, size_t num_heads,
                                                  size_t num_kv_heads, size_t head_dim, void* d_workspace,
                                                  size_t workspace_bytes, b2_stream_t stream_handle) {
    b2::RaggedCall c{};
    c.q = d_q;
    c.q_seq_stride = q_seq_stride;
    c.k_cache = d_k_cache;
    c.v_cache = d_v_cache;
    c.cache_seq_stride = cache_seq_stride;
    c.kv_len = d_pos;
    c.kv_len_bias = 1;
    c.max_kv_len = max_kv_len;
    c.out = d_out;
    c.out_seq_stride = out_seq_stride;
    c.num_seqs = num_seqs;
    c.num_heads = num_heads;
    c.num_kv_heads = num_kv_heads;
    c.head_dim = head_dim;
    c.workspace = d_workspace;
    c.workspace_bytes = workspace_bytes;
    c.step = true;
    c.k_new = d_k_new;
    c.v_new = d_v_new;
    c.kv_new_stride = kv_new_stride;
    c.cos = d_cos;
    c.sin = d_sin;
    c.rope_rows = rope_rows;
    c.rotate = apply_rotation;
    return b2::launch_ragged(c, reinterpret_cast<cudaStream_t>(stream_handle));
}
