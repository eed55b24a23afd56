// Causal GQA prefill on the 5th-generation tensor cores (tcgen05 + TMA + TMEM).
//
// Computes what src/kernels/causal_attention.hip.cpp:271-374 computes
// (out[t][h] = softmax_{j<=t}(q_t . k_j / sqrt(d)) V, GQA kv head h/group,
// packed fp16 output) for head_dim 128, with the Blackwell dense-GEMM
// treatment instead of the reference's scalar 8x8 tiles:
//
// * one CTA per (128-query tile, query head, sequence), heaviest (most KV
//   tiles) first; KV tiles strictly above the diagonal are never touched
//   (causal tile skipping), only the diagonal tile is masked;
// * warp 0: TMA producer -- Q tile once, then K and V 128x128 tiles through a
//   2-stage ring each (128-byte swizzle, tensor maps over the caller's rows, so
//   the interleaved [Q|K|V] layout and the KV cache are read in place);
// * warp 1: allocates TMEM and issues tcgen05.mma from one thread:
//   S_j = Q K_j^T into one of two TMEM S buffers (128 fp32 columns each), then
//   O += P_j V_j with P_j read straight from TMEM (kind::f16, f32 accumulate);
//   S_{j+1} is issued before waiting for P_j so the tensor core works on the
//   next tile while the softmax warps handle this one;
// * warps 4-7: one query row per thread: tcgen05.ld the S row, online softmax
//   in the log2 domain with a lazily moved running max (O in TMEM is rescaled
//   only when a row max grows by more than 2^8), P packed to fp16 and
//   tcgen05.st over the S buffer; finally O / l to fp16 rows in global memory.
// All mbarrier waits are bounded (b2_ptx.cuh) and every issued copy and MMA is
// drained before TMEM is freed.
#include <math.h>

#include <atomic>

#include "b2_common.cuh"
#include "b2_ptx.cuh"
#include "prefill.h"
#include "tcgen05.cuh"

namespace b2 {
namespace {

constexpr int kThreads = 256;
constexpr uint32_t kTileBytes = 128 * 128 * 2;  // one 128x128 fp16 tile (two 64-column swizzle boxes)
constexpr uint32_t kBoxBytes = kTileBytes / 2;
constexpr int kStages = 2;
constexpr uint32_t kSmemTiles = (1 + 2 * kStages) * kTileBytes;  // Q + K ring + V ring
constexpr uint32_t kSmemBytes = kSmemTiles + 1024 /*barriers*/ + 1024 /*alignment slack*/;
constexpr uint32_t kTmemCols = 512;   // S0 [0,128), S1 [128,256), O [256,384)
constexpr float kRescaleThreshold = 8.f;

struct Bars {
    uint64_t q_full;
    uint64_t k_full[kStages], k_empty[kStages];
    uint64_t v_full[kStages], v_empty[kStages];
    uint64_t s_full[2], p_full[2];
    uint64_t o_done;
    uint64_t drain;
    uint32_t tmem_base;
    uint32_t abort;
};

__device__ __forceinline__ float ex2f(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// This CTA's work item. The grid is (q tiles, head units, sequences) and CTAs
// start in linear block order, so the linear index is dealt longest-first
// over the whole grid: every sequence's and head unit's last q tile (the most
// KV tiles) first, then the next, ... -- the lightest items run last, and no
// heavy tile of a late head unit starts near the end of the launch.
__device__ __forceinline__ void prefill_item(uint32_t num_q_tiles, uint32_t& qt, uint32_t& unit, uint32_t& b) {
    const uint32_t units = gridDim.y * gridDim.z;
    const uint32_t id = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
    const uint32_t level = id / units, r = id - level * units;
    qt = num_q_tiles - 1 - level;
    unit = r % gridDim.y;
    b = r / gridDim.y;
}

__global__ void __launch_bounds__(kThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                      const __grid_constant__ CUtensorMap map_v, const PrefillArgs a, const uint32_t num_q_tiles) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* sq = smem;
    uint8_t* sk = smem + kTileBytes;                       // [kStages] tiles
    uint8_t* sv = smem + (1 + kStages) * kTileBytes;       // [kStages] tiles
    Bars* bars = reinterpret_cast<Bars*>(smem + kSmemTiles);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint32_t qt, h, b;
    prefill_item(num_q_tiles, qt, h, b);
    const uint32_t kvh = h / a.group;
    const uint32_t q_row0 = qt * 128;
    const uint32_t n_kv = qt + 1;                          // causal: KV tiles 0..qt

    if (threadIdx.x == 0) {
        mbar_init(&bars->q_full, 1);
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&bars->k_full[s], 1);
            mbar_init(&bars->k_empty[s], 1);
            mbar_init(&bars->v_full[s], 1);
            mbar_init(&bars->v_empty[s], 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(&bars->s_full[s], 1);
            mbar_init(&bars->p_full[s], 4);
        }
        mbar_init(&bars->o_done, 1);
        mbar_init(&bars->drain, 1);
        bars->abort = 0;
        fence_mbarrier_init();
    }
    if (warp == 1) tc::tmem_alloc(&bars->tmem_base, kTmemCols);
    pdl_wait_primary();  // Q/K/V may be written by the previous kernel (RoPE / append)
    pdl_launch_dependents();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tbase = bars->tmem_base;

    if (warp == 0) {
        // ---------------- TMA producer
        if (lane == 0) {
            tc::prefetch_tensormap(&map_q);
            tc::prefetch_tensormap(&map_k);
            tc::prefetch_tensormap(&map_v);
            const int32_t qx = static_cast<int32_t>(h * 128), kx = static_cast<int32_t>(kvh * 128);
            mbar_arrive_expect_tx(&bars->q_full, kTileBytes);
            tc::tma_load_3d(sq, &map_q, qx, q_row0, b, &bars->q_full);
            tc::tma_load_3d(sq + kBoxBytes, &map_q, qx + 64, q_row0, b, &bars->q_full);
            uint32_t issued_k = 0, issued_v = 0;
            bool ok = true;
            for (uint32_t j = 0; j < n_kv && ok; ++j) {
                const uint32_t s = j % kStages, r = j / kStages;
                const int32_t y = static_cast<int32_t>(j * 128);
                if (r > 0 && !(ok = mbar_wait(&bars->k_empty[s], (r - 1) & 1))) break;
                mbar_arrive_expect_tx(&bars->k_full[s], kTileBytes);
                tc::tma_load_3d(sk + s * kTileBytes, &map_k, kx, y, b, &bars->k_full[s]);
                tc::tma_load_3d(sk + s * kTileBytes + kBoxBytes, &map_k, kx + 64, y, b, &bars->k_full[s]);
                issued_k = j + 1;
                if (r > 0 && !(ok = mbar_wait(&bars->v_empty[s], (r - 1) & 1))) break;
                mbar_arrive_expect_tx(&bars->v_full[s], kTileBytes);
                tc::tma_load_3d(sv + s * kTileBytes, &map_v, kx, y, b, &bars->v_full[s]);
                tc::tma_load_3d(sv + s * kTileBytes + kBoxBytes, &map_v, kx + 64, y, b, &bars->v_full[s]);
                issued_v = j + 1;
            }
            if (!ok) bars->abort = 1;
            // drain: every issued copy lands before the CTA can exit
            (void)mbar_wait(&bars->q_full, 0);
            for (uint32_t j = issued_k > kStages ? issued_k - kStages : 0; j < issued_k; ++j)
                (void)mbar_wait(&bars->k_full[j % kStages], (j / kStages) & 1);
            for (uint32_t j = issued_v > kStages ? issued_v - kStages : 0; j < issued_v; ++j)
                (void)mbar_wait(&bars->v_full[j % kStages], (j / kStages) & 1);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (one thread)
        if (lane == 0) {
            constexpr uint32_t id_s = tc::idesc_f16_f32(128, 128, false, false);
            constexpr uint32_t id_o = tc::idesc_f16_f32(128, 128, false, true);
            const uint32_t tmem_o = tbase + 256;
            bool ok = mbar_wait(&bars->q_full, 0);
            auto issue_s = [&](uint32_t j) -> bool {
                const uint32_t s = j % kStages;
                if (!mbar_wait(&bars->k_full[s], (j / kStages) & 1)) return false;
                tc::fence_after_sync();
                const uint32_t kbase = smem_u32(sk + s * kTileBytes), qbase = smem_u32(sq);
#pragma unroll
                for (uint32_t ks = 0; ks < 8; ++ks) {
                    const uint32_t off = (ks >> 2) * kBoxBytes + (ks & 3) * 32;
                    tc::mma_ss(tbase + (j & 1) * 128, tc::desc_kmajor_sw128(qbase + off),
                               tc::desc_kmajor_sw128(kbase + off), id_s, ks > 0);
                }
                tc::commit(&bars->s_full[j & 1]);
                tc::commit(&bars->k_empty[s]);
                return true;
            };
            if (ok) ok = issue_s(0);
            for (uint32_t j = 0; j < n_kv && ok; ++j) {
                if (j + 1 < n_kv && !(ok = issue_s(j + 1))) break;
                if (!(ok = mbar_wait(&bars->p_full[j & 1], (j >> 1) & 1))) break;
                const uint32_t s = j % kStages;
                if (!(ok = mbar_wait(&bars->v_full[s], (j / kStages) & 1))) break;
                tc::fence_after_sync();
                const uint32_t vbase = smem_u32(sv + s * kTileBytes);
#pragma unroll
                for (uint32_t ks = 0; ks < 8; ++ks)
                    tc::mma_ts(tmem_o, tbase + (j & 1) * 128 + ks * 8, tc::desc_mnmajor_sw128(vbase + ks * 2048, kBoxBytes),
                               id_o, (j > 0 || ks > 0) ? 1u : 0u);
                tc::commit(&bars->v_empty[s]);
                tc::commit(&bars->o_done);
            }
            if (!ok) bars->abort = 1;
            // every issued MMA completes before TMEM is released
            tc::commit(&bars->drain);
            (void)mbar_wait(&bars->drain, 0);
        }
    } else if (warp >= 4) {
        // ---------------- softmax: one query row per thread
        const uint32_t quarter = warp - 4;
        const uint32_t r = quarter * 32 + lane;        // row within the tile == TMEM lane
        const uint32_t lane_addr = (quarter * 32) << 16;
        const uint32_t grow = q_row0 + r;              // query position
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        for (uint32_t j = 0; j < n_kv; ++j) {
            const uint32_t buf = j & 1;
            if (!(ok = mbar_wait(&bars->s_full[buf], (j >> 1) & 1))) break;
            tc::fence_after_sync();
            float s[128];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                uint32_t raw[32];
                tc::tmem_ld32(tbase + lane_addr + buf * 128 + c * 32, raw);
                tc::tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i) s[c * 32 + i] = __uint_as_float(raw[i]) * a.scale_log2;
            }
            if (j == qt) {  // diagonal tile: keys after the query are masked
#pragma unroll
                for (int c = 0; c < 128; ++c)
                    if (j * 128 + c > grow) s[c] = -INFINITY;
            }
            float mx = s[0];
#pragma unroll
            for (int c = 1; c < 128; ++c) mx = fmaxf(mx, s[c]);
            const bool need = mx > m + kRescaleThreshold;
            if (__any_sync(0xffffffffu, need)) {
                const float mn = fmaxf(m, mx);
                const float alpha = ex2f(m - mn);  // 0 for the first tile
                if (j > 0) {
                    // O holds sum_{<j} P V: rescale it once PV_{j-1} is done
                    if (!(ok = mbar_wait(&bars->o_done, (j - 1) & 1))) break;
                    tc::fence_after_sync();
#pragma unroll 1
                    for (int c = 0; c < 4; ++c) {
                        uint32_t raw[32];
                        const uint32_t addr = tbase + lane_addr + 256 + c * 32;
                        tc::tmem_ld32(addr, raw);
                        tc::tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; ++i) raw[i] = __float_as_uint(__uint_as_float(raw[i]) * alpha);
                        tc::tmem_st32(addr, raw);
                    }
                    tc::tmem_wait_st();
                }
                l *= alpha;
                m = mn;
            }
            uint32_t packed[64];
            float rs = 0.f;
#pragma unroll
            for (int c = 0; c < 64; ++c) {
                const float p0 = ex2f(s[2 * c] - m), p1 = ex2f(s[2 * c + 1] - m);
                rs += p0 + p1;
                packed[c] = pack_half2(p0, p1);
            }
            l += rs;
            tc::tmem_st32(tbase + lane_addr + buf * 128, *reinterpret_cast<const uint32_t(*)[32]>(&packed[0]));
            tc::tmem_st32(tbase + lane_addr + buf * 128 + 32, *reinterpret_cast<const uint32_t(*)[32]>(&packed[32]));
            tc::tmem_wait_st();
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->p_full[buf]);
        }
        if (ok) ok = mbar_wait(&bars->o_done, (n_kv - 1) & 1);
        if (ok) {
            tc::fence_after_sync();
            const float inv = 1.f / l;
            __half* orow = a.out + static_cast<uint64_t>(b) * a.out_batch_stride +
                           static_cast<uint64_t>(grow) * a.out_stride + static_cast<uint64_t>(h) * 128;
#pragma unroll 1
            for (int c = 0; c < 4; ++c) {
                uint32_t raw[32];
                tc::tmem_ld32(tbase + lane_addr + 256 + c * 32, raw);
                tc::tmem_wait_ld();
                uint32_t o16[16];
#pragma unroll
                for (int i = 0; i < 16; ++i)
                    o16[i] = pack_half2(__uint_as_float(raw[2 * i]) * inv, __uint_as_float(raw[2 * i + 1]) * inv);
                if (grow < a.seq_len) {
                    uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        dst[i] = make_uint4(o16[4 * i], o16[4 * i + 1], o16[4 * i + 2], o16[4 * i + 3]);
                }
            }
        } else {
            bars->abort = 1;
        }
        tc::fence_before_sync();
    }
    __syncthreads();
    if (bars->abort && threadIdx.x == 0) atomicOr(&g_device_error, kErrWaitTimeout);
    if (warp == 1) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tbase, kTmemCols);
    }
}

// ---------------------------------------------------------------------------
// Head-pair kernel: one CTA per (128-query tile, two query heads of one GQA
// group, sequence). Both heads read the same K/V tiles, so each tile is
// staged once for twice the math, and the tensor core alternates between the
// two heads' MMAs while each head's softmax warpgroup works on its own S:
//   TMEM: S_A [0,128), S_B [128,256), O_A [256,384), O_B [384,512)
//   MMA order per KV tile j: PV_A(j-1)... i.e.
//     S_A(0) S_B(0) | PV_A(0) S_A(1) PV_B(0) S_B(1) | PV_A(1) S_A(2) ...
//   (P_A is read from S_A by PV_A(j) before S_A(j+1) overwrites it: the MMAs
//   of one thread execute in issue order). A commit after S_X(j) also covers
//   PV_X(j-1), so the softmax warps may rescale O_X as soon as S_X(j) is
//   complete.
// Warps: 0 TMA producer, 1 TMEM + MMA, 4-7 softmax of head A, 8-11 of head B
// (warp w reads TMEM lanes 32 * (w % 4) ...).
constexpr int kPairThreads = 384;
constexpr int kRegsCtl = 88;       // per thread, producer / MMA warpgroup
constexpr int kRegsSoftmax = 200;  // per thread, each softmax warpgroup
static_assert(4 * 32 * (kRegsCtl + 2 * kRegsSoftmax) <= kPairThreads * 168, "register split above the launch's");

constexpr uint32_t kPairSmemTiles = (2 + 2 * kStages) * kTileBytes;  // Q_A, Q_B, K ring, V ring
constexpr uint32_t kPairSmemBytes = kPairSmemTiles + 1024 + 1024;

struct PairBars {
    uint64_t q_full;
    uint64_t k_full[kStages], k_empty[kStages];
    uint64_t v_full[kStages], v_empty[kStages];
    uint64_t s_full[2], p_full[2], o_done[2];
    uint64_t drain;
    uint32_t tmem_base;
    uint32_t abort;
};

// ---- softmax arithmetic on packed fp32 pairs (sm_100 f32x2 instructions) ----
__device__ __forceinline__ void ffma2(float& d0, float& d1, float a0, float a1, float b0, float b1, float c0,
                                      float c1) {
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "mov.b64 rc, {%6, %7};\n\tfma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d0), "=f"(d1)
        : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}
__device__ __forceinline__ void fadd2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
    asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d0), "=f"(d1)
        : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// Softmax warpgroup of one head: rows of the 128-query tile, one per thread.
__device__ __forceinline__ bool pair_softmax(const PrefillArgs& a, PairBars* bars, uint32_t tbase, uint32_t x,
                                             uint32_t h, uint32_t b, uint32_t qt, uint32_t n_kv, uint32_t quarter,
                                             uint32_t lane) {
    const uint32_t r = quarter * 32 + lane;
    const uint32_t lane_addr = (quarter * 32) << 16;
    const uint32_t s_col = x * 128, o_col = 256 + x * 128;
    const uint32_t grow = qt * 128 + r;
    float m = -INFINITY, l = 0.f;
    for (uint32_t j = 0; j < n_kv; ++j) {
        if (!mbar_wait(&bars->s_full[x], j & 1)) return false;
        tc::fence_after_sync();
        // the whole S row: four loads in flight, one wait
        uint32_t sr[128];
#pragma unroll
        for (int c = 0; c < 4; ++c) tc::tmem_ld32_at(tbase + lane_addr + s_col + c * 32, sr + 32 * c);
        tc::tmem_wait_ld();
        if (j == qt) {  // diagonal tile: keys after the query are masked
#pragma unroll
            for (int c = 0; c < 128; ++c)
                if (j * 128 + c > grow) sr[c] = 0xff800000u;  // -inf
        }
        // row max of the raw scores with 8 independent chains (no 128-long dependency)
        float mk[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) mk[k] = fmax3(__uint_as_float(sr[k]), __uint_as_float(sr[8 + k]),
                                                  __uint_as_float(sr[16 + k]));
#pragma unroll
        for (int c = 24; c < 128; c += 16) {
#pragma unroll
            for (int k = 0; k < 8; ++k)
                mk[k] = fmax3(mk[k], __uint_as_float(sr[c + k]), __uint_as_float(sr[c + 8 + k]));
        }
        const float mx = fmax3(fmax3(mk[0], mk[1], mk[2]), fmax3(mk[3], mk[4], mk[5]), fmaxf(mk[6], mk[7])) *
                         a.scale_log2;
        const bool need = mx > m + kRescaleThreshold;
        if (__any_sync(0xffffffffu, need)) {
            const float mn = fmaxf(m, mx);
            const float alpha = ex2f(m - mn);  // 0 for the first tile
            if (j > 0) {
                // O_x holds sum_{<j} P V (PV_x(j-1) completed before S_x(j))
#pragma unroll 1
                for (int c = 0; c < 4; ++c) {
                    uint32_t raw[32];
                    const uint32_t addr = tbase + lane_addr + o_col + c * 32;
                    tc::tmem_ld32(addr, raw);
                    tc::tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) raw[i] = __float_as_uint(__uint_as_float(raw[i]) * alpha);
                    tc::tmem_st32(addr, raw);
                }
            }
            l *= alpha;
            m = mn;
        }
        // p = 2^(s * scale - m) (one packed FMA per pair), sums in 8 chains
        float rsum[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        const float sc = a.scale_log2, nm = -m;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
            uint32_t packed[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                float x0, x1;
                ffma2(x0, x1, __uint_as_float(sr[64 * c + 2 * i]), __uint_as_float(sr[64 * c + 2 * i + 1]), sc, sc,
                      nm, nm);
                const float p0 = ex2f(x0), p1 = ex2f(x1);
                fadd2(rsum[(i & 3) * 2], rsum[(i & 3) * 2 + 1], rsum[(i & 3) * 2], rsum[(i & 3) * 2 + 1], p0, p1);
                packed[i] = pack_half2(p0, p1);
            }
            tc::tmem_st32(tbase + lane_addr + s_col + c * 32, packed);
        }
        const float rs = ((rsum[0] + rsum[1]) + (rsum[2] + rsum[3])) + ((rsum[4] + rsum[5]) + (rsum[6] + rsum[7]));
        l += rs;
        tc::tmem_wait_st();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->p_full[x]);
    }
    if (!mbar_wait(&bars->o_done[x], 0)) return false;
    tc::fence_after_sync();
    const float inv = 1.f / l;
    __half* orow = a.out + static_cast<uint64_t>(b) * a.out_batch_stride + static_cast<uint64_t>(grow) * a.out_stride +
                   static_cast<uint64_t>(h) * 128;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
        uint32_t raw[32];
        tc::tmem_ld32(tbase + lane_addr + o_col + c * 32, raw);
        tc::tmem_wait_ld();
        uint32_t o16[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
            o16[i] = pack_half2(__uint_as_float(raw[2 * i]) * inv, __uint_as_float(raw[2 * i + 1]) * inv);
        if (grow < a.seq_len) {
            uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
            for (int i = 0; i < 4; ++i) dst[i] = make_uint4(o16[4 * i], o16[4 * i + 1], o16[4 * i + 2], o16[4 * i + 3]);
        }
    }
    return true;
}

__global__ void __launch_bounds__(kPairThreads, 1)
    prefill_pair_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                        const __grid_constant__ CUtensorMap map_v, const PrefillArgs a, const uint32_t num_q_tiles) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* sq = smem;                                     // Q_A, Q_B
    uint8_t* sk = smem + 2 * kTileBytes;                    // [kStages] tiles
    uint8_t* sv = smem + (2 + kStages) * kTileBytes;        // [kStages] tiles
    PairBars* bars = reinterpret_cast<PairBars*>(smem + kPairSmemTiles);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint32_t qt, hp, b;
    prefill_item(num_q_tiles, qt, hp, b);
    const uint32_t h0 = hp * 2;                             // heads h0, h0 + 1 (same KV head)
    const uint32_t kvh = h0 / a.group;
    const uint32_t q_row0 = qt * 128;
    const uint32_t n_kv = qt + 1;

    if (threadIdx.x == 0) {
        mbar_init(&bars->q_full, 1);
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&bars->k_full[s], 1);
            mbar_init(&bars->k_empty[s], 1);
            mbar_init(&bars->v_full[s], 1);
            mbar_init(&bars->v_empty[s], 1);
        }
        for (int x = 0; x < 2; ++x) {
            mbar_init(&bars->s_full[x], 1);
            mbar_init(&bars->p_full[x], 4);
            mbar_init(&bars->o_done[x], 1);
        }
        mbar_init(&bars->drain, 1);
        bars->abort = 0;
        fence_mbarrier_init();
    }
    if (warp == 1) tc::tmem_alloc(&bars->tmem_base, kTmemCols);
    pdl_wait_primary();  // Q/K/V may be written by the previous kernel (RoPE / append)
    pdl_launch_dependents();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tbase = bars->tmem_base;

    // Registers: the launch gives 384 x 168 per CTA; the producer / MMA
    // warpgroup hands most of its share to the two softmax warpgroups
    // (4 x 32 x (kRegsCtl + 2 * kRegsSoftmax) <= 384 x 168).
    if (warp < 4) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsCtl));
        if (warp == 0) {
            // ---------------- TMA producer
            if (lane == 0) {
                tc::prefetch_tensormap(&map_q);
                tc::prefetch_tensormap(&map_k);
                tc::prefetch_tensormap(&map_v);
                const int32_t kx = static_cast<int32_t>(kvh * 128);
                mbar_arrive_expect_tx(&bars->q_full, 2 * kTileBytes);
                for (int x = 0; x < 2; ++x) {
                    const int32_t qx = static_cast<int32_t>((h0 + x) * 128);
                    tc::tma_load_3d(sq + x * kTileBytes, &map_q, qx, q_row0, b, &bars->q_full);
                    tc::tma_load_3d(sq + x * kTileBytes + kBoxBytes, &map_q, qx + 64, q_row0, b, &bars->q_full);
                }
                uint32_t issued_k = 0, issued_v = 0;
                bool ok = true;
                for (uint32_t j = 0; j < n_kv && ok; ++j) {
                    const uint32_t s = j % kStages, r = j / kStages;
                    const int32_t y = static_cast<int32_t>(j * 128);
                    if (r > 0 && !(ok = mbar_wait(&bars->k_empty[s], (r - 1) & 1))) break;
                    mbar_arrive_expect_tx(&bars->k_full[s], kTileBytes);
                    tc::tma_load_3d(sk + s * kTileBytes, &map_k, kx, y, b, &bars->k_full[s]);
                    tc::tma_load_3d(sk + s * kTileBytes + kBoxBytes, &map_k, kx + 64, y, b, &bars->k_full[s]);
                    issued_k = j + 1;
                    if (r > 0 && !(ok = mbar_wait(&bars->v_empty[s], (r - 1) & 1))) break;
                    mbar_arrive_expect_tx(&bars->v_full[s], kTileBytes);
                    tc::tma_load_3d(sv + s * kTileBytes, &map_v, kx, y, b, &bars->v_full[s]);
                    tc::tma_load_3d(sv + s * kTileBytes + kBoxBytes, &map_v, kx + 64, y, b, &bars->v_full[s]);
                    issued_v = j + 1;
                }
                if (!ok) bars->abort = 1;
                (void)mbar_wait(&bars->q_full, 0);
                for (uint32_t j = issued_k > kStages ? issued_k - kStages : 0; j < issued_k; ++j)
                    (void)mbar_wait(&bars->k_full[j % kStages], (j / kStages) & 1);
                for (uint32_t j = issued_v > kStages ? issued_v - kStages : 0; j < issued_v; ++j)
                    (void)mbar_wait(&bars->v_full[j % kStages], (j / kStages) & 1);
            }
        } else if (warp == 1) {
            // ---------------- MMA issuer (one thread)
            if (lane == 0) {
                constexpr uint32_t id_s = tc::idesc_f16_f32(128, 128, false, false);
                constexpr uint32_t id_o = tc::idesc_f16_f32(128, 128, false, true);
                bool ok = mbar_wait(&bars->q_full, 0);
                // S_x(j) = Q_x K_j^T
                auto issue_s = [&](uint32_t j, uint32_t x) {
                    const uint32_t s = j % kStages;
                    const uint32_t kbase = smem_u32(sk + s * kTileBytes), qbase = smem_u32(sq + x * kTileBytes);
    #pragma unroll
                    for (uint32_t ks = 0; ks < 8; ++ks) {
                        const uint32_t off = (ks >> 2) * kBoxBytes + (ks & 3) * 32;
                        tc::mma_ss(tbase + x * 128, tc::desc_kmajor_sw128(qbase + off), tc::desc_kmajor_sw128(kbase + off),
                                   id_s, ks > 0);
                    }
                    tc::commit(&bars->s_full[x]);
                };
                // O_x += P_x(j) V_j
                auto issue_pv = [&](uint32_t j, uint32_t x) {
                    const uint32_t vbase = smem_u32(sv + (j % kStages) * kTileBytes);
    #pragma unroll
                    for (uint32_t ks = 0; ks < 8; ++ks)
                        tc::mma_ts(tbase + 256 + x * 128, tbase + x * 128 + ks * 8,
                                   tc::desc_mnmajor_sw128(vbase + ks * 2048, kBoxBytes), id_o, (j > 0 || ks > 0) ? 1u : 0u);
                };
                if (ok && (ok = mbar_wait(&bars->k_full[0], 0))) {
                    tc::fence_after_sync();
                    issue_s(0, 0);
                    issue_s(0, 1);
                    tc::commit(&bars->k_empty[0]);
                }
                for (uint32_t j = 0; j < n_kv && ok; ++j) {
                    const uint32_t s = j % kStages;
                    const bool more = j + 1 < n_kv;
                    if (!(ok = mbar_wait(&bars->v_full[s], (j / kStages) & 1))) break;
                    if (more && !(ok = mbar_wait(&bars->k_full[(j + 1) % kStages], ((j + 1) / kStages) & 1))) break;
                    for (uint32_t x = 0; x < 2 && ok; ++x) {
                        if (!(ok = mbar_wait(&bars->p_full[x], j & 1))) break;
                        tc::fence_after_sync();
                        issue_pv(j, x);
                        if (!more) tc::commit(&bars->o_done[x]);
                        if (x == 1) tc::commit(&bars->v_empty[s]);
                        if (more) {
                            issue_s(j + 1, x);
                            if (x == 1) tc::commit(&bars->k_empty[(j + 1) % kStages]);
                        }
                    }
                }
                if (!ok) bars->abort = 1;
                tc::commit(&bars->drain);
                (void)mbar_wait(&bars->drain, 0);
            }
        }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsSoftmax));
        const uint32_t x = (warp - 4) / 4;  // 0: head h0 (warps 4-7), 1: head h0 + 1 (warps 8-11)
        if (!pair_softmax(a, bars, tbase, x, h0 + x, b, qt, n_kv, warp & 3, lane)) bars->abort = 1;
        tc::fence_before_sync();
    }
    __syncthreads();
    if (bars->abort && threadIdx.x == 0) atomicOr(&g_device_error, kErrWaitTimeout);
    if (warp == 1) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tbase, kTmemCols);
    }
}

int ensure_smem_attr() {
    static std::atomic<uint64_t> done{0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return B2_ERR_CUDA;
    const uint64_t bit = 1ull << (dev & 63);
    if (done.load() & bit) return B2_OK;
    int st = cuda_status(
        cudaFuncSetAttribute(prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
    if (st == B2_OK)
        st = cuda_status(
            cudaFuncSetAttribute(prefill_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPairSmemBytes));
    if (st == B2_OK) done.fetch_or(bit);
    return st;
}

}  // namespace

unsigned int device_error_prefill() {
    unsigned int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v)) != cudaSuccess) return 0;
    return v;
}

int clear_device_error_prefill() {
    const unsigned int zero = 0;
    return cuda_status(cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero)));
}

int launch_prefill_sm100(const PrefillArgs& a, uint32_t batch, cudaStream_t stream) {
    if (a.head_dim != 128 || a.start_pos != 0) return B2_ERR_UNSUPPORTED;
    // tensor maps: 16-byte aligned bases and row / batch strides
    if (!aligned16(a.q) || !aligned16(a.k) || !aligned16(a.v) || !aligned16(a.out)) return B2_ERR_UNSUPPORTED;
    if (a.q_stride % 8 || a.kv_stride % 8 || a.out_stride % 8) return B2_ERR_UNSUPPORTED;
    if (batch > 1 && (a.q_batch_stride % 8 || a.kv_batch_stride % 8 || a.out_batch_stride % 8))
        return B2_ERR_UNSUPPORTED;
    int st = ensure_smem_attr();
    if (st != B2_OK) return st;
    CUtensorMap mq, mk, mv;
    const uint64_t S = a.seq_len;
    if (encode_tensor_map_3d_f16(&mq, a.q, static_cast<uint64_t>(a.num_heads) * 128, S, batch, a.q_stride * 2,
                                 a.q_batch_stride * 2, 64, 128) != 0 ||
        encode_tensor_map_3d_f16(&mk, a.k, static_cast<uint64_t>(a.num_kv_heads) * 128, S, batch, a.kv_stride * 2,
                                 a.kv_batch_stride * 2, 64, 128) != 0 ||
        encode_tensor_map_3d_f16(&mv, a.v, static_cast<uint64_t>(a.num_kv_heads) * 128, S, batch, a.kv_stride * 2,
                                 a.kv_batch_stride * 2, 64, 128) != 0)
        return B2_ERR_UNSUPPORTED;
    const uint32_t q_tiles = (a.seq_len + 127) / 128;
    if (a.group % 2 == 0)  // head pairs of one GQA group share every K/V tile
        return launch_pdl(prefill_pair_kernel, dim3(q_tiles, a.num_heads / 2, batch), dim3(kPairThreads),
                          kPairSmemBytes, stream, mq, mk, mv, a, q_tiles);
    return launch_pdl(prefill_tc_kernel, dim3(q_tiles, a.num_heads, batch), dim3(kThreads), kSmemBytes, stream, mq,
                      mk, mv, a, q_tiles);
}

}  // namespace b2
