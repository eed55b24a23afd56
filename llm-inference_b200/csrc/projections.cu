// The two projections either side of the attention path, as persistent
// tcgen05 GEMMs with fused epilogues (FP16 in and out, FP32 accumulation):
//
// QKV projection, the producer (src/kernels/qkv_gemm.hip.cpp:7-115,
// launch_qkv_gemm / launch_qkv_decode): qkv[t][n] = sum_k x[t][k] W[n][k],
// x [seq][hidden] (the normed hidden states), W [q_dim + 2 kv_dim][hidden]
// (Q, then K, then V weights, PyTorch [out, in]), qkv [seq][q_dim + 2 kv_dim]
// -- the [t][Q | K | V] rows the RoPE/append and prefill kernels read. The
// fused form also does the engine's next step, launch_rope_and_store_kv
// (include/model_inference.hpp:266-281), in the GEMM epilogue: each output
// element is rounded to FP16 as the plain GEMM stores it, Q is rotated in
// place, K is kept as is in the row and rotated into the cache row start_pos
// + t, V is copied to its cache row. The result is bit-identical to the plain
// GEMM followed by the RoPE/append kernel, without the second pass over the
// rows.
//
// Attention output projection, the consumer
// (src/kernels/attention_out_projection.hip.cpp:8-58, launch_attention_out_
// projection and its decode form): out[t][n] = sum_k attn[t][k] W[n][k] +
// beta * out[t][n], attn [seq][num_heads * head_dim] (the packed rows the
// prefill and decode kernels write), W [hidden][num_heads * head_dim], out
// [seq][hidden] holding the residual on entry when beta != 0. beta == 0 never
// reads out.
//
// Prefill (seq > 128): clusters of two CTAs own output tiles of 256 tokens x
// 256 columns (tcgen05.mma.cta_group::2, M 256, N 256, K 16; f16 in, f32
// accumulate), K in 64-element steps: each CTA's warp 0 streams its 128 rows
// of A (activations) and its half of B (weights) into a 6-stage ring
// (128-byte swizzle, 32 KB a stage), the leader's warp 1 issues the MMAs into
// one of two 256-column TMEM accumulators in each CTA, and each CTA's warps
// 4-7 drain their 128 rows through the epilogue while the next tile's MMAs
// run. Up to 128 tokens (or where pairs cannot be scheduled) one CTA owns a
// 128 x 256 tile with a 4-stage ring of 48 KB. Both operands K-major, as the
// reference's rocBLAS calls (transpose W, keep X).
// Decode (seq 1): a bandwidth-bound GEMV (the reference's
// launch_matrix_vector_mul), one warp per output row, 16-byte loads of W
// issued before the dependency wait.
// Other shapes (N not a multiple of 256, K not a multiple of 64, unaligned
// rows) take a plain SIMT kernel; a QKV shape the fused epilogue does not
// cover takes the GEMM followed by the RoPE/append kernel.
#include <math.h>

#include <atomic>

#include "b2_common.cuh"
#include "b2_ptx.cuh"
#include "tcgen05.cuh"

namespace b2 {
namespace {

constexpr uint32_t kBM = 128, kBN = 256, kBK = 64;
constexpr uint32_t kStages = 4;
constexpr uint32_t kABytes = kBM * kBK * 2;   // 16 KB
constexpr uint32_t kBBytes = kBN * kBK * 2;   // 32 KB
constexpr uint32_t kStageBytes = kABytes + kBBytes;
constexpr uint32_t kGemmSmem = kStages * kStageBytes + 1024 /*barriers*/ + 1024 /*alignment*/;
constexpr int kGemmThreads = 256;             // 0 TMA, 1 MMA, 2-3 idle, 4-7 epilogue

struct GemmArgs {
    const __half* residual;  // = out (read only when beta != 0)
    __half* out;
    uint32_t M, N, K;
    uint32_t tiles_m, tiles_n;
    float beta;
    // QKV epilogue: out = the [t][Q | K | V] rows, N = q_dim + 2 kv_dim
    __half* k_cache;    // [max_seq][kv_dim], row start_pos + t
    __half* v_cache;
    const __half* cos;  // [max_seq][head_dim / 2]
    const __half* sin;
    uint32_t q_dim, kv_dim, head_dim, start_pos;
    uint32_t rotate;    // 0 = NoPE layer: K stored as is
};

enum : int { kEpiResidual = 0, kEpiQkvRope = 1 };

struct GemmBars {
    uint64_t full[kStages], empty[kStages];
    uint64_t acc_full[2], acc_empty[2];
    uint32_t tmem_base;
    uint32_t abort;
};

// Stores of 32 FP16 values (4 x 16 B) of one output row.
__device__ __forceinline__ void store32(__half* dst, const uint4 (&v)[4]) {
    uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int i = 0; i < 4; ++i) d[i] = v[i];
}

// 32 accumulator columns rounded to FP16, as the GEMM stores them.
__device__ __forceinline__ void round32(const uint32_t (&raw)[32], uint4 (&v)[4]) {
#pragma unroll
    for (int i = 0; i < 4; ++i)
        v[i] = make_uint4(pack_half2(__uint_as_float(raw[8 * i]), __uint_as_float(raw[8 * i + 1])),
                          pack_half2(__uint_as_float(raw[8 * i + 2]), __uint_as_float(raw[8 * i + 3])),
                          pack_half2(__uint_as_float(raw[8 * i + 4]), __uint_as_float(raw[8 * i + 5])),
                          pack_half2(__uint_as_float(raw[8 * i + 6]), __uint_as_float(raw[8 * i + 7])));
}

// Out-projection epilogue of one accumulator tile (256 columns from n0) for
// this thread's row: + beta * residual, FP16 stores.
__device__ __forceinline__ void residual_epilogue(const GemmArgs& g, uint32_t tacc, uint32_t row, uint32_t n0,
                                                  bool live) {
    const uint64_t base = static_cast<uint64_t>(row) * g.N + n0;
#pragma unroll 1
    for (uint32_t half = 0; half < 2; ++half) {
        // this half's 128 residual values in flight before the TMEM loads
        uint4 res[16];
        if (g.beta != 0.f && live) {
#pragma unroll
            for (int v = 0; v < 16; ++v)
                res[v] = *reinterpret_cast<const uint4*>(g.residual + base + half * 128 + v * 8);
        }
#pragma unroll
        for (uint32_t c = 0; c < 4; ++c) {
            uint32_t raw[32];
            tc::tmem_ld32(tacc + half * 128 + c * 32, raw);
            tc::tmem_wait_ld();
            uint32_t o16[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                float lo = __uint_as_float(raw[2 * j]), hi = __uint_as_float(raw[2 * j + 1]);
                if (g.beta != 0.f && live) {
                    const uint32_t w = (&res[c * 4].x)[j];
                    const __half2 r2 = *reinterpret_cast<const __half2*>(&w);
                    const float2 rf = __half22float2(r2);
                    lo = fmaf(g.beta, rf.x, lo);
                    hi = fmaf(g.beta, rf.y, hi);
                }
                o16[j] = pack_half2(lo, hi);
            }
            if (live) {
                uint4* dst = reinterpret_cast<uint4*>(g.out + base + half * 128 + c * 32);
#pragma unroll
                for (int v = 0; v < 4; ++v)
                    dst[v] = make_uint4(o16[4 * v], o16[4 * v + 1], o16[4 * v + 2], o16[4 * v + 3]);
            }
        }
    }
}

// QKV epilogue of one accumulator tile (256 columns starting at n0, all of Q,
// all of K or all of V since q_dim and kv_dim are multiples of 256) for this
// thread's row: the steps of launch_rope_and_store_kv
// (src/kernels/rope.hip.cpp:61-134) on the rounded GEMM outputs. A rotated
// head is taken 32 frequency pairs at a time: columns [c, c + 32) and
// [c + d/2, c + d/2 + 32) of the head, with cos/sin of frequencies c..c+32 at
// the row's position.
__device__ __forceinline__ void qkv_rope_epilogue(const GemmArgs& g, uint32_t tacc, uint32_t row, uint32_t n0,
                                                  bool live) {
    __half* qrow = g.out + static_cast<uint64_t>(row) * g.N + n0;
    const bool is_q = n0 < g.q_dim;
    const bool is_k = !is_q && n0 < g.q_dim + g.kv_dim;
    const uint64_t pos = static_cast<uint64_t>(g.start_pos) + row;
    __half* crow = nullptr;
    if (!is_q)
        crow = (is_k ? g.k_cache : g.v_cache) + pos * g.kv_dim + (n0 - g.q_dim - (is_k ? 0u : g.kv_dim));
    if (g.rotate && (is_q || is_k)) {
        const uint32_t hd = g.head_dim >> 1;
        const __half* cs = g.cos + pos * hd;
        const __half* sn = g.sin + pos * hd;
#pragma unroll 1
        for (uint32_t hb = 0; hb < kBN; hb += g.head_dim) {
#pragma unroll 1
            for (uint32_t c = 0; c < hd; c += 32) {
                uint4 cv[4], sv[4];
                if (live) {
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        cv[i] = __ldg(reinterpret_cast<const uint4*>(cs + c) + i);
                        sv[i] = __ldg(reinterpret_cast<const uint4*>(sn + c) + i);
                    }
                }
                uint32_t lo_raw[32], hi_raw[32];
                tc::tmem_ld32(tacc + hb + c, lo_raw);
                tc::tmem_ld32(tacc + hb + hd + c, hi_raw);
                tc::tmem_wait_ld();
                if (!live) continue;
                uint4 lo[4], hi[4];
                round32(lo_raw, lo);
                round32(hi_raw, hi);
                if (is_k) {  // the row keeps K as the GEMM wrote it
                    store32(qrow + hb + c, lo);
                    store32(qrow + hb + hd + c, hi);
                }
#pragma unroll
                for (int i = 0; i < 4; ++i) rot8_pairs(lo[i], hi[i], cv[i], sv[i]);
                __half* dst = is_q ? qrow : crow;
                store32(dst + hb + c, lo);
                store32(dst + hb + hd + c, hi);
            }
        }
    } else {
#pragma unroll 1
        for (uint32_t c = 0; c < kBN; c += 32) {
            uint32_t raw[32];
            tc::tmem_ld32(tacc + c, raw);
            tc::tmem_wait_ld();
            if (!live) continue;
            uint4 v[4];
            round32(raw, v);
            store32(qrow + c, v);
            if (crow) store32(crow + c, v);
        }
    }
}

template <int kEpi>
__device__ __forceinline__ void proj_gemm_body(const CUtensorMap* map_a, const CUtensorMap* map_b,
                                               const GemmArgs& g) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    GemmBars* bars = reinterpret_cast<GemmBars*>(smem + kStages * kStageBytes);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t ntiles = g.tiles_m * g.tiles_n;
    const uint32_t kb_count = g.K / kBK;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < kStages; ++s) {
            mbar_init(&bars->full[s], 1);
            mbar_init(&bars->empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&bars->acc_full[b], 1);
            mbar_init(&bars->acc_empty[b], 4);
        }
        bars->abort = 0;
        fence_mbarrier_init();
    }
    if (warp == 1) tc::tmem_alloc(&bars->tmem_base, 512);
    pdl_wait_primary();  // attn rows and the residual come from earlier kernels
    pdl_launch_dependents();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tbase = bars->tmem_base;

    if (warp == 0) {
        if (lane == 0) {
            tc::prefetch_tensormap(map_a);
            tc::prefetch_tensormap(map_b);
            uint32_t i = 0;
            bool ok = true;
            for (uint32_t tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
                // N-fastest order: consecutive CTAs share the A rows (L2 reuse)
                const int32_t m0 = static_cast<int32_t>((tile / g.tiles_n) * kBM);
                const int32_t n0 = static_cast<int32_t>((tile % g.tiles_n) * kBN);
                for (uint32_t kb = 0; kb < kb_count; ++kb, ++i) {
                    const uint32_t s = i % kStages, r = i / kStages;
                    if (r > 0 && !(ok = mbar_wait(&bars->empty[s], (r - 1) & 1))) break;
                    uint8_t* st = smem + s * kStageBytes;
                    mbar_arrive_expect_tx(&bars->full[s], kStageBytes);
                    tc::tma_load_3d(st, map_a, static_cast<int32_t>(kb * kBK), m0, 0, &bars->full[s]);
                    tc::tma_load_3d(st + kABytes, map_b, static_cast<int32_t>(kb * kBK), n0, 0, &bars->full[s]);
                }
            }
            if (!ok) bars->abort = 1;
            // never leave with copies in flight into shared memory
            for (uint32_t j = i > kStages ? i - kStages : 0; j < i; ++j)
                (void)mbar_wait(&bars->full[j % kStages], (j / kStages) & 1);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = tc::idesc_f16_f32(kBM, kBN, false, false);
            uint32_t i = 0, t = 0;
            bool ok = true;
            for (uint32_t tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++t) {
                const uint32_t buf = t & 1;
                // the epilogue has drained this accumulator (tile t - 2)
                if (t >= 2 && !(ok = mbar_wait(&bars->acc_empty[buf], ((t >> 1) - 1) & 1))) break;
                tc::fence_after_sync();
                const uint32_t d = tbase + buf * kBN;
                for (uint32_t kb = 0; kb < kb_count; ++kb, ++i) {
                    const uint32_t s = i % kStages;
                    if (!(ok = mbar_wait(&bars->full[s], (i / kStages) & 1))) break;
                    tc::fence_after_sync();
                    const uint32_t a = smem_u32(smem + s * kStageBytes), b = a + kABytes;
#pragma unroll
                    for (uint32_t ks = 0; ks < kBK / 16; ++ks)
                        tc::mma_ss(d, tc::desc_kmajor_sw128(a + ks * 32), tc::desc_kmajor_sw128(b + ks * 32), idesc,
                                   (kb | ks) != 0 ? 1u : 0u);
                    tc::commit(&bars->empty[s]);  // the stage is free once these MMAs have read it
                }
                if (ok) tc::commit(&bars->acc_full[buf]);
            }
            if (!ok) bars->abort = 1;
        }
    } else if (warp >= 4) {
        const uint32_t quarter = static_cast<uint32_t>(warp) & 3;
        const uint32_t lane_addr = (quarter * 32) << 16;
        uint32_t t = 0;
        bool ok = true;
        for (uint32_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++t) {
            const uint32_t buf = t & 1;
            const uint32_t row = (tile / g.tiles_n) * kBM + quarter * 32 + lane;
            const uint32_t n0 = (tile % g.tiles_n) * kBN;
            const bool live = row < g.M;
            if (!(ok = mbar_wait(&bars->acc_full[buf], (t >> 1) & 1))) break;
            tc::fence_after_sync();
            if constexpr (kEpi == kEpiQkvRope)
                qkv_rope_epilogue(g, tbase + lane_addr + buf * kBN, row, n0, live);
            else
                residual_epilogue(g, tbase + lane_addr + buf * kBN, row, n0, live);
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->acc_empty[buf]);
        }
        if (!ok) bars->abort = 1;
    }
    __syncthreads();
    if (bars->abort && threadIdx.x == 0) atomicOr(&g_device_error, kErrWaitTimeout);
    if (warp == 1) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tbase, 512);
    }
}

__global__ void __launch_bounds__(kGemmThreads, 1)
    out_proj_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                         const GemmArgs g) {
    proj_gemm_body<kEpiResidual>(&map_a, &map_b, g);
}

__global__ void __launch_bounds__(kGemmThreads, 1)
    qkv_rope_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                         const GemmArgs g) {
    proj_gemm_body<kEpiQkvRope>(&map_a, &map_b, g);
}

// ---- CTA-pair form -----------------------------------------------------------
// Output tiles of 256 tokens x 256 columns per cluster of two CTAs
// (tcgen05.mma.cta_group::2, M 256, N 256, K 16): each CTA loads its own 128
// rows of A and its half (128 rows) of B per 64-wide K slice, so a stage is
// 32 KB instead of 48 KB and six stages fit (3,072 MMA cycles in flight per SM
// against 2,048 for the single-CTA form), and each SM pulls 64 B per MMA cycle
// from L2 instead of 96. The leader (cluster rank 0) issues the MMAs; both
// CTAs' copies complete on the leader's stage barrier; the leader's commits
// release the stage and signal the accumulator in both CTAs; each CTA drains
// its own 128 TMEM lanes with the same epilogues, and both CTAs' epilogue warps
// arrive on the leader's accumulator-free barrier.
constexpr uint32_t kPairStages = 6;
constexpr uint32_t kPairABytes = 128 * kBK * 2;   // this CTA's 128 rows of A
constexpr uint32_t kPairBBytes = 128 * kBK * 2;   // this CTA's 128 rows (half) of B
constexpr uint32_t kPairStageBytes = kPairABytes + kPairBBytes;
constexpr uint32_t kPairSmem = kPairStages * kPairStageBytes + 1024 + 1024;

struct PairBars {
    uint64_t full[kPairStages], empty[kPairStages];
    uint64_t acc_full[2], acc_empty[2];
    uint32_t tmem_base;
    uint32_t abort;
};

template <int kEpi>
__device__ __forceinline__ void proj_gemm_pair_body(const CUtensorMap* map_a, const CUtensorMap* map_b,
                                                    const GemmArgs& g) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    PairBars* bars = reinterpret_cast<PairBars*>(smem + kPairStages * kPairStageBytes);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = tc::cluster_rank();
    const bool leader = rank == 0;
    const uint32_t pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
    const uint32_t ntiles = g.tiles_m * g.tiles_n;  // tiles_m counts 256-row blocks here
    const uint32_t kb_count = g.K / kBK;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < kPairStages; ++s) {
            mbar_init(&bars->full[s], 1);
            mbar_init(&bars->empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&bars->acc_full[b], 1);
            mbar_init(&bars->acc_empty[b], 8);  // 4 epilogue warps x 2 CTAs
        }
        bars->abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) tc::tmem_alloc_pair(&bars->tmem_base, 512);
    // the peer's barriers are initialised before any copy or arrive reaches them
    tc::fence_before_sync();
    tc::cluster_sync();
    tc::fence_after_sync();
    pdl_wait_primary();  // activations and the residual come from earlier kernels
    pdl_launch_dependents();
    const uint32_t tbase = bars->tmem_base;

    if (warp == 0) {
        if (lane == 0) {
            tc::prefetch_tensormap(map_a);
            tc::prefetch_tensormap(map_b);
            uint32_t i = 0;
            bool ok = true;
            for (uint32_t tile = pair; tile < ntiles && ok; tile += npairs) {
                const int32_t m0 = static_cast<int32_t>((tile / g.tiles_n) * 256 + rank * 128);
                const int32_t n0 = static_cast<int32_t>((tile % g.tiles_n) * kBN + rank * 128);
                for (uint32_t kb = 0; kb < kb_count; ++kb, ++i) {
                    const uint32_t s = i % kPairStages, r = i / kPairStages;
                    // released by the leader's commit once the pair MMAs have read it
                    if (r > 0 && !(ok = mbar_wait(&bars->empty[s], (r - 1) & 1))) break;
                    uint8_t* st = smem + s * kPairStageBytes;
                    if (leader) mbar_arrive_expect_tx(&bars->full[s], 2 * kPairStageBytes);
                    const uint32_t fb = tc::cluster_addr(&bars->full[s], 0);
                    tc::tma_load_3d_pair(st, map_a, static_cast<int32_t>(kb * kBK), m0, 0, fb);
                    tc::tma_load_3d_pair(st + kPairABytes, map_b, static_cast<int32_t>(kb * kBK), n0, 0, fb);
                }
            }
            if (!ok) bars->abort = 1;
            // The copies complete on the leader's barriers; the leader's MMA
            // thread waits for every stage it consumes, and this CTA leaves only
            // after the cluster barrier below, which the leader reaches after
            // its MMA loop.
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            constexpr uint32_t idesc = tc::idesc_f16_f32(256, kBN, false, false);
            uint32_t i = 0, t = 0;
            bool ok = true;
            for (uint32_t tile = pair; tile < ntiles && ok; tile += npairs, ++t) {
                const uint32_t buf = t & 1;
                // both CTAs' epilogues have drained this accumulator (tile t - 2)
                if (t >= 2 && !(ok = mbar_wait(&bars->acc_empty[buf], ((t >> 1) - 1) & 1))) break;
                tc::fence_after_sync();
                const uint32_t d = tbase + buf * kBN;
                for (uint32_t kb = 0; kb < kb_count; ++kb, ++i) {
                    const uint32_t s = i % kPairStages;
                    if (!(ok = mbar_wait(&bars->full[s], (i / kPairStages) & 1))) break;
                    tc::fence_after_sync();
                    const uint32_t a = smem_u32(smem + s * kPairStageBytes), b = a + kPairABytes;
#pragma unroll
                    for (uint32_t ks = 0; ks < kBK / 16; ++ks)
                        tc::mma_ss_pair(d, tc::desc_kmajor_sw128(a + ks * 32), tc::desc_kmajor_sw128(b + ks * 32),
                                        idesc, (kb | ks) != 0 ? 1u : 0u);
                    tc::commit_pair(&bars->empty[s], 0x3);  // the stage is free in both CTAs
                }
                if (ok) tc::commit_pair(&bars->acc_full[buf], 0x3);
            }
            if (!ok) bars->abort = 1;
        }
    } else if (warp >= 4) {
        const uint32_t quarter = static_cast<uint32_t>(warp) & 3;
        const uint32_t lane_addr = (quarter * 32) << 16;
        uint32_t t = 0;
        bool ok = true;
        for (uint32_t tile = pair; tile < ntiles; tile += npairs, ++t) {
            const uint32_t buf = t & 1;
            const uint32_t row = (tile / g.tiles_n) * 256 + rank * 128 + quarter * 32 + lane;
            const uint32_t n0 = (tile % g.tiles_n) * kBN;
            const bool live = row < g.M;
            if (!(ok = mbar_wait(&bars->acc_full[buf], (t >> 1) & 1))) break;
            tc::fence_after_sync();
            if constexpr (kEpi == kEpiQkvRope)
                qkv_rope_epilogue(g, tbase + lane_addr + buf * kBN, row, n0, live);
            else
                residual_epilogue(g, tbase + lane_addr + buf * kBN, row, n0, live);
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive_cluster(tc::cluster_addr(&bars->acc_empty[buf], 0));
        }
        if (!ok) bars->abort = 1;
    }
    // Neither CTA leaves while the other may still signal its barriers or
    // read its shared memory through the pair MMAs.
    tc::fence_before_sync();
    __syncthreads();
    tc::cluster_sync();
    tc::fence_after_sync();
    if (bars->abort && threadIdx.x == 0) atomicOr(&g_device_error, kErrWaitTimeout);
    if (warp == 1) tc::tmem_dealloc_pair(tbase, 512);
}

__global__ void __launch_bounds__(kGemmThreads, 1)
    out_proj_gemm_pair_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                              const GemmArgs g) {
    proj_gemm_pair_body<kEpiResidual>(&map_a, &map_b, g);
}

__global__ void __launch_bounds__(kGemmThreads, 1)
    qkv_rope_gemm_pair_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                              const GemmArgs g) {
    proj_gemm_pair_body<kEpiQkvRope>(&map_a, &map_b, g);
}

// Decode GEMV: out[n] = W[n] . x + beta * out[n], one warp per row, K a
// multiple of 256 and at most kGemvMaxK (each lane holds 8 halves of the row
// per 256). The weights do not depend on the kernel this one follows on the
// stream, so the row is loaded before the dependency wait: with programmatic
// dependent launch the 8 MB weight stream overlaps the previous kernel's
// tail, and only x and the residual are read after it.
constexpr int kGemvWarps = 8;
constexpr uint32_t kGemvMaxK = 4096;
__global__ void __launch_bounds__(kGemvWarps * 32)
    out_proj_gemv_kernel(const __half* __restrict__ x, const __half* __restrict__ w, __half* out, uint32_t N,
                         uint32_t K, float beta) {
    constexpr int kMaxV = kGemvMaxK / 256;
    pdl_launch_dependents();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t n = blockIdx.x * kGemvWarps + warp;
    const bool live = n < N;
    const __half* row = w + static_cast<uint64_t>(live ? n : 0) * K;
    const uint32_t nv = K / 256;
    uint4 wv[kMaxV];
#pragma unroll
    for (int u = 0; u < kMaxV; ++u)
        wv[u] = (live && static_cast<uint32_t>(u) < nv) ? ldg_nc_v4(row + u * 256 + lane * 8)
                                                          : make_uint4(0u, 0u, 0u, 0u);
    pdl_wait_primary();  // x and the residual may come from the previous kernel
    if (!live) return;
    // the residual load goes out with the x loads, not after the reduction
    const float resid = (lane == 0 && beta != 0.f) ? __half2float(out[n]) : 0.f;
    float acc = 0.f;
#pragma unroll
    for (int u = 0; u < kMaxV; ++u) {
        if (static_cast<uint32_t>(u) < nv) {
            const uint4 xv = *reinterpret_cast<const uint4*>(x + u * 256 + lane * 8);
            const __half2* a = reinterpret_cast<const __half2*>(&wv[u]);
            const __half2* b = reinterpret_cast<const __half2*>(&xv);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float2 fa = __half22float2(a[j]), fb = __half22float2(b[j]);
                acc = fmaf(fa.x, fb.x, acc);
                acc = fmaf(fa.y, fb.y, acc);
            }
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) {
        if (beta != 0.f) acc = fmaf(beta, resid, acc);
        out[n] = __float2half_rn(acc);
    }
}

// Any shape: one thread per output element, FP32 accumulation.
__global__ void out_proj_simt_kernel(const __half* __restrict__ x, const __half* __restrict__ w, __half* out,
                                     uint32_t M, uint32_t N, uint32_t K, float beta) {
    pdl_wait_primary();
    pdl_launch_dependents();
    const uint64_t idx = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<uint64_t>(M) * N) return;
    const uint32_t m = static_cast<uint32_t>(idx / N), n = static_cast<uint32_t>(idx % N);
    const __half* a = x + static_cast<uint64_t>(m) * K;
    const __half* b = w + static_cast<uint64_t>(n) * K;
    float acc = 0.f;
    for (uint32_t k = 0; k < K; ++k) acc = fmaf(__half2float(a[k]), __half2float(b[k]), acc);
    if (beta != 0.f) acc = fmaf(beta, __half2float(out[idx]), acc);
    out[idx] = __float2half_rn(acc);
}

int sm_count() {
    static std::atomic<int> cached{0};
    int v = cached.load();
    if (v > 0) return v;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) !=
                                                  cudaSuccess || v <= 0)
        v = 148;
    cached.store(v);
    return v;
}

int ensure_gemm_smem() {
    static std::atomic<uint64_t> done{0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return B2_ERR_CUDA;
    const uint64_t bit = 1ull << (dev & 63);
    if (done.load() & bit) return B2_OK;
    int st =
        cuda_status(cudaFuncSetAttribute(out_proj_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemmSmem));
    if (st == B2_OK)
        st = cuda_status(
            cudaFuncSetAttribute(qkv_rope_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemmSmem));
    if (st == B2_OK)
        st = cuda_status(cudaFuncSetAttribute(out_proj_gemm_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              kPairSmem));
    if (st == B2_OK)
        st = cuda_status(cudaFuncSetAttribute(qkv_rope_gemm_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              kPairSmem));
    if (st == B2_OK) done.fetch_or(bit);
    return st;
}

// Tensor maps of the two K-major operands: activations [M][K] (128-row
// boxes), weights [N][K] (b_rows-row boxes: 256 for one CTA, 128 for a pair).
int gemm_maps(CUtensorMap* ma, CUtensorMap* mb, const __half* x, const __half* w, size_t M, size_t N, size_t K,
              uint32_t b_rows) {
    if (encode_tensor_map_3d_f16(ma, x, K, M, 1, K * 2, 0, kBK, kBM) != 0 ||
        encode_tensor_map_3d_f16(mb, w, K, N, 1, K * 2, 0, kBK, b_rows) != 0)
        return B2_ERR_UNSUPPORTED;
    return B2_OK;
}

// Two-CTA clusters of a pair kernel that fit on the GPU at once (0: use the
// single-CTA kernel). Cached per device and kernel as the count + 1.
template <typename Kern>
uint32_t pair_clusters(Kern kernel, std::atomic<int>* cache) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    const int v = cache[dev].load();
    if (v > 0) return static_cast<uint32_t>(v - 1);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(2 * static_cast<uint32_t>(sm_count() / 2));
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = kPairSmem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess) {
        (void)cudaGetLastError();
        n = 0;
    }
    if (n < 0) n = 0;
    cache[dev].store(n + 1);
    return static_cast<uint32_t>(n);
}

std::atomic<int> g_pair_clusters_oproj[64], g_pair_clusters_qkv[64];  // zero: not queried yet

// Launch a pair kernel as `clusters` clusters of two CTAs, with programmatic
// dependent launch allowed (as launch_pdl).
template <typename... KArgs, typename... Args>
int launch_pdl_pairs(void (*kernel)(KArgs...), uint32_t clusters, size_t smem, cudaStream_t stream,
                     Args&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(2 * clusters);
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 2;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        note_cuda_error(e);
        return B2_ERR_CUDA;
    }
    return launch_status();
}

// The persistent GEMM over g (tiles_m / tiles_n filled in here): CTA pairs of
// 256-row tiles when the prompt spans more than one 128-row tile and pairs
// can be scheduled, else one CTA per 128-row tile.
template <int kEpi>
int launch_gemm(const __half* x, const __half* w, GemmArgs g, cudaStream_t stream) {
    int st = ensure_gemm_smem();
    if (st != B2_OK) return st;
    CUtensorMap ma, mb;
    g.tiles_n = g.N / kBN;
    auto pair_kernel = kEpi == kEpiQkvRope ? qkv_rope_gemm_pair_kernel : out_proj_gemm_pair_kernel;
    const uint32_t max_clusters =
        g.M > kBM ? pair_clusters(pair_kernel, kEpi == kEpiQkvRope ? g_pair_clusters_qkv : g_pair_clusters_oproj)
                  : 0u;
    if (max_clusters > 0) {
        if ((st = gemm_maps(&ma, &mb, x, w, g.M, g.N, g.K, kBN / 2)) != B2_OK) return st;
        g.tiles_m = (g.M + 255) / 256;
        const uint32_t clusters = std::min<uint32_t>(g.tiles_m * g.tiles_n, max_clusters);
        return launch_pdl_pairs(pair_kernel, clusters, kPairSmem, stream, ma, mb, g);
    }
    if ((st = gemm_maps(&ma, &mb, x, w, g.M, g.N, g.K, kBN)) != B2_OK) return st;
    g.tiles_m = (g.M + kBM - 1) / kBM;
    const uint32_t grid = std::min<uint32_t>(g.tiles_m * g.tiles_n, static_cast<uint32_t>(sm_count()));
    return launch_pdl(kEpi == kEpiQkvRope ? qkv_rope_gemm_kernel : out_proj_gemm_kernel, dim3(grid),
                      dim3(kGemmThreads), kGemmSmem, stream, ma, mb, g);
}

int launch_out_proj(const void* d_in, void* d_out, const void* d_w, size_t M, size_t N, size_t K, float beta,
                    cudaStream_t stream, bool decode_form) {
    if (M == 0 || N == 0 || K == 0) return B2_NOTHING_TO_DO;
    if (!d_in || !d_out || !d_w) return B2_ERR_INVALID_ARG;
    if (M > 0x7fffffffull || N > 0x7fffffffull || K > 0x7fffffffull) return B2_ERR_UNSUPPORTED;
    const auto* x = static_cast<const __half*>(d_in);
    const auto* w = static_cast<const __half*>(d_w);
    auto* out = static_cast<__half*>(d_out);
    const uint32_t m = static_cast<uint32_t>(M), n = static_cast<uint32_t>(N), k = static_cast<uint32_t>(K);
    const bool aligned = aligned16(x) && aligned16(w) && aligned16(out);
    if (decode_form || M == 1) {
        if (aligned && K % 256 == 0 && K <= kGemvMaxK && M == 1)
            return launch_pdl(out_proj_gemv_kernel, dim3((n + kGemvWarps - 1) / kGemvWarps), dim3(kGemvWarps * 32),
                              0, stream, x, w, out, n, k, beta);
    } else if (aligned && N % kBN == 0 && K % kBK == 0) {
        GemmArgs g{};
        g.residual = out;
        g.out = out;
        g.M = m;
        g.N = n;
        g.K = k;
        g.beta = beta;
        return launch_gemm<kEpiResidual>(x, w, g, stream);
    }
    const uint64_t total = static_cast<uint64_t>(m) * n;
    return launch_pdl(out_proj_simt_kernel, dim3(static_cast<uint32_t>((total + 255) / 256)), dim3(256), 0, stream,
                      x, w, out, m, n, k, beta);
}

// launch_qkv_gemm + launch_rope_and_store_kv in one kernel where the epilogue
// covers the shape (more than one token; head_dim 64, 128 or 256; q_dim and
// kv_dim multiples of the 256-column tile; K a multiple of 64; 16-byte
// aligned operands), else the two launches.
int launch_qkv_rope(const void* d_in, void* d_qkv, const void* d_w, void* d_k_cache, void* d_v_cache,
                    const void* d_cos, const void* d_sin, size_t M, size_t hidden, size_t H, size_t KVH, size_t d,
                    size_t start_pos, bool rotate, cudaStream_t stream) {
    if (M == 0) return B2_NOTHING_TO_DO;
    if (!d_in || !d_qkv || !d_w || !d_k_cache || !d_v_cache || H == 0 || KVH == 0 || d == 0 || hidden == 0)
        return B2_ERR_INVALID_ARG;
    if (rotate && (!d_cos || !d_sin)) return B2_ERR_INVALID_ARG;
    if (d % 2 != 0 || H % KVH != 0) return B2_ERR_INVALID_ARG;
    const size_t q_dim = H * d, kv_dim = KVH * d, N = q_dim + 2 * kv_dim;
    if (M > 0x7fffffffull || N > 0x7fffffffull || hidden > 0x7fffffffull || start_pos + M > 0x7fffffffull)
        return B2_ERR_UNSUPPORTED;
    // one token: the GEMV (a 128-row tile would stream the weights for one
    // row's worth of work) and the RoPE kernel
    const bool fused = M > 1 && (d == 64 || d == 128 || d == 256) && q_dim % kBN == 0 && kv_dim % kBN == 0 &&
                       hidden % kBK == 0 && aligned16(d_in) && aligned16(d_w) && aligned16(d_qkv) &&
                       aligned16(d_k_cache) && aligned16(d_v_cache) &&
                       (!rotate || (aligned16(d_cos) && aligned16(d_sin)));
    if (!fused) {
        int st = launch_out_proj(d_in, d_qkv, d_w, M, N, hidden, 0.f, stream, false);
        if (st != B2_OK) return st;
        auto* qkv = static_cast<__half*>(d_qkv);
        return b2_launch_rope_and_store_kv(qkv, qkv + q_dim, qkv + q_dim + kv_dim, d_k_cache, d_v_cache, d_cos, d_sin,
                                           M, H, KVH, d, N, N, start_pos, rotate,
                                           reinterpret_cast<b2_stream_t>(stream));
    }
    GemmArgs g{};
    g.out = static_cast<__half*>(d_qkv);
    g.M = static_cast<uint32_t>(M);
    g.N = static_cast<uint32_t>(N);
    g.K = static_cast<uint32_t>(hidden);
    g.k_cache = static_cast<__half*>(d_k_cache);
    g.v_cache = static_cast<__half*>(d_v_cache);
    g.cos = static_cast<const __half*>(d_cos);
    g.sin = static_cast<const __half*>(d_sin);
    g.q_dim = static_cast<uint32_t>(q_dim);
    g.kv_dim = static_cast<uint32_t>(kv_dim);
    g.head_dim = static_cast<uint32_t>(d);
    g.start_pos = static_cast<uint32_t>(start_pos);
    g.rotate = rotate ? 1u : 0u;
    return launch_gemm<kEpiQkvRope>(static_cast<const __half*>(d_in), static_cast<const __half*>(d_w), g, stream);
}

}  // namespace

unsigned int device_error_proj() {
    unsigned int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v)) != cudaSuccess) return 0;
    return v;
}

int clear_device_error_proj() {
    const unsigned int zero = 0;
    return cuda_status(cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero)));
}

}  // namespace b2

extern "C" int b2_launch_attention_out_projection(const void* d_in, void* d_out, const void* d_o_proj_weights,
                                                  size_t seq_len, size_t hidden_size, size_t num_heads,
                                                  size_t head_dim, float beta, b2_stream_t stream) {
    return b2::launch_out_proj(d_in, d_out, d_o_proj_weights, seq_len, hidden_size, num_heads * head_dim, beta,
                               reinterpret_cast<cudaStream_t>(stream), false);
}

extern "C" int b2_launch_attention_out_projection_decode(const void* d_in, void* d_out, const void* d_o_proj_weights,
                                                         size_t hidden_size, size_t num_heads, size_t head_dim,
                                                         float beta, b2_stream_t stream) {
    return b2::launch_out_proj(d_in, d_out, d_o_proj_weights, 1, hidden_size, num_heads * head_dim, beta,
                               reinterpret_cast<cudaStream_t>(stream), true);
}

extern "C" int b2_launch_qkv_gemm(const void* d_input_norm, void* d_qkv_out, const void* d_qkv_weights,
                                  size_t seq_len, size_t hidden_size, size_t total_qkv_dim, b2_stream_t stream) {
    return b2::launch_out_proj(d_input_norm, d_qkv_out, d_qkv_weights, seq_len, total_qkv_dim, hidden_size, 0.f,
                               reinterpret_cast<cudaStream_t>(stream), false);
}

extern "C" int b2_launch_qkv_decode(const void* d_input_norm, void* d_qkv_out, const void* d_qkv_weights,
                                    size_t hidden_size, size_t total_qkv_dim, b2_stream_t stream) {
    return b2::launch_out_proj(d_input_norm, d_qkv_out, d_qkv_weights, 1, total_qkv_dim, hidden_size, 0.f,
                               reinterpret_cast<cudaStream_t>(stream), true);
}

extern "C" int b2_launch_qkv_gemm_rope_store_kv(const void* d_input_norm, void* d_qkv_out, const void* d_qkv_weights,
                                                void* d_k_cache, void* d_v_cache, const void* d_cos,
                                                const void* d_sin, size_t seq_len, size_t hidden_size,
                                                size_t num_heads, size_t num_kv_heads, size_t head_dim,
                                                size_t start_pos, bool apply_rotary, b2_stream_t stream) {
    return b2::launch_qkv_rope(d_input_norm, d_qkv_out, d_qkv_weights, d_k_cache, d_v_cache, d_cos, d_sin, seq_len,
                               hidden_size, num_heads, num_kv_heads, head_dim, start_pos, apply_rotary,
                               reinterpret_cast<cudaStream_t>(stream));
}
