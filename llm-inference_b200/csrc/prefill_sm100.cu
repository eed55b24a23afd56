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
    const uint32_t qt = num_q_tiles - 1 - blockIdx.x;     // heaviest tiles first
    const uint32_t h = blockIdx.y;
    const uint32_t b = blockIdx.z;
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

int ensure_smem_attr() {
    static std::atomic<uint64_t> done{0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return B2_ERR_CUDA;
    const uint64_t bit = 1ull << (dev & 63);
    if (done.load() & bit) return B2_OK;
    const int st = cuda_status(
        cudaFuncSetAttribute(prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
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
    return launch_pdl(prefill_tc_kernel, dim3(q_tiles, a.num_heads, batch), dim3(kThreads), kSmemBytes, stream, mq,
                      mk, mv, a, q_tiles);
}

}  // namespace b2
