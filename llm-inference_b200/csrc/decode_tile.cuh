// Tile math shared by the flash-decode kernels (sm_100a): mma.sync m16n8k16
// score / P.V tiles with tokens as M, the lazily rescaled online softmax,
// fragment loads and the cross-warp combine of split states.
#pragma once

#include <cuda_fp16.h>
#include <math.h>
#include <stdint.h>

#include "b2_common.cuh"

namespace b2 {

constexpr int kChunk = 256;  // KV_CHUNK
constexpr int kTile = 16;    // tokens per MMA tile
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

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

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// The running max only moves when a tile's max exceeds it by more than this
// (log2 units): P stays <= 2^8 (exact enough in fp16) and most tiles skip
// rescaling O.
constexpr float kRescaleThreshold = 8.f;

// Scores of one 16-token tile, S^T fragment in the log2 domain. ka/kb: K rows
// g and g+8 (4 x 16 B at 32j + 8t). With kPartial, rows at or past `valid`
// (zero in ka/kb) are masked to -inf.
template <bool kPartial>
__device__ __forceinline__ void tile_scores(float (&s)[4], const uint4 (&ka)[4], const uint4 (&kb)[4],
                                            const uint32_t (&qf)[8][2], uint32_t g, uint32_t valid,
                                            float scale_log2) {
    float s2[4] = {0.f, 0.f, 0.f, 0.f};  // two accumulation chains halve the MMA latency
    s[0] = s[1] = s[2] = s[3] = 0.f;
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
#pragma unroll
    for (int i = 0; i < 4; ++i) s[i] = (s[i] + s2[i]) * scale_log2;
    if (kPartial) {
        if (g >= valid) s[0] = s[1] = -INFINITY;  // g: the token held by MMA row g
        if (g + 8 >= valid) s[2] = s[3] = -INFINITY;
    }
}

// Online softmax + O^T += V^T . P^T for one tile. va: V rows 2t, 2t+1, 2t+8,
// 2t+9 (2 x 16 B at 64b + 8g); masked rows must hold zeros.
__device__ __forceinline__ void tile_softmax_pv(WarpState& st, const float (&s)[4], const uint4 (&va)[4][2], int g,
                                                int t) {
    float mx0 = fmaxf(s[0], s[2]), mx1 = fmaxf(s[1], s[3]);
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
    }
    const bool grow = (mx0 > st.m0 + kRescaleThreshold) || (mx1 > st.m1 + kRescaleThreshold);
    if (__any_sync(0xffffffffu, grow)) {
        const float mn0 = fmaxf(st.m0, mx0), mn1 = fmaxf(st.m1, mx1);
        const float al0 = ex2(st.m0 - mn0), al1 = ex2(st.m1 - mn1);  // 0 on the first tile
        st.l0 *= al0;
        st.l1 *= al1;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            st.o[i][0] *= al0;
            st.o[i][1] *= al1;
            st.o[i][2] *= al0;
            st.o[i][3] *= al1;
        }
        st.m0 = mn0;
        st.m1 = mn1;
    }
    const float p0 = ex2(s[0] - st.m0), p1 = ex2(s[1] - st.m1);
    const float p2 = ex2(s[2] - st.m0), p3 = ex2(s[3] - st.m1);
    st.l0 += p0 + p2;
    st.l1 += p1 + p3;

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

// Load K (rows g, g+8) or V (rows 2t, 2t+1, 2t+8, 2t+9) fragments of one
// tile from a row-major tile whose rows are `row_bytes` apart; rows at or
// past `valid` read as zero when kPartial.
template <bool kPartial>
__device__ __forceinline__ void load_k_frags(const uint8_t* kt, uint32_t row_bytes, int g, int t, uint32_t valid,
                                             uint4 (&ka)[4], uint4 (&kb)[4]) {
    const uint4 zero4 = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint8_t* pa = kt + g * row_bytes + (32 * j + 8 * t) * 2;
        ka[j] = (!kPartial || static_cast<uint32_t>(g) < valid) ? *reinterpret_cast<const uint4*>(pa) : zero4;
        kb[j] = (!kPartial || static_cast<uint32_t>(g + 8) < valid)
                    ? *reinterpret_cast<const uint4*>(pa + 8 * row_bytes)
                    : zero4;
    }
}

template <bool kPartial>
__device__ __forceinline__ void load_v_frags(const uint8_t* vt, uint32_t row_bytes, int g, int t, uint32_t valid,
                                             uint4 (&va)[4][2]) {
    const uint4 zero4 = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const uint32_t row = 2 * t + (r & 1) + (r >> 1) * 8;
#pragma unroll
        for (int b = 0; b < 2; ++b)
            va[r][b] = (!kPartial || row < valid)
                           ? *reinterpret_cast<const uint4*>(vt + row * row_bytes + (64 * b + 8 * g) * 2)
                           : zero4;
    }
}

// Write one warp's state (after state_finish) as partial p of its KV head's
// query heads head0 .. head0 + group - 1: o of (head, p) at
// po + head * o_hs + p * o_ps, dims 0..63 there and dims 64..127 o_half
// floats later (64 for contiguous rows), m (natural log) and l at
// pm / pl + head * ml_hs + p * ml_ps.
__device__ __forceinline__ void store_warp_partial(const WarpState& st, float* po, float* pm, float* pl,
                                                   uint64_t o_hs, uint64_t o_ps, uint64_t o_half, uint64_t ml_hs,
                                                   uint64_t ml_ps, uint32_t p, uint32_t head0, uint32_t group, int g,
                                                   int t) {
#pragma unroll
    for (int hsel = 0; hsel < 2; ++hsel) {
        const uint32_t hh = 2 * t + hsel;
        if (hh >= group) continue;
        const uint32_t head = head0 + hh;
        float* o = po + head * o_hs + p * o_ps;
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
            const int d = 8 * g + 2 * (mt & 3);  // within the half mt >> 2
            *reinterpret_cast<float2*>(o + (mt >> 2) * o_half + d) =
                hsel == 0 ? make_float2(st.o[mt][0], st.o[mt][2]) : make_float2(st.o[mt][1], st.o[mt][3]);
        }
        if (g == 0) {
            const float m = hsel == 0 ? st.m0 : st.m1;
            pm[head * ml_hs + p * ml_ps] = m == -INFINITY ? -INFINITY : m * kLn2;
            pl[head * ml_hs + p * ml_ps] = hsel == 0 ? st.l0 : st.l1;
        }
    }
}

// ---- Tiles staged column block by column block with 128-byte swizzling
// ([block][16 rows][128 B], chunk c of row r at c ^ (r & 7); two blocks per KV
// head). MMA row m (and P.V contraction index m) holds token tile_token(m):
// odd rows are exchanged with the row 4 away, so the two rows a quarter-warp
// reads land on disjoint 16-byte slots for the K fragments, and the four rows
// of each V fragment load on disjoint slot pairs (no bank conflicts).
__device__ __forceinline__ uint32_t tile_token(uint32_t m) { return m ^ ((m & 1u) << 2); }

// K fragments of one head: kt = the head's 16 rows in its first column block,
// the second block kBlk bytes further (blocks of more than 16 rows when a
// stage carries several 16-token sub-tiles).
template <bool kPartial, uint32_t kBlk = kTile * 128>
__device__ __forceinline__ void load_k_frags_sw(const uint8_t* kt, int g, int t, uint32_t valid, uint4 (&ka)[4],
                                                uint4 (&kb)[4]) {
    const uint4 zero4 = make_uint4(0u, 0u, 0u, 0u);
    const uint32_t tok = tile_token(static_cast<uint32_t>(g));
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t chunk = ((j & 1) * 4 + t) ^ tok;
        const uint8_t* pa = kt + (j >> 1) * kBlk + tok * 128 + chunk * 16;
        ka[j] = (!kPartial || tok < valid) ? *reinterpret_cast<const uint4*>(pa) : zero4;
        kb[j] = (!kPartial || tok + 8 < valid) ? *reinterpret_cast<const uint4*>(pa + 8 * 128) : zero4;
    }
}

// V fragments of one head: contraction rows 2t, 2t+1, 2t+8, 2t+9 (their
// tokens via tile_token), head_dim halves 64b + 8g.
template <bool kPartial, uint32_t kBlk = kTile * 128>
__device__ __forceinline__ void load_v_frags_sw(const uint8_t* vt, int g, int t, uint32_t valid,
                                                uint4 (&va)[4][2]) {
    const uint4 zero4 = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const uint32_t tok = tile_token(2 * t + (r & 1)) + (r >> 1) * 8;
#pragma unroll
        for (int b = 0; b < 2; ++b)
            va[r][b] = (!kPartial || tok < valid)
                           ? *reinterpret_cast<const uint4*>(vt + b * kBlk + tok * 128 +
                                                             ((static_cast<uint32_t>(g) ^ (tok & 7u)) << 4))
                           : zero4;
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

// Combine scratch in shared memory: m/l [slot][8 heads], o [slot][8 heads][kOStride].
// The 129-float head stride spreads a warp's fragment stores over the banks
// (a 128 stride puts the 4 lanes of a row group on one bank).
constexpr int kOStride = 129;

// Store one warp's state into slot `slot`.
__device__ __forceinline__ void state_to_smem(const WarpState& st, int slot, float* sm_m, float* sm_l, float* sm_o,
                                              int g, int t) {
    if (g == 0) {
        sm_m[slot * 8 + 2 * t] = st.m0;
        sm_m[slot * 8 + 2 * t + 1] = st.m1;
        sm_l[slot * 8 + 2 * t] = st.l0;
        sm_l[slot * 8 + 2 * t + 1] = st.l1;
    }
    float* o0 = sm_o + (slot * 8 + 2 * t) * kOStride;
    float* o1 = o0 + kOStride;
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
        const int d = 64 * (mt >> 2) + 8 * g + 2 * (mt & 3);
        o0[d] = st.o[mt][0];
        o1[d] = st.o[mt][1];
        o0[d + 1] = st.o[mt][2];
        o1[d + 1] = st.o[mt][3];
    }
}

// Combine `nslots` warp states of one KV head (slots first, first+stride, ...)
// into the partial of (head kvh*group + hh, split), idx = hh*128 + d (the
// per-chunk split kernel; the persistent kernels fold warp states in
// registers instead).
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
        O = fmaf(sc, sm_o[(sl * 8 + hh) * kOStride + d], O);
    }
    const uint64_t state = static_cast<uint64_t>(kvh * group + hh) * splits + split;
    po[state * 128 + d] = O;
    if (d == 0) {
        pm[state] = M == -INFINITY ? -INFINITY : M * kLn2;
        pl[state] = L;
    }
}

}  // namespace b2
