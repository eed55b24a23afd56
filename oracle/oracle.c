/*
 * CPU oracle for the GQA attention hot path -- TEST INFRASTRUCTURE ONLY.
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load
 * this file's library, and only as the checker or the timed CPU baseline.
 * See oracle.h for the reference file:line each function restates.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ---------------------------------------------------------------- fp16 */

float or_half_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t exp = (h >> 10) & 0x1fu;
    const uint32_t man = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0x1fu) {
        bits = sign | 0x7f800000u | (man << 13);
    } else if (exp != 0) {
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    } else if (man == 0) {
        bits = sign;
    } else {
        /* subnormal: value = man * 2^-24, exact in binary32 */
        float f = (float)man * 5.9604644775390625e-08f;
        memcpy(&bits, &f, 4);
        bits |= sign;
    }
    float out;
    memcpy(&out, &bits, 4);
    return out;
}

uint16_t or_float_to_half(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) /* inf / nan (quiet) */
        return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
    if (ax >= 0x477ff000u) /* >= 65520 rounds to infinity */
        return (uint16_t)(sign | 0x7c00u);
    if (ax < 0x38800000u) { /* below 2^-14: subnormal half or zero */
        float af;
        memcpy(&af, &ax, 4);
        /* af * 2^24 is exact; round half to even in the default mode */
        const float m = nearbyintf(af * 16777216.0f);
        return (uint16_t)(sign | (uint16_t)m); /* m == 1024 encodes 2^-14 */
    }
    const uint32_t man = ax & 0x7fffffu;
    const uint32_t exp = (ax >> 23) - 112u;
    uint32_t h = (exp << 10) | (man >> 13);
    const uint32_t rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u)))
        ++h;
    return (uint16_t)(sign | h);
}

void or_halves_to_floats(const uint16_t* src, float* dst, size_t n) {
    for (size_t i = 0; i < n; ++i) dst[i] = or_half_to_float(src[i]);
}

void or_floats_to_halves(const float* src, uint16_t* dst, size_t n) {
    for (size_t i = 0; i < n; ++i) dst[i] = or_float_to_half(src[i]);
}

/* ---------------------------------------------------------------- RoPE */

void or_inverse_frequencies(size_t head_dim, float rope_theta, float* inv_freq) {
    const size_t half_dim = head_dim / 2;
    for (size_t i = 0; i < half_dim; ++i) {
        const float exponent = (float)(2 * i) / (float)head_dim;
        inv_freq[i] = 1.0f / powf(rope_theta, exponent);
    }
}

void or_fill_rope_tables(size_t max_seq_len, size_t head_dim, float rope_theta,
                         uint16_t* cos_table, uint16_t* sin_table) {
    const size_t half_dim = head_dim / 2;
    float* inv_freq = (float*)malloc(sizeof(float) * (half_dim ? half_dim : 1));
    or_inverse_frequencies(head_dim, rope_theta, inv_freq);
    for (size_t pos = 0; pos < max_seq_len; ++pos) {
        for (size_t i = 0; i < half_dim; ++i) {
            const float angle = (float)pos * inv_freq[i];
            cos_table[pos * half_dim + i] = or_float_to_half(cosf(angle));
            sin_table[pos * half_dim + i] = or_float_to_half(sinf(angle));
        }
    }
    free(inv_freq);
}

/* rope.hip.cpp:44-58 rotate_pair: fp32 products, no fused multiply-add
 * (the library compiles -ffp-contract=off). */
static void rotate_head(const uint16_t* src, uint16_t* dst, const uint16_t* cs,
                        const uint16_t* sn, size_t half_dim) {
    for (size_t i = 0; i < half_dim; ++i) {
        const float c = or_half_to_float(cs[i]);
        const float s = or_half_to_float(sn[i]);
        const float x0 = or_half_to_float(src[i]);
        const float x1 = or_half_to_float(src[i + half_dim]);
        const float a = x0 * c;
        const float b = x1 * s;
        const float e = x1 * c;
        const float g = x0 * s;
        dst[i] = or_float_to_half(a - b);
        dst[i + half_dim] = or_float_to_half(e + g);
    }
}

int or_rope_and_store_kv(uint16_t* q, uint16_t* k, const uint16_t* v,
                         uint16_t* k_cache, uint16_t* v_cache,
                         const uint16_t* cos_table, const uint16_t* sin_table,
                         size_t seq_len, size_t num_heads, size_t num_kv_heads,
                         size_t head_dim, size_t q_stride, size_t k_stride,
                         size_t start_pos, int apply_rotation) {
    if (seq_len == 0) return 0; /* rope.hip.cpp:156 */
    const size_t half_dim = head_dim / 2;
    const size_t kv_dim = num_kv_heads * head_dim;
    if (q_stride == 0) q_stride = num_heads * head_dim;
    if (k_stride == 0) k_stride = kv_dim;
    if (apply_rotation) {
        uint16_t* tmp = (uint16_t*)malloc(sizeof(uint16_t) * head_dim);
        for (size_t t = 0; t < seq_len; ++t) {
            const uint16_t* cs = cos_table + (start_pos + t) * half_dim;
            const uint16_t* sn = sin_table + (start_pos + t) * half_dim;
            for (size_t h = 0; h < num_heads; ++h) {
                uint16_t* head = q + t * q_stride + h * head_dim;
                rotate_head(head, tmp, cs, sn, half_dim);
                memcpy(head, tmp, sizeof(uint16_t) * head_dim);
            }
            for (size_t j = 0; j < num_kv_heads; ++j) {
                const size_t src = t * k_stride + j * head_dim;
                const size_t dst = (start_pos + t) * kv_dim + j * head_dim;
                rotate_head(k + src, tmp, cs, sn, half_dim);
                if (k_cache == NULL) { /* rope.hip.cpp:121-125 */
                    memcpy(k + src, tmp, sizeof(uint16_t) * head_dim);
                    continue;
                }
                memcpy(k_cache + dst, tmp, sizeof(uint16_t) * head_dim);
                memcpy(v_cache + dst, v + src, sizeof(uint16_t) * head_dim);
            }
        }
        free(tmp);
        return 0;
    }
    if (k_cache == NULL || v_cache == NULL) return -1;
    for (size_t t = 0; t < seq_len; ++t) { /* rope.hip.cpp:9-42 */
        const size_t src = t * k_stride;
        const size_t dst = (start_pos + t) * kv_dim;
        memcpy(k_cache + dst, k + src, sizeof(uint16_t) * kv_dim);
        memcpy(v_cache + dst, v + src, sizeof(uint16_t) * kv_dim);
    }
    return 0;
}

/* ----------------------------------------------------------- attention */

static void set_threads(int num_threads) {
#ifdef _OPENMP
    if (num_threads > 0) omp_set_num_threads(num_threads);
#else
    (void)num_threads;
#endif
}

void or_causal_attention_rows(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                              size_t seq_len, size_t start_pos,
                              size_t num_heads, size_t num_kv_heads, size_t head_dim,
                              size_t q_stride, size_t kv_stride,
                              const int64_t* rows, size_t num_rows,
                              uint16_t* out16, float* out32, size_t out_stride,
                              int num_threads) {
    if (seq_len == 0 || num_kv_heads == 0 || num_heads % num_kv_heads) return;
    const size_t group = num_heads / num_kv_heads;
    if (q_stride == 0) q_stride = num_heads * head_dim;
    if (kv_stride == 0) kv_stride = num_kv_heads * head_dim;
    if (out_stride == 0) out_stride = num_heads * head_dim;
    const size_t n_rows = rows ? num_rows : seq_len;
    const size_t kv_total = start_pos + seq_len;
    const double scale = 1.0 / sqrt((double)head_dim);
    set_threads(num_threads);
    const long long work = (long long)(n_rows * num_heads);
#pragma omp parallel
    {
        double* qf = (double*)malloc(sizeof(double) * head_dim);
        double* acc = (double*)malloc(sizeof(double) * head_dim);
        double* sc = (double*)malloc(sizeof(double) * kv_total);
#pragma omp for schedule(dynamic, 4)
        for (long long w = 0; w < work; ++w) {
            const size_t r = (size_t)w / num_heads;
            const size_t h = (size_t)w % num_heads;
            const size_t i = rows ? (size_t)rows[r] : r;
            const size_t kvh = h / group;
            const size_t n_keys = start_pos + i + 1;
            const uint16_t* qrow = q + i * q_stride + h * head_dim;
            for (size_t c = 0; c < head_dim; ++c) qf[c] = or_half_to_float(qrow[c]);
            double mx = -INFINITY;
            for (size_t j = 0; j < n_keys; ++j) {
                const uint16_t* krow = k + j * kv_stride + kvh * head_dim;
                double dot = 0.0;
                for (size_t c = 0; c < head_dim; ++c) dot += qf[c] * or_half_to_float(krow[c]);
                sc[j] = dot * scale;
                if (sc[j] > mx) mx = sc[j];
            }
            double den = 0.0;
            for (size_t j = 0; j < n_keys; ++j) { sc[j] = exp(sc[j] - mx); den += sc[j]; }
            for (size_t c = 0; c < head_dim; ++c) acc[c] = 0.0;
            for (size_t j = 0; j < n_keys; ++j) {
                const uint16_t* vrow = v + j * kv_stride + kvh * head_dim;
                const double p = sc[j];
                for (size_t c = 0; c < head_dim; ++c) acc[c] += p * or_half_to_float(vrow[c]);
            }
            for (size_t c = 0; c < head_dim; ++c) {
                const float val = (float)(acc[c] / den);
                const size_t o = r * out_stride + h * head_dim + c;
                if (out16) out16[o] = or_float_to_half(val);
                if (out32) out32[o] = val;
            }
        }
        free(qf);
        free(acc);
        free(sc);
    }
}

void or_decode_partials(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                        size_t kv_len, size_t num_heads, size_t num_kv_heads,
                        size_t head_dim, size_t kv_stride, size_t chunk,
                        float* partial_o, float* partial_m, float* partial_l,
                        int num_threads) {
    if (kv_len == 0 || num_kv_heads == 0 || num_heads % num_kv_heads || chunk == 0) return;
    const size_t group = num_heads / num_kv_heads;
    if (kv_stride == 0) kv_stride = num_kv_heads * head_dim;
    const size_t chunks = (kv_len + chunk - 1) / chunk;
    const float rs = 1.0f / sqrtf((float)head_dim);
    set_threads(num_threads);
    const long long work = (long long)(num_heads * chunks);
#pragma omp parallel
    {
        float* sc = (float*)malloc(sizeof(float) * chunk);
        float* qf = (float*)malloc(sizeof(float) * head_dim);
#pragma omp for schedule(static)
        for (long long w = 0; w < work; ++w) {
            const size_t h = (size_t)w / chunks;
            const size_t c = (size_t)w % chunks;
            const size_t kvh = h / group;
            const size_t t0 = c * chunk;
            const size_t t1 = t0 + chunk < kv_len ? t0 + chunk : kv_len;
            for (size_t e = 0; e < head_dim; ++e) qf[e] = or_half_to_float(q[h * head_dim + e]);
            float mx = -INFINITY;
            for (size_t t = t0; t < t1; ++t) {
                const uint16_t* krow = k + t * kv_stride + kvh * head_dim;
                float dot = 0.f;
                for (size_t e = 0; e < head_dim; ++e) dot += qf[e] * or_half_to_float(krow[e]);
                sc[t - t0] = dot * rs;
                if (sc[t - t0] > mx) mx = sc[t - t0];
            }
            float l = 0.f;
            for (size_t t = t0; t < t1; ++t) { sc[t - t0] = expf(sc[t - t0] - mx); l += sc[t - t0]; }
            float* o = partial_o + (h * chunks + c) * head_dim;
            for (size_t e = 0; e < head_dim; ++e) o[e] = 0.f;
            for (size_t t = t0; t < t1; ++t) {
                const uint16_t* vrow = v + t * kv_stride + kvh * head_dim;
                const float p = sc[t - t0];
                for (size_t e = 0; e < head_dim; ++e) o[e] += p * or_half_to_float(vrow[e]);
            }
            partial_m[h * chunks + c] = mx;
            partial_l[h * chunks + c] = l;
        }
        free(sc);
        free(qf);
    }
}

void or_merge_partials(const float* partial_o, const float* partial_m,
                       const float* partial_l, size_t num_heads,
                       size_t num_chunks, size_t head_dim,
                       uint16_t* out16, float* out32) {
    for (size_t h = 0; h < num_heads; ++h) {
        float gmax = -INFINITY;
        for (size_t c = 0; c < num_chunks; ++c)
            if (partial_m[h * num_chunks + c] > gmax) gmax = partial_m[h * num_chunks + c];
        double den = 0.0;
        for (size_t c = 0; c < num_chunks; ++c)
            den += exp((double)partial_m[h * num_chunks + c] - gmax) * partial_l[h * num_chunks + c];
        for (size_t e = 0; e < head_dim; ++e) {
            double num = 0.0;
            for (size_t c = 0; c < num_chunks; ++c)
                num += exp((double)partial_m[h * num_chunks + c] - gmax) *
                       partial_o[(h * num_chunks + c) * head_dim + e];
            const float val = (float)(num / den);
            if (out16) out16[h * head_dim + e] = or_float_to_half(val);
            if (out32) out32[h * head_dim + e] = val;
        }
    }
}

void or_decode_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                         size_t kv_len, size_t num_heads, size_t num_kv_heads,
                         size_t head_dim, size_t kv_stride,
                         uint16_t* out16, float* out32, int num_threads) {
    if (kv_len == 0 || num_kv_heads == 0 || num_heads % num_kv_heads) return;
    const size_t group = num_heads / num_kv_heads;
    if (kv_stride == 0) kv_stride = num_kv_heads * head_dim;
    const double scale = 1.0 / sqrt((double)head_dim);
    set_threads(num_threads);
    /* Each (head, key block) contributes an exact partial; combined below.
     * Blocks make the work parallel for long caches. */
    const size_t block = 4096;
    const size_t blocks = (kv_len + block - 1) / block;
    double* bm = (double*)malloc(sizeof(double) * num_heads * blocks);
    double* bl = (double*)malloc(sizeof(double) * num_heads * blocks);
    double* bo = (double*)malloc(sizeof(double) * num_heads * blocks * head_dim);
    const long long work = (long long)(num_heads * blocks);
#pragma omp parallel
    {
        double* sc = (double*)malloc(sizeof(double) * block);
        double* qf = (double*)malloc(sizeof(double) * head_dim);
#pragma omp for schedule(dynamic, 1)
        for (long long w = 0; w < work; ++w) {
            const size_t h = (size_t)w / blocks;
            const size_t b = (size_t)w % blocks;
            const size_t kvh = h / group;
            const size_t t0 = b * block;
            const size_t t1 = t0 + block < kv_len ? t0 + block : kv_len;
            for (size_t e = 0; e < head_dim; ++e) qf[e] = or_half_to_float(q[h * head_dim + e]);
            double mx = -INFINITY;
            for (size_t t = t0; t < t1; ++t) {
                const uint16_t* krow = k + t * kv_stride + kvh * head_dim;
                double dot = 0.0;
                for (size_t e = 0; e < head_dim; ++e) dot += qf[e] * or_half_to_float(krow[e]);
                sc[t - t0] = dot * scale;
                if (sc[t - t0] > mx) mx = sc[t - t0];
            }
            double l = 0.0;
            for (size_t t = t0; t < t1; ++t) { sc[t - t0] = exp(sc[t - t0] - mx); l += sc[t - t0]; }
            double* o = bo + (h * blocks + b) * head_dim;
            for (size_t e = 0; e < head_dim; ++e) o[e] = 0.0;
            for (size_t t = t0; t < t1; ++t) {
                const uint16_t* vrow = v + t * kv_stride + kvh * head_dim;
                const double p = sc[t - t0];
                for (size_t e = 0; e < head_dim; ++e) o[e] += p * or_half_to_float(vrow[e]);
            }
            bm[h * blocks + b] = mx;
            bl[h * blocks + b] = l;
        }
        free(sc);
        free(qf);
    }
    for (size_t h = 0; h < num_heads; ++h) {
        double gmax = -INFINITY;
        for (size_t b = 0; b < blocks; ++b) if (bm[h * blocks + b] > gmax) gmax = bm[h * blocks + b];
        double den = 0.0;
        for (size_t b = 0; b < blocks; ++b) den += exp(bm[h * blocks + b] - gmax) * bl[h * blocks + b];
        for (size_t e = 0; e < head_dim; ++e) {
            double num = 0.0;
            for (size_t b = 0; b < blocks; ++b)
                num += exp(bm[h * blocks + b] - gmax) * bo[(h * blocks + b) * head_dim + e];
            const float val = (float)(num / den);
            if (out16) out16[h * head_dim + e] = or_float_to_half(val);
            if (out32) out32[h * head_dim + e] = val;
        }
    }
    free(bm);
    free(bl);
    free(bo);
}
