/*
 * CPU oracle for the int8 GEMM + DynamicQuantizeLinear path. TEST INFRASTRUCTURE ONLY: see og_oracle.h for what may
 * use it and which reference file each function restates. Build with -ffp-contract=off so that no multiply and add
 * are fused, as in the C# references.
 */
#include "og_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* Int8Tests.cs:36-47: s = seed * 2654435761 + 7, then s = s * 1664525 + 1013904223 per byte, byte = s >> 24. */
void og_oracle_bytes(uint8_t* out, int64_t length, int32_t seed) {
    uint32_t s = (uint32_t)seed * 2654435761u + 7u;
    for (int64_t i = 0; i < length; i++) {
        s = s * 1664525u + 1013904223u;
        out[i] = (uint8_t)(s >> 24);
    }
}

/* Rig.cs:8-19: lo + (hi - lo) * ((s >> 8) / 2^24), every step rounded to binary32. */
void og_oracle_random(float* out, int64_t n, int32_t seed, float lo, float hi) {
    uint32_t s = (uint32_t)seed * 2654435761u + 12345u;
    for (int64_t i = 0; i < n; i++) {
        s = s * 1664525u + 1013904223u;
        float u = (float)(s >> 8) / 16777216.0f;
        float w = hi - lo;
        float t = w * u;
        out[i] = lo + t;
    }
}

/* Int8Tests.cs:632-647: the seven input distributions of DynamicQuantizeIsBitExact. */
void og_oracle_dq_input(float* out, int64_t count, int32_t seed, int32_t kind) {
    uint32_t s = (uint32_t)seed * 2654435761u + 99u;
    for (int64_t i = 0; i < count; i++) {
        s = s * 1664525u + 1013904223u;
        float q = (float)(s >> 8) / 16777216.0f;
        float q2 = q * 2.0f;
        float u = q2 - 1.0f;
        float v;
        switch (kind) {
            case 0: v = u * 4.7f; break;
            case 1: { float t = u + 1.0f; v = t * 3.3f; } break;
            case 2: { float t = u + 1.0f; float w = t * 0.0123f; v = -w; } break;
            case 3: { float c = u * u; c = c * u; c = c * 100.0f; v = c + 0.001f; } break;
            case 4: { float t = u * 127.0f; t = nearbyintf(t); v = t * 0.125f; } break;
            case 5: v = 0.0f; break;
            default: v = u * 1e-3f; break;
        }
        out[i] = v;
    }
}

static inline int32_t val8(uint8_t v, int32_t is_signed) { return is_signed ? (int32_t)(int8_t)v : (int32_t)v; }

typedef struct gemm_job {
    const og_oracle_problem* p;
    const uint8_t *a, *b, *za, *zb;
    int32_t a_signed, b_signed, za_vector, zb_vector;
    int32_t* c;
    int64_t row_begin, row_end;
} gemm_job;

/* Int8Tests.cs:52-82 for rows [row_begin, row_end) of the Batch*M rows. The sums are formed in uint32 so that they wrap
 * like the C# unchecked int; integer addition is exact modulo 2^32 in any order, so k runs in the outer loop of each row
 * to keep B's rows streaming through the cache. */
static void* gemm_rows(void* arg) {
    const gemm_job* j = (const gemm_job*)arg;
    const og_oracle_problem* p = j->p;
    const int64_t M = p->m, N = p->n, K = p->k;
    const int64_t lda = p->lda == 0 ? K : p->lda;
    const int64_t ldb = p->ldb == 0 ? (p->transpose_b ? K : N) : p->ldb;
    int32_t* arow = (int32_t*)malloc(sizeof(int32_t) * (size_t)(K > 0 ? K : 1));
    int32_t* zbv = (int32_t*)malloc(sizeof(int32_t) * (size_t)(N > 0 ? N : 1));
    uint32_t* acc = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)(N > 0 ? N : 1));
    for (int64_t n = 0; n < N; n++) zbv[n] = j->zb ? val8(j->zb[j->zb_vector ? n : 0], j->b_signed) : 0;
    for (int64_t row = j->row_begin; row < j->row_end; row++) {
        const int64_t bt = row / M, m = row % M;
        const int32_t zA = j->za ? val8(j->za[j->za_vector ? m : 0], j->a_signed) : 0;
        const uint8_t* ap = j->a + p->offset_a + bt * (int64_t)p->stride_a + m * lda;
        for (int64_t k = 0; k < K; k++) arow[k] = val8(ap[k], j->a_signed) - zA;
        const uint8_t* bp = j->b + p->offset_b + bt * (int64_t)p->stride_b;
        memset(acc, 0, sizeof(uint32_t) * (size_t)N);
        if (!p->transpose_b) {
            for (int64_t k = 0; k < K; k++) {
                const int32_t av = arow[k];
                const uint8_t* brow = bp + k * ldb;
                if (j->b_signed) {
                    for (int64_t n = 0; n < N; n++) acc[n] += (uint32_t)(av * ((int32_t)(int8_t)brow[n] - zbv[n]));
                } else {
                    for (int64_t n = 0; n < N; n++) acc[n] += (uint32_t)(av * ((int32_t)brow[n] - zbv[n]));
                }
            }
        } else {
            for (int64_t n = 0; n < N; n++) {
                const uint8_t* bcol = bp + n * ldb;
                uint32_t s = 0;
                for (int64_t k = 0; k < K; k++) s += (uint32_t)(arow[k] * (val8(bcol[k], j->b_signed) - zbv[n]));
                acc[n] = s;
            }
        }
        int32_t* crow = j->c + row * N;
        for (int64_t n = 0; n < N; n++) crow[n] = (int32_t)acc[n];
    }
    free(arow);
    free(zbv);
    free(acc);
    return NULL;
}

void og_oracle_int8_gemm(const og_oracle_problem* p, const uint8_t* a, int32_t a_signed, const uint8_t* b,
                         int32_t b_signed, const uint8_t* za, int32_t za_vector, const uint8_t* zb, int32_t zb_vector,
                         int32_t* c, int32_t threads) {
    const int64_t rows = (int64_t)p->batch * p->m;
    if (rows <= 0 || p->n <= 0) return;
    if (threads < 1) threads = 1;
    if (threads > rows) threads = (int32_t)rows;
    gemm_job jobs[256];
    pthread_t tids[256];
    if (threads > 256) threads = 256;
    for (int32_t t = 0; t < threads; t++) {
        jobs[t] = (gemm_job){p, a, b, za, zb, a_signed, b_signed, za_vector, zb_vector, c,
                             rows * t / threads, rows * (t + 1) / threads};
    }
    if (threads == 1) {
        gemm_rows(&jobs[0]);
        return;
    }
    for (int32_t t = 0; t < threads; t++) pthread_create(&tids[t], NULL, gemm_rows, &jobs[t]);
    for (int32_t t = 0; t < threads; t++) pthread_join(tids[t], NULL);
}

/* Int8GemmDot.hlsl:4-10 and Put (:134-140): an unsigned byte u is staged as u xor 0x80 = u - 128 and its zero point z
 * moves to z - 128; then sum (s - z')(t - w') = sum s*t - w' * sum s - z' * sum t + K z' w', all modulo 2^32. */
void og_oracle_int8_gemm_signed_domain(const og_oracle_problem* p, const uint8_t* a, int32_t a_signed,
                                       const uint8_t* b, int32_t b_signed, const uint8_t* za, int32_t za_vector,
                                       const uint8_t* zb, int32_t zb_vector, int32_t* c) {
    const int64_t M = p->m, N = p->n, K = p->k;
    const int64_t lda = p->lda == 0 ? K : p->lda;
    const int64_t ldb = p->ldb == 0 ? (p->transpose_b ? K : N) : p->ldb;
    for (int64_t bt = 0; bt < p->batch; bt++) {
        for (int64_t m = 0; m < M; m++) {
            const int32_t zpa = za ? val8(za[za_vector ? m : 0], a_signed) : 0;
            const int32_t zsa = a_signed ? zpa : zpa - 128;
            for (int64_t n = 0; n < N; n++) {
                const int32_t zpb = zb ? val8(zb[zb_vector ? n : 0], b_signed) : 0;
                const int32_t zsb = b_signed ? zpb : zpb - 128;
                uint32_t dot = 0, sa = 0, sb = 0;
                for (int64_t k = 0; k < K; k++) {
                    uint8_t av = a[p->offset_a + bt * (int64_t)p->stride_a + m * lda + k];
                    uint8_t bv = b[p->offset_b + bt * (int64_t)p->stride_b + (p->transpose_b ? n * ldb + k : k * ldb + n)];
                    int32_t s = (int32_t)(int8_t)(a_signed ? av : (uint8_t)(av ^ 0x80u));
                    int32_t t = (int32_t)(int8_t)(b_signed ? bv : (uint8_t)(bv ^ 0x80u));
                    dot += (uint32_t)(s * t);
                    sa += (uint32_t)s;
                    sb += (uint32_t)t;
                }
                uint32_t r = dot - (uint32_t)zsb * sa - (uint32_t)zsa * sb + (uint32_t)K * (uint32_t)zsa * (uint32_t)zsb;
                c[(bt * M + m) * N + n] = (int32_t)r;
            }
        }
    }
}

/* .NET Math.Clamp(float value, float min, float max). */
static float net_clamp(float v, float lo, float hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* Int8Tests.cs:84-97. */
int32_t og_oracle_requant(int32_t acc, float mult, int32_t zero, int32_t is_unsigned) {
    const int32_t lo = is_unsigned ? 0 : -128;
    const int32_t hi = is_unsigned ? 255 : 127;
    float v = (float)acc * mult;
    if (isnan(v)) return lo;
    float r = nearbyintf(v);
    r = net_clamp(r, (float)(lo - zero), (float)(hi - zero));
    return (int32_t)r + zero;
}

/* Int8Tests.cs:356-373: acc (+ int bias, wrapping), then float(acc) * scale rounded, then + float bias rounded. */
float og_oracle_float_epilogue(int32_t acc, int32_t has_int_bias, int32_t int_bias, float scale, int32_t has_float_bias,
                               float float_bias) {
    if (has_int_bias) acc = (int32_t)((uint32_t)acc + (uint32_t)int_bias);
    float f = (float)acc * scale;
    if (has_float_bias) f = f + float_bias;
    return f;
}

/* .NET Math.Min / Math.Max for float: NaN propagates, -0 orders below +0. */
static float net_min(float x, float y) {
    if (isnan(x)) return x;
    if (isnan(y)) return y;
    if (x < y) return x;
    if (y < x) return y;
    return signbit(x) ? x : y;
}
static float net_max(float x, float y) {
    if (isnan(x)) return x;
    if (isnan(y)) return y;
    if (x > y) return x;
    if (y > x) return y;
    return signbit(x) ? y : x;
}

/* Int8Tests.cs:577-615 (onemodel's DynamicQuantizeLinear). */
void og_oracle_dynamic_quantize(const float* x, int64_t count, uint8_t* y, float* scale_out, uint8_t* zero_point) {
    float mn = INFINITY, mx = -INFINITY;
    for (int64_t i = 0; i < count; i++) {
        float v = x[i];
        if (v < mn) mn = v;
        if (v > mx) mx = v;
    }
    float lo = net_min(0.0f, mn), hi = net_max(0.0f, mx);
    float range = hi - lo;
    float scale = range / 255.0f;
    int32_t zp = 0;
    if (scale != 0.0f && isfinite(scale)) {
        float q = lo / scale;
        float z = nearbyintf(0.0f - q);
        zp = z < 0.0f ? 0 : (z > 255.0f ? 255 : (int32_t)z);
    }
    if (scale == 0.0f) {
        memset(y, 0, (size_t)count);
        *scale_out = 1.0f;
        *zero_point = 0;
        return;
    }
    const float zf = (float)zp;
    for (int64_t i = 0; i < count; i++) {
        float q = x[i] / scale;
        float v = nearbyintf(q) + zf;
        y[i] = isnan(v) ? 0 : (v < 0.0f ? 0 : (v > 255.0f ? 255 : (uint8_t)(int32_t)v));
    }
    *scale_out = scale;
    *zero_point = (uint8_t)zp;
}

static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* DivExact.hlsli:4-21 (Unpack): 24-bit mantissa with the top bit set, subnormals normalised. */
static void unpack(uint32_t bits, uint32_t* m, int32_t* e) {
    *e = (int32_t)((bits >> 23) & 255u);
    *m = bits & 0x7FFFFFu;
    if (*e == 0) {
        *e = 1;
        while (*m < 0x800000u) { *m <<= 1; *e -= 1; }
    } else {
        *m |= 0x800000u;
    }
}

/* DivExact.hlsli:28-99: x / s by long division of the mantissas (26 quotient bits + sticky), round to nearest even;
 * zeros, infinities, NaNs and results outside the normal range fall back to the plain division. */
float og_oracle_div_exact(float x, float s) {
    const uint32_t xb = f2u(x), sb = f2u(s);
    const uint32_t xa = xb & 0x7FFFFFFFu, sa = sb & 0x7FFFFFFFu;
    if (xa == 0u && sa != 0u && sa <= 0x7F800000u) return u2f((xb ^ sb) & 0x80000000u);
    if (xa == 0u || sa == 0u || xa >= 0x7F800000u || sa >= 0x7F800000u) return x / s;
    uint32_t ma, mb;
    int32_t ea, eb;
    unpack(xa, &ma, &ea);
    unpack(sa, &mb, &eb);
    uint32_t r = ma, q = 0u;
    if (r >= mb) { q = 1u; r -= mb; }
    for (int i = 0; i < 26; i++) {
        r <<= 1;
        q <<= 1;
        if (r >= mb) { q |= 1u; r -= mb; }
    }
    int32_t e = ea - eb + 127;
    uint32_t shift = 2u;
    if (q >= 0x4000000u) shift = 3u; else e -= 1;
    uint32_t m = q >> shift;
    uint32_t rest = q & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1u);
    int sticky = r != 0u;
    if (rest > half || (rest == half && (sticky || (m & 1u) != 0u))) {
        m += 1u;
        if (m == 0x1000000u) { m >>= 1; e += 1; }
    }
    if (e < 1 || e > 254) return x / s;
    return u2f(((xb ^ sb) & 0x80000000u) | ((uint32_t)e << 23) | (m & 0x7FFFFFu));
}
