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

/* The blocking of the reference's portable kernel, Int8GemmTiled (src/RecursiveAI.OneGpu.Kernels/Shaders/
 * Int8GemmKernel.hlsl:98-244), restated for the host's cores as the second CPU baseline: 64 x 64 output tiles, K in
 * chunks of 16 staged as float (A - za) and (B - zb) (zeros past M, N or K), the products accumulated in float per
 * tile element and folded into a wrapping int32 every 8 chunks (128 k) and at the end. Every partial sum is an integer
 * below 2^24 in magnitude (|a - za| and |b - zb| are at most 255, 128 products), so the float sums are exact and the
 * result equals og_oracle_int8_gemm bit for bit. Tiles are dealt to `threads` POSIX threads in turn. */
#define TB 64
#define TK 16
typedef struct tiled_job {
    const og_oracle_problem* p;
    const uint8_t *a, *b, *za, *zb;
    int32_t a_signed, b_signed, za_vector, zb_vector;
    int32_t* c;
    int64_t tile_begin, tile_end;
} tiled_job;

static void* gemm_tiles(void* arg) {
    const tiled_job* j = (const tiled_job*)arg;
    const og_oracle_problem* p = j->p;
    const int64_t M = p->m, N = p->n, K = p->k;
    const int64_t lda = p->lda == 0 ? K : p->lda;
    const int64_t ldb = p->ldb == 0 ? (p->transpose_b ? K : N) : p->ldb;
    const int64_t tm_count = (M + TB - 1) / TB, tn_count = (N + TB - 1) / TB;
    float as[TK][TB], bs[TK][TB], acc[TB][TB];
    uint32_t isum[TB][TB];
    for (int64_t t = j->tile_begin; t < j->tile_end; t++) {
        const int64_t bt = t / (tm_count * tn_count), r = t % (tm_count * tn_count);
        const int64_t m0 = (r / tn_count) * TB, n0 = (r % tn_count) * TB;
        const uint8_t* ab = j->a + p->offset_a + bt * (int64_t)p->stride_a;
        const uint8_t* bb = j->b + p->offset_b + bt * (int64_t)p->stride_b;
        memset(acc, 0, sizeof(acc));
        memset(isum, 0, sizeof(isum));
        for (int64_t k0 = 0; k0 < K; k0 += TK) {
            for (int kk = 0; kk < TK; kk++) {
                const int64_t k = k0 + kk;
                for (int i = 0; i < TB; i++) {
                    const int64_t m = m0 + i, n = n0 + i;
                    float av = 0.0f, bv = 0.0f;
                    if (m < M && k < K) {
                        const int32_t z = j->za ? val8(j->za[j->za_vector ? m : 0], j->a_signed) : 0;
                        av = (float)(val8(ab[m * lda + k], j->a_signed) - z);
                    }
                    if (n < N && k < K) {
                        const int32_t z = j->zb ? val8(j->zb[j->zb_vector ? n : 0], j->b_signed) : 0;
                        bv = (float)(val8(bb[p->transpose_b ? n * ldb + k : k * ldb + n], j->b_signed) - z);
                    }
                    as[kk][i] = av;
                    bs[kk][i] = bv;
                }
            }
            for (int kk = 0; kk < TK; kk++)
                for (int i = 0; i < TB; i++) {
                    const float av = as[kk][i];
                    for (int q = 0; q < TB; q++) acc[i][q] += av * bs[kk][q];
                }
            if (((k0 / TK) & 7) == 7) {
                for (int i = 0; i < TB; i++)
                    for (int q = 0; q < TB; q++) {
                        isum[i][q] += (uint32_t)(int32_t)acc[i][q];
                        acc[i][q] = 0.0f;
                    }
            }
        }
        for (int i = 0; i < TB; i++) {
            const int64_t m = m0 + i;
            if (m >= M) break;
            int32_t* crow = j->c + (bt * M + m) * N;
            for (int q = 0; q < TB && n0 + q < N; q++) crow[n0 + q] = (int32_t)(isum[i][q] + (uint32_t)(int32_t)acc[i][q]);
        }
    }
    return NULL;
}

void og_oracle_int8_gemm_tiled(const og_oracle_problem* p, const uint8_t* a, int32_t a_signed, const uint8_t* b,
                               int32_t b_signed, const uint8_t* za, int32_t za_vector, const uint8_t* zb,
                               int32_t zb_vector, int32_t* c, int32_t threads) {
    const int64_t tiles = (int64_t)p->batch * ((p->m + TB - 1) / TB) * ((p->n + TB - 1) / TB);
    if (tiles <= 0) return;
    if (threads < 1) threads = 1;
    if (threads > tiles) threads = (int32_t)tiles;
    if (threads > 256) threads = 256;
    tiled_job jobs[256];
    pthread_t tids[256];
    for (int32_t t = 0; t < threads; t++)
        jobs[t] = (tiled_job){p, a, b, za, zb, a_signed, b_signed, za_vector, zb_vector, c,
                              tiles * t / threads, tiles * (t + 1) / threads};
    if (threads == 1) {
        gemm_tiles(&jobs[0]);
        return;
    }
    for (int32_t t = 0; t < threads; t++) pthread_create(&tids[t], NULL, gemm_tiles, &jobs[t]);
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

/* IEEE 754 binary32 -> binary16, round to nearest even (the C# (Half) cast): overflow to infinity, results below
 * the smallest normal become subnormals or zero, NaN stays NaN (quiet, top payload bits kept). */
uint16_t og_oracle_float_to_half(float f) {
    const uint32_t x = f2u(f);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t exp = (x >> 23) & 0xFFu;
    uint32_t man = x & 0x7FFFFFu;
    if (exp == 0xFFu) return (uint16_t)(sign | 0x7C00u | (man != 0u ? 0x200u | (man >> 13) : 0u));
    const int32_t e = (int32_t)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        man |= 0x800000u;
        const uint32_t shift = (uint32_t)(14 - e);
        uint32_t h = man >> shift;
        const uint32_t rest = man & ((1u << shift) - 1u), half = 1u << (shift - 1u);
        if (rest > half || (rest == half && (h & 1u))) h++;
        return (uint16_t)(sign | h);
    }
    uint32_t h = sign | ((uint32_t)e << 10) | (man >> 13);
    const uint32_t rest = man & 0x1FFFu;
    if (rest > 0x1000u || (rest == 0x1000u && (h & 1u))) h++;  /* a carry moves into the exponent (or to infinity) */
    return (uint16_t)h;
}

/* IEEE 754 binary16 -> binary32, exact. */
float og_oracle_half_to_float(uint16_t h) {
    const uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    const uint32_t exp = ((uint32_t)h >> 10) & 0x1Fu;
    uint32_t man = (uint32_t)h & 0x3FFu;
    if (exp == 0x1Fu) return u2f(sign | 0x7F800000u | (man << 13));
    if (exp != 0u) return u2f(sign | ((exp - 15u + 127u) << 23) | (man << 13));
    if (man == 0u) return u2f(sign);
    int32_t e = -1;
    do {
        e++;
        man <<= 1;
    } while ((man & 0x400u) == 0u);
    return u2f(sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3FFu) << 13));
}

static inline int32_t quant_value(int32_t kind, const void* p, int64_t i) {
    if (kind == 0) return (int32_t)((const uint8_t*)p)[i];
    if (kind == 1) return (int32_t)((const int8_t*)p)[i];
    return ((const int32_t*)p)[i];
}

/* DequantizeTests.cs:57-68: want = (float)unchecked(x - zp) * scale, then (Half)want for half outputs. */
void og_oracle_dequantize(int32_t kind, const void* x, int64_t count, int32_t per_axis, int64_t axis_len, int64_t inner,
                          const float* scale, const void* zero_point, int32_t half_out, void* out) {
    for (int64_t j = 0; j < count; j++) {
        const int64_t a = per_axis ? (j / inner) % axis_len : 0;
        const int32_t zp = zero_point != NULL ? quant_value(kind, zero_point, a) : 0;
        const int32_t d = (int32_t)((uint32_t)quant_value(kind, x, j) - (uint32_t)zp);
        const float want = (float)d * scale[a];
        if (half_out) ((uint16_t*)out)[j] = og_oracle_float_to_half(want);
        else ((float*)out)[j] = want;
    }
}

/* DequantizeTests.cs:138-148 (QuantizeOne): v = MathF.Round(x / scale) + zeroPoint in binary32, NaN -> lo, clamp. */
void og_oracle_quantize(int32_t is_signed, int32_t half_in, const void* x, int64_t count, int32_t per_axis,
                        int64_t axis_len, int64_t inner, const float* scale, const uint8_t* zero_point, uint8_t* out) {
    const int32_t lo = is_signed ? -128 : 0, hi = is_signed ? 127 : 255;
    for (int64_t j = 0; j < count; j++) {
        const int64_t a = per_axis ? (j / inner) % axis_len : 0;
        const int32_t zp = zero_point != NULL ? val8(zero_point[a], is_signed) : 0;
        const float xv = half_in ? og_oracle_half_to_float(((const uint16_t*)x)[j]) : ((const float*)x)[j];
        const float q = xv / scale[a];
        const float v = nearbyintf(q) + (float)zp;
        int32_t r;
        if (isnan(v)) r = lo;
        else r = v < (float)lo ? lo : (v > (float)hi ? hi : (int32_t)v);
        out[j] = (uint8_t)(r & 0xFF);
    }
}

/* ConvProblem.OutHeight / OutWidth (GpuWindow.OutputExtent without auto padding or ceil mode). */
int32_t og_oracle_conv_out_extent(int32_t input, int32_t kernel, int32_t stride, int32_t dilation, int32_t pad_begin,
                                  int32_t pad_end) {
    if (input < 1 || kernel < 1 || stride < 1 || dilation < 1) return 0;
    const int64_t effective = (int64_t)dilation * (kernel - 1) + 1;
    const int64_t span = (int64_t)input + pad_begin + pad_end - effective;
    if (span < 0) return 0;
    const int64_t extent = span / stride + 1;
    return extent > 2147483647 ? 0 : (int32_t)extent;
}

typedef struct conv_job {
    const og_oracle_conv* p;
    const uint8_t *x, *w, *xz, *wz;
    int32_t xs, ws, wz_vector;
    int32_t* y;
    int64_t row0, row1;  /* rows (image, output channel) of this thread */
} conv_job;

static void* conv_rows(void* arg) {
    const conv_job* j = (const conv_job*)arg;
    const og_oracle_conv* p = j->p;
    const int32_t oh = og_oracle_conv_out_extent(p->h, p->kh, p->stride_h, p->dilation_h, p->pad_top, p->pad_bottom);
    const int32_t ow = og_oracle_conv_out_extent(p->w, p->kw, p->stride_w, p->dilation_w, p->pad_left, p->pad_right);
    const int32_t cin_g = p->cin / p->groups, cout_g = p->cout / p->groups;
    const int32_t xzv = j->xz != NULL ? val8(j->xz[0], j->xs) : 0;
    for (int64_t row = j->row0; row < j->row1; row++) {
        const int64_t n = row / p->cout, m = row % p->cout, g = m / cout_g;
        const int32_t wzv = j->wz != NULL ? val8(j->wz[j->wz_vector ? m : 0], j->ws) : 0;
        for (int32_t i = 0; i < oh; i++) {
            for (int32_t jj = 0; jj < ow; jj++) {
                uint32_t acc = 0;
                for (int32_t c = 0; c < cin_g; c++) {
                    for (int32_t kh = 0; kh < p->kh; kh++) {
                        const int64_t ih = (int64_t)i * p->stride_h + (int64_t)kh * p->dilation_h - p->pad_top;
                        if (ih < 0 || ih >= p->h) continue;
                        for (int32_t kw = 0; kw < p->kw; kw++) {
                            const int64_t iw = (int64_t)jj * p->stride_w + (int64_t)kw * p->dilation_w - p->pad_left;
                            if (iw < 0 || iw >= p->w) continue;
                            const int64_t xi = p->offset_x + ((((n * p->cin) + g * cin_g + c) * p->h + ih) * p->w + iw);
                            const int64_t wi = p->offset_w + ((((m * cin_g) + c) * p->kh + kh) * p->kw + kw);
                            const int32_t xv = val8(j->x[xi], j->xs) - xzv;
                            const int32_t wv = val8(j->w[wi], j->ws) - wzv;
                            acc += (uint32_t)xv * (uint32_t)wv;
                        }
                    }
                }
                j->y[((n * p->cout + m) * oh + i) * ow + jj] = (int32_t)acc;
            }
        }
    }
    return NULL;
}

/* ConvIntegerTests.cs:41-88 (Reference), rows (image, output channel) split over POSIX threads. */
void og_oracle_conv_integer(const og_oracle_conv* p, const uint8_t* x, int32_t x_signed, const uint8_t* w,
                            int32_t w_signed, const uint8_t* xz, const uint8_t* wz, int32_t wz_vector, int32_t* y,
                            int32_t threads) {
    const int64_t rows = (int64_t)p->batch * p->cout;
    if (rows <= 0) return;
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    if (threads > rows) threads = (int32_t)rows;
    conv_job jobs[256];
    pthread_t tids[256];
    for (int32_t t = 0; t < threads; t++)
        jobs[t] = (conv_job){p, x, w, xz, wz, x_signed, w_signed, wz_vector, y, rows * t / threads,
                             rows * (t + 1) / threads};
    if (threads == 1) {
        conv_rows(&jobs[0]);
        return;
    }
    for (int32_t t = 0; t < threads; t++) pthread_create(&tids[t], NULL, conv_rows, &jobs[t]);
    for (int32_t t = 0; t < threads; t++) pthread_join(tids[t], NULL);
}
