/*
 * tn_oracle.c -- CPU restatement of torchnative's Q4_0 linear and SDPA
 * arithmetic. TEST INFRASTRUCTURE ONLY (the parity checker and the timed CPU
 * baseline); see tn_oracle.h for what pins it and who may call it.
 *
 * Compiled with -ffp-contract=off so that every `a * b + c` below rounds twice,
 * as the Rust source it restates does (Rust never contracts to FMA).
 * Paths cited are relative to the reference project root.
 */
#include "tn_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* IEEE 754 binary16 / bfloat16 conversions, round to nearest even.         */
/* The reference uses the `half` crate (f16::from_f32, bf16::from_f32),      */
/* which rounds to nearest even and keeps subnormals.                        */
/* ------------------------------------------------------------------------ */

uint16_t tno_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t exp = (x >> 23) & 0xffu;
    uint32_t man = x & 0x7fffffu;
    if (exp == 0xffu) {
        if (man) return (uint16_t)(sign | 0x7e00u | (man >> 13));
        return (uint16_t)(sign | 0x7c00u);
    }
    int32_t e = (int32_t)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        /* binary16 subnormal: value = h * 2^-24, h = m >> (14 - e). */
        if (e < -10) return (uint16_t)sign;
        uint32_t m = man | 0x800000u;
        int shift = 14 - e;
        uint32_t h = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (h & 1u))) h++;
        return (uint16_t)(sign | h);
    }
    uint32_t h = ((uint32_t)e << 10) | (man >> 13);
    uint32_t rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++; /* carry may reach inf: correct */
    return (uint16_t)(sign | h);
}

float tno_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t exp = ((uint32_t)h >> 10) & 0x1fu;
    uint32_t man = (uint32_t)h & 0x3ffu;
    uint32_t x;
    if (exp == 0) {
        if (man == 0) {
            x = sign;
        } else {
            float v = (float)man * 5.9604644775390625e-08f; /* man * 2^-24, exact */
            memcpy(&x, &v, 4);
            x |= sign;
        }
    } else if (exp == 31) {
        x = sign | 0x7f800000u | (man << 13);
    } else {
        x = sign | ((exp + 112u) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

uint16_t tno_f32_to_bf16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40u);
    x += 0x7fffu + ((x >> 16) & 1u);
    return (uint16_t)(x >> 16);
}

float tno_bf16_to_f32(uint16_t b) {
    uint32_t x = (uint32_t)b << 16;
    float f;
    memcpy(&f, &x, 4);
    return f;
}

/* Rust `f as u8` / `f as i8`: truncate toward zero, saturate, NaN -> 0. */
static uint8_t sat_u8(float v) {
    if (!(v == v)) return 0;
    if (v <= 0.0f) return 0;
    if (v >= 255.0f) return 255;
    return (uint8_t)v;
}
static int8_t sat_i8(float v) {
    if (!(v == v)) return 0;
    if (v <= -128.0f) return -128;
    if (v >= 127.0f) return 127;
    return (int8_t)v;
}

static void put_u16(uint8_t *p, uint16_t v) {
    p[0] = (uint8_t)(v & 0xff);
    p[1] = (uint8_t)(v >> 8);
}
static uint16_t get_u16(const uint8_t *p) { return (uint16_t)(p[0] | ((uint16_t)p[1] << 8)); }

/* ------------------------------------------------------------------------ */
/* Q4_0: 18-byte block = f16 d, then 16 bytes; element j is (qs[j] & 15) - 8,
 * element j + 16 is (qs[j] >> 4) - 8 (k_quants.rs:79-83, 219-239).        */
/* ------------------------------------------------------------------------ */

void tno_q4_0_quantize(const float *x, uint8_t *blob, int64_t n) {
    /* k_quants.rs:241-277: signed maximum (first of equal magnitudes wins),
     * d = max / -8, q = min(15, (x * (1/d) + 8.5) as u8). */
    for (int64_t i = 0; i < n / 32; ++i) {
        const float *xs = x + i * 32;
        uint8_t *out = blob + i * 18;
        float amax = 0.0f, max = 0.0f;
        for (int j = 0; j < 32; ++j) {
            float a = fabsf(xs[j]);
            if (amax < a) {
                amax = a;
                max = xs[j];
            }
        }
        float d = max / -8.0f;
        float id = (d != 0.0f) ? 1.0f / d : 0.0f;
        put_u16(out, tno_f32_to_f16(d));
        for (int j = 0; j < 16; ++j) {
            float x0 = xs[j] * id;
            float x1 = xs[16 + j] * id;
            uint8_t q0 = sat_u8(x0 + 8.5f);
            uint8_t q1 = sat_u8(x1 + 8.5f);
            if (q0 > 15) q0 = 15;
            if (q1 > 15) q1 = 15;
            out[2 + j] = (uint8_t)(q0 | (q1 << 4));
        }
    }
}

void tno_q4_0_dequantize(const uint8_t *blob, float *y, int64_t n) {
    for (int64_t i = 0; i < n / 32; ++i) {
        const uint8_t *b = blob + i * 18;
        float d = tno_f16_to_f32(get_u16(b));
        for (int j = 0; j < 16; ++j) {
            int x0 = (b[2 + j] & 0x0f) - 8;
            int x1 = (b[2 + j] >> 4) - 8;
            y[i * 32 + j] = (float)x0 * d;
            y[i * 32 + j + 16] = (float)x1 * d;
        }
    }
}

/* Q8_0: 34-byte block = f16 d, then 32 int8 (k_quants.rs:115-119). */
void tno_q8_0_quantize(const float *x, uint8_t *blob, int64_t n) {
    /* k_quants.rs:676-706: d = amax / 127, q = round(x * (1/d)) as i8,
     * round half away from zero (f32::round). */
    for (int64_t i = 0; i < n / 32; ++i) {
        const float *xs = x + i * 32;
        uint8_t *out = blob + i * 34;
        float amax = 0.0f;
        for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(xs[j]));
        float d = amax / 127.0f;
        float id = (d != 0.0f) ? 1.0f / d : 0.0f;
        put_u16(out, tno_f32_to_f16(d));
        for (int j = 0; j < 32; ++j) {
            int8_t q = sat_i8(roundf(xs[j] * id));
            out[2 + j] = (uint8_t)q;
        }
    }
}

void tno_q8_0_dequantize(const uint8_t *blob, float *y, int64_t n) {
    for (int64_t i = 0; i < n / 32; ++i) {
        const uint8_t *b = blob + i * 34;
        float d = tno_f16_to_f32(get_u16(b));
        for (int j = 0; j < 32; ++j) y[i * 32 + j] = (float)(int8_t)b[2 + j] * d;
    }
}

float tno_q4_0_q8_0_dot(const uint8_t *w, const uint8_t *xq, int64_t nblocks) {
    /* k_quants.rs:312-330, in its order: integer block sum, then
     * sumf += (sum_i as f32 * d_w) * d_x, block after block. */
    float sumf = 0.0f;
    for (int64_t b = 0; b < nblocks; ++b) {
        const uint8_t *wb = w + b * 18;
        const uint8_t *xb = xq + b * 34;
        int32_t sum_i = 0;
        for (int j = 0; j < 16; ++j) {
            int32_t v0 = (int32_t)(wb[2 + j] & 0x0f) - 8;
            int32_t v1 = (int32_t)(wb[2 + j] >> 4) - 8;
            sum_i += v0 * (int32_t)(int8_t)xb[2 + j] + v1 * (int32_t)(int8_t)xb[2 + 16 + j];
        }
        float dw = tno_f16_to_f32(get_u16(wb));
        float dx = tno_f16_to_f32(get_u16(xb));
        sumf += (float)sum_i * dw * dx;
    }
    return sumf;
}

float tno_q8_0_q8_0_dot(const uint8_t *w, const uint8_t *xq, int64_t nblocks) {
    /* BlockQ8_0::vec_dot_unopt, k_quants.rs:737-756: the same order as the
     * Q4_0 dot above -- integer block sum of signed codes, then
     * sumf += (sum_i as f32 * d_w) * d_x, block after block. */
    float sumf = 0.0f;
    for (int64_t b = 0; b < nblocks; ++b) {
        const uint8_t *wb = w + b * 34;
        const uint8_t *xb = xq + b * 34;
        int32_t sum_i = 0;
        for (int j = 0; j < 32; ++j) sum_i += (int32_t)(int8_t)wb[2 + j] * (int32_t)(int8_t)xb[2 + j];
        float dw = tno_f16_to_f32(get_u16(wb));
        float dx = tno_f16_to_f32(get_u16(xb));
        sumf += (float)sum_i * dw * dx;
    }
    return sumf;
}

/* ---- Q4_K weights with Q8_K activations ----------------------------------
 * BlockQ4K (vendor/candle-core/src/quantized/k_quants.rs:153-159): 144 bytes
 * per 256 elements -- f16 d, f16 dmin, 12 bytes of 6-bit sub-block scales and
 * mins, 128 bytes of nibbles (qs[32c..32c+32] holds sub-block 2c in the low
 * nibbles and 2c+1 in the high ones). BlockQ8K (:185-190): f32 d, 256 int8
 * codes, 16 int16 sums of 16 codes: 292 bytes. */

static void q4k_scale_min(int j, const uint8_t *q, int *sc, int *m) {
    /* get_scale_min_k4, quantized/utils.rs:50-60 */
    if (j < 4) {
        *sc = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

void tno_q4_k_dequantize(const uint8_t *blob, float *y, int64_t n) {
    /* BlockQ4K::to_float, k_quants.rs:1722-1748: y = d*sc * q - dmin*m, each
     * product rounded to f32, then the subtraction */
    for (int64_t b = 0; b < n / 256; ++b) {
        const uint8_t *blk = blob + b * 144;
        const float d = tno_f16_to_f32(get_u16(blk)), mn = tno_f16_to_f32(get_u16(blk + 2));
        const uint8_t *sc = blk + 4, *qs = blk + 16;
        float *o = y + b * 256;
        for (int c = 0; c < 4; ++c) {
            int s0, m0, s1, m1;
            q4k_scale_min(2 * c, sc, &s0, &m0);
            q4k_scale_min(2 * c + 1, sc, &s1, &m1);
            const float d1 = d * (float)s0, mm1 = mn * (float)m0, d2 = d * (float)s1, mm2 = mn * (float)m1;
            for (int l = 0; l < 32; ++l) o[64 * c + l] = d1 * (float)(qs[32 * c + l] & 0xF) - mm1;
            for (int l = 0; l < 32; ++l) o[64 * c + 32 + l] = d2 * (float)(qs[32 * c + l] >> 4) - mm2;
        }
    }
}

static float round_half_away(float v) { return roundf(v); }

void tno_q8_k_quantize(const float *x, uint8_t *blob, int64_t n) {
    /* BlockQ8K::from_float, k_quants.rs:2376-2410: the signed value of largest
     * magnitude (first one), iscale = -127/max, q = clamp(round(iscale*x)),
     * bsums of 16, d = 1/iscale; an all-zero block is d = 0, codes 0 */
    for (int64_t b = 0; b < n / 256; ++b) {
        const float *xs = x + b * 256;
        uint8_t *blk = blob + b * 292;
        float mx = 0.0f, amax = 0.0f;
        for (int j = 0; j < 256; ++j)
            if (amax < fabsf(xs[j])) {
                amax = fabsf(xs[j]);
                mx = xs[j];
            }
        int8_t q[256];
        int16_t bs[16];
        float d = 0.0f;
        memset(q, 0, sizeof q);
        memset(bs, 0, sizeof bs);
        if (amax != 0.0f) {
            const float iscale = -127.0f / mx;
            for (int j = 0; j < 256; ++j) {
                float v = round_half_away(iscale * xs[j]);
                v = v < -128.0f ? -128.0f : (v > 127.0f ? 127.0f : v);
                q[j] = (int8_t)v;
            }
            for (int j = 0; j < 16; ++j) {
                int s = 0;
                for (int i = 0; i < 16; ++i) s += q[16 * j + i];
                bs[j] = (int16_t)s;
            }
            d = 1.0f / iscale;
        }
        memcpy(blk, &d, 4);
        memcpy(blk + 4, q, 256);
        memcpy(blk + 260, bs, 32);
    }
}

float tno_q4_k_q8_k_dot(const uint8_t *w, const uint8_t *xq, int64_t nsb) {
    /* BlockQ4K::vec_dot_unopt, k_quants.rs:1478-1544, in its order: per
     * super-block eight i32 lanes aux[l] += sc * (q8 * q4) over the elements
     * l mod 8, sums[l] += (d_w*d_x) * aux[l], sumf -= (dmin_w*d_x) * sum(bsums *
     * mins); the result is sumf + (sums[0] + ... + sums[7]). */
    float sumf = 0.0f, sums[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int64_t b = 0; b < nsb; ++b) {
        const uint8_t *wb = w + b * 144, *xb = xq + b * 292;
        const uint8_t *qs = wb + 16;
        int8_t a[256];
        for (int c = 0; c < 4; ++c)
            for (int l = 0; l < 32; ++l) {
                a[64 * c + l] = (int8_t)(qs[32 * c + l] & 0xF);
                a[64 * c + 32 + l] = (int8_t)(qs[32 * c + l] >> 4);
            }
        int sc[8], mn[8];
        for (int j = 0; j < 8; ++j) q4k_scale_min(j, wb + 4, &sc[j], &mn[j]);
        int16_t bs[16];
        memcpy(bs, xb + 260, 32);
        int32_t sumi = 0;
        for (int j = 0; j < 16; ++j) sumi += (int32_t)bs[j] * mn[j / 2];
        int32_t aux[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        const int8_t *q8 = (const int8_t *)(xb + 4);
        for (int s = 0; s < 8; ++s)
            for (int g = 0; g < 4; ++g)
                for (int l = 0; l < 8; ++l) {
                    const int e = 32 * s + 8 * g + l;
                    aux[l] += sc[s] * (int32_t)(int16_t)(q8[e] * a[e]);
                }
        float dx;
        memcpy(&dx, xb, 4);
        const float d = tno_f16_to_f32(get_u16(wb)) * dx;
        for (int l = 0; l < 8; ++l) sums[l] += d * (float)aux[l];
        const float dmin = tno_f16_to_f32(get_u16(wb + 2)) * dx;
        sumf -= dmin * (float)sumi;
    }
    float t = 0.0f;
    for (int l = 0; l < 8; ++l) t += sums[l];
    return sumf + t;
}

void tno_q4_k_linear(const float *x, const uint8_t *w_blob, const float *bias, float *y,
                     int64_t M, int64_t N, int64_t K, int threads) {
    /* the same matmul steps (k_quants.rs:2430-2580) with Q8_K activations */
    const int64_t nsb = K / 256;
    uint8_t *xq = (uint8_t *)malloc((size_t)(M * nsb * 292 + 1));
    for (int64_t r = 0; r < M; ++r) tno_q8_k_quantize(x + r * K, xq + r * nsb * 292, K);
    (void)threads;
    for (int64_t r = 0; r < M; ++r)
        for (int64_t c = 0; c < N; ++c) y[r * N + c] = tno_q4_k_q8_k_dot(w_blob + c * nsb * 144, xq + r * nsb * 292, nsb);
    free(xq);
    if (bias)
        for (int64_t r = 0; r < M; ++r)
            for (int64_t c = 0; c < N; ++c) y[r * N + c] = y[r * N + c] + bias[c];
}

/* ---- the matmul: quads of output columns split across workers ----------- */

typedef float (*dot_fn)(const uint8_t *, const uint8_t *, int64_t);

typedef struct {
    const uint8_t *xq;
    const uint8_t *w;
    float *y;
    int64_t M, N, nb;
    int64_t quad_begin, quad_end;
    dot_fn dot;
    int64_t wblock; /* bytes per weight block: 18 (Q4_0) or 34 (Q8_0) */
} lin_job;

static void *lin_worker(void *arg) {
    lin_job *j = (lin_job *)arg;
    const int64_t row_tile = 16; /* k_quants.rs:2522 ROW_TILE */
    for (int64_t r0 = 0; r0 < j->M; r0 += row_tile) {
        int64_t r1 = r0 + row_tile < j->M ? r0 + row_tile : j->M;
        for (int64_t q = j->quad_begin; q < j->quad_end; ++q) {
            for (int64_t r = r0; r < r1; ++r) {
                const uint8_t *xr = j->xq + r * j->nb * 34;
                for (int c = 0; c < 4; ++c) {
                    int64_t col = q * 4 + c;
                    j->y[r * j->N + col] = j->dot(j->w + col * j->nb * j->wblock, xr, j->nb);
                }
            }
        }
    }
    return NULL;
}

static void q_linear(const float *x, const uint8_t *w_blob, const float *bias, float *y, int64_t M, int64_t N,
                     int64_t K, int threads, dot_fn dot, int64_t wblock) {
    int64_t nb = K / 32;
    uint8_t *xq = (uint8_t *)malloc((size_t)(M * nb * 34 + 1));
    for (int64_t r = 0; r < M; ++r) tno_q8_0_quantize(x + r * K, xq + r * nb * 34, K);
    int64_t quads = N / 4;
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    int64_t per = (quads + threads - 1) / threads;
    pthread_t tid[256];
    int created[256];
    lin_job jobs[256];
    for (int t = 0; t < threads; ++t) {
        int64_t qb = t * per, qe = qb + per < quads ? qb + per : quads;
        created[t] = 0;
        if (qb >= qe) continue;
        jobs[t] = (lin_job){xq, w_blob, y, M, N, nb, qb, qe, dot, wblock};
        if (t + 1 < threads && pthread_create(&tid[t], NULL, lin_worker, &jobs[t]) == 0)
            created[t] = 1;
        else
            lin_worker(&jobs[t]);
    }
    for (int t = 0; t < threads; ++t)
        if (created[t]) pthread_join(tid[t], NULL);
    /* the column tail (k_quants.rs:2555-2575): the same dot, one column at a time */
    for (int64_t r = 0; r < M; ++r)
        for (int64_t col = quads * 4; col < N; ++col)
            y[r * N + col] = dot(w_blob + col * nb * wblock, xq + r * nb * 34, nb);
    free(xq);
    if (bias)
        for (int64_t r = 0; r < M; ++r)
            for (int64_t col = 0; col < N; ++col) y[r * N + col] = y[r * N + col] + bias[col];
}

void tno_q4_0_linear(const float *x, const uint8_t *w_blob, const float *bias, float *y,
                     int64_t M, int64_t N, int64_t K, int threads) {
    q_linear(x, w_blob, bias, y, M, N, K, threads, tno_q4_0_q8_0_dot, 18);
}

void tno_q8_0_linear(const float *x, const uint8_t *w_blob, const float *bias, float *y,
                     int64_t M, int64_t N, int64_t K, int threads) {
    q_linear(x, w_blob, bias, y, M, N, K, threads, tno_q8_0_q8_0_dot, 34);
}

/* ------------------------------------------------------------------------ */
/* scaled_dot_product_attention, sdpa_flash_cpu's default branch           */
/* (torch_c/src/aten.rs:10327-10420):                                       */
/*   scores = q k^T (f32 for f32/f16/bf16, f64 for f64)                     */
/*   causal (upper-left, aten.rs:10038-10041): key j > row i gets           */
/*     s*scale + (-inf), every other element s*scale + 0.0                 */
/*   non-causal: s*scale + 0.0 (affine(scale, 0.0))                         */
/*   + attn_mask; max; w = exp(s - max); sum; p = w / sum; out = p v        */
/*   logsumexp = log(sum) + max; out narrowed to the input dtype.           */
/* ------------------------------------------------------------------------ */

typedef struct {
    const void *q, *k, *v, *mask;
    int mask_dtype;
    const int64_t *ms, *qs, *ks, *vs;
    void *out, *lse;
    int dtype;
    int64_t B, Hq, Hkv, L, S, D;
    int causal;
    double scale;
    int64_t bh_begin, bh_end;
} sdpa_job;

static double load_elem(const void *p, int dtype, int64_t i) {
    switch (dtype) {
    case 0: return (double)((const float *)p)[i];
    case 1: return (double)tno_f16_to_f32(((const uint16_t *)p)[i]);
    case 2: return (double)tno_bf16_to_f32(((const uint16_t *)p)[i]);
    default: return ((const double *)p)[i];
    }
}

/* The key/value rows of one head, widened to the accumulate type once per
 * (b, h) so the score and output loops read contiguous memory; the
 * arithmetic and its order are unchanged (each load_elem widening is exact). */
static void widen_head(const sdpa_job *j, int64_t b, int64_t hk, float *kf, float *vf) {
    for (int64_t t = 0; t < j->S; ++t)
        for (int64_t d = 0; d < j->D; ++d) {
            kf[t * j->D + d] = (float)load_elem(j->k, j->dtype, b * j->ks[0] + hk * j->ks[1] + t * j->ks[2] + d * j->ks[3]);
            vf[t * j->D + d] = (float)load_elem(j->v, j->dtype, b * j->vs[0] + hk * j->vs[1] + t * j->vs[2] + d * j->vs[3]);
        }
}

/* A row whose every score is -inf (no key to attend) answers zeros and a
 * logsumexp of 0: upstream's CPU flash kernel and the reference's blocked
 * kernel (torch_c/src/flash.rs:758-776: row_max -inf -> 0, row_sum 0 -> 1).
 * The default branch as written would form exp(-inf - (-inf)) = NaN there. */
static void sdpa_head_f32(const sdpa_job *j, int64_t b, int64_t h, float *sc, float *kf, float *vf, float *qf,
                          float *of) {
    int64_t rep = j->Hq / j->Hkv, hk = h / rep;
    float scale = (float)j->scale; /* candle's affine casts its f64 multiplier to the dtype */
    widen_head(j, b, hk, kf, vf);
    for (int64_t i = 0; i < j->L; ++i) {
        for (int64_t d = 0; d < j->D; ++d)
            qf[d] = (float)load_elem(j->q, j->dtype, b * j->qs[0] + h * j->qs[1] + i * j->qs[2] + d * j->qs[3]);
        for (int64_t t = 0; t < j->S; ++t) {
            const float *kr = kf + t * j->D;
            float s = 0.0f;
            for (int64_t d = 0; d < j->D; ++d) s += qf[d] * kr[d];
            if (j->causal && t > i)
                s = s * scale + (-INFINITY);
            else
                s = s * scale + 0.0f;
            if (j->mask)
                s = s + (float)load_elem(j->mask, j->mask_dtype,
                                         b * j->ms[0] + h * j->ms[1] + i * j->ms[2] + t * j->ms[3]);
            sc[t] = s;
        }
        float mx = -INFINITY;
        for (int64_t t = 0; t < j->S; ++t) mx = sc[t] > mx ? sc[t] : mx;
        int64_t orow = ((b * j->Hq + h) * j->L + i) * j->D;
        float sum = 0.0f;
        if (mx == -INFINITY) {
            for (int64_t d = 0; d < j->D; ++d) of[d] = 0.0f;
        } else {
            for (int64_t t = 0; t < j->S; ++t) {
                sc[t] = expf(sc[t] - mx);
                sum += sc[t];
            }
            for (int64_t t = 0; t < j->S; ++t) sc[t] = sc[t] / sum;
            for (int64_t d = 0; d < j->D; ++d) of[d] = 0.0f;
            for (int64_t t = 0; t < j->S; ++t) {
                const float *vr = vf + t * j->D;
                for (int64_t d = 0; d < j->D; ++d) of[d] += sc[t] * vr[d];
            }
        }
        for (int64_t d = 0; d < j->D; ++d) {
            if (j->dtype == 0)
                ((float *)j->out)[orow + d] = of[d];
            else if (j->dtype == 1)
                ((uint16_t *)j->out)[orow + d] = tno_f32_to_f16(of[d]);
            else
                ((uint16_t *)j->out)[orow + d] = tno_f32_to_bf16(of[d]);
        }
        ((float *)j->lse)[(b * j->Hq + h) * j->L + i] = (mx == -INFINITY) ? 0.0f : logf(sum) + mx;
    }
}

static void sdpa_head_f64(const sdpa_job *j, int64_t b, int64_t h, double *sc, double *of) {
    int64_t rep = j->Hq / j->Hkv, hk = h / rep;
    double scale = j->scale;
    for (int64_t i = 0; i < j->L; ++i) {
        for (int64_t t = 0; t < j->S; ++t) {
            double s = 0.0;
            for (int64_t d = 0; d < j->D; ++d)
                s += load_elem(j->q, 3, b * j->qs[0] + h * j->qs[1] + i * j->qs[2] + d * j->qs[3]) *
                     load_elem(j->k, 3, b * j->ks[0] + hk * j->ks[1] + t * j->ks[2] + d * j->ks[3]);
            if (j->causal && t > i)
                s = s * scale + (-INFINITY);
            else
                s = s * scale + 0.0;
            if (j->mask)
                s = s + load_elem(j->mask, j->mask_dtype, b * j->ms[0] + h * j->ms[1] + i * j->ms[2] + t * j->ms[3]);
            sc[t] = s;
        }
        double mx = -INFINITY;
        for (int64_t t = 0; t < j->S; ++t) mx = sc[t] > mx ? sc[t] : mx;
        double sum = 0.0;
        int64_t orow = ((b * j->Hq + h) * j->L + i) * j->D;
        for (int64_t d = 0; d < j->D; ++d) of[d] = 0.0;
        if (mx != -INFINITY) {
            for (int64_t t = 0; t < j->S; ++t) {
                sc[t] = exp(sc[t] - mx);
                sum += sc[t];
            }
            for (int64_t t = 0; t < j->S; ++t) sc[t] = sc[t] / sum;
            for (int64_t t = 0; t < j->S; ++t)
                for (int64_t d = 0; d < j->D; ++d)
                    of[d] += sc[t] * load_elem(j->v, 3, b * j->vs[0] + hk * j->vs[1] + t * j->vs[2] + d * j->vs[3]);
        }
        for (int64_t d = 0; d < j->D; ++d) ((double *)j->out)[orow + d] = of[d];
        ((double *)j->lse)[(b * j->Hq + h) * j->L + i] = (mx == -INFINITY) ? 0.0 : log(sum) + mx;
    }
}

static void *sdpa_worker(void *arg) {
    sdpa_job *j = (sdpa_job *)arg;
    const size_t S1 = (size_t)(j->S > 0 ? j->S : 1), D1 = (size_t)(j->D > 0 ? j->D : 1);
    void *sc = malloc(S1 * 8);
    double *of64 = (double *)malloc(D1 * 8);
    float *kf = NULL, *vf = NULL, *qf = (float *)malloc(D1 * 4), *of = (float *)malloc(D1 * 4);
    if (j->dtype != 3) {
        kf = (float *)malloc(S1 * D1 * 4);
        vf = (float *)malloc(S1 * D1 * 4);
    }
    for (int64_t bh = j->bh_begin; bh < j->bh_end; ++bh) {
        int64_t b = bh / j->Hq, h = bh % j->Hq;
        if (j->dtype == 3)
            sdpa_head_f64(j, b, h, (double *)sc, of64);
        else
            sdpa_head_f32(j, b, h, (float *)sc, kf, vf, qf, of);
    }
    free(sc);
    free(of64);
    free(kf);
    free(vf);
    free(qf);
    free(of);
    return NULL;
}

void tno_sdpa(const void *q, const void *k, const void *v, const void *mask, int mask_dtype,
              const int64_t *mask_strides, void *out, void *lse, int dtype, int64_t B, int64_t Hq,
              int64_t Hkv, int64_t L, int64_t S, int64_t D, const int64_t *q_strides,
              const int64_t *k_strides, const int64_t *v_strides, int is_causal, double scale,
              int threads) {
    static const int64_t zero[4] = {0, 0, 0, 0};
    int64_t total = B * Hq;
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    if (threads > total) threads = (int)(total > 0 ? total : 1);
    int64_t per = (total + threads - 1) / threads;
    pthread_t tid[256];
    int created[256];
    sdpa_job jobs[256];
    for (int t = 0; t < threads; ++t) {
        created[t] = 0;
        int64_t b0 = t * per, b1 = b0 + per < total ? b0 + per : total;
        if (b0 >= b1) continue;
        jobs[t] = (sdpa_job){q, k, v, mask, mask_dtype, mask_strides ? mask_strides : zero,
                             q_strides, k_strides, v_strides, out, lse, dtype, B, Hq, Hkv, L, S, D,
                             is_causal, scale, b0, b1};
        if (t + 1 < threads && pthread_create(&tid[t], NULL, sdpa_worker, &jobs[t]) == 0)
            created[t] = 1;
        else
            sdpa_worker(&jobs[t]);
    }
    for (int t = 0; t < threads; ++t)
        if (created[t]) pthread_join(tid[t], NULL);
}
