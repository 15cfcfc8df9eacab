/*
 * mimoracle.c -- CPU restatement of mimir-model's quantized decode path.
 *
 * TEST INFRASTRUCTURE, NOT PRODUCT: the checker for the GPU library and the
 * timed CPU baseline.  See mimoracle.h for the contract and the rule that
 * only tests, smoke() and bench.py's CPU legs may use it.
 *
 * Compile with -ffp-contract=off (the Makefile does): every a*b+c below is
 * two roundings unless written as fmaf().
 */
#include "mimoracle.h"

#include <math.h>
#include <stdint.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ */
/* small helpers                                                        */
/* ------------------------------------------------------------------ */

static inline uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint16_t le16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static inline void put16(uint8_t *p, uint16_t v) { p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); }

typedef void (*range_fn)(void *ctx, int64_t lo, int64_t hi);
typedef struct { range_fn fn; void *ctx; int64_t lo, hi; } range_job;

/* A persistent pool of worker threads, like the reference's worker pool
 * (interp/pool.go): created on first use, each product wakes them with a
 * new generation of jobs instead of creating threads.  One product uses the
 * pool at a time (pool_mu); no job calls parallel_for itself. */
#define POOL_MAX 256
static pthread_mutex_t pool_mu = PTHREAD_MUTEX_INITIALIZER;
static pthread_mutex_t pool_lk = PTHREAD_MUTEX_INITIALIZER;
static pthread_cond_t pool_go = PTHREAD_COND_INITIALIZER, pool_done = PTHREAD_COND_INITIALIZER;
static int pool_n = 0;              /* workers created (ids 1..pool_n) */
static unsigned long pool_gen = 0;  /* generation of the jobs in pool_jobs */
static int pool_active = 0;         /* jobs of this generation (job 0 is the caller's) */
static int pool_pending = 0;        /* worker jobs of this generation not finished */
static range_job pool_jobs[POOL_MAX];

static void *pool_worker(void *arg) {
    const int id = (int)(intptr_t)arg;
    unsigned long seen = 0;
    pthread_mutex_lock(&pool_lk);
    for (;;) {
        while (pool_gen == seen) pthread_cond_wait(&pool_go, &pool_lk);
        seen = pool_gen;
        /* a generation's workers all finish it before the next one starts */
        if (id < pool_active) {
            const range_job j = pool_jobs[id];
            pthread_mutex_unlock(&pool_lk);
            if (j.lo < j.hi) j.fn(j.ctx, j.lo, j.hi);
            pthread_mutex_lock(&pool_lk);
            if (--pool_pending == 0) pthread_cond_signal(&pool_done);
        }
    }
    return NULL;
}

/* A forked child has none of the workers: it starts with an empty pool (the
 * locks are held across the fork, so none is left locked by a thread the
 * child does not have). */
static void pool_prefork(void) {
    pthread_mutex_lock(&pool_mu);
    pthread_mutex_lock(&pool_lk);
}
static void pool_postfork_parent(void) {
    pthread_mutex_unlock(&pool_lk);
    pthread_mutex_unlock(&pool_mu);
}
static void pool_postfork_child(void) {
    pool_n = 0;
    pool_active = pool_pending = 0;
    pthread_cond_init(&pool_go, NULL);
    pthread_cond_init(&pool_done, NULL);
    pthread_mutex_unlock(&pool_lk);
    pthread_mutex_unlock(&pool_mu);
}
static pthread_once_t pool_once = PTHREAD_ONCE_INIT;
static void pool_register(void) { pthread_atfork(pool_prefork, pool_postfork_parent, pool_postfork_child); }

/* Runs fn over [0, n) split into nthreads contiguous pieces, like the
 * reference's parallel() over output rows (interp/pool.go:33-66). */
static void parallel_for(int64_t n, int nthreads, range_fn fn, void *ctx) {
    if (nthreads > POOL_MAX) nthreads = POOL_MAX;
    if (nthreads > n) nthreads = (int)n;
    if (nthreads <= 1) { fn(ctx, 0, n); return; }
    pthread_once(&pool_once, pool_register);
    pthread_mutex_lock(&pool_mu);
    pthread_mutex_lock(&pool_lk);
    while (pool_n < nthreads - 1) {
        pthread_t th;
        if (pthread_create(&th, NULL, pool_worker, (void *)(intptr_t)(pool_n + 1)) != 0) break;
        pthread_detach(th);
        pool_n++;
    }
    const int use = pool_n + 1 < nthreads ? pool_n + 1 : nthreads;
    const int64_t per = (n + use - 1) / use;
    for (int t = 0; t < use; t++) {
        const int64_t lo = t * per < n ? t * per : n, hi = lo + per < n ? lo + per : n;
        pool_jobs[t] = (range_job){fn, ctx, lo, hi};
    }
    const range_job mine = pool_jobs[0];
    pool_active = use;
    pool_pending = use - 1;
    if (pool_pending > 0) {
        pool_gen++;
        pthread_cond_broadcast(&pool_go);
    }
    pthread_mutex_unlock(&pool_lk);
    if (mine.lo < mine.hi) fn(ctx, mine.lo, mine.hi);
    pthread_mutex_lock(&pool_lk);
    while (pool_pending > 0) pthread_cond_wait(&pool_done, &pool_lk);
    pthread_mutex_unlock(&pool_lk);
    pthread_mutex_unlock(&pool_mu);
}

/* ------------------------------------------------------------------ */
/* f16 <-> f32, float.go:24-88                                          */
/* ------------------------------------------------------------------ */

float mo_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000) << 16;
    uint32_t exp = (h >> 10) & 0x1F, mant = h & 0x3FF;
    if (exp == 0) {
        if (mant == 0) return bits_f32(sign);
        /* subnormal: mant * 2^-24, renormalised */
        uint32_t e = 127 - 15 + 1;
        while ((mant & 0x400) == 0) { mant <<= 1; e--; }
        return bits_f32(sign | (e << 23) | ((mant & 0x3FF) << 13));
    }
    if (exp == 0x1F) return bits_f32(sign | 0x7F800000u | (mant << 13));
    return bits_f32(sign | ((exp + 127 - 15) << 23) | (mant << 13));
}

uint16_t mo_f32_to_f16(float f) {
    uint32_t b = f32_bits(f);
    uint16_t sign = (uint16_t)((b >> 16) & 0x8000);
    int32_t exp = (int32_t)((b >> 23) & 0xFF);
    uint32_t mant = b & 0x7FFFFF;
    if (exp == 0xFF) {
        if (mant == 0) return sign | 0x7C00;
        return (uint16_t)(sign | 0x7E00 | (mant >> 13)); /* quiet NaN, top payload kept */
    }
    int32_t e = exp - 127 + 15;
    if (e >= 0x1F) return sign | 0x7C00;
    if (e <= 0) {
        if (e < -11) return sign;
        mant |= 0x800000;
        uint32_t shift = (uint32_t)(14 - e);
        uint32_t half = 1u << (shift - 1);
        uint32_t rem = mant & ((half << 1) - 1);
        uint32_t q = mant >> shift;
        if (rem > half || (rem == half && (q & 1))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t q = ((uint32_t)e << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1FFF;
    if (rem > 0x1000 || (rem == 0x1000 && (q & 1))) q++;
    return (uint16_t)(sign | q);
}

void mo_cast_f16(const float *x, uint16_t *y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = mo_f32_to_f16(x[i]);
}

/* ------------------------------------------------------------------ */
/* sizes, dtype.go:48-129                                               */
/* ------------------------------------------------------------------ */

int64_t mo_row_bytes(int dt, int64_t k) {
    switch (dt) {
    case MO_F32: return 4 * k;
    case MO_F16: return 2 * k;
    case MO_Q8_0: return k % 32 ? 0 : k / 32 * 34;
    case MO_Q4_K: return k % 256 ? 0 : k / 256 * 144;
    case MO_Q6_K: return k % 256 ? 0 : k / 256 * 210;
    }
    return 0;
}

/* ------------------------------------------------------------------ */
/* decoders, quant.go:197-344                                           */
/* ------------------------------------------------------------------ */

/* Q8_0: y = d*q, quant.go:197-206 */
static void deq_q8_0(const uint8_t *src, float *dst, int64_t nb) {
    for (int64_t b = 0; b < nb; b++) {
        const uint8_t *blk = src + 34 * b;
        float d = mo_f16_to_f32(le16(blk));
        for (int j = 0; j < 32; j++) dst[32 * b + j] = d * (float)(int8_t)blk[2 + j];
    }
}

/* getScaleMinK4, quant.go:246-254 */
static inline void scale_min_k4(int j, const uint8_t *q, uint8_t *sc, uint8_t *m) {
    if (j < 4) { *sc = q[j] & 63; *m = q[j + 4] & 63; return; }
    *sc = (uint8_t)((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
    *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
}

/* Q4_K: y = (d*sc)*n - dmin*m, each product rounded, quant.go:260-289 */
static void deq_q4_k(const uint8_t *src, float *dst, int64_t nb) {
    for (int64_t b = 0; b < nb; b++) {
        const uint8_t *blk = src + 144 * b;
        float d = mo_f16_to_f32(le16(blk)), dmin = mo_f16_to_f32(le16(blk + 2));
        const uint8_t *scales = blk + 4, *q = blk + 16;
        float *y = dst + 256 * b;
        for (int c = 0; c < 4; c++) {
            uint8_t sc, m;
            scale_min_k4(2 * c, scales, &sc, &m);
            float d1 = d * (float)sc, m1 = dmin * (float)m;
            scale_min_k4(2 * c + 1, scales, &sc, &m);
            float d2 = d * (float)sc, m2 = dmin * (float)m;
            for (int l = 0; l < 32; l++) y[64 * c + l] = d1 * (float)(q[32 * c + l] & 0xF) - m1;
            for (int l = 0; l < 32; l++) y[64 * c + 32 + l] = d2 * (float)(q[32 * c + l] >> 4) - m2;
        }
    }
}

/* Q6_K: y = (d*sc)*(q-32), quant.go:294-321 */
static void deq_q6_k(const uint8_t *src, float *dst, int64_t nb) {
    for (int64_t b = 0; b < nb; b++) {
        const uint8_t *blk = src + 210 * b;
        float d = mo_f16_to_f32(le16(blk + 208));
        for (int h = 0; h < 2; h++) {
            const uint8_t *ql = blk + 64 * h, *qh = blk + 128 + 32 * h;
            const int8_t *sc = (const int8_t *)(blk + 192 + 8 * h);
            float *y = dst + 256 * b + 128 * h;
            for (int l = 0; l < 32; l++) {
                int is = l / 16;
                int q1 = (int)((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
                int q2 = (int)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                int q3 = (int)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                int q4 = (int)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                y[l] = (d * (float)sc[is + 0]) * (float)q1;
                y[l + 32] = (d * (float)sc[is + 2]) * (float)q2;
                y[l + 64] = (d * (float)sc[is + 4]) * (float)q3;
                y[l + 96] = (d * (float)sc[is + 6]) * (float)q4;
            }
        }
    }
}

int mo_dequantize(int dt, const uint8_t *src, float *dst, int64_t n) {
    switch (dt) {
    case MO_F32: memcpy(dst, src, 4 * (size_t)n); return 0;
    case MO_F16:
        for (int64_t i = 0; i < n; i++) dst[i] = mo_f16_to_f32(le16(src + 2 * i));
        return 0;
    case MO_Q8_0: if (n % 32) return -1; deq_q8_0(src, dst, n / 32); return 0;
    case MO_Q4_K: if (n % 256) return -1; deq_q4_k(src, dst, n / 256); return 0;
    case MO_Q6_K: if (n % 256) return -1; deq_q6_k(src, dst, n / 256); return 0;
    }
    return -1;
}

/* ------------------------------------------------------------------ */
/* encoders                                                             */
/* ------------------------------------------------------------------ */

/* quantizeQ8_0, quant.go:208-228 (roundf: half away from zero) */
void mo_quantize_q8_0(const float *x, uint8_t *dst, int64_t n) {
    for (int64_t b = 0; b < n / 32; b++) {
        const float *xb = x + 32 * b;
        float amax = 0;
        for (int j = 0; j < 32; j++) { float a = fabsf(xb[j]); if (a > amax) amax = a; }
        float d = amax / 127.0f, id = d != 0 ? 1.0f / d : 0.0f;
        uint8_t *blk = dst + 34 * b;
        put16(blk, mo_f32_to_f16(d));
        for (int j = 0; j < 32; j++) blk[2 + j] = (uint8_t)(int8_t)roundf(xb[j] * id);
    }
}

static inline float f16_round(float f) { return mo_f16_to_f32(mo_f32_to_f16(f)); }
static inline int clampi(int v, int lo, int hi) { return v < lo ? lo : v > hi ? hi : v; }

/* Q4_K encoder (this project's own; min/max fit per sub-block of 32).
 * Sub-block j covers [-dmin*m_j, d*sc_j*15 - dmin*m_j]; d and dmin are the
 * largest sub-block step and offset over 63, rounded to f16; sc, m are
 * 6-bit; quants are the nearest of 0..15 under the decoded step. */
static void enc_q4_k_block(const float *x, uint8_t *blk) {
    float step[8], off[8], maxstep = 0, maxoff = 0;
    for (int j = 0; j < 8; j++) {
        float lo = 0, hi = 0;
        for (int i = 0; i < 32; i++) {
            float v = x[32 * j + i];
            if (v < lo) lo = v;
            if (v > hi) hi = v;
        }
        step[j] = (hi - lo) / 15.0f;
        off[j] = -lo;
        if (step[j] > maxstep) maxstep = step[j];
        if (off[j] > maxoff) maxoff = off[j];
    }
    float d = f16_round(maxstep / 63.0f), dmin = f16_round(maxoff / 63.0f);
    uint8_t sc[8], m[8];
    for (int j = 0; j < 8; j++) {
        sc[j] = (uint8_t)(d > 0 ? clampi((int)lrintf(step[j] / d), 0, 63) : 0);
        m[j] = (uint8_t)(dmin > 0 ? clampi((int)lrintf(off[j] / dmin), 0, 63) : 0);
    }
    memset(blk, 0, 144);
    put16(blk, mo_f32_to_f16(d));
    put16(blk + 2, mo_f32_to_f16(dmin));
    uint8_t *s = blk + 4;
    for (int j = 0; j < 4; j++) {
        s[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
        s[j + 4] = (uint8_t)((m[j] & 63) | ((m[j + 4] >> 4) << 6));
        s[j + 8] = (uint8_t)((sc[j + 4] & 0xF) | ((m[j + 4] & 0xF) << 4));
    }
    uint8_t q[256];
    for (int j = 0; j < 8; j++) {
        float ds = d * (float)sc[j], dm = dmin * (float)m[j];
        for (int i = 0; i < 32; i++)
            q[32 * j + i] = (uint8_t)(ds > 0 ? clampi((int)lrintf((x[32 * j + i] + dm) / ds), 0, 15) : 0);
    }
    for (int c = 0; c < 4; c++)
        for (int l = 0; l < 32; l++)
            blk[16 + 32 * c + l] = (uint8_t)(q[64 * c + l] | (q[64 * c + 32 + l] << 4));
}

void mo_quantize_q4_k(const float *x, uint8_t *dst, int64_t n) {
    for (int64_t b = 0; b < n / 256; b++) enc_q4_k_block(x + 256 * b, dst + 144 * b);
}

/* Q6_K encoder (this project's own).  Group g of 16 elements uses scale
 * sc[g]: the element of largest magnitude maps to -32, the scales are
 * 8-bit signed under one f16 d. */
static void enc_q6_k_block(const float *x, uint8_t *blk) {
    float gs[16], maxs = 0;
    for (int g = 0; g < 16; g++) {
        float vmax = 0, amax = 0;
        for (int i = 0; i < 16; i++) {
            float v = x[16 * g + i];
            if (fabsf(v) > amax) { amax = fabsf(v); vmax = v; }
        }
        gs[g] = vmax / -32.0f;
        if (fabsf(gs[g]) > maxs) maxs = fabsf(gs[g]);
    }
    float d = f16_round(maxs / 127.0f);
    int8_t sc[16];
    for (int g = 0; g < 16; g++) sc[g] = (int8_t)(d > 0 ? clampi((int)lrintf(gs[g] / d), -128, 127) : 0);
    uint8_t q[256];
    for (int g = 0; g < 16; g++) {
        float ds = d * (float)sc[g];
        for (int i = 0; i < 16; i++)
            q[16 * g + i] = (uint8_t)(ds != 0 ? clampi((int)lrintf(x[16 * g + i] / ds), -32, 31) + 32 : 32);
    }
    memset(blk, 0, 210);
    for (int h = 0; h < 2; h++) {
        uint8_t *ql = blk + 64 * h, *qh = blk + 128 + 32 * h;
        const uint8_t *y = q + 128 * h;
        for (int l = 0; l < 32; l++) {
            uint8_t q1 = y[l], q2 = y[l + 32], q3 = y[l + 64], q4 = y[l + 96];
            ql[l] = (uint8_t)((q1 & 0xF) | ((q3 & 0xF) << 4));
            ql[l + 32] = (uint8_t)((q2 & 0xF) | ((q4 & 0xF) << 4));
            qh[l] = (uint8_t)((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
        }
    }
    memcpy(blk + 192, sc, 16);
    put16(blk + 208, mo_f32_to_f16(d));
}

void mo_quantize_q6_k(const float *x, uint8_t *dst, int64_t n) {
    for (int64_t b = 0; b < n / 256; b++) enc_q6_k_block(x + 256 * b, dst + 210 * b);
}

int mo_quantize(int dt, const float *x, uint8_t *dst, int64_t n) {
    switch (dt) {
    case MO_Q8_0: if (n % 32) return -1; mo_quantize_q8_0(x, dst, n); return 0;
    case MO_Q4_K: if (n % 256) return -1; mo_quantize_q4_k(x, dst, n); return 0;
    case MO_Q6_K: if (n % 256) return -1; mo_quantize_q6_k(x, dst, n); return 0;
    case MO_F32: memcpy(dst, x, 4 * (size_t)n); return 0;
    case MO_F16: for (int64_t i = 0; i < n; i++) put16(dst + 2 * i, mo_f32_to_f16(x[i])); return 0;
    }
    return -1;
}

/* ---- seeded synthetic values ---- */

static inline uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* Element i of stream `seed`: Box-Muller on two 53-bit uniforms. */
static inline double normal_at(uint64_t seed, uint64_t i) {
    uint64_t a = mix64(seed ^ mix64(2 * i)), b = mix64(seed ^ mix64(2 * i + 1));
    double u1 = ((double)(a >> 11) + 1.0) * 0x1p-53; /* (0, 1] */
    double u2 = (double)(b >> 11) * 0x1p-53;         /* [0, 1) */
    return sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
}

void mo_gen_normal(uint64_t seed, int64_t n, float mean, float sigma, float *x) {
    for (int64_t i = 0; i < n; i++) x[i] = (float)(mean + sigma * normal_at(seed, (uint64_t)i));
}

typedef struct { int dt; uint64_t seed; int64_t k, row0; float sigma; uint8_t *dst; } gen_ctx;

static void gen_rows(void *p, int64_t lo, int64_t hi) {
    gen_ctx *c = (gen_ctx *)p;
    float *row = (float *)malloc(sizeof(float) * (size_t)c->k);
    int64_t rb = mo_row_bytes(c->dt, c->k);
    for (int64_t r = lo; r < hi; r++) {
        const int64_t g = c->row0 + r; /* the row of the whole tensor */
        for (int64_t i = 0; i < c->k; i++) row[i] = (float)(c->sigma * normal_at(c->seed, (uint64_t)(g * c->k + i)));
        mo_quantize(c->dt, row, c->dst + r * rb, c->k);
    }
    free(row);
}

int mo_gen_weight_rows(int dt, uint64_t seed, int64_t row0, int64_t n, int64_t k, float sigma, uint8_t *dst,
                       int nthreads) {
    if (mo_row_bytes(dt, k) == 0 || row0 < 0) return -1;
    gen_ctx c = {dt, seed, k, row0, sigma, dst};
    parallel_for(n, nthreads, gen_rows, &c);
    return 0;
}

int mo_gen_weight(int dt, uint64_t seed, int64_t n, int64_t k, float sigma, uint8_t *dst, int nthreads) {
    return mo_gen_weight_rows(dt, seed, 0, n, k, sigma, dst, nthreads);
}

/* ------------------------------------------------------------------ */
/* 8-bit activations, internal/kernels/q8.go:50-97, 237-273             */
/* ------------------------------------------------------------------ */

int mo_q8_quantize(const float *x, int64_t k, int block, int8_t *q, float *d32, int16_t *xs, int16_t *m32) {
    if (k == 0 || (block != 32 && block != 256) || k % block) return 0;
    for (int64_t b = 0; b < k / block; b++) {
        const float *xb = x + block * b;
        int8_t *qb = q + block * b;
        /* amaxQ8Go: refuse NaN and |x| > 2^60 */
        float amax = 0;
        for (int i = 0; i < block; i++) {
            float a = bits_f32(f32_bits(xb[i]) & 0x7FFFFFFFu);
            if (!(a <= 0x1p60f)) return 0;
            if (a > amax) amax = a;
        }
        if (amax == 0) memset(qb, 0, (size_t)block);
        else
            for (int i = 0; i < block; i++) /* quantQ8Go: RoundToEven in float64 */
                qb[i] = (int8_t)rint(127.0 * (double)xb[i] / (double)amax);
        for (int r = 0; r < block / 32; r++) {
            int16_t s = 0;
            for (int i = 0; i < 32; i++) s = (int16_t)(s + qb[32 * r + i]);
            if (xs) xs[block * b / 32 + r] = s;
        }
        if (m32)
            for (int i = 0; i < block / 2; i++)
                m32[block * b / 2 + i] = (int16_t)(32 * ((int16_t)qb[2 * i] + (int16_t)qb[2 * i + 1]));
        float d = amax / 127.0f;
        for (int r = 0; r < block / 32; r++) d32[block * b / 32 + r] = d;
    }
    return 1;
}

static inline int f16_finite(const uint8_t *p) { return (le16(p) & 0x7C00) != 0x7C00; }

/* The block sums of dotQ8KRef are exact integers, so any summation order
 * gives the same S: besides the scalar loops below (the checker) the block
 * sums have an AVX2 form, as the reference computes them on amd64
 * (dotQ4KQ8KAVX2 / dotQ6KQ8KAVX2, internal/kernels/kernels_amd64.s:
 * 1045-1510): VPMADDUBSW of the unsigned quants with the int8 activations
 * (no saturation for these ranges: |pair| <= 15*127*2 for Q4_K, 63*127*2
 * for Q6_K), VPMADDWD with the sub-block scales, int32 lanes summed at the
 * end.  mo_set_simd(0) selects the scalar loops. */
static int g_simd = 1;

void mo_set_simd(int on) { g_simd = on != 0; }

int mo_simd_active(void) {
#if defined(__AVX2__)
    return g_simd;
#else
    return 0;
#endif
}

#if defined(__AVX2__)
#include <immintrin.h>

static inline int32_t hsum_i32x8(__m256i v) {
    __m128i s = _mm_add_epi32(_mm256_castsi256_si128(v), _mm256_extracti128_si256(v, 1));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0x4E));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0xB1));
    return _mm_cvtsi128_si32(s);
}

/* S = sum_c sc[2c] * sum(lo nibbles of qs[32c..] * y[64c..]) + sc[2c+1] * sum(hi * y[64c+32..]) */
static int32_t q4k_block_s_avx2(const uint8_t *qs, const int8_t *y, const int32_t sc[8]) {
    const __m256i m4 = _mm256_set1_epi8(0x0F);
    __m256i acc = _mm256_setzero_si256();
    for (int c = 0; c < 4; c++) {
        const __m256i v = _mm256_loadu_si256((const __m256i *)(qs + 32 * c));
        const __m256i lo = _mm256_and_si256(v, m4);
        const __m256i hi = _mm256_and_si256(_mm256_srli_epi16(v, 4), m4);
        const __m256i p0 = _mm256_maddubs_epi16(lo, _mm256_loadu_si256((const __m256i *)(y + 64 * c)));
        const __m256i p1 = _mm256_maddubs_epi16(hi, _mm256_loadu_si256((const __m256i *)(y + 64 * c + 32)));
        acc = _mm256_add_epi32(acc, _mm256_madd_epi16(p0, _mm256_set1_epi16((short)sc[2 * c])));
        acc = _mm256_add_epi32(acc, _mm256_madd_epi16(p1, _mm256_set1_epi16((short)sc[2 * c + 1])));
    }
    return hsum_i32x8(acc);
}

/* S of a Q6_K block: per half h, per quarter k of 32 elements, the 6-bit
 * quants r (q = r - 32) times y, scales sc[8h + 2k + (l >= 16)]. */
static int32_t q6k_block_s_avx2(const uint8_t *blk, const int8_t *y) {
    const __m256i m4 = _mm256_set1_epi8(0x0F), m2 = _mm256_set1_epi8(0x03), c32 = _mm256_set1_epi8(32);
    __m256i acc = _mm256_setzero_si256();
    for (int h = 0; h < 2; h++) {
        const uint8_t *ql = blk + 64 * h, *qh = blk + 128 + 32 * h;
        const int8_t *sc = (const int8_t *)(blk + 192 + 8 * h);
        const int8_t *yh = y + 128 * h;
        const __m256i la = _mm256_loadu_si256((const __m256i *)ql);
        const __m256i lb = _mm256_loadu_si256((const __m256i *)(ql + 32));
        const __m256i hv = _mm256_loadu_si256((const __m256i *)qh);
        __m256i r[4];
        r[0] = _mm256_or_si256(_mm256_and_si256(la, m4), _mm256_slli_epi16(_mm256_and_si256(hv, m2), 4));
        r[1] = _mm256_or_si256(_mm256_and_si256(lb, m4),
                               _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(hv, 2), m2), 4));
        r[2] = _mm256_or_si256(_mm256_and_si256(_mm256_srli_epi16(la, 4), m4),
                               _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(hv, 4), m2), 4));
        r[3] = _mm256_or_si256(_mm256_and_si256(_mm256_srli_epi16(lb, 4), m4),
                               _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(hv, 6), m2), 4));
        for (int k = 0; k < 4; k++) {
            const __m256i yk = _mm256_loadu_si256((const __m256i *)(yh + 32 * k));
            /* (r - 32) y in pairs: r y - 32 y, each term within int16 */
            const __m256i pk = _mm256_sub_epi16(_mm256_maddubs_epi16(r[k], yk), _mm256_maddubs_epi16(c32, yk));
            const __m256i s16 = _mm256_set_m128i(_mm_set1_epi16(sc[2 * k + 1]), _mm_set1_epi16(sc[2 * k]));
            acc = _mm256_add_epi32(acc, _mm256_madd_epi16(pk, s16));
        }
    }
    return hsum_i32x8(acc);
}
#endif

int mo_dot_q8k_ref(int dt, const uint8_t *row, const int8_t *q, const float *d32, const int16_t *xs, int64_t k,
                   float *out) {
    float tot = 0, off = 0;
    for (int64_t b = 0; b < k / 256; b++) {
        const int8_t *y = q + 256 * b;
        float dx = d32[8 * b];
        if (dt == MO_Q4_K) {
            const uint8_t *blk = row + 144 * b;
            if (!f16_finite(blk) || !f16_finite(blk + 2)) return 0;
            float d = mo_f16_to_f32(le16(blk)), dmin = mo_f16_to_f32(le16(blk + 2));
            int32_t sc[8], m[8];
            const uint8_t *s = blk + 4;
            for (int j = 0; j < 4; j++) {
                sc[j] = s[j] & 63;
                m[j] = s[j + 4] & 63;
                sc[4 + j] = (s[j + 8] & 0xF) | ((s[j] >> 6) << 4);
                m[4 + j] = (s[j + 8] >> 4) | ((s[j + 4] >> 6) << 4);
            }
            int32_t S = 0, M = 0;
#if defined(__AVX2__)
            if (g_simd) {
                S = q4k_block_s_avx2(blk + 16, y, sc);
            } else
#endif
            for (int c = 0; c < 4; c++) {
                int32_t lo = 0, hi = 0;
                for (int i = 0; i < 32; i++) {
                    uint8_t v = blk[16 + 32 * c + i];
                    lo += (int32_t)(v & 15) * y[64 * c + i];
                    hi += (int32_t)(v >> 4) * y[64 * c + 32 + i];
                }
                S += sc[2 * c] * lo + sc[2 * c + 1] * hi;
            }
            for (int j = 0; j < 8; j++) M += m[j] * (int32_t)xs[8 * b + j];
            tot = fmaf((float)S, d * dx, tot);
            off = fmaf((float)M, dmin * dx, off);
            continue;
        }
        const uint8_t *blk = row + 210 * b;
        if (!f16_finite(blk + 208)) return 0;
        float d = mo_f16_to_f32(le16(blk + 208));
        int32_t S = 0;
#if defined(__AVX2__)
        if (g_simd) {
            tot = fmaf((float)q6k_block_s_avx2(blk, y), d * dx, tot);
            continue;
        }
#endif
        for (int h = 0; h < 2; h++) {
            const uint8_t *ql = blk + 64 * h, *qh = blk + 128 + 32 * h;
            const int8_t *sc = (const int8_t *)(blk + 192 + 8 * h);
            const int8_t *yh = y + 128 * h;
            for (int l = 0; l < 32; l++) {
                int is = l / 16;
                int32_t q1 = (int32_t)((ql[l] & 0xF) | ((qh[l] & 3) << 4)) - 32;
                int32_t q2 = (int32_t)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                int32_t q3 = (int32_t)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                int32_t q4 = (int32_t)((ql[l + 32] >> 4) | ((qh[l] >> 6) << 4)) - 32;
                S += sc[is] * q1 * yh[l] + sc[is + 2] * q2 * yh[l + 32] + sc[is + 4] * q3 * yh[l + 64] +
                     sc[is + 6] * q4 * yh[l + 96];
            }
        }
        tot = fmaf((float)S, d * dx, tot);
    }
    *out = tot - off;
    return 1;
}

/* The block-32 kernels (dequant_matmul_a8.v1) exist only as AVX2 assembly in
 * the reference; their float operations are restated here lane by lane.  A
 * vector register is 8 f32 lanes; each lane's integer value is exact in
 * int32 (VPMADDUBSW/VPMADDWD cannot saturate for these operand ranges:
 * |nibble*q| pairs <= 3810, |q6*q| pairs <= 16002, |w8*q| pairs <= 32512 with
 * q in [-127, 127]), so a lane is the plain integer sum over its 4 elements.
 *
 * HSUM1, internal/kernels/kernels_amd64.s:408-413: VEXTRACTF128 + VADDPS give
 * a_i = v_i + v_{i+4}; two VHADDPS give (a0 + a1) + (a2 + a3). */
static float hsum1(const float v[8]) {
    float a0 = v[0] + v[4], a1 = v[1] + v[5], a2 = v[2] + v[6], a3 = v[3] + v[7];
    return (a0 + a1) + (a2 + a3);
}

/* dotQ4KQ8AVX2, internal/kernels/kernels_amd64.s:441-562.  Per block: the
 * offsets lane s (sub-block s) gets fma(f32(dmin*m_s), dbs_s, Y3_s) with
 * dbs_s = f32(dx_s * xs_s) (q8.go:93-96); chunk c = sub-blocks 2c and 2c+1,
 * lane j = elements 4j..4j+3 of each: Y0_j = fma(dx_2c, sc_2c * S_lo, Y0_j),
 * Y1_j = fma(dx_2c+1, sc_2c+1 * S_hi, Y1_j); then Y2 = fma(d, Y0 + Y1, Y2).
 * The row's value is HSUM1(Y2 - Y3). */
static int dot_q4k_q8_b32(const uint8_t *row, const int8_t *q, const float *d32, const int16_t *xs, int64_t nb,
                          float *out) {
    float y2[8] = {0}, y3[8] = {0};
    for (int64_t b = 0; b < nb; b++) {
        const uint8_t *blk = row + 144 * b;
        const int8_t *y = q + 256 * b;
        const float *dx = d32 + 8 * b;
        if (!f16_finite(blk) || !f16_finite(blk + 2)) return 0;
        float d = mo_f16_to_f32(le16(blk)), dmin = mo_f16_to_f32(le16(blk + 2));
        int32_t sc[8], m[8];
        const uint8_t *s = blk + 4;
        for (int j = 0; j < 4; j++) {
            sc[j] = s[j] & 63;
            m[j] = s[j + 4] & 63;
            sc[4 + j] = (s[j + 8] & 0xF) | ((s[j] >> 6) << 4);
            m[4 + j] = (s[j + 8] >> 4) | ((s[j + 4] >> 6) << 4);
        }
        for (int l = 0; l < 8; l++) {
            float dm = dmin * (float)m[l];
            float dbs = dx[l] * (float)xs[8 * b + l];
            y3[l] = fmaf(dm, dbs, y3[l]);
        }
        float y0[8] = {0}, y1[8] = {0};
        for (int c = 0; c < 4; c++)
            for (int l = 0; l < 8; l++) {
                int32_t lo = 0, hi = 0;
                for (int e = 4 * l; e < 4 * l + 4; e++) {
                    uint8_t v = blk[16 + 32 * c + e];
                    lo += (int32_t)(v & 15) * y[64 * c + e];
                    hi += (int32_t)(v >> 4) * y[64 * c + 32 + e];
                }
                y0[l] = fmaf(dx[2 * c], (float)(sc[2 * c] * lo), y0[l]);
                y1[l] = fmaf(dx[2 * c + 1], (float)(sc[2 * c + 1] * hi), y1[l]);
            }
        for (int l = 0; l < 8; l++) y2[l] = fmaf(d, y0[l] + y1[l], y2[l]);
    }
    float v[8];
    for (int l = 0; l < 8; l++) v[l] = y2[l] - y3[l];
    *out = hsum1(v);
    return 1;
}

/* dotQ6KQ8AVX2, internal/kernels/kernels_amd64.s:763-853.  Per half h and
 * quarter j (32 elements), lane l = elements 4l..4l+3 with the scale
 * sc[8h + 2j + (l >= 4)] (the q6scales shuffle masks): the lane value is
 * sc * sum (q6 - 32) * y (VPMADDUBSW, then VPSUBW of the m32 pair sums), and
 * acc_l = fma(dx_{4h+j}, value, acc_l) with acc = Y0 for even j, Y1 for odd
 * j; per block Y2 = fma(d, Y0 + Y1, Y2).  The row's value is HSUM1(Y2). */
static int dot_q6k_q8_b32(const uint8_t *row, const int8_t *q, const float *d32, int64_t nb, float *out) {
    float y2[8] = {0};
    for (int64_t b = 0; b < nb; b++) {
        const uint8_t *blk = row + 210 * b;
        if (!f16_finite(blk + 208)) return 0;
        float d = mo_f16_to_f32(le16(blk + 208));
        float acc[2][8] = {{0}};
        for (int h = 0; h < 2; h++) {
            const uint8_t *ql = blk + 64 * h, *qh = blk + 128 + 32 * h;
            const int8_t *sc = (const int8_t *)(blk + 192 + 8 * h);
            const int8_t *yh = q + 256 * b + 128 * h;
            for (int j = 0; j < 4; j++)
                for (int l = 0; l < 8; l++) {
                    int32_t S = 0;
                    for (int e = 4 * l; e < 4 * l + 4; e++) {
                        int low = (j & 1) ? ql[e + 32] : ql[e];
                        low = (j >> 1) ? (low >> 4) : (low & 15);
                        int32_t qv = low | (((qh[e] >> (2 * j)) & 3) << 4);
                        S += (qv - 32) * yh[32 * j + e];
                    }
                    int32_t scl = sc[2 * j + (l >= 4)];
                    acc[j & 1][l] = fmaf(d32[8 * b + 4 * h + j], (float)(scl * S), acc[j & 1][l]);
                }
        }
        for (int l = 0; l < 8; l++) y2[l] = fmaf(d, acc[0][l] + acc[1][l], y2[l]);
    }
    *out = hsum1(y2);
    return 1;
}

/* dotQ8_0Q8AVX2, internal/kernels/kernels_amd64.s:1007-1040.  Per block of
 * 32: the scale f32(d_w * dx) (VMULSS), lane l = sum of w*y over elements
 * 4l..4l+3 (VPSIGNB/VPABSB make |w| the unsigned operand; exact for
 * q in [-127, 127]), Y0_l = fma(scale, lane, Y0_l).  The value is HSUM1(Y0). */
static int dot_q80_q8_b32(const uint8_t *row, const int8_t *q, const float *d32, int64_t nb, float *out) {
    float y0[8] = {0};
    for (int64_t b = 0; b < nb; b++) {
        const uint8_t *blk = row + 34 * b;
        if (!f16_finite(blk)) return 0;
        float scale = mo_f16_to_f32(le16(blk)) * d32[b];
        const int8_t *w = (const int8_t *)(blk + 2);
        for (int l = 0; l < 8; l++) {
            int32_t S = 0;
            for (int e = 4 * l; e < 4 * l + 4; e++) S += (int32_t)w[e] * q[32 * b + e];
            y0[l] = fmaf(scale, (float)S, y0[l]);
        }
    }
    *out = hsum1(y0);
    return 1;
}

/* RowDot.DotQ8 with blocks of 32, internal/kernels/q8.go:143-151. */
int mo_dot_q8_b32(int dt, const uint8_t *row, const int8_t *q, const float *d32, const int16_t *xs, int64_t k,
                  float *out) {
    switch (dt) {
    case MO_Q4_K: return dot_q4k_q8_b32(row, q, d32, xs, k / 256, out);
    case MO_Q6_K: return dot_q6k_q8_b32(row, q, d32, k / 256, out);
    case MO_Q8_0: return dot_q80_q8_b32(row, q, d32, k / 32, out);
    }
    return 0;
}

float mo_dot_f32(const float *a, const float *b, int64_t n) {
    float s0 = 0, s1 = 0, s2 = 0, s3 = 0;
    int64_t i = 0;
    for (; i + 4 <= n; i += 4) {
        s0 += a[i] * b[i];
        s1 += a[i + 1] * b[i + 1];
        s2 += a[i + 2] * b[i + 2];
        s3 += a[i + 3] * b[i + 3];
    }
    for (; i < n; i++) s0 += a[i] * b[i];
    return (s0 + s1) + (s2 + s3);
}

/* ------------------------------------------------------------------ */
/* matrix products                                                      */
/* ------------------------------------------------------------------ */

typedef struct {
    const float *x; int64_t rows, k; int dt; const uint8_t *w; int64_t n; const float *bias; float *y;
    int block;
    /* a8 state */
    const int8_t *q; const float *d32; const int16_t *xs; const uint8_t *quantized;
} mm_ctx;

/* linearCols, interp/fast.go:180-196 (purego RowDot: decode, then dotF32Go) */
static void mm_f32_cols(void *p, int64_t lo, int64_t hi) {
    mm_ctx *c = (mm_ctx *)p;
    int64_t rb = mo_row_bytes(c->dt, c->k);
    float *buf = (float *)malloc(sizeof(float) * (size_t)(c->k ? c->k : 1));
    for (int64_t j = lo; j < hi; j++) {
        mo_dequantize(c->dt, c->w + j * rb, buf, c->k);
        for (int64_t i = 0; i < c->rows; i++) {
            float s = mo_dot_f32(c->x + i * c->k, buf, c->k);
            if (c->bias) s += c->bias[j];
            c->y[i * c->n + j] = s;
        }
    }
    free(buf);
}

int mo_dequant_matmul(const float *x, int64_t rows, int64_t k, int dt, const uint8_t *w, int64_t n,
                      const float *bias, float *y, int nthreads) {
    if (mo_row_bytes(dt, k) == 0 && k != 0) return -1;
    mm_ctx c = {x, rows, k, dt, w, n, bias, y, 0, NULL, NULL, NULL, NULL};
    parallel_for(n, nthreads, mm_f32_cols, &c);
    return 0;
}

/* linearA8's loop over weight rows, interp/fast.go:324-377: the 8-bit
 * kernel for quantized rows, the f32 kernel for rows it refuses and for the
 * whole weight row once a block scale is found not finite. */
static void mm_a8_cols(void *p, int64_t lo, int64_t hi) {
    mm_ctx *c = (mm_ctx *)p;
    int64_t rb = mo_row_bytes(c->dt, c->k);
    float *buf = (float *)malloc(sizeof(float) * (size_t)c->k);
    for (int64_t j = lo; j < hi; j++) {
        const uint8_t *row = c->w + j * rb;
        int q8 = 1, loaded = 0;
        for (int64_t i = 0; i < c->rows; i++) {
            float s = 0;
            if (q8 && c->quantized[i])
                q8 = (c->block == 32 ? mo_dot_q8_b32 : mo_dot_q8k_ref)(c->dt, row, c->q + i * c->k, c->d32 + i * (c->k / 32),
                                                                      c->xs + i * (c->k / 32), c->k, &s);
            if (!q8 || !c->quantized[i]) {
                if (!loaded) { mo_dequantize(c->dt, row, buf, c->k); loaded = 1; }
                s = mo_dot_f32(c->x + i * c->k, buf, c->k);
            }
            if (c->bias) s += c->bias[j];
            c->y[i * c->n + j] = s;
        }
    }
    free(buf);
}

typedef struct { const float *x; int64_t k; int block; int8_t *q; float *d32; int16_t *xs; uint8_t *ok; } q8_ctx;

static void q8_rows(void *p, int64_t lo, int64_t hi) {
    q8_ctx *c = (q8_ctx *)p;
    for (int64_t i = lo; i < hi; i++)
        c->ok[i] = (uint8_t)mo_q8_quantize(c->x + i * c->k, c->k, c->block, c->q + i * c->k, c->d32 + i * (c->k / 32),
                                           c->xs + i * (c->k / 32), NULL);
}

int mo_dequant_matmul_a8(const float *x, int64_t rows, int64_t k, int dt, const uint8_t *w, int64_t n,
                         const float *bias, int block, float *y, int nthreads) {
    if (block != 32 && block != 256) return -1;
    /* FusedQ8Blocks (q8.go:104-115): blocks of 256 for Q4_K and Q6_K, blocks
     * of 32 for Q4_K, Q6_K and Q8_0 (the AVX2 kernels, the path every amd64
     * host with AVX2 and F16C takes); everything else is the exact f32
     * product (fast.go:254-258). */
    int fused = (dt == MO_Q4_K || dt == MO_Q6_K) || (block == 32 && dt == MO_Q8_0);
    if (!fused || k == 0) return mo_dequant_matmul(x, rows, k, dt, w, n, bias, y, nthreads);
    if (k % (dt == MO_Q8_0 ? 32 : 256)) return -1;
    int8_t *q = (int8_t *)malloc((size_t)(rows * k));
    float *d32 = (float *)malloc(sizeof(float) * (size_t)(rows * k / 32));
    int16_t *xs = (int16_t *)malloc(sizeof(int16_t) * (size_t)(rows * k / 32));
    uint8_t *ok = (uint8_t *)malloc((size_t)rows + 1);
    q8_ctx qc = {x, k, block, q, d32, xs, ok};
    parallel_for(rows, nthreads, q8_rows, &qc);
    mm_ctx c = {x, rows, k, dt, w, n, bias, y, block, q, d32, xs, ok};
    parallel_for(n, nthreads, mm_a8_cols, &c);
    free(q); free(d32); free(xs); free(ok);
    return 0;
}

/* ------------------------------------------------------------------ */
/* per-token operators                                                  */
/* ------------------------------------------------------------------ */

void mo_rms_norm(const float *x, int64_t rows, int64_t n, const float *scale, double eps, float *y) {
    if (n == 0) return;
    float epsf = (float)eps;
    for (int64_t r = 0; r < rows; r++) {
        const float *src = x + r * n;
        float *row = y + r * n;
        double ss = 0;
        for (int64_t j = 0; j < n; j++) ss += (double)src[j] * (double)src[j];
        float inv = (float)(1.0 / sqrt((double)(float)(ss / (double)n) + (double)epsf));
        for (int64_t j = 0; j < n; j++) {
            float v = src[j] * inv;
            if (scale) v = v * scale[j];
            row[j] = v;
        }
    }
}

int mo_rope(const float *x, int B, int H, int T, int D, const int64_t *pos, int pos_rows, double theta,
            int rotary, int interleaved, float *y) {
    if (rotary <= 0 || rotary % 2 || rotary > D) return -1;
    int h = rotary / 2;
    double *inv = (double *)malloc(sizeof(double) * (size_t)h);
    float *cs = (float *)malloc(sizeof(float) * 2 * (size_t)h);
    for (int i = 0; i < h; i++) inv[i] = pow(theta, -2.0 * (double)i / (double)rotary);
    for (int b = 0; b < B; b++)
        for (int t = 0; t < T; t++) {
            int pb = pos_rows != 1 ? b : 0;
            double pp = (double)pos[pb * T + t];
            for (int i = 0; i < h; i++) {
                double ang = pp * inv[i];
                cs[2 * i] = (float)(cos(ang) * 1.0);
                cs[2 * i + 1] = (float)(sin(ang) * 1.0);
            }
            for (int hd = 0; hd < H; hd++) {
                int64_t at = (((int64_t)b * H + hd) * T + t) * D;
                const float *src = x + at;
                float *row = y + at;
                memcpy(row, src, sizeof(float) * (size_t)D);
                for (int i = 0; i < h; i++) {
                    int i1 = interleaved ? 2 * i : i, i2 = interleaved ? 2 * i + 1 : i + h;
                    float x1 = src[i1], x2 = src[i2], c = cs[2 * i], s = cs[2 * i + 1];
                    row[i1] = x1 * c - x2 * s;
                    row[i2] = x2 * c + x1 * s;
                }
            }
        }
    free(inv); free(cs);
    return 0;
}

/* ------------------------------------------------------------------ */
/* the amd64 vector kernels of internal/kernels/attn_amd64.s            */
/* ------------------------------------------------------------------ */

/* exp(t) as expSumF32AVX2 computes it (attn_amd64.s:82-237): Cephes' expf
 * in float32 -- t = f*ln2 + r with f = RoundToEven(t*log2e), r by two fused
 * steps, a degree-5 polynomial in r evaluated with fused multiply-adds,
 * times 2^f -- and 0 below the limit (where VCMPPS GE_OQ is false; NaN too).
 * The constants are the kernel's `expc` table. */
static inline float expf_amd64(float t) {
    const float lo = bits_f32(0xc2aeac4fu), log2e = bits_f32(0x3fb8aa3bu);
    const float c1 = bits_f32(0x3f318000u), c2 = bits_f32(0xb95e8083u);
    const float p0 = bits_f32(0x39506967u), p1 = bits_f32(0x3ab743ceu), p2 = bits_f32(0x3c088908u);
    const float p3 = bits_f32(0x3d2aa9c1u), p4 = bits_f32(0x3e2aaaaau), p5 = bits_f32(0x3f000000u);
    const int valid = t >= lo;
    const float u = t > lo ? t : lo; /* VMAXPS: the second operand on NaN or equality */
    const float f = rintf(u * log2e);
    float r = fmaf(-f, c1, u);
    r = fmaf(-f, c2, r);
    const float r2 = r * r;
    float p = p0;
    p = fmaf(r, p, p1);
    p = fmaf(r, p, p2);
    p = fmaf(r, p, p3);
    p = fmaf(r, p, p4);
    p = fmaf(r, p, p5);
    p = fmaf(r2, p, r);
    p = p + 1.0f;
    const float y = p * bits_f32((uint32_t)((int)f + 127) << 23);
    return valid ? y : 0.0f;
}

/* silu(a)*b as siluMulF32AVX2 computes it (attn_amd64.s:465-527):
 * h = exp(-|a|/2), silu = a/(1+h*h) for a >= 0, (a*h)*h/(1+h*h) below. */
static inline float silu_mul_amd64(float a, float b) {
    const float t = bits_f32(f32_bits(a) | 0x80000000u) * 0.5f;
    const float h = expf_amd64(t);
    const float den = h * h + 1.0f;
    const float num = a >= 0.0f ? a : (a * h) * h;
    return (num / den) * b;
}

/* one key/value row as f32 (f16 converts exactly) */
static const float *kv_row(const void *base, int dt, int64_t j, int d, float *buf) {
    if (dt == MO_F32) return (const float *)base + j * d;
    const uint8_t *p = (const uint8_t *)base + 2 * j * d;
    for (int i = 0; i < d; i++) buf[i] = mo_f16_to_f32(le16(p + 2 * i));
    return buf;
}

/* attendRow, interp/fast.go:728-751, with the amd64 kernels of attn.go
 * (d a multiple of 8, as for every llama head size):
 *   ScoresF16/F32 -> scoresF16AVX2/scoresF32AVX2 (attn_amd64.s:12-80, 308-385):
 *     8 fused-multiply-add accumulators a[l] over elements 8c+l; keys in
 *     groups of four combine ((a0+a1)+(a2+a3))+((a4+a5)+(a6+a7)), the last
 *     n%4 keys ((a0+a4)+(a1+a5))+((a2+a6)+(a3+a7)); then times scale;
 *   ExpSumF32 (attn.go:41-56): the first n&~7 through expSumF32AVX2 with
 *     8 lane sums combined ((S0+S4)+(S1+S5))+((S2+S6)+(S3+S7)), the rest
 *     float32(math.Exp(float64)) added in order (all of them when n < 8);
 *   WeightedSumF16/F32 -> wsum*AVX2: one fused multiply-add per element and
 *     key, in key order;
 *   o = acc / sum.
 * Returns 0 (caller takes the scalar path) when the largest score is not finite. */
static int attend_row(const float *q, const void *kb, const void *vb, int dt, int64_t st, int64_t n, int d,
                      float scale, float *sc, float *acc, float *o, float *buf) {
    const int64_t n4 = n & ~(int64_t)3;
    for (int64_t j = 0; j < n; j++) {
        const float *kr = kv_row(kb, dt, st + j, d, buf);
        float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int c = 0; c < d / 8; c++)
            for (int l = 0; l < 8; l++) a[l] = fmaf(q[8 * c + l], kr[8 * c + l], a[l]);
        const float v = j < n4 ? ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]))
                               : ((a[0] + a[4]) + (a[1] + a[5])) + ((a[2] + a[6]) + (a[3] + a[7]));
        sc[j] = v * scale;
    }
    float mx = -INFINITY;
    for (int64_t j = 0; j < n; j++) if (sc[j] > mx || sc[j] != sc[j]) mx = sc[j];
    if (isinf(mx) || mx != mx) return 0;
    float sum = 0;
    int64_t j = 0;
    if (n >= 8) {
        const int64_t n8 = n & ~(int64_t)7;
        float S[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (; j < n8; j++) {
            const float e = expf_amd64(sc[j] - mx);
            sc[j] = e;
            S[j & 7] += e;
        }
        sum = ((S[0] + S[4]) + (S[1] + S[5])) + ((S[2] + S[6]) + (S[3] + S[7]));
    }
    for (; j < n; j++) {
        const float e = (float)exp((double)(sc[j] - mx));
        sc[j] = e;
        sum += e;
    }
    for (int i = 0; i < d; i++) acc[i] = 0;
    for (int64_t jj = 0; jj < n; jj++) {
        const float *vr = kv_row(vb, dt, st + jj, d, buf);
        for (int i = 0; i < d; i++) acc[i] = fmaf(sc[jj], vr[i], acc[i]);
    }
    for (int i = 0; i < d; i++) o[i] = acc[i] / sum;
    return 1;
}

int mo_attention(const float *q, int B, int Hq, int Tq, int D, const void *k, const void *v, int kv_dtype,
                 int Hkv, int Tk, const uint8_t *mask, const int *mask_shape, double scale_d, int causal,
                 float *out) {
    if (Hkv <= 0 || Hq % Hkv) return -1;
    if (kv_dtype != MO_F32 && kv_dtype != MO_F16) return -1;
    int G = Hq / Hkv;
    float scale = (float)scale_d;
    int64_t mst[4] = {0, 0, 0, 0};
    if (mask) {
        int64_t acc = 1;
        for (int i = 3; i >= 0; i--) { if (mask_shape[i] != 1) mst[i] = acc; acc *= mask_shape[i]; }
    }
    int esz = kv_dtype == MO_F32 ? 4 : 2;
    float *sc = (float *)malloc(sizeof(float) * (size_t)(Tk ? Tk : 1));
    float *acc = (float *)malloc(sizeof(float) * (size_t)D);
    float *buf = (float *)malloc(sizeof(float) * (size_t)D);
    int rows_in_order = !mask || mst[3] == 1;
    for (int b = 0; b < B; b++)
        for (int h = 0; h < Hq; h++) {
            int kvh = b * Hkv + h / G;
            const uint8_t *kb = (const uint8_t *)k + (int64_t)kvh * Tk * D * esz;
            const uint8_t *vb = (const uint8_t *)v + (int64_t)kvh * Tk * D * esz;
            for (int i = 0; i < Tq; i++) {
                const float *qi = q + (((int64_t)b * Hq + h) * Tq + i) * D;
                float *o = out + (((int64_t)b * Hq + h) * Tq + i) * D;
                const uint8_t *mrow = mask ? mask + b * mst[0] + h * mst[1] + i * mst[2] : NULL;
                int64_t end = Tk, st = 0;
                if (mask && rows_in_order) {
                    /* ends/starts of a boolean mask row, interp/fast.go:606-636 */
                    end = Tk;
                    while (end > 0 && mrow[end - 1] == 0) end--;
                    while (st < end && mrow[st] == 0) st++;
                }
                if (causal) { int64_t lim = i + (Tk - Tq) + 1; if (lim < end) end = lim; if (end < 0) end = 0; }
                if (rows_in_order && st < end) {
                    int hole = 0;
                    if (mask) for (int64_t j = st; j < end; j++) if (mrow[j] == 0) { hole = 1; break; }
                    if (!hole && attend_row(qi, kb, vb, kv_dtype, st, end - st, D, scale, sc, acc, o, buf)) continue;
                }
                /* scalar path, interp/fast.go:661-716 */
                float mx = -INFINITY;
                for (int64_t j = 0; j < end; j++) {
                    float s = -INFINITY;
                    int allowed = !causal || j <= i + (Tk - Tq);
                    if (mask) allowed = allowed && mrow[j * mst[3]] != 0;
                    if (allowed) s = mo_dot_f32(qi, kv_row(kb, kv_dtype, j, D, buf), D) * scale + 0.0f;
                    sc[j] = s;
                    if (s > mx || s != s) mx = s;
                }
                float sum = 0;
                for (int64_t j = 0; j < end; j++) {
                    if (isinf(sc[j]) && sc[j] < 0 && !(isinf(mx) && mx < 0)) { sc[j] = 0; continue; }
                    float e = (float)exp((double)(sc[j] - mx));
                    sc[j] = e;
                    sum += e;
                }
                for (int d = 0; d < D; d++) acc[d] = 0;
                for (int64_t j = 0; j < end; j++) {
                    if (sc[j] == 0) continue;
                    const float *vr = kv_row(vb, kv_dtype, j, D, buf);
                    for (int d = 0; d < D; d++) acc[d] += sc[j] * vr[d];
                }
                for (int d = 0; d < D; d++) o[d] = acc[d] / sum;
            }
        }
    free(sc); free(acc); free(buf);
    return 0;
}

/* SiluMulF32 (attn.go:59-73): siluMulF32AVX2 on the first n&~7 elements,
 * float64 on the rest.  fastSwiglu (interp/fast.go:487-498) hands it pieces
 * of n/(8*GOMAXPROCS) elements; for the llama shapes on the reference's
 * 4-core benchmark machine every piece is a multiple of 8. */
void mo_swiglu(const float *a, const float *b, int64_t n, float *y) {
    const int64_t n8 = n & ~(int64_t)7;
    for (int64_t i = 0; i < n8; i++) y[i] = silu_mul_amd64(a[i], b[i]);
    for (int64_t i = n8; i < n; i++) y[i] = (float)((double)a[i] / (1.0 + exp(-(double)a[i])) * (double)b[i]);
}

int mo_embedding(int dt, const uint8_t *table, int64_t V, int64_t E, const int32_t *ids, int64_t n, float *y) {
    int64_t rb = mo_row_bytes(dt, E);
    if (rb == 0) return -1;
    for (int64_t i = 0; i < n; i++) {
        int64_t id = ids[i];
        if (id >= 0 && id < V) mo_dequantize(dt, table + id * rb, y + i * E, E);
        else memset(y + i * E, 0, sizeof(float) * (size_t)E);
    }
    return 0;
}

int32_t mo_argmax(const float *v, int64_t n) {
    int64_t best = 0;
    for (int64_t i = 0; i < n; i++) if (v[i] > v[best]) best = i;
    return (int32_t)best;
}

/* ------------------------------------------------------------------ */
/* llama graph, importer/llama.go:400-534                               */
/* ------------------------------------------------------------------ */

typedef struct { int dt; const uint8_t *p; } wref;
/* bq, bk, bv: the query/key/value biases of a Qwen 2 graph (f32), or none */
typedef struct { wref attn_norm, q, k, v, o, ffn_norm, gate, up, down, bq, bk, bv; void *ck, *cv; } layer_w;

struct mo_llama {
    mo_llama_config c;
    wref embd, out_norm, out;
    layer_w *L;
};

mo_llama *mo_llama_new(const mo_llama_config *c) {
    if (c->layers <= 0 || c->heads <= 0 || c->kv_heads <= 0 || c->heads % c->kv_heads) return NULL;
    mo_llama *m = (mo_llama *)calloc(1, sizeof(mo_llama));
    m->c = *c;
    if (m->c.nthreads <= 0) m->c.nthreads = 1;
    m->L = (layer_w *)calloc((size_t)c->layers, sizeof(layer_w));
    size_t cache = (size_t)c->kv_heads * c->context * c->head_dim * (c->cache_f16 ? 2 : 4);
    for (int l = 0; l < c->layers; l++) { m->L[l].ck = calloc(1, cache); m->L[l].cv = calloc(1, cache); }
    return m;
}

void mo_llama_free(mo_llama *m) {
    if (!m) return;
    for (int l = 0; l < m->c.layers; l++) { free(m->L[l].ck); free(m->L[l].cv); }
    free(m->L);
    free(m);
}

void mo_llama_reset(mo_llama *m) {
    size_t cache = (size_t)m->c.kv_heads * m->c.context * m->c.head_dim * (m->c.cache_f16 ? 2 : 4);
    for (int l = 0; l < m->c.layers; l++) { memset(m->L[l].ck, 0, cache); memset(m->L[l].cv, 0, cache); }
}

int mo_llama_set_weight(mo_llama *m, const char *name, int dt, const void *data) {
    wref w = {dt, (const uint8_t *)data};
    if (!strcmp(name, "token_embd.weight")) { m->embd = w; return 0; }
    if (!strcmp(name, "output_norm.weight")) { m->out_norm = w; return 0; }
    if (!strcmp(name, "output.weight")) { m->out = w; return 0; }
    int l = 0, used = 0;
    char rest[64];
    if (sscanf(name, "blk.%d.%63s%n", &l, rest, &used) != 2 || l < 0 || l >= m->c.layers) return -1;
    layer_w *L = &m->L[l];
    if (!strcmp(rest, "attn_norm.weight")) L->attn_norm = w;
    else if (!strcmp(rest, "attn_q.weight")) L->q = w;
    else if (!strcmp(rest, "attn_k.weight")) L->k = w;
    else if (!strcmp(rest, "attn_v.weight")) L->v = w;
    else if (!strcmp(rest, "attn_output.weight")) L->o = w;
    else if (!strcmp(rest, "ffn_norm.weight")) L->ffn_norm = w;
    else if (!strcmp(rest, "ffn_gate.weight")) L->gate = w;
    else if (!strcmp(rest, "ffn_up.weight")) L->up = w;
    else if (!strcmp(rest, "ffn_down.weight")) L->down = w;
    else if (!strcmp(rest, "attn_q.bias") && dt == MO_F32) L->bq = w;
    else if (!strcmp(rest, "attn_k.bias") && dt == MO_F32) L->bk = w;
    else if (!strcmp(rest, "attn_v.bias") && dt == MO_F32) L->bv = w;
    else return -1;
    return 0;
}

/* matmulBias, importer/llama.go:243-268: a8.v2 block 256 for K-quants when
   a8; the bias (Qwen 2's query/key/value projections) as the optional third
   input */
static int mmb(mo_llama *m, const float *x, int64_t rows, int64_t k, wref w, int64_t n, wref b, float *y) {
    if (!w.p) return -1;
    const float *bias = (const float *)b.p;
    if (m->c.a8) return mo_dequant_matmul_a8(x, rows, k, w.dt, w.p, n, bias, 256, y, m->c.nthreads);
    return mo_dequant_matmul(x, rows, k, w.dt, w.p, n, bias, y, m->c.nthreads);
}

static int mm(mo_llama *m, const float *x, int64_t rows, int64_t k, wref w, int64_t n, float *y) {
    const wref none = {0, NULL};
    return mmb(m, x, rows, k, w, n, none, y);
}

int mo_llama_forward(mo_llama *m, const int32_t *tokens, const int64_t *positions, int T, float *logits, int all_rows) {
    const mo_llama_config *c = &m->c;
    int E = c->embed, H = c->heads, Hkv = c->kv_heads, D = c->head_dim, F = c->ffn, C = c->context;
    int64_t KV = (int64_t)Hkv * D;
    if (!m->embd.p || !m->out_norm.p) return -1;
    for (int t = 0; t < T; t++) if (positions[t] < 0 || positions[t] >= C) return -1;
    float *x = (float *)malloc(sizeof(float) * (size_t)T * E);
    float *h = (float *)malloc(sizeof(float) * (size_t)T * E);
    float *q = (float *)malloc(sizeof(float) * (size_t)T * E);
    float *kk = (float *)malloc(sizeof(float) * (size_t)T * KV);
    float *vv = (float *)malloc(sizeof(float) * (size_t)T * KV);
    float *qh = (float *)malloc(sizeof(float) * (size_t)T * E);
    float *kh = (float *)malloc(sizeof(float) * (size_t)T * KV);
    float *vh = (float *)malloc(sizeof(float) * (size_t)T * KV);
    float *att = (float *)malloc(sizeof(float) * (size_t)T * E);
    float *o = (float *)malloc(sizeof(float) * (size_t)T * E);
    float *g = (float *)malloc(sizeof(float) * (size_t)T * F);
    float *u = (float *)malloc(sizeof(float) * (size_t)T * F);
    float *a = (float *)malloc(sizeof(float) * (size_t)T * F);
    uint8_t *mask = (uint8_t *)malloc((size_t)T * C);
    int rc = 0;
    mo_embedding(m->embd.dt, m->embd.p, c->vocab, E, tokens, T, x);
    for (int t = 0; t < T; t++)
        for (int j = 0; j < C; j++) mask[(int64_t)t * C + j] = (uint8_t)(j <= positions[t]);
    int mshape[4] = {1, 1, T, C};
    int esz = c->cache_f16 ? 2 : 4;
    for (int l = 0; l < c->layers && rc == 0; l++) {
        layer_w *L = &m->L[l];
        mo_rms_norm(x, T, E, (const float *)L->attn_norm.p, c->norm_eps, h);
        rc |= mmb(m, h, T, E, L->q, E, L->bq, q);
        rc |= mmb(m, h, T, E, L->k, KV, L->bk, kk);
        rc |= mmb(m, h, T, E, L->v, KV, L->bv, vv);
        /* [1,T,n,D] -> [1,n,T,D] */
        for (int t = 0; t < T; t++)
            for (int hd = 0; hd < H; hd++)
                memcpy(qh + ((int64_t)hd * T + t) * D, q + (int64_t)t * E + (int64_t)hd * D, sizeof(float) * D);
        for (int t = 0; t < T; t++)
            for (int hd = 0; hd < Hkv; hd++) {
                memcpy(kh + ((int64_t)hd * T + t) * D, kk + (int64_t)t * KV + (int64_t)hd * D, sizeof(float) * D);
                memcpy(vh + ((int64_t)hd * T + t) * D, vv + (int64_t)t * KV + (int64_t)hd * D, sizeof(float) * D);
            }
        mo_rope(qh, 1, H, T, D, positions, 1, c->rope_theta, c->rope_dims, c->interleaved, q);
        mo_rope(kh, 1, Hkv, T, D, positions, 1, c->rope_theta, c->rope_dims, c->interleaved, kk);
        /* cast (f16 cache) and scatter at the positions, interp/prim.go:76-96, 278 */
        for (int hd = 0; hd < Hkv; hd++)
            for (int t = 0; t < T; t++) {
                const float *kr = kk + ((int64_t)hd * T + t) * D, *vr = vh + ((int64_t)hd * T + t) * D;
                int64_t at = ((int64_t)hd * C + positions[t]) * D;
                if (esz == 2) {
                    mo_cast_f16(kr, (uint16_t *)L->ck + at, D);
                    mo_cast_f16(vr, (uint16_t *)L->cv + at, D);
                } else {
                    memcpy((float *)L->ck + at, kr, sizeof(float) * D);
                    memcpy((float *)L->cv + at, vr, sizeof(float) * D);
                }
            }
        mo_attention(q, 1, H, T, D, L->ck, L->cv, c->cache_f16 ? MO_F16 : MO_F32, Hkv, C, mask, mshape,
                     1.0 / sqrt((double)D), 0, att);
        for (int t = 0; t < T; t++)
            for (int hd = 0; hd < H; hd++)
                memcpy(o + (int64_t)t * E + (int64_t)hd * D, att + ((int64_t)hd * T + t) * D, sizeof(float) * D);
        rc |= mm(m, o, T, E, L->o, E, h);
        for (int64_t i = 0; i < (int64_t)T * E; i++) x[i] = x[i] + h[i];
        mo_rms_norm(x, T, E, (const float *)L->ffn_norm.p, c->norm_eps, h);
        rc |= mm(m, h, T, E, L->gate, F, g);
        rc |= mm(m, h, T, E, L->up, F, u);
        mo_swiglu(g, u, (int64_t)T * F, a);
        rc |= mm(m, a, T, F, L->down, E, h);
        for (int64_t i = 0; i < (int64_t)T * E; i++) x[i] = x[i] + h[i];
    }
    if (rc == 0) {
        wref head = m->out.p ? m->out : m->embd; /* tied embeddings when output.weight is absent */
        int first = all_rows ? 0 : T - 1;
        mo_rms_norm(x + (int64_t)first * E, T - first, E, (const float *)m->out_norm.p, c->norm_eps, h);
        rc |= mm(m, h, T - first, E, head, c->vocab, logits);
    }
    free(x); free(h); free(q); free(kk); free(vv); free(qh); free(kh); free(vh); free(att); free(o);
    free(g); free(u); free(a); free(mask);
    return rc ? -1 : 0;
}
