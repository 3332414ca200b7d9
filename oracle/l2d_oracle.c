/*
 * l2d_oracle.c -- CPU oracle for the L2-domain-aware GEMV (test infrastructure only).
 *
 * Build flags matter: -O3 -ffp-contract=off, so `sum += a[k]*x[k]` rounds the product and the
 * sum separately, exactly as the reference's host check loop does when nvcc's host compiler
 * targets baseline x86-64 (no FMA).  See oracle/Makefile.
 */
#include "l2d_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <pthread.h>
#include <unistd.h>

/* ------------------------------------------------------------------------------------------ */
/* Reference-mode generator.                                                                   */
/* ------------------------------------------------------------------------------------------ */

/* gemv_k1024_persistent_subwarp.cu:56-63 (also gemv_cublas_benchmark.cu:18-25). */
uint32_t or_mix32(uint32_t x) {
    x ^= x >> 16;
    x *= 0x7feb352du;
    x ^= x >> 15;
    x *= 0x846ca68bu;
    x ^= x >> 16;
    return x;
}

/* gemv_k1024_persistent_subwarp.cu:118-139.  The flat index is truncated to 32 bits before the
 * xor with the seed (`static_cast<uint32_t>(i) ^ seed`), so values repeat with period 2^32. */
void or_ref_fill(float *out, uint64_t first, uint64_t n, uint32_t seed, int stream, int integer_mode) {
    uint32_t s = stream == 0 ? seed : seed + 0x9e37u;
    for (uint64_t j = 0; j < n; ++j) {
        uint32_t h = or_mix32((uint32_t)(first + j) ^ s);
        if (integer_mode) {
            out[j] = stream == 0 ? (float)((int)(h % 17u) - 8) : (float)((int)(h % 7u) - 3);
        } else {
            out[j] = (float)(h & 0xffu) / 255.0f - 0.5f;
        }
    }
}

/* ------------------------------------------------------------------------------------------ */
/* BASELINE-config generator.  Only integer ops and IEEE +,-,*,/,sqrt in double, written without */
/* contraction, so the device generator in the library reproduces every value bit for bit.    */
/* ------------------------------------------------------------------------------------------ */

uint64_t or_splitmix64(uint64_t z) {
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

uint64_t or_rng_u64(uint64_t seed, uint64_t stream, uint64_t index, uint32_t sub) {
    uint64_t key = or_splitmix64(seed ^ (stream * 0xd1342543de82ef95ull) ^ 0x243f6a8885a308d3ull);
    return or_splitmix64(key + 2u * index + sub);
}

/* log(u) = e*ln2 + 2*atanh(s), s = (m-1)/(m+1), m in [sqrt(1/2), sqrt(2)). */
double or_log_pos(double u) {
    uint64_t bits;
    memcpy(&bits, &u, sizeof bits);
    int e = (int)((bits >> 52) & 0x7ff) - 1023;
    uint64_t mbits = (bits & 0x000fffffffffffffull) | 0x3ff0000000000000ull;
    double m;
    memcpy(&m, &mbits, sizeof m);
    if (m > 1.4142135623730951) {
        m = m * 0.5;
        e = e + 1;
    }
    double s = (m - 1.0) / (m + 1.0);
    double s2 = s * s;
    double p = 1.0 / 23.0;
    p = p * s2 + 1.0 / 21.0;
    p = p * s2 + 1.0 / 19.0;
    p = p * s2 + 1.0 / 17.0;
    p = p * s2 + 1.0 / 15.0;
    p = p * s2 + 1.0 / 13.0;
    p = p * s2 + 1.0 / 11.0;
    p = p * s2 + 1.0 / 9.0;
    p = p * s2 + 1.0 / 7.0;
    p = p * s2 + 1.0 / 5.0;
    p = p * s2 + 1.0 / 3.0;
    p = p * s2 + 1.0;
    double lm = 2.0 * s * p;
    return (double)e * 0.6931471805599453 + lm;
}

static double or_cos_series(double x) {
    /* sum_k (-1)^k x^(2k) / (2k)!, k = 0..9, Horner in x^2 */
    double x2 = x * x;
    double p = -1.0 / 6402373705728000.0; /* -1/18! */
    p = p * x2 + 1.0 / 20922789888000.0;  /* +1/16! */
    p = p * x2 - 1.0 / 87178291200.0;     /* -1/14! */
    p = p * x2 + 1.0 / 479001600.0;       /* +1/12! */
    p = p * x2 - 1.0 / 3628800.0;         /* -1/10! */
    p = p * x2 + 1.0 / 40320.0;           /* +1/8! */
    p = p * x2 - 1.0 / 720.0;             /* -1/6! */
    p = p * x2 + 1.0 / 24.0;              /* +1/4! */
    p = p * x2 - 0.5;
    p = p * x2 + 1.0;
    return p;
}

static double or_sin_series(double x) {
    /* x * sum_k (-1)^k x^(2k) / (2k+1)!, k = 0..9 */
    double x2 = x * x;
    double p = -1.0 / 121645100408832000.0; /* -1/19! */
    p = p * x2 + 1.0 / 355687428096000.0;   /* +1/17! */
    p = p * x2 - 1.0 / 1307674368000.0;     /* -1/15! */
    p = p * x2 + 1.0 / 6227020800.0;        /* +1/13! */
    p = p * x2 - 1.0 / 39916800.0;          /* -1/11! */
    p = p * x2 + 1.0 / 362880.0;            /* +1/9! */
    p = p * x2 - 1.0 / 5040.0;              /* -1/7! */
    p = p * x2 + 1.0 / 120.0;               /* +1/5! */
    p = p * x2 - 1.0 / 6.0;
    p = p * x2 + 1.0;
    return p * x;
}

/* cos(2*pi*u), u in [0,1): fold to w in [0, 1/4] by symmetry, then pick the cos or sin series
 * on an angle in [0, pi/4]. */
double or_cos_2pi(double u) {
    double w = u - 0.5; /* cos(2*pi*u) = -cos(2*pi*w) */
    double sign = -1.0;
    if (w < 0.0) w = -w;
    if (w > 0.25) {
        w = 0.5 - w;
        sign = -sign;
    }
    if (w > 0.125) {
        double a = (0.25 - w) * 6.283185307179586;
        return sign * or_sin_series(a);
    }
    return sign * or_cos_series(w * 6.283185307179586);
}

float or_cfg_value(uint64_t seed, uint64_t stream, uint64_t index, int dist, float p0, float p1) {
    uint64_t r0 = or_rng_u64(seed, stream, index, 0);
    if (dist == OR_DIST_UNIFORM) {
        float u = (float)(uint32_t)(r0 >> 40) * 0x1p-24f;
        float span = p1 - p0;
        float t = span * u;
        return p0 + t;
    }
    uint64_t r1 = or_rng_u64(seed, stream, index, 1);
    double u1 = (double)((r0 >> 11) + 1u) * 0x1p-53; /* (0, 1] */
    double u2 = (double)(r1 >> 11) * 0x1p-53;        /* [0, 1) */
    double l = or_log_pos(u1);
    double r = sqrt(-2.0 * l);
    double z = r * or_cos_2pi(u2);
    double v = (double)p1 * z;
    v = v + (double)p0;
    return (float)v;
}

void or_cfg_fill(float *out, uint64_t first, uint64_t n, uint64_t seed, uint64_t stream, int dist, float p0, float p1) {
    for (uint64_t j = 0; j < n; ++j) out[j] = or_cfg_value(seed, stream, first + j, dist, p0, p1);
}

typedef struct {
    float *out;
    uint64_t first, n, seed, stream;
    int dist;
    float p0, p1;
} or_fill_job;

static void *or_fill_worker(void *arg) {
    or_fill_job *j = (or_fill_job *)arg;
    or_cfg_fill(j->out, j->first, j->n, j->seed, j->stream, j->dist, j->p0, j->p1);
    return NULL;
}

/* or_cfg_fill with the index range split over `threads` POSIX threads (0 = all online cores);
 * every value depends on its index only, so the output equals the single-threaded fill. */
void or_cfg_fill_mt(float *out, uint64_t first, uint64_t n, uint64_t seed, uint64_t stream, int dist, float p0, float p1,
                    int threads) {
    int nt = threads > 0 ? threads : (int)sysconf(_SC_NPROCESSORS_ONLN);
    if (nt < 1) nt = 1;
    if (nt > 256) nt = 256;
    if ((uint64_t)nt > n / 65536 + 1) nt = (int)(n / 65536 + 1);
    or_fill_job jobs[256];
    pthread_t tids[256];
    int started[256];
    for (int t = 0; t < nt; ++t) {
        const uint64_t lo = n * (uint64_t)t / (uint64_t)nt, hi = n * (uint64_t)(t + 1) / (uint64_t)nt;
        or_fill_job j = {out + lo, first + lo, hi - lo, seed, stream, dist, p0, p1};
        jobs[t] = j;
        started[t] = t > 0 && pthread_create(&tids[t], NULL, or_fill_worker, &jobs[t]) == 0;
    }
    or_fill_worker(&jobs[0]);
    for (int t = 1; t < nt; ++t) {
        if (started[t]) pthread_join(tids[t], NULL);
        else or_fill_worker(&jobs[t]);
    }
}

/* ------------------------------------------------------------------------------------------ */
/* Storage formats.                                                                            */
/* ------------------------------------------------------------------------------------------ */

uint16_t or_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t a = x & 0x7fffffffu;
    if (a >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (a > 0x7f800000u ? 0x200u : 0u));
    if (a >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* >= 65520 rounds to inf */
    if (a < 0x38800000u) {                                 /* below 2^-14: subnormal or zero */
        uint32_t e = a >> 23;
        if (e < 102u) return (uint16_t)sign;
        uint32_t mant = (a & 0x7fffffu) | 0x800000u;
        uint32_t shift = 126u - e;
        uint32_t q = mant >> shift;
        uint32_t rem = mant & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t e = (a >> 23) - 127u + 15u;
    uint32_t mant = a & 0x7fffffu;
    uint32_t q = (e << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
    return (uint16_t)(sign | q);
}

float or_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t e = ((uint32_t)h >> 10) & 0x1fu;
    uint32_t m = (uint32_t)h & 0x3ffu;
    uint32_t x;
    if (e == 0) {
        if (m == 0) {
            x = sign;
        } else {
            int shift = 0;
            while (!(m & 0x400u)) {
                m <<= 1;
                shift++;
            }
            m &= 0x3ffu;
            x = sign | ((uint32_t)(127 - 15 - shift + 1) << 23) | (m << 13);
        }
    } else if (e == 31) {
        x = sign | 0x7f800000u | (m << 13);
    } else {
        x = sign | ((e - 15u + 127u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

uint16_t or_f32_to_bf16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40u);
    uint32_t r = x + 0x7fffu + ((x >> 16) & 1u);
    return (uint16_t)(r >> 16);
}

float or_bf16_to_f32(uint16_t h) {
    uint32_t x = (uint32_t)h << 16;
    float f;
    memcpy(&f, &x, 4);
    return f;
}

void or_round_array(const float *in, void *out, uint64_t n, int dtype) {
    if (dtype == OR_F32) {
        memcpy(out, in, n * sizeof(float));
    } else if (dtype == OR_F16) {
        uint16_t *o = (uint16_t *)out;
        for (uint64_t i = 0; i < n; ++i) o[i] = or_f32_to_f16(in[i]);
    } else {
        uint16_t *o = (uint16_t *)out;
        for (uint64_t i = 0; i < n; ++i) o[i] = or_f32_to_bf16(in[i]);
    }
}

static float g_f16_table[65536];
static int g_f16_table_ready = 0;

static void or_init_f16_table(void) {
    if (g_f16_table_ready) return;
    for (uint32_t i = 0; i < 65536u; ++i) g_f16_table[i] = or_f16_to_f32((uint16_t)i);
    g_f16_table_ready = 1;
}

void or_widen_array(const void *in, float *out, uint64_t n, int dtype) {
    if (dtype == OR_F32) {
        memcpy(out, in, n * sizeof(float));
        return;
    }
    const uint16_t *h = (const uint16_t *)in;
    if (dtype == OR_F16) {
        or_init_f16_table();
        for (uint64_t i = 0; i < n; ++i) out[i] = g_f16_table[h[i]];
    } else {
        for (uint64_t i = 0; i < n; ++i) out[i] = or_bf16_to_f32(h[i]);
    }
}

/* ------------------------------------------------------------------------------------------ */
/* GEMV oracles.                                                                               */
/* ------------------------------------------------------------------------------------------ */

void or_gemv_seq_f32(const float *A, const float *x, float *y, int64_t M, int64_t N, int64_t lda) {
    for (int64_t row = 0; row < M; ++row) {
        float sum = 0.0f;
        const float *a = A + row * lda;
        for (int64_t k = 0; k < N; ++k) sum += a[k] * x[k];
        y[row] = sum;
    }
}

static inline float or_load(const void *p, int dtype, int64_t i) {
    if (dtype == OR_F32) return ((const float *)p)[i];
    uint16_t h = ((const uint16_t *)p)[i];
    return dtype == OR_F16 ? g_f16_table[h] : or_bf16_to_f32(h);
}

static void or_gemv_rows(const void *A, int dtype, const float *xf, float *y, int64_t r0, int64_t r1, int64_t N,
                         int64_t lda) {
    for (int64_t row = r0; row < r1; ++row) {
        float sum = 0.0f;
        if (dtype == OR_F32) {
            const float *a = (const float *)A + row * lda;
            for (int64_t k = 0; k < N; ++k) sum += a[k] * xf[k];
        } else if (dtype == OR_F16) {
            const uint16_t *a = (const uint16_t *)A + row * lda;
            for (int64_t k = 0; k < N; ++k) sum += g_f16_table[a[k]] * xf[k];
        } else {
            const uint16_t *a = (const uint16_t *)A + row * lda;
            for (int64_t k = 0; k < N; ++k) sum += or_bf16_to_f32(a[k]) * xf[k];
        }
        y[row] = sum;
    }
}

void or_gemv_seq_any(const void *A, int dtype, const void *x, float *y, int64_t M, int64_t N, int64_t lda) {
    or_init_f16_table();
    float xf_stack[16384];
    float *xf = xf_stack;
    float *heap = NULL;
    if (N > 16384) {
        heap = (float *)malloc((size_t)N * sizeof(float));
        xf = heap;
    }
    for (int64_t k = 0; k < N; ++k) xf[k] = or_load(x, dtype, k);
    or_gemv_rows(A, dtype, xf, y, 0, M, N, lda);
    free(heap);
}

int or_max_threads(void) {
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}

typedef struct {
    const void *A;
    int dtype;
    const float *xf;
    float *y;
    int64_t r0, r1, N, lda;
} or_rows_job;

static void *or_rows_worker(void *arg) {
    or_rows_job *j = (or_rows_job *)arg;
    or_gemv_rows(j->A, j->dtype, j->xf, j->y, j->r0, j->r1, j->N, j->lda);
    return NULL;
}

/* Row-parallel form of the same per-row loop: each thread owns a contiguous block of rows, so
 * every y[row] is bit-identical to the single-threaded result. */
void or_gemv_omp_any(const void *A, int dtype, const void *x, float *y, int64_t M, int64_t N, int64_t lda, int threads) {
    or_init_f16_table();
    float *xf = (float *)malloc((size_t)(N > 0 ? N : 1) * sizeof(float));
    for (int64_t k = 0; k < N; ++k) xf[k] = or_load(x, dtype, k);
    int nt = threads > 0 ? threads : or_max_threads();
    if (nt > 1024) nt = 1024;
    if ((int64_t)nt > M) nt = M > 0 ? (int)M : 1;
    or_rows_job jobs[1024];
    pthread_t tids[1024];
    int started[1024];
    for (int t = 0; t < nt; ++t) {
        jobs[t].A = A;
        jobs[t].dtype = dtype;
        jobs[t].xf = xf;
        jobs[t].y = y;
        jobs[t].r0 = M * t / nt;
        jobs[t].r1 = M * (t + 1) / nt;
        jobs[t].N = N;
        jobs[t].lda = lda;
        started[t] = t > 0 && pthread_create(&tids[t], NULL, or_rows_worker, &jobs[t]) == 0;
    }
    or_rows_worker(&jobs[0]);
    for (int t = 1; t < nt; ++t) {
        if (started[t]) pthread_join(tids[t], NULL);
        else or_rows_worker(&jobs[t]);
    }
    free(xf);
}

void or_gemv_f64(const void *A, int dtype, const void *x, double *y, int64_t M, int64_t N, int64_t lda) {
    or_init_f16_table();
    for (int64_t row = 0; row < M; ++row) {
        double sum = 0.0;
        for (int64_t k = 0; k < N; ++k) sum += (double)or_load(A, dtype, row * lda + k) * (double)or_load(x, dtype, k);
        y[row] = sum;
    }
}

double or_max_abs_err(const double *ref, const float *y, int64_t n) {
    double m = 0.0;
    for (int64_t i = 0; i < n; ++i) {
        double d = fabs((double)y[i] - ref[i]);
        if (d > m || d != d) m = d;
    }
    return m;
}

double or_rel_l2(const double *ref, const float *y, int64_t n) {
    double num = 0.0, den = 0.0;
    for (int64_t i = 0; i < n; ++i) {
        double d = (double)y[i] - ref[i];
        num += d * d;
        den += ref[i] * ref[i];
    }
    if (den == 0.0) return num == 0.0 ? 0.0 : INFINITY;
    return sqrt(num / den);
}

float or_max_abs_err_f32(const float *ref, const float *y, int64_t n) {
    float err = 0.0f;
    for (int64_t i = 0; i < n; ++i) {
        float d = fabsf(y[i] - ref[i]);
        err = err > d ? err : d;
    }
    return err;
}

/* ------------------------------------------------------------------------------------------ */
/* Predictor and placement.                                                                    */
/* ------------------------------------------------------------------------------------------ */

int or_predict_far(int side, uint32_t mask, uint64_t addr, int attr) {
    uint32_t bits = (uint32_t)addr;
    int parity = __builtin_popcount(bits & mask) & 1;
    return parity ^ side ^ attr;
}

int or_predict_addr_side(uint64_t base, uint32_t mask, const int *attr, uint64_t addr) {
    uint64_t page = (addr - base) / (2ull * 1024ull * 1024ull);
    return or_predict_far(0, mask, addr, attr[page]) & 1;
}

void or_partition_rows(uint64_t base, uint64_t row_bytes, int64_t M, uint32_t mask, const int *attr,
                       int32_t *side0, int64_t *n0, int32_t *side1, int64_t *n1,
                       int32_t *base0, int64_t *nb0, int32_t *base1, int64_t *nb1) {
    int64_t c0 = 0, c1 = 0, b0 = 0, b1 = 0;
    for (int64_t row = 0; row < M; ++row) {
        uint64_t addr = base + (uint64_t)row * row_bytes;
        int side = or_predict_addr_side(base, mask, attr, addr);
        if (side) side1[c1++] = (int32_t)row;
        else side0[c0++] = (int32_t)row;
        if (row & 1) base1[b1++] = (int32_t)row;
        else base0[b0++] = (int32_t)row;
    }
    *n0 = c0;
    *n1 = c1;
    *nb0 = b0;
    *nb1 = b1;
}

/* ------------------------------------------------------------------------------------------ */
/* Reference probe classification rules.                                                       */
/* ------------------------------------------------------------------------------------------ */

int or_ref_smid_side(const uint32_t *lat, int n) {
    uint32_t max_latency = 0, min_latency = 1024;
    for (int i = 0; i < n; ++i) {
        uint32_t cur = lat[i];
        max_latency = cur > max_latency ? cur : max_latency;
        min_latency = cur < min_latency ? cur : min_latency;
    }
    return (uint32_t)(max_latency - min_latency) > 100u;
}

uint32_t or_ref_mask_from_exp2(const uint32_t *lat14, float *exp2_avg, int *base_attr) {
    float avg = 0.0f;
    for (int i = 0; i < 14; ++i) avg += (float)lat14[i];
    avg /= 14.0f;
    int battr = (float)lat14[0] > avg;
    uint32_t mask = 0;
    for (int i = 0; i < 14; ++i) {
        int cur = (float)lat14[i] > avg;
        if (cur != battr) mask |= 1u << (i + 7);
    }
    if (exp2_avg) *exp2_avg = avg;
    if (base_attr) *base_attr = battr;
    return mask;
}
