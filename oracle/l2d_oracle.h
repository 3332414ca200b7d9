/*
 * l2d_oracle.h -- CPU oracle for the L2-domain-aware GEMV hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is a plain-C restatement of the reference
 * algorithm (LyleLuo/L2Domain, applications/gemv + utility/latopt.cuh) used as
 * the checker by tests/, __graft_entry__.smoke() and the cpu_baseline leg of
 * bench.py.  Nothing in the product library links or calls it.
 *
 * Parity pins: mix32 and the domain predictor are checked against the
 * reference's own host-callable functions compiled from its sources
 * (oracle/Makefile target `ref`, fixtures in tests/golden/); the GEMV check
 * loop is pinned by the reference's exact-integer input mode, for which every
 * summation order yields the same fp32 result.
 */
#ifndef L2D_ORACLE_H
#define L2D_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { OR_F32 = 0, OR_F16 = 1, OR_BF16 = 2 };
enum { OR_DIST_UNIFORM = 0, OR_DIST_NORMAL = 1 };

/* ---- reference-mode generator (gemv_k1024_persistent_subwarp.cu:56-63, :118-139) ---- */
uint32_t or_mix32(uint32_t x);
/* A[i] (or x[i]) for flat indices [first, first+n); stream 0 = A (seed), 1 = x (seed+0x9e37). */
void or_ref_fill(float *out, uint64_t first, uint64_t n, uint32_t seed, int stream, int integer_mode);

/* ---- BASELINE-config generator: counter-based splitmix64, exact on host and device ---- */
uint64_t or_splitmix64(uint64_t z);
uint64_t or_rng_u64(uint64_t seed, uint64_t stream, uint64_t index, uint32_t sub);
double or_log_pos(double u);     /* natural log for u in (0, 1], textbook atanh series */
double or_cos_2pi(double u);     /* cos(2*pi*u) for u in [0, 1), Taylor series after octant reduction */
/* dist UNIFORM: p0 + (p1 - p0) * u;  dist NORMAL: p1 * N(0,1) + p0 (p0 = mean, p1 = sigma). */
float or_cfg_value(uint64_t seed, uint64_t stream, uint64_t index, int dist, float p0, float p1);
void or_cfg_fill(float *out, uint64_t first, uint64_t n, uint64_t seed, uint64_t stream, int dist, float p0, float p1);
/* The same values, computed by `threads` threads (0 = all online cores). */
void or_cfg_fill_mt(float *out, uint64_t first, uint64_t n, uint64_t seed, uint64_t stream, int dist, float p0, float p1,
                    int threads);

/* ---- storage formats (IEEE round-to-nearest-even, integer code) ---- */
uint16_t or_f32_to_f16(float f);
float or_f16_to_f32(uint16_t h);
uint16_t or_f32_to_bf16(float f);
float or_bf16_to_f32(uint16_t h);
void or_round_array(const float *in, void *out, uint64_t n, int dtype);   /* f32 -> dtype storage */
void or_widen_array(const void *in, float *out, uint64_t n, int dtype);   /* dtype storage -> f32 */

/* ---- GEMV oracles ---- */
/* gemv_k1024_persistent_subwarp.cu:383-390: sequential fp32 `sum += a[k]*x[k]`, no contraction. */
void or_gemv_seq_f32(const float *A, const float *x, float *y, int64_t M, int64_t N, int64_t lda);
/* Same loop over dtype storage widened to fp32 element by element (fp16/bf16 CPU check). */
void or_gemv_seq_any(const void *A, int dtype, const void *x, float *y, int64_t M, int64_t N, int64_t lda);
/* Same per-row loop, rows split over `threads` POSIX threads (0 = all online cores). */
void or_gemv_omp_any(const void *A, int dtype, const void *x, float *y, int64_t M, int64_t N, int64_t lda, int threads);
/* fp64 accumulation of the same (already rounded) inputs. */
void or_gemv_f64(const void *A, int dtype, const void *x, double *y, int64_t M, int64_t N, int64_t lda);
int or_max_threads(void);

double or_max_abs_err(const double *ref, const float *y, int64_t n);
double or_rel_l2(const double *ref, const float *y, int64_t n);
/* gemv_k1024_persistent_subwarp.cu:391-397 (max |y - ref| in fp32). */
float or_max_abs_err_f32(const float *ref, const float *y, int64_t n);

/* ---- domain predictor and row placement ---- */
/* latopt.cuh:255-263 */
int or_predict_far(int side, uint32_t mask, uint64_t addr, int attr);
/* gemv_k1024_persistent_subwarp.cu:105-108; attr indexed by 2 MiB page relative to base. */
int or_predict_addr_side(uint64_t base, uint32_t mask, const int *attr, uint64_t addr);
/* gemv_k1024_persistent_subwarp.cu:261-273: rows to side lists by the predicted side of the
 * row start; baseline lists by row parity.  Outputs must hold M entries each; counts returned. */
void or_partition_rows(uint64_t base, uint64_t row_bytes, int64_t M, uint32_t mask, const int *attr,
                       int32_t *side0, int64_t *n0, int32_t *side1, int64_t *n1,
                       int32_t *base0, int64_t *nb0, int32_t *base1, int64_t *nb1);

/* ---- the reference's probe classification rules (restated for synthetic-latency tests) ---- */
/* latopt.cuh:517-528: side = (max - min) > 100 over the 16 probe latencies. */
int or_ref_smid_side(const uint32_t *lat, int n);
/* latopt.cuh:732-746: exp2 series over bits 7..20 -> mask, base attr and the mean. */
uint32_t or_ref_mask_from_exp2(const uint32_t *lat14, float *exp2_avg, int *base_attr);

#ifdef __cplusplus
}
#endif
#endif
