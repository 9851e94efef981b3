/*
 * drift_oracle.h — CPU restatement of drift's emulated-matmul arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY. This is the oracle the CUDA engine is compared
 * against (tests, smoke check, and the CPU-baseline leg of the benchmark). No
 * product code links, loads or calls it.
 *
 * Enum values and the policy struct come from the engine's public header so
 * both sides read the same policy bytes.
 */
#ifndef DRIFT_ORACLE_H
#define DRIFT_ORACLE_H

#include <stdint.h>
#include "../include/drift_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Format constants (MiniFloat ctor, java/.../fmt/MiniFloat.java:70-107). */
int o_format_info(int fmt, double *max_finite, double *min_normal,
                  double *min_subnormal, int32_t *width);

/* splitmix64 (java/.../fmt/Rng.java:17-27). */
uint64_t o_rng_next_long(uint64_t *state);
double o_rng_next_double(uint64_t *state);

/* MiniFloat.encode / decode / quantize, element-wise over arrays. Return a
 * drift status; on error the arrays are partially written (as Java throws
 * midway). */
int o_encode(int fmt, int rm, const double *v, int32_t *codes, int64_t n,
             uint64_t *rng_state /* may be NULL */);
int o_decode(int fmt, const int32_t *codes, double *v, int64_t n);

/* Dot.round over an array (java/.../kernel/Dot.java:141-182). */
int o_acc_round(int acc, int rm, const double *x, double *y, int64_t n,
                uint64_t *rng_state);

/* Quant (java/.../kernel/Quant.java). */
double o_amax(const double *x, int64_t n);
double o_per_tensor_scale(int fmt, double amax);
int o_quantize(const drift_policy *p, int fmt, int rm, const double *src,
               double *dst, int64_t n, double scale, uint64_t *rng_state,
               int64_t *clamped);

/* Dot.dot (java/.../kernel/Dot.java:26-121). status via *err. */
double o_dot(const double *a, int64_t a_off, int64_t a_stride,
             const double *b, int64_t b_off, int64_t b_stride, int64_t n,
             const drift_policy *p, uint64_t *rng_state, int *err);

/* The (i, o) double loop over Dot.dot that Pass / the sweeps run
 * (java/.../train/Pass.java:200-232). Rows are split over `threads` host
 * threads when the accumulator draws no random numbers. */
int o_gemm(const drift_policy *p, int64_t M, int64_t N, int64_t K,
           const double *A, int64_t a_off, int64_t a_rs, int64_t a_ks,
           const double *B, int64_t b_off, int64_t b_rs, int64_t b_ks,
           const double *bias, double *C, int64_t c_rs, uint64_t *rng_state,
           int threads);

/* The (t, i, o) loops of AttnPass over Dot.dot
 * (java/.../train/AttnPass.java:245-290, :373-427) for one drift_contraction:
 * row i's window, 0.0 for causal o > i, the score scale, the accumulating
 * add of dInput (:478-484). */
int o_contract(const drift_policy *p, const drift_contraction *op, const double *A,
               const double *B, double *C, uint64_t *rng_state);

/* java.util.Random as specified by its Javadoc (LCG 0x5DEECE66D, polar
 * nextGaussian with StrictMath.sqrt/log), used to regenerate the reference's
 * DotSweep inputs (java/.../tools/DotSweep.java:124-130). log and exp come
 * from the host libm, which can differ from the JVM's by an ulp. */
typedef struct o_jrandom {
    uint64_t seed;
    int have_next_gaussian;
    double next_gaussian;
} o_jrandom;
void o_jrandom_init(o_jrandom *r, int64_t seed);
int32_t o_jrandom_next(o_jrandom *r, int bits);
double o_jrandom_next_double(o_jrandom *r);
double o_jrandom_next_gaussian(o_jrandom *r);
int32_t o_jrandom_next_int(o_jrandom *r, int32_t bound);
/* DotSweep.fill(a, b, seed) (java/.../tools/DotSweep.java:124-130). */
/* StrictMath.log: fdlibm 5.3's logarithm, restated (drift_oracle.c). */
double o_strict_log(double x);
void o_dotsweep_fill(double *a, double *b, int64_t n, int64_t seed);

#ifdef __cplusplus
}
#endif
#endif
