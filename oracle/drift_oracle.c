/*
 * drift_oracle.c — CPU restatement of drift's emulated-matmul arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY: the oracle for the CUDA engine. Only the tests,
 * the smoke check and the benchmark's CPU-baseline leg load it.
 *
 * Every function follows the Java source line by line (IEEE binary64, round
 * to nearest even, no FMA contraction: build with -ffp-contract=off and no
 * fast-math). Citations are relative to the reference project's root; the
 * Java package prefix java/src/main/java/io/drift/ is written as "..".
 */
#include "drift_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------ formats */

enum { SP_IEEE = 0, SP_FN = 1, SP_FINITE = 2 };

typedef struct {
    int exp_bits, mant_bits, bias, specials;
    int width, mant_mask, max_exp_field, exp_mask, sign_bit, code_mask;
    int min_normal_exp;
    double max_finite, min_normal, min_subnormal;
} ofmt;

static ofmt g_fmt[DRIFT_NUM_FORMATS];
static int g_fmt_ready = 0;

/* MiniFloat constructor (../fmt/MiniFloat.java:70-107). */
static void fmt_make(ofmt *f, int e, int m, int bias, int sp) {
    f->exp_bits = e;
    f->mant_bits = m;
    f->bias = bias;
    f->specials = sp;
    f->width = 1 + e + m;
    f->mant_mask = (1 << m) - 1;
    f->max_exp_field = (1 << e) - 1;
    f->exp_mask = f->max_exp_field << m;
    f->sign_bit = 1 << (e + m);
    f->code_mask = (1 << f->width) - 1;
    f->min_normal_exp = 1 - bias;
    f->min_normal = scalbn(1.0, f->min_normal_exp);
    f->min_subnormal = scalbn(1.0, f->min_normal_exp - m);
    int top_exp, top_mant;
    switch (sp) {
        case SP_IEEE: top_exp = f->max_exp_field - 1; top_mant = f->mant_mask; break;
        case SP_FN: top_exp = f->max_exp_field; top_mant = f->mant_mask - 1; break;
        default: top_exp = f->max_exp_field; top_mant = f->mant_mask; break;
    }
    f->max_finite = scalbn(1.0 + (double)top_mant / (1 << m), top_exp - bias);
}

/* Formats table (../fmt/Formats.java:20-45); all SATURATE. */
static void fmt_init(void) {
    if (g_fmt_ready) return;
    fmt_make(&g_fmt[DRIFT_E4M3], 4, 3, 7, SP_FN);
    fmt_make(&g_fmt[DRIFT_E5M2], 5, 2, 15, SP_IEEE);
    fmt_make(&g_fmt[DRIFT_E2M1], 2, 1, 1, SP_FINITE);
    fmt_make(&g_fmt[DRIFT_E3M2], 3, 2, 3, SP_FINITE);
    fmt_make(&g_fmt[DRIFT_E2M3], 2, 3, 1, SP_FINITE);
    fmt_make(&g_fmt[DRIFT_FP16], 5, 10, 15, SP_IEEE);
    fmt_make(&g_fmt[DRIFT_BF16], 8, 7, 127, SP_IEEE);
    g_fmt_ready = 1;
}

static const ofmt *fmt_get(int id) {
    fmt_init();
    if (id < 0 || id >= DRIFT_NUM_FORMATS) return NULL;
    return &g_fmt[id];
}

int o_format_info(int fmt, double *max_finite, double *min_normal,
                  double *min_subnormal, int32_t *width) {
    const ofmt *f = fmt_get(fmt);
    if (!f) return DRIFT_EINVAL;
    if (max_finite) *max_finite = f->max_finite;
    if (min_normal) *min_normal = f->min_normal;
    if (min_subnormal) *min_subnormal = f->min_subnormal;
    if (width) *width = f->width;
    return DRIFT_OK;
}

/* ------------------------------------------------------------ Java math */

/* Math.getExponent(double): unbiased exponent field, -1023 for zero and
 * subnormals, 1024 for Inf/NaN. */
static int j_get_exponent(double d) {
    uint64_t b;
    memcpy(&b, &d, 8);
    return (int)((b >> 52) & 0x7FF) - 1023;
}

/* ------------------------------------------------------------ Rng */

/* Rng.nextLong (../fmt/Rng.java:17-22). */
uint64_t o_rng_next_long(uint64_t *state) {
    uint64_t z = (*state += 0x9E3779B97F4A7C15ULL);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

/* Rng.nextDouble (../fmt/Rng.java:25-27). */
double o_rng_next_double(uint64_t *state) {
    return (double)(o_rng_next_long(state) >> 11) * 0x1.0p-53;
}

/* ------------------------------------------------------------ MiniFloat */

/* MiniFloat.roundToIntegral (../fmt/MiniFloat.java:258-278). */
static int64_t round_to_integral(double scaled, int rm, uint64_t *rng, int *err) {
    switch (rm) {
        case DRIFT_NEAREST_EVEN:
            return (int64_t)rint(scaled);
        case DRIFT_TRUNCATE:
            return (int64_t)floor(scaled);
        case DRIFT_STOCHASTIC: {
            double fl = floor(scaled);
            double frac = scaled - fl;
            if (frac == 0.0) return (int64_t)fl;
            if (rng == NULL) {
                *err = DRIFT_EINVAL;
                return 0;
            }
            return (int64_t)fl + (o_rng_next_double(rng) < frac ? 1 : 0);
        }
        default:
            *err = DRIFT_EINVAL;
            return 0;
    }
}

static int top_binade_allows(const ofmt *f, int mant_field) {
    switch (f->specials) {
        case SP_IEEE: return 0;
        case SP_FN: return mant_field < f->mant_mask;
        default: return 1;
    }
}

static int max_finite_bits(const ofmt *f) {
    switch (f->specials) {
        case SP_IEEE: return ((f->max_exp_field - 1) << f->mant_bits) | f->mant_mask;
        case SP_FN: return (f->max_exp_field << f->mant_bits) | (f->mant_mask - 1);
        default: return (f->max_exp_field << f->mant_bits) | f->mant_mask;
    }
}

/* Every format in Formats.java saturates, so overflowBits is maxFiniteBits
 * (../fmt/MiniFloat.java:239-248). */
static int overflow_bits(const ofmt *f) { return max_finite_bits(f); }

/* MiniFloat.nanBits (../fmt/MiniFloat.java:231-237). */
static int nan_bits(const ofmt *f) {
    return f->specials == SP_IEEE ? (f->exp_mask | 1) : (f->exp_mask | f->mant_mask);
}

/* MiniFloat.encode (../fmt/MiniFloat.java:156-211). */
static int encode1(const ofmt *f, double v, int rm, uint64_t *rng, int *err) {
    if (isnan(v)) {
        if (f->specials == SP_FINITE) {
            *err = DRIFT_ENAN_FINITE;
            return 0;
        }
        return nan_bits(f);
    }
    int sign = (v < 0.0 || (v == 0.0 && signbit(v))) ? f->sign_bit : 0;
    double a = fabs(v);
    if (a == 0.0) return sign;
    if (isinf(a)) return sign | overflow_bits(f);

    int e = j_get_exponent(a);
    if (e == -1023 || e < f->min_normal_exp) e = f->min_normal_exp;
    int quantum_exp = e - f->mant_bits;
    double scaled = scalbn(a, -quantum_exp);
    int64_t m = round_to_integral(scaled, rm, rng, err);
    if (*err) return 0;

    int64_t normal_base = (int64_t)1 << f->mant_bits;
    if (m < normal_base) return sign | (int)m;
    if (m >= (normal_base << 1)) {
        m >>= 1;
        e += 1;
    }
    int exp_field = e + f->bias;
    int mant_field = (int)(m - normal_base);
    if (exp_field > f->max_exp_field ||
        (exp_field == f->max_exp_field && !top_binade_allows(f, mant_field))) {
        return sign | overflow_bits(f);
    }
    return sign | (exp_field << f->mant_bits) | mant_field;
}

/* MiniFloat.decode (../fmt/MiniFloat.java:117-142). */
static double decode1(const ofmt *f, int bits) {
    int exp_field = (bits & f->exp_mask) >> f->mant_bits;
    int mant = bits & f->mant_mask;
    double sign = (bits & f->sign_bit) ? -1.0 : 1.0;
    if (exp_field == f->max_exp_field) {
        if (f->specials == SP_IEEE) return mant == 0 ? sign * INFINITY : NAN;
        if (f->specials == SP_FN && mant == f->mant_mask) return NAN;
    }
    if (exp_field == 0) return sign * scalbn((double)mant, f->min_normal_exp - f->mant_bits);
    double significand = 1.0 + (double)mant / (1 << f->mant_bits);
    return sign * scalbn(significand, exp_field - f->bias);
}

/* MiniFloat.quantize(v, rm, rng) (../fmt/MiniFloat.java:219-221). */
static double quantize1(const ofmt *f, double v, int rm, uint64_t *rng, int *err) {
    int c = encode1(f, v, rm, rng, err);
    if (*err) return 0.0;
    return decode1(f, c);
}

int o_encode(int fmt, int rm, const double *v, int32_t *codes, int64_t n,
             uint64_t *rng_state) {
    const ofmt *f = fmt_get(fmt);
    if (!f) return DRIFT_EINVAL;
    int err = 0;
    for (int64_t i = 0; i < n; i++) {
        codes[i] = encode1(f, v[i], rm, rng_state, &err);
        if (err) return err;
    }
    return DRIFT_OK;
}

int o_decode(int fmt, const int32_t *codes, double *v, int64_t n) {
    const ofmt *f = fmt_get(fmt);
    if (!f) return DRIFT_EINVAL;
    for (int64_t i = 0; i < n; i++) {
        if (codes[i] & ~f->code_mask) return DRIFT_EINVAL;
        v[i] = decode1(f, codes[i]);
    }
    return DRIFT_OK;
}

/* ------------------------------------------------------------ Dot.round */

/* Dot.round (../kernel/Dot.java:141-182). */
static double acc_round1(double x, int acc, int rm, uint64_t *rng, int *err) {
    int mant, min_exp;
    double max;
    if (acc == DRIFT_ACC_FP16) {
        mant = 10;
        min_exp = -14;
        max = 65504.0;
    } else {
        mant = 7;
        min_exp = -126;
        max = scalbn(255.0, 120);
    }
    if (x == 0.0 || isnan(x)) return x;
    double ax = fabs(x);
    if (isinf(ax)) return copysign(max, x);
    int e = j_get_exponent(ax);
    if (e < min_exp) e = min_exp;
    int q = e - mant;
    double scaled = scalbn(ax, -q);
    double m;
    switch (rm) {
        case DRIFT_NEAREST_EVEN: m = rint(scaled); break;
        case DRIFT_TRUNCATE: m = floor(scaled); break;
        default: {
            double fl = floor(scaled);
            double frac = scaled - fl;
            if (frac == 0.0) {
                m = fl;
            } else {
                if (rng == NULL) {
                    *err = DRIFT_EINVAL;
                    return 0.0;
                }
                m = fl + (o_rng_next_double(rng) < frac ? 1 : 0);
            }
        }
    }
    double r = scalbn(m, q);
    if (r > max) r = max;
    return copysign(r, x);
}

int o_acc_round(int acc, int rm, const double *x, double *y, int64_t n,
                uint64_t *rng_state) {
    if (acc != DRIFT_ACC_FP16 && acc != DRIFT_ACC_BF16) return DRIFT_EINVAL;
    if (rm < 0 || rm > 2) return DRIFT_EINVAL;
    int err = 0;
    for (int64_t i = 0; i < n; i++) {
        y[i] = acc_round1(x[i], acc, rm, rng_state, &err);
        if (err) return err;
    }
    return DRIFT_OK;
}

/* ------------------------------------------------------------ Quant */

/* Quant.amax (../kernel/Quant.java:25-34). */
double o_amax(const double *x, int64_t n) {
    double m = 0.0;
    for (int64_t i = 0; i < n; i++) {
        double v = fabs(x[i]);
        if (v > m) m = v;
    }
    return m;
}

/* Quant.perTensorScale (../kernel/Quant.java:37-42). */
double o_per_tensor_scale(int fmt, double amax) {
    const ofmt *f = fmt_get(fmt);
    if (!f) return 1.0;
    if (amax == 0.0 || !isfinite(amax)) return 1.0;
    return f->max_finite / amax;
}

/* Quant.quantizeMx (../kernel/Quant.java:95-123). */
static int64_t quantize_mx(const double *src, double *dst, int64_t n,
                           const ofmt *f, const drift_policy *p, int rm,
                           uint64_t *rng, int *err) {
    int64_t block = p->scale_block;
    int emax_elem = j_get_exponent(f->max_finite);
    int64_t clamped = 0;
    for (int64_t start = 0; start < n; start += block) {
        int64_t len = block < n - start ? block : n - start;
        double block_amax = o_amax(src + start, len);
        if (block_amax == 0.0 || !isfinite(block_amax)) {
            for (int64_t i = 0; i < len; i++) dst[start + i] = 0.0;
            continue;
        }
        int shared = j_get_exponent(block_amax) - emax_elem + p->mx_headroom;
        shared = shared < -127 ? -127 : (shared > 127 ? 127 : shared);
        for (int64_t i = 0; i < len; i++) {
            double scaled = scalbn(src[start + i], -shared);
            if (fabs(scaled) > f->max_finite) clamped++;
            double q = quantize1(f, scaled, rm, rng, err);
            if (*err) return clamped;
            dst[start + i] = scalbn(q, shared);
        }
    }
    return clamped;
}

/* Quant.quantize (../kernel/Quant.java:56-82). */
int o_quantize(const drift_policy *p, int fmt, int rm, const double *src,
               double *dst, int64_t n, double scale, uint64_t *rng_state,
               int64_t *clamped_out) {
    int64_t clamped = 0;
    int err = 0;
    if (fmt == DRIFT_FMT_NONE) {
        memmove(dst, src, (size_t)n * sizeof(double));
        if (clamped_out) *clamped_out = 0;
        return DRIFT_OK;
    }
    const ofmt *f = fmt_get(fmt);
    if (!f || rm < 0 || rm > 2) return DRIFT_EINVAL;
    switch (p->scaling) {
        case DRIFT_SCALE_NONE:
            for (int64_t i = 0; i < n && !err; i++) {
                double v = src[i];
                if (fabs(v) > f->max_finite) clamped++;
                dst[i] = quantize1(f, v, rm, rng_state, &err);
            }
            break;
        case DRIFT_PER_TENSOR: {
            double inv = 1.0 / scale;
            for (int64_t i = 0; i < n && !err; i++) {
                double up = src[i] * scale;
                if (fabs(up) > f->max_finite) clamped++;
                dst[i] = quantize1(f, up, rm, rng_state, &err) * inv;
            }
            break;
        }
        case DRIFT_MX_BLOCK:
            if (p->scale_block <= 0) return DRIFT_EINVAL;
            clamped = quantize_mx(src, dst, n, f, p, rm, rng_state, &err);
            break;
        default:
            return DRIFT_EINVAL;
    }
    if (clamped_out) *clamped_out = clamped;
    return err;
}

/* ------------------------------------------------------------ Dot */

typedef struct {
    const double *a;
    int64_t a_off, a_stride;
    const double *b;
    int64_t b_off, b_stride;
    const drift_policy *p;
    uint64_t *rng;
    int *err;
} dotargs;

/* Dot.forward (../kernel/Dot.java:37-68). */
static double dot_forward(const dotargs *d, int64_t from, int64_t count) {
    int64_t ia = d->a_off + from * d->a_stride;
    int64_t ib = d->b_off + from * d->b_stride;
    switch (d->p->acc) {
        case DRIFT_ACC_FP64: {
            double s = 0.0;
            for (int64_t i = 0; i < count; i++, ia += d->a_stride, ib += d->b_stride)
                s += d->a[ia] * d->b[ib];
            return s;
        }
        case DRIFT_ACC_FP32: {
            float s = 0.0f;
            for (int64_t i = 0; i < count; i++, ia += d->a_stride, ib += d->b_stride)
                s = (float)((double)s + d->a[ia] * d->b[ib]);
            return s;
        }
        default: {
            double s = 0.0;
            for (int64_t i = 0; i < count; i++, ia += d->a_stride, ib += d->b_stride) {
                s = acc_round1(s + d->a[ia] * d->b[ib], d->p->acc, d->p->acc_rounding, d->rng, d->err);
                if (*d->err) return 0.0;
            }
            return s;
        }
    }
}

/* Dot.backward (../kernel/Dot.java:70-84). */
static double dot_backward(const dotargs *d, int64_t n) {
    double s = 0.0;
    float f = 0.0f;
    for (int64_t i = n - 1; i >= 0; i--) {
        double prod = d->a[d->a_off + i * d->a_stride] * d->b[d->b_off + i * d->b_stride];
        switch (d->p->acc) {
            case DRIFT_ACC_FP64: s += prod; break;
            case DRIFT_ACC_FP32: f = (float)((double)f + prod); break;
            default:
                s = acc_round1(s + prod, d->p->acc, d->p->acc_rounding, d->rng, d->err);
                if (*d->err) return 0.0;
        }
    }
    return d->p->acc == DRIFT_ACC_FP32 ? (double)f : s;
}

/* Dot.pairwise with PAIRWISE_BASE 8 (../kernel/Dot.java:86-102). */
static double dot_pairwise(const dotargs *d, int64_t from, int64_t count) {
    if (count <= 8) return dot_forward(d, from, count);
    int64_t half = (int64_t)((uint64_t)count >> 1);
    double left = dot_pairwise(d, from, half);
    double right = dot_pairwise(d, from + half, count - half);
    if (*d->err) return 0.0;
    switch (d->p->acc) {
        case DRIFT_ACC_FP64: return left + right;
        case DRIFT_ACC_FP32: return (float)(left + right);
        default: return acc_round1(left + right, d->p->acc, d->p->acc_rounding, d->rng, d->err);
    }
}

/* Dot.blocked (../kernel/Dot.java:104-121). */
static double dot_blocked(const dotargs *d, int64_t n) {
    int64_t block = d->p->acc_block > 1 ? d->p->acc_block : 1;
    if (d->p->acc == DRIFT_ACC_FP64) {
        double total = 0.0;
        for (int64_t start = 0; start < n; start += block)
            total += dot_forward(d, start, block < n - start ? block : n - start);
        return total;
    }
    float total = 0.0f;
    for (int64_t start = 0; start < n; start += block) {
        double partial = dot_forward(d, start, block < n - start ? block : n - start);
        total = (float)((double)total + partial);
    }
    return total;
}

/* Dot.dot (../kernel/Dot.java:26-35). */
double o_dot(const double *a, int64_t a_off, int64_t a_stride,
             const double *b, int64_t b_off, int64_t b_stride, int64_t n,
             const drift_policy *p, uint64_t *rng_state, int *err) {
    dotargs d = {a, a_off, a_stride, b, b_off, b_stride, p, rng_state, err};
    *err = 0;
    if (p->acc < 0 || p->acc > 3 || p->order < 0 || p->order > 3) {
        *err = DRIFT_EINVAL;
        return 0.0;
    }
    switch (p->order) {
        case DRIFT_SEQUENTIAL: return dot_forward(&d, 0, n);
        case DRIFT_REVERSED: return dot_backward(&d, n);
        case DRIFT_PAIRWISE: return dot_pairwise(&d, 0, n);
        default: return dot_blocked(&d, n);
    }
}

/* ------------------------------------------------------------ GEMM loop */

typedef struct {
    const drift_policy *p;
    int64_t M, N, K;
    const double *A;
    int64_t a_off, a_rs, a_ks;
    const double *B;
    int64_t b_off, b_rs, b_ks;
    const double *bias;
    double *C;
    int64_t c_rs;
    uint64_t *rng;
    int64_t row_begin, row_end;
    int err;
} gemmjob;

/* The (i, o) loop with the bias add of ../train/Pass.java:200-204; without
 * a bias the dot is stored as is (adding 0.0 would turn -0.0 into +0.0). */
static void *gemm_rows(void *arg) {
    gemmjob *j = (gemmjob *)arg;
    for (int64_t i = j->row_begin; i < j->row_end && !j->err; i++) {
        for (int64_t o = 0; o < j->N && !j->err; o++) {
            int err = 0;
            double v = o_dot(j->A, j->a_off + i * j->a_rs, j->a_ks, j->B,
                             j->b_off + o * j->b_rs, j->b_ks, j->K, j->p, j->rng, &err);
            if (err) {
                j->err = err;
                break;
            }
            j->C[i * j->c_rs + o] = j->bias ? v + j->bias[o] : v;
        }
    }
    return NULL;
}

int o_gemm(const drift_policy *p, int64_t M, int64_t N, int64_t K,
           const double *A, int64_t a_off, int64_t a_rs, int64_t a_ks,
           const double *B, int64_t b_off, int64_t b_rs, int64_t b_ks,
           const double *bias, double *C, int64_t c_rs, uint64_t *rng_state,
           int threads) {
    gemmjob base = {p, M, N, K, A, a_off, a_rs, a_ks, B, b_off, b_rs, b_ks,
                    bias, C, c_rs, rng_state, 0, M, 0};
    int draws = (p->acc == DRIFT_ACC_FP16 || p->acc == DRIFT_ACC_BF16) &&
                p->acc_rounding == DRIFT_STOCHASTIC;
    if (threads <= 1 || draws || M < 2) {
        gemm_rows(&base);
        return base.err;
    }
    if (threads > M) threads = (int)M;
    gemmjob *jobs = (gemmjob *)calloc((size_t)threads, sizeof(gemmjob));
    pthread_t *tids = (pthread_t *)calloc((size_t)threads, sizeof(pthread_t));
    int64_t per = (M + threads - 1) / threads;
    int started = 0;
    for (int t = 0; t < threads; t++) {
        jobs[t] = base;
        jobs[t].row_begin = t * per;
        jobs[t].row_end = (t + 1) * per < M ? (t + 1) * per : M;
        if (jobs[t].row_begin >= jobs[t].row_end) break;
        pthread_create(&tids[t], NULL, gemm_rows, &jobs[t]);
        started++;
    }
    int err = 0;
    for (int t = 0; t < started; t++) {
        pthread_join(tids[t], NULL);
        if (!err && jobs[t].err) err = jobs[t].err;
    }
    free(jobs);
    free(tids);
    return err;
}

/* ------------------------------------------------------------ attention loops */

/* AttnPass's score loop (../train/AttnPass.java:245-255): dot over the whole
 * depth for s <= i, times scoreScale, 0.0 for s > i; dProb (:373-381) the
 * same without the scale. Context and dq (:283-288, :412-417): n = i + 1
 * from k = 0. dv and dk (:382-388, :419-424): n = t - s from k = s. The
 * dInput accumulation (:478-484): dx += dot. */
int o_contract(const drift_policy *p, const drift_contraction *op, const double *A,
               const double *B, double *C, uint64_t *rng_state) {
    for (int64_t t = 0; t < op->batch; t++) {
        for (int64_t i = 0; i < op->rows; i++) {
            for (int64_t o = 0; o < op->cols; o++) {
                double *c = C + op->c_off + t * op->c_batch + i * op->c_row + o * op->c_col;
                if (op->causal && o > i) {
                    *c = 0.0;
                    continue;
                }
                int64_t lo = 0, n = op->depth;
                if (op->window == DRIFT_WINDOW_PREFIX) n = i + 1;
                if (op->window == DRIFT_WINDOW_SUFFIX) {
                    lo = i;
                    n = op->depth - i;
                }
                int err = 0;
                double v = o_dot(A, op->a_off + t * op->a_batch + i * op->a_row + lo * op->a_k,
                                 op->a_k, B,
                                 op->b_off + t * op->b_batch + o * op->b_col + lo * op->b_k,
                                 op->b_k, n, p, rng_state, &err);
                if (err) return err;
                if (op->alpha != 1.0) v = v * op->alpha;
                *c = op->accumulate ? *c + v : v;
            }
        }
    }
    return DRIFT_OK;
}

/* ------------------------------------------------------------ StrictMath.log */
/*
 * java.util.Random.nextGaussian calls StrictMath.log, which the Java platform
 * specifies as fdlibm 5.3's logarithm (the "Freely Distributable LIBM" of Sun
 * Microsystems, e_log.c). Host libm's log differs from it by an ulp on some
 * arguments, and that alone kept half of DotSweep's (n, seed) input groups
 * from regenerating. This restates fdlibm's published method with its
 * published constants, in its order of operations:
 *   x = 2^k (1 + f) with sqrt(2)/2 <= 1 + f < sqrt(2);
 *   s = f / (2 + f), so log(1 + f) = 2s + s R(s^2), R a degree-14 Remez
 *   polynomial with coefficients Lg1..Lg7;
 *   log(x) = k ln2_hi + (f - (hfsq - (s (hfsq + R) + k ln2_lo))), hfsq = f^2/2,
 *   with ln2 split so k ln2_hi is exact; tiny f and the upper part of each
 *   binade take the shorter forms below.
 * Only positive normal and subnormal arguments reach it from nextGaussian
 * (0 < s < 1); zero, negatives, Inf and NaN follow fdlibm's returns too.
 */
static uint32_t hi_word(double x) {
    uint64_t b;
    memcpy(&b, &x, 8);
    return (uint32_t)(b >> 32);
}

static uint32_t lo_word(double x) {
    uint64_t b;
    memcpy(&b, &x, 8);
    return (uint32_t)b;
}

static double set_hi_word(double x, uint32_t h) {
    uint64_t b;
    memcpy(&b, &x, 8);
    b = ((uint64_t)h << 32) | (b & 0xFFFFFFFFULL);
    memcpy(&x, &b, 8);
    return x;
}

static double from_bits(uint64_t b) {
    double d;
    memcpy(&d, &b, 8);
    return d;
}

double o_strict_log(double x) {
    const double ln2_hi = from_bits(0x3FE62E42FEE00000ULL);   /* 6.93147180369123816490e-01 */
    const double ln2_lo = from_bits(0x3DEA39EF35793C76ULL);   /* 1.90821492927058770002e-10 */
    const double two54 = 18014398509481984.0;
    const double Lg1 = from_bits(0x3FE5555555555593ULL), Lg2 = from_bits(0x3FD999999997FA04ULL),
                 Lg3 = from_bits(0x3FD2492494229359ULL), Lg4 = from_bits(0x3FCC71C51D8E78AFULL),
                 Lg5 = from_bits(0x3FC7466496CB03DEULL), Lg6 = from_bits(0x3FC39A09D078C69FULL),
                 Lg7 = from_bits(0x3FC2F112DF3E5244ULL);
    int32_t hx = (int32_t)hi_word(x);
    int k = 0;
    if (hx < 0x00100000) {                        /* subnormal, zero or negative */
        if (((hx & 0x7fffffff) | lo_word(x)) == 0) return -two54 / 0.0;
        if (hx < 0) return (x - x) / 0.0;
        k -= 54;
        x *= two54;
        hx = (int32_t)hi_word(x);
    }
    if (hx >= 0x7ff00000) return x + x;
    k += (hx >> 20) - 1023;
    hx &= 0x000fffff;
    int32_t i = (hx + 0x95f64) & 0x100000;        /* 1 when the significand is >= sqrt(2) */
    x = set_hi_word(x, (uint32_t)(hx | (i ^ 0x3ff00000)));
    k += i >> 20;
    const double f = x - 1.0;
    const double dk = (double)k;
    if ((0x000fffff & (2 + hx)) < 3) {           /* |f| < 2^-20 */
        if (f == 0.0) return k == 0 ? 0.0 : dk * ln2_hi + dk * ln2_lo;
        const double R = f * f * (0.5 - 0.33333333333333333 * f);
        return k == 0 ? f - R : dk * ln2_hi - ((R - dk * ln2_lo) - f);
    }
    const double s = f / (2.0 + f);
    const double z = s * s;
    const double w = z * z;
    const int32_t upper = (hx - 0x6147a) | (0x6b851 - hx);
    const double t1 = w * (Lg2 + w * (Lg4 + w * Lg6));
    const double t2 = z * (Lg1 + w * (Lg3 + w * (Lg5 + w * Lg7)));
    const double R = t2 + t1;
    if (upper > 0) {
        const double hfsq = 0.5 * f * f;
        if (k == 0) return f - (hfsq - s * (hfsq + R));
        return dk * ln2_hi - ((hfsq - (s * (hfsq + R) + dk * ln2_lo)) - f);
    }
    if (k == 0) return f - s * (f - R);
    return dk * ln2_hi - ((s * (f - R) - dk * ln2_lo) - f);
}

/* ------------------------------------------------------------ java.util.Random */

#define JR_MULT 0x5DEECE66DULL
#define JR_MASK ((1ULL << 48) - 1)

void o_jrandom_init(o_jrandom *r, int64_t seed) {
    r->seed = ((uint64_t)seed ^ JR_MULT) & JR_MASK;
    r->have_next_gaussian = 0;
    r->next_gaussian = 0.0;
}

int32_t o_jrandom_next(o_jrandom *r, int bits) {
    r->seed = (r->seed * JR_MULT + 0xBULL) & JR_MASK;
    return (int32_t)(uint32_t)(r->seed >> (48 - bits));
}

double o_jrandom_next_double(o_jrandom *r) {
    int64_t hi = (int64_t)(uint32_t)o_jrandom_next(r, 26);
    int64_t lo = (int64_t)(uint32_t)o_jrandom_next(r, 27);
    return (double)((hi << 27) + lo) * 0x1.0p-53;
}

double o_jrandom_next_gaussian(o_jrandom *r) {
    if (r->have_next_gaussian) {
        r->have_next_gaussian = 0;
        return r->next_gaussian;
    }
    double v1, v2, s;
    do {
        v1 = 2 * o_jrandom_next_double(r) - 1;
        v2 = 2 * o_jrandom_next_double(r) - 1;
        s = v1 * v1 + v2 * v2;
    } while (s >= 1 || s == 0);
    double multiplier = sqrt(-2 * o_strict_log(s) / s);  /* StrictMath.sqrt / StrictMath.log */
    r->next_gaussian = v2 * multiplier;
    r->have_next_gaussian = 1;
    return v1 * multiplier;
}

int32_t o_jrandom_next_int(o_jrandom *r, int32_t bound) {
    int32_t rr = o_jrandom_next(r, 31);
    int32_t m = bound - 1;
    if ((bound & m) == 0) return (int32_t)(((int64_t)bound * (int64_t)rr) >> 31);
    for (int32_t u = rr; (int32_t)((uint32_t)u - (uint32_t)(rr = u % bound) + (uint32_t)m) < 0;
         u = o_jrandom_next(r, 31)) {
    }
    return rr;
}

/* DotSweep.fill (java/.../tools/DotSweep.java:124-130). Math.exp is host
 * libm's here: the JVM's exp differs from it by an ulp on rare arguments, so
 * a few (n, seed) groups still do not regenerate (565 of the 600 in
 * results/dot_sweep.csv do). */
void o_dotsweep_fill(double *a, double *b, int64_t n, int64_t seed) {
    o_jrandom r;
    o_jrandom_init(&r, seed);
    for (int64_t i = 0; i < n; i++) {
        double g = o_jrandom_next_gaussian(&r);
        a[i] = g * exp(o_jrandom_next_gaussian(&r) * 0.8);
        g = o_jrandom_next_gaussian(&r);
        b[i] = g * exp(o_jrandom_next_gaussian(&r) * 0.8);
    }
}
