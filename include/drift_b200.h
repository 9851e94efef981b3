/*
 * drift_b200.h — C ABI of the B200 emulated-matmul engine.
 *
 * The engine reproduces, bit for bit, drift's policy-parameterised matmul
 * arithmetic: cast to a minifloat format (MiniFloat), per-tensor / MX scaling
 * (Quant), and the accumulator/order engine (Dot). Every entry point here
 * replaces a loop of the Java reference that calls those static methods; the
 * comment above each one cites the Java interface it stands in for (paths are
 * relative to the reference project's root).
 *
 * Conventions
 *  - Plain C: no C++ or torch types cross this boundary. Sizes are int64_t.
 *  - Every function returns a drift status (DRIFT_OK == 0). drift_last_error()
 *    gives the message of the calling thread's most recent failure.
 *  - Host entry points take HOST pointers (Java MemorySegment / off-heap
 *    arrays). They copy to the device, run, copy back, and return only when
 *    the result is in the caller's buffer. They never keep a pointer.
 *  - *_dev entry points take DEVICE pointers and a cudaStream_t passed as
 *    void*, used as given (NULL is the CUDA default stream). They are
 *    asynchronous with respect to the host unless noted.
 *  - rng_state is the Java Rng.state() long (java/src/main/java/io/drift/fmt/
 *    Rng.java:29-31). On return it holds the state the Java Rng would hold
 *    after the same calls, so callers can interleave engine calls with Java
 *    code that shares the stream.
 *  - One drift_ctx per host thread. A context owns a CUDA stream and a
 *    device workspace; it is not safe to use one context from two threads at
 *    once. Different contexts share nothing.
 */
#ifndef DRIFT_B200_H
#define DRIFT_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define DRIFT_API __attribute__((visibility("default")))
#else
#define DRIFT_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- status */
#define DRIFT_OK            0
/* Bad enum, shape, stride or null pointer; or stochastic rounding that
 * needed a draw with no rng (java/.../fmt/MiniFloat.java:270-272). */
#define DRIFT_EINVAL        1
/* NaN cast into a format with no NaN: Java throws ArithmeticException
 * (java/.../fmt/MiniFloat.java:157-160). */
#define DRIFT_ENAN_FINITE   2
/* A CUDA runtime call failed. */
#define DRIFT_ECUDA         3
/* A bounded device-side wait gave up. */
#define DRIFT_ETIMEOUT      4
/* A valid policy this engine does not implement yet. */
#define DRIFT_EUNSUPPORTED  5
/* Device memory could not be obtained. */
#define DRIFT_ENOMEM        6

/* ------------------------------------------------ enums (Java ordinals) */
/* Formats.ALL order (java/.../fmt/Formats.java:20-48). */
#define DRIFT_FMT_NONE  (-1)   /* NumericPolicy.inputFormat == null: no cast */
#define DRIFT_E4M3      0
#define DRIFT_E5M2      1
#define DRIFT_E2M1      2
#define DRIFT_E3M2      3
#define DRIFT_E2M3      4
#define DRIFT_FP16      5
#define DRIFT_BF16      6
#define DRIFT_NUM_FORMATS 7

/* Rounding (java/.../fmt/Rounding.java:14-20). -1 in a policy's grad_rounding
 * means "same as input_rounding" (NumericPolicy.gradCastRounding). */
#define DRIFT_ROUND_INHERIT   (-1)
#define DRIFT_NEAREST_EVEN    0
#define DRIFT_STOCHASTIC      1
#define DRIFT_TRUNCATE        2

/* NumericPolicy.Scaling (java/.../kernel/NumericPolicy.java:56-63). */
#define DRIFT_SCALE_NONE      0
#define DRIFT_PER_TENSOR      1
#define DRIFT_MX_BLOCK        2

/* NumericPolicy.Acc (java/.../kernel/NumericPolicy.java:26-41). */
#define DRIFT_ACC_FP64        0
#define DRIFT_ACC_FP32        1
#define DRIFT_ACC_FP16        2
#define DRIFT_ACC_BF16        3

/* NumericPolicy.Order (java/.../kernel/NumericPolicy.java:44-53). */
#define DRIFT_SEQUENTIAL      0
#define DRIFT_REVERSED        1
#define DRIFT_PAIRWISE        2
#define DRIFT_BLOCKED         3

/*
 * NumericPolicy flattened to a POD (java/.../kernel/NumericPolicy.java:58-96).
 * A Java caller fills it from the policy object; NumericPolicy.Builder and the
 * named registry stay on the Java side. Formats are DRIFT_* ids or
 * DRIFT_FMT_NONE; grad_format DRIFT_FMT_NONE with a non-null input format
 * means "same as input" (NumericPolicy.gradCastFormat), exactly as a null
 * gradFormat does in Java.
 */
typedef struct drift_policy {
    int32_t input_format;
    int32_t grad_format;
    int32_t input_rounding;
    int32_t grad_rounding;
    int32_t scaling;
    int32_t scale_block;     /* MX block length, Builder default 32 */
    int32_t amax_history;    /* delayed scaling window, 0 = current */
    int32_t mx_headroom;     /* added to the OCP shared exponent */
    int32_t acc;
    int32_t order;
    int32_t acc_block;       /* BLOCKED chunk length, Builder default 32 */
    int32_t acc_rounding;
    int32_t master_fp32;
    int32_t cast_scores;
    int32_t cast_probs;
    int32_t reserved;        /* must be 0 */
} drift_policy;

typedef struct drift_ctx drift_ctx;

/* ------------------------------------------------------------ lifecycle */
/* Opens a context on CUDA device `device` with its own stream. */
DRIFT_API int drift_open(int device, drift_ctx **out);
DRIFT_API int drift_close(drift_ctx *ctx);
/* Message for the calling thread's most recent non-OK status. */
DRIFT_API const char *drift_last_error(void);
/* Build identification string (arch, version). */
DRIFT_API const char *drift_version(void);

/* --------------------------------------------------------- format layer */
/* MiniFloat.maxFinite / minSubnormal of a format
 * (java/.../fmt/MiniFloat.java:61-68, :106). Pure host arithmetic. */
DRIFT_API int drift_format_info(int fmt, double *max_finite, double *min_normal,
                      double *min_subnormal, int32_t *width);

/* MiniFloat.encode(v, rm, rng) over an array, element order
 * (java/.../fmt/MiniFloat.java:156-211). codes[i] is the bit pattern. */
DRIFT_API int drift_encode(drift_ctx *ctx, int fmt, int rounding, const double *v,
                 int32_t *codes, int64_t n, uint64_t *rng_state);

/* MiniFloat.decode(bits) over an array (java/.../fmt/MiniFloat.java:117-142).
 * A code wider than the format is DRIFT_EINVAL, as Java throws. */
DRIFT_API int drift_decode(drift_ctx *ctx, int fmt, const int32_t *codes, double *v,
                 int64_t n);

/*
 * DumpTables (java/.../tools/DumpTables.java:61-124) from the device codec.
 * drift_value_table: the raw double bits of decode(c) for every code c of the
 * format, `bits` holding 2^width entries (values_<fmt>.csv, :61-79).
 * drift_pair_table: rows first .. first+n-1 of pairs_<fmt>.csv, the
 * nearest-even code of the exact product and of the exact sum of a code
 * pair. DRIFT_PAIRS_EXHAUSTIVE: row p is (p / codes, p % codes), p < codes^2
 * (:87-100). DRIFT_PAIRS_SAMPLED: row p uses the Rng draws 2p and 2p+1 of a
 * stream seeded `seed`, each taken as (nextLong() >>> 1) % codes
 * (:106-124; DumpTables seeds 0x51ED1EA5). `a` and `b` may be NULL.
 */
#define DRIFT_PAIRS_EXHAUSTIVE 0
#define DRIFT_PAIRS_SAMPLED    1
DRIFT_API int drift_value_table(drift_ctx *ctx, int fmt, uint64_t *bits);
DRIFT_API int drift_pair_table(drift_ctx *ctx, int fmt, int mode, uint64_t seed, int64_t first,
                     int64_t n, int32_t *a, int32_t *b, int32_t *prod, int32_t *sum);
DRIFT_API int drift_value_table_dev(drift_ctx *ctx, int fmt, uint64_t *d_bits, void *stream);
DRIFT_API int drift_pair_table_dev(drift_ctx *ctx, int fmt, int mode, uint64_t seed,
                         int64_t first, int64_t n, int32_t *d_a, int32_t *d_b,
                         int32_t *d_prod, int32_t *d_sum, void *stream);

/* Dot.round(x, acc, rm, rng) over an array, element order
 * (java/.../kernel/Dot.java:141-182). acc is DRIFT_ACC_FP16 or _BF16. */
DRIFT_API int drift_acc_round(drift_ctx *ctx, int acc, int rounding, const double *x,
                    double *y, int64_t n, uint64_t *rng_state);

/* ---------------------------------------------------------- quant layer */
/* Quant.amax (java/.../kernel/Quant.java:25-34). NaN is ignored. */
DRIFT_API int drift_amax(drift_ctx *ctx, const double *x, int64_t n, double *amax_out);

/* Quant.perTensorScale (java/.../kernel/Quant.java:37-42). Host arithmetic. */
DRIFT_API int drift_per_tensor_scale(int fmt, double amax, double *scale_out);

/*
 * Quant.quantize(src, 0, dst, 0, n, f, p, rm, scale, rng)
 * (java/.../kernel/Quant.java:56-82, MX at :95-123). fmt DRIFT_FMT_NONE copies.
 * clamped_out (may be NULL) receives the Java return value, widened to int64.
 * rng_state may be NULL when no draw is needed; a needed draw with a NULL
 * rng_state is DRIFT_EINVAL (Java: IllegalArgumentException).
 */
DRIFT_API int drift_quantize(drift_ctx *ctx, const drift_policy *p, int fmt,
                   int rounding, const double *src, double *dst, int64_t n,
                   double scale, uint64_t *rng_state, int64_t *clamped_out);

/* ------------------------------------------------------------ dot layer */
/*
 * C[i*c_row_stride + o] = Dot.dot(A, a_off + i*a_row_stride, a_k_stride,
 *                                 B, b_off + o*b_row_stride, b_k_stride,
 *                                 K, p, rng) (+ bias[o] when bias != NULL)
 * for i in [0,M), o in [0,N): the double loops of
 * java/.../train/Pass.java:200-204 (forward), :222-226 (dgrad, B strided),
 * :228-232 (wgrad, both strided), java/.../tools/DotSweep.java:121 (M=N=1)
 * and java/.../tools/RealDotSweep.java:132-139. Dot.dot itself is
 * java/.../kernel/Dot.java:26-121. Strides may be any non-negative values.
 * With a STOCHASTIC accumulator the dots draw from *rng_state in (i, o) order
 * and in each dot's evaluation order, only for inexact sums, exactly as the
 * Java loop does; on return *rng_state is advanced past every draw. A NULL
 * rng_state is DRIFT_EINVAL only if some draw was needed.
 */
DRIFT_API int drift_gemm(drift_ctx *ctx, const drift_policy *p, int64_t M, int64_t N,
               int64_t K, const double *A, int64_t a_off, int64_t a_row_stride,
               int64_t a_k_stride, const double *B, int64_t b_off,
               int64_t b_row_stride, int64_t b_k_stride, const double *bias,
               double *C, int64_t c_row_stride, uint64_t *rng_state);

/* ------------------------------------------ device-resident entry points */
/* As drift_amax; amax lands in the device double *d_amax. */
DRIFT_API int drift_amax_dev(drift_ctx *ctx, const double *d_x, int64_t n,
                   double *d_amax, void *stream);

/*
 * As drift_quantize on device buffers. The per-tensor scale is read from the
 * device double *d_scale when non-NULL, else `scale` is used. Clamp counts are
 * ADDED to the device int64 *d_clamped (may be NULL). For stochastic rounding
 * the Rng state lives in the device uint64 *d_rng_state, which the call
 * advances on the device (no host round trip). Errors raised on the device
 * (NaN into a finite format, a needed draw with d_rng_state NULL) are reported
 * by drift_check_dev.
 */
DRIFT_API int drift_quantize_dev(drift_ctx *ctx, const drift_policy *p, int fmt,
                       int rounding, const double *d_src, double *d_dst,
                       int64_t n, const double *d_scale, double scale,
                       uint64_t *d_rng_state, int64_t *d_clamped,
                       void *stream);

/*
 * `rows` tensors of `len` doubles each (row r at d_src + r*len), each cast as
 * drift_quantize_dev casts one tensor, with its own per-tensor scale
 * (Quant.perTensorScale of the row's own amax) under PER_TENSOR scaling:
 * DotSweep.run's cast of every vector (java/.../tools/DotSweep.java:112-122),
 * one launch for all of them. Clamps are added to d_clamped[r] (int64, may
 * be NULL). Nearest-even or truncate only, and no MX scaling: DRIFT_EINVAL
 * otherwise (cast such rows one by one).
 */
DRIFT_API int drift_quantize_rows_dev(drift_ctx *ctx, const drift_policy *p, int fmt,
                            int rounding, const double *d_src, double *d_dst,
                            int64_t rows, int64_t len, int64_t *d_clamped, void *stream);

/*
 * The number of Rng draws drift_quantize_dev would take for the same
 * arguments, written to the device int64 *d_draws, without casting: one read
 * of d_src. 0 for a rounding other than stochastic. A tensor cast in element
 * order across ranks (one shard per rank, MX blocks not split) starts rank
 * r's stream after the draws of shards 0..r-1: the Rng state advanced by k
 * draws is state + k * 0x9E3779B97F4A7C15 (Rng.java:17-22).
 */
DRIFT_API int drift_quantize_draws_dev(drift_ctx *ctx, const drift_policy *p, int fmt,
                             int rounding, const double *d_src, int64_t n,
                             const double *d_scale, double scale, int64_t *d_draws,
                             void *stream);

/* Quant.perTensorScale (java/.../kernel/Quant.java:37-42) from a device amax
 * into a device scale, so a cast can follow an amax without a host trip. */
DRIFT_API int drift_per_tensor_scale_dev(drift_ctx *ctx, int fmt,
                                         const double *d_amax, double *d_scale,
                                         void *stream);

/*
 * drift_quantize_dev for callers that cannot allocate device memory. No
 * counterpart in the reference: it exists for host programs that reserve all
 * device memory up front under a fixed budget and do not let a library
 * allocate while they run (a cudaMalloc can fail once the budget is spent, and
 * cudaMalloc/cudaFree synchronise the device, stalling the caller's other
 * streams). It takes no drift_ctx, since opening one allocates.
 *
 * The cast is the same as drift_quantize_dev's, bit for bit. Stochastic
 * rounding needs scratch space; it comes from one array of about 1 MiB that
 * the library declares statically, which every GPU that loads the library
 * holds until the process exits. That bounds one stochastic call to
 * DRIFT_NOALLOC_MAX_ITEMS items (groups of 32 elements, or MX blocks of
 * scale_block elements): n up to 8,388,608 elements for an element-wise cast
 * with 32-element items. Larger stochastic calls return DRIFT_ENOMEM and do
 * nothing. Nearest-even and truncating casts use no scratch and have no such
 * limit.
 *
 * The first call on each device that casts (any format but none, any
 * rounding, any n) looks up the array's device address with that device
 * current; make that first call before any stream capture. CUDA loads the
 * library's device code and this array onto a device lazily, when the
 * library first launches work there, unless the process runs with
 * CUDA_MODULE_LOADING=EAGER; a caller whose budget must also cover that load
 * makes one small call (for example a stochastic cast of 32 elements) on
 * each device before its budgeted region. All calls share the array, so
 * calls that overlap on the GPU (other streams, or other threads on the same
 * device) race and must be serialised by the caller. Device-side errors (NaN
 * into a format without NaN, a needed draw with d_rng_state NULL) are ORed
 * into the caller's device int *d_err, which the caller clears and reads.
 * Nothing is allocated or freed by the call.
 */
#define DRIFT_NOALLOC_MAX_ITEMS (1 << 18)
DRIFT_API int drift_quantize_dev_noalloc(const drift_policy *p, int fmt,
                                         int rounding, const double *d_src,
                                         double *d_dst, int64_t n,
                                         const double *d_scale, double scale,
                                         uint64_t *d_rng_state,
                                         int64_t *d_clamped, int *d_err,
                                         void *stream);

/* As drift_gemm on device buffers (offsets folded into the pointers). With a
 * STOCHASTIC accumulator the Rng state is the device uint64 *d_rng_state
 * (required then, ignored otherwise), advanced on the device; that case
 * synchronises the stream once per settling pass. */
DRIFT_API int drift_gemm_dev(drift_ctx *ctx, const drift_policy *p, int64_t M,
                   int64_t N, int64_t K, const double *d_A,
                   int64_t a_row_stride, int64_t a_k_stride, const double *d_B,
                   int64_t b_row_stride, int64_t b_k_stride,
                   const double *d_bias, double *d_C, int64_t c_row_stride,
                   uint64_t *d_rng_state, void *stream);

/* Which path the context's most recent drift_gemm / drift_gemm_dev with a
 * non-stochastic accumulator took (for a host-buffer call that travelled in
 * row chunks, its last chunk):
 *   DRIFT_ROUTE_DOUBLE   0  the double-precision contraction (one launch);
 *   DRIFT_ROUTE_FP32     1  the FP32 pipe: an FP32 accumulator, sequential,
 *                          reversed or blocked in chunks of a multiple of 16,
 *                          at least 2^27 multiply-accumulates, and every
 *                          product of the two operands an exact fp32 number,
 *                          so that Dot.java's (float)(s + a*b) is one fp32 FMA;
 *   DRIFT_ROUTE_SCANNED  2  a candidate for the FP32 pipe whose operand scan
 *                          kept it on the double-precision contraction;
 *   DRIFT_ROUTE_STAGED   3  one output per thread with the operands staged in
 *                          shared memory (one launch): a call too thin for
 *                          the tiled kernel (drift_set_thin_tiles);
 *   DRIFT_ROUTE_PROVEN   4  the double-precision contraction of an FP32 or
 *                          BF16 accumulator without its per-step range
 *                          checks: a scan of both operands proved that every
 *                          partial sum stays in the accumulator's normal range
 *                          below its top binade (nonzero |a|·|b| >= 2^-74, no
 *                          Inf, NaN or subnormal, and the largest magnitudes
 *                          bound K sums below 2^126).
 * Every route gives the same bits; the route is a performance fact.
 * Waits for `stream`. */
#define DRIFT_ROUTE_DOUBLE 0
#define DRIFT_ROUTE_FP32 1
#define DRIFT_ROUTE_SCANNED 2
#define DRIFT_ROUTE_STAGED 3
#define DRIFT_ROUTE_PROVEN 4
DRIFT_API int drift_gemm_route(drift_ctx *ctx, int *route, void *stream);

/* No counterpart in the reference (a performance fact): the number of kernels
 * the context's most recent drift_gemm_dev (or the last chunk of a drift_gemm)
 * with a non-stochastic accumulator queued: the contraction, plus the
 * operand scans, decisions and second contraction builds of the FP32-pipe and
 * range-proof routes (the build the scan does not pick leaves at once). */
DRIFT_API int drift_gemm_launches(drift_ctx *ctx, int *launches);

/* No counterpart in the reference (a tuning knob; results do not change):
 * drift_gemm / drift_gemm_dev calls whose M x N outputs make fewer than
 * `tiles` 64 x 64 tiles run one output per thread instead of on the tiled
 * kernel, so that a thin call (a batch-64 linear layer) still reaches every
 * SM. Negative restores the default, measured per policy: below two thirds
 * of a tile per SM (98 tiles on a B200) for sequential, reversed and
 * 32-aligned blocked orders with an FP32/FP16/BF16 accumulator, below a third
 * (49) otherwise. 0 sends every call to the tiled kernel. */
DRIFT_API int drift_set_thin_tiles(drift_ctx *ctx, int64_t tiles);

/* Error sums of RealDotSweep's RMS ratio
 * (java/.../tools/RealDotSweep.java:130-142): ADDS sum((got-exact)^2) to
 * d_sums[0] and sum(exact^2) to d_sums[1]. */
DRIFT_API int drift_error_sums_dev(drift_ctx *ctx, const double *d_got,
                                   const double *d_exact, int64_t n,
                                   double *d_sums, void *stream);

/*
 * Exact order statistics of the relative error |got - exact| / |exact| over
 * all n outputs (the medians of java/.../tools/DotSweep.java:152-153 and
 * RealDotSweep.java:140-141), by radix selection on the double's bits in
 * DRIFT_RADIX_PASSES passes. d_state holds two uint64: the digits chosen so
 * far (start at 0) and the 0-based rank sought (start at k). Each pass:
 * drift_radix_hist_dev clears d_hist (DRIFT_RADIX_BINS uint64) and counts the
 * next digit of the elements still in play; several ranks may then sum their
 * d_hist (all-reduce) so the selection runs over all of their outputs; then
 * drift_radix_select_dev picks the digit. After the last pass d_state[0] is
 * the bit pattern of the k-th smallest relative error (NaN, from 0/0, sorts
 * after +Inf as Java's sort places it).
 */
#define DRIFT_RADIX_PASSES 6
#define DRIFT_RADIX_BINS 2048
DRIFT_API int drift_radix_hist_dev(drift_ctx *ctx, const double *d_got,
                                   const double *d_exact, int64_t n, int pass,
                                   const uint64_t *d_state, uint64_t *d_hist,
                                   void *stream);
DRIFT_API int drift_radix_select_dev(drift_ctx *ctx, int pass,
                                     const uint64_t *d_hist, uint64_t *d_state,
                                     void *stream);

/*
 * The same order statistic within each of `groups` groups of n outputs
 * (group g holds d_got[g*n .. g*n+n) and the same span of d_exact): writes
 * the k-th smallest relative error of group g (0 <= k < n) to d_out[g], NaN
 * sorting after +Inf. One launch for many small groups, such as the
 * per-(policy, length) medians over DotSweep's seeds
 * (java/.../tools/DotSweep.java:152-153). n <= DRIFT_GROUP_MAX.
 */
#define DRIFT_GROUP_MAX 4096
DRIFT_API int drift_group_kth_rel_error_dev(drift_ctx *ctx, const double *d_got,
                                            const double *d_exact, int64_t groups,
                                            int64_t n, int64_t k, double *d_out,
                                            void *stream);

/*
 * RealDotSweep's per-policy loop (java/.../tools/RealDotSweep.java:119-142) in
 * one call on host tensors: X (M x K) and W (N x K), row-major, cross to the
 * device once; the exact FP64 contraction (:88-95); then for each of
 * n_policies policies, in order: an Rng seeded rng_seed (:122), the
 * whole-tensor per-tensor scales (Quant.perTensorScale of Quant.amax, :125-126;
 * computed only under PER_TENSOR scaling, the one that reads them), the casts
 * of X then W (Quant.quantize with the policy's input format, rounding and
 * scaling, :127-128), the contraction (Dot.dot over every (row of X, row of W)
 * pair, :132-139), and its statistics against the exact outputs.
 * stats_out[4p .. 4p+3] receives, for policy p: the true median of
 * |got - exact| / |exact| (the mean of the two middle values, :140-141), the
 * RMS ratio sqrt(sum (got-exact)^2 / sum exact^2) (:142, :149-155; a parallel
 * sum, so equal to the sequential one to rounding), the clamp count of X's
 * cast and of W's. Only the statistics come back. Returns when they are in
 * stats_out.
 */
DRIFT_API int drift_real_dot_sweep(drift_ctx *ctx, const drift_policy *policies,
                                   int n_policies, int64_t M, int64_t N, int64_t K,
                                   const double *X, const double *W, uint64_t rng_seed,
                                   double *stats_out);

/* ----------------------------------------------------------- diagnostics */
/*
 * A batched contraction with per-row windows: the attention matmuls of
 * AttnPass (java/.../train/AttnPass.java:245-290, :373-427), and a batched
 * drift_gemm. For t < batch, i < rows, o < cols the output
 *   C[c_off + t*c_batch + i*c_row + o*c_col]
 * is Dot.dot(A, a_off + t*a_batch + i*a_row + lo*a_k, a_k,
 *            B, b_off + t*b_batch + o*b_col + lo*b_k, b_k, n, p, rng)
 * times alpha (when alpha != 1: the score scale, :248), added into C when
 * `accumulate` is set (dInput into dx, :478-484). The window (lo, n) of row i:
 *   DRIFT_WINDOW_FULL    lo = 0, n = depth (scores, dProb: :245-255, :373-381)
 *   DRIFT_WINDOW_PREFIX  lo = 0, n = i + 1 (context, dq: :283-288, :412-417)
 *   DRIFT_WINDOW_SUFFIX  lo = i, n = depth - i (dv, dk: :382-388, :419-424)
 * PREFIX and SUFFIX need rows <= depth. With `causal` set, outputs with
 * o > i are written 0.0 and take no dot (and no draws). Dots run, and a
 * stochastic accumulator draws, in (t, i, o) order. C must not overlap A or B.
 */
#define DRIFT_WINDOW_FULL   0
#define DRIFT_WINDOW_PREFIX 1
#define DRIFT_WINDOW_SUFFIX 2
typedef struct drift_contraction {
    int64_t batch, rows, cols, depth;
    int64_t a_off, a_batch, a_row, a_k;
    int64_t b_off, b_batch, b_col, b_k;
    int64_t c_off, c_batch, c_row, c_col;
    double alpha;
    int32_t window;
    int32_t causal;
    int32_t accumulate;
    int32_t reserved;    /* must be 0 */
} drift_contraction;

/* Host buffers a[a_len], b[b_len], c[c_len] (Java arrays): every element the
 * contraction reaches must lie inside them, or DRIFT_EINVAL. c is read
 * (accumulate) and written in place. The Rng state travels as with
 * drift_gemm. */
DRIFT_API int drift_contract(drift_ctx *ctx, const drift_policy *p, const drift_contraction *op,
                   const double *a, int64_t a_len, const double *b, int64_t b_len,
                   double *c, int64_t c_len, uint64_t *rng_state);
/* Device buffers on `stream`; the Rng state is the device uint64
 * *d_rng_state, needed only by a stochastic accumulator. */
DRIFT_API int drift_contract_dev(drift_ctx *ctx, const drift_policy *p,
                       const drift_contraction *op, const double *d_a,
                       const double *d_b, double *d_c, uint64_t *d_rng_state,
                       void *stream);

/* ---------------------------------------- device-resident training step */
/*
 * The arithmetic of Pass/Trainer around the casts and contractions
 * (java/.../train/Pass.java, Trainer.java), on device buffers, so a training
 * step keeps its weights, casts, gradients and Adam moments on the GPU. Each
 * keeps the Java loop order; results equal the host loops bit for bit.
 */
/* Pass.forward's lookup (Pass.java:122-126): out row r = table row
 * tokens[r], rows of `width`. A token outside [0, vocab) is reported by
 * drift_check_dev as DRIFT_EINVAL. */
DRIFT_API int drift_embed_gather_dev(drift_ctx *ctx, const int32_t *d_tokens, int64_t n_tok,
                           const double *d_table, int64_t vocab, int64_t width,
                           double *d_out, void *stream);
/* Pass.backward's embedding gradient (Pass.java:168-179): table_grad row v
 * += rows[r] for every r with tokens[r] == v, in increasing r. */
DRIFT_API int drift_embed_grad_dev(drift_ctx *ctx, const int32_t *d_tokens, int64_t n_tok,
                         const double *d_rows, int64_t width, double *d_table_grad,
                         int64_t vocab, void *stream);
/* Pass.linearBackward's bias gradient (Pass.java:234-240): db[o] = the sum
 * of dy[i*cols + o] over i in order. */
DRIFT_API int drift_bias_grad_dev(drift_ctx *ctx, const double *d_dy, int64_t rows,
                        int64_t cols, double *d_db, void *stream);
/* Pass.tanhBackward (Pass.java:279-283): grad[i] *= 1 - out[i]^2. */
DRIFT_API int drift_tanh_backward_dev(drift_ctx *ctx, const double *d_out, double *d_grad,
                            int64_t n, void *stream);
/* Pass.scaleFor with an amax history (Pass.java:249-271): the scale from the
 * largest of the last min(count, len) amaxes (this step's when count is 0),
 * then this step's amax recorded and *d_count advanced. */
DRIFT_API int drift_scale_for_dev(drift_ctx *ctx, int fmt, const double *d_amax_now,
                        double *d_history, int32_t history_len, int64_t *d_count,
                        double *d_scale, void *stream);
/* Trainer.adam for one tensor at `step` (1-based; Trainer.java:246-269),
 * FP32 masters rounding weight and moments to float. */
DRIFT_API int drift_adam_dev(drift_ctx *ctx, double *d_param, const double *d_grad,
                   double *d_m, double *d_v, int64_t n, int32_t step, double lr,
                   int32_t fp32_master, void *stream);

/* No counterpart in the reference: measures the FP64 pipe's DMUL+DADD issue
 * rate on the context's device (operations per second), the denominator of
 * the contraction's roofline. Takes a few milliseconds. */
DRIFT_API int drift_probe_fp64(drift_ctx *ctx, double *ops_per_s);

/* No counterpart in the reference: measures the FP32 pipe's FFMA issue rate
 * (fused multiply-adds per second), the denominator of the FP32-pipe
 * contraction's roofline (drift_gemm_route). Takes a few milliseconds. */
DRIFT_API int drift_probe_fp32(drift_ctx *ctx, double *fma_per_s);

/*
 * Synchronises `stream` and returns the first device-side error raised since
 * the last check on this context (DRIFT_ENAN_FINITE, DRIFT_EINVAL,
 * DRIFT_ETIMEOUT), clearing it.
 */
DRIFT_API int drift_check_dev(drift_ctx *ctx, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* DRIFT_B200_H */
