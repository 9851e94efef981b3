// gemm.cu — the emulated contraction: C[i,o] = Dot.dot(A row i, B row o, K).
//
// Device form of the (i, o) loops of java/src/main/java/io/drift/train/
// Pass.java:200-232 over Dot.dot (java/src/main/java/io/drift/kernel/
// Dot.java:26-121). Tensor cores are not used: the order of the additions is
// the quantity under study, so every output runs its own scalar chain in
// exactly the Java order, and parallelism comes only from independent outputs.
//
// Per multiply-accumulate: one DMUL and one DADD (never fused: Java rounds the
// product to double before the add, Dot.java:46/:54/:63) and, for the FP32,
// FP16 and BF16 accumulators, the fast rounding of codec.cuh (FastForm: one
// LOP3 and two DFMAs), its range words folded and checked once per group of
// eight or sixteen of a thread's outputs.
//
// Tiling. A CTA of 256 threads owns a 64x64 output tile; thread (ty, tx) owns
// rows ty + 16i and columns tx + 16j (i, j < 4), so the sixteen threads that
// share a row read sixteen consecutive B rows. K advances in tiles of 16
// through a 3-stage shared-memory ring laid out [row][18]: 16 k values and a
// 2-double pad, so consecutive rows start 4 banks apart. (Measured on B200,
// this layout takes a quarter fewer shared-memory wavefronts per load than a
// dense swizzled or k-pair-planar tile.)
//
// K-contiguous operands with 16-byte-aligned rows are fetched by the Tensor
// Memory Accelerator: one elected thread issues one cp.async.bulk.tensor.2d per
// operand per stage with a box 18 doubles wide, which lands directly in the
// padded layout (the two extra doubles are the next tile's first k values, or
// zero fill past K); completion is counted on the stage's mbarrier
// (expect_tx), and the other threads spend no instructions on loads. (On B200
// this beat per-thread cp.async staging for every accumulator: +10% for FP64,
// +3% for FP32, +12% for pairwise.) Other strides (the dgrad / wgrad
// operands, Pass.java:224, :230) go through a register loader that writes the
// same layout. The summation order never depends on the staging.
//
// Every wait on an mbarrier is bounded: a stage that does not arrive within
// the limit raises DEV_ERR_TIMEOUT in the context's error word and the CTA
// leaves together (the decision is made CTA-wide), instead of spinning.
//
// Orders. SEQUENTIAL and REVERSED walk k up or down. BLOCKED folds each
// acc_block chunk into an FP32 total (FP64 for FP64 accumulation,
// Dot.java:104-121). PAIRWISE follows Dot.pairwise (half = count >>> 1,
// leaves of at most 8, Dot.java:86-102). When acc_block is a multiple of 16,
// or K is a power of two >= 16 (every leaf 8 long, every split exact), chunk
// and leaf boundaries fall on tile boundaries and all segment work happens
// once per tile: a 16-wide tile is one level-1 node of the pairwise tree and
// the tiles combine as a perfect binary tree (ctz(t+1) merges after tile t).
// Other shapes use a leaf schedule built on the host from the same recursion,
// checked once per k. Either way the schedule is the same for every output,
// so control flow is uniform across the CTA.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <type_traits>
#include <vector>

#include <cuda.h>

#include "codec.cuh"
#include "internal.h"
#include "tma.cuh"

namespace drift {

constexpr int BM = 64, BN = 64, BK = 16, TM = 4, TN = 4, GEMM_THREADS = 256;
constexpr int STAGES = 3;
constexpr int LDK = BK + 2;                      // padded row length, in doubles
constexpr int STAGE_DOUBLES = (BM + BN) * LDK;   // one A tile and one B tile
constexpr int TILE_BYTES = BM * LDK * (int)sizeof(double);  // 9 KiB per operand per stage
// Stages plus the stage barriers.
constexpr int GEMM_SMEM = STAGES * STAGE_DOUBLES * (int)sizeof(double) + 64;
// Pairwise leaves over a full tile are validated once per tile (mac16_run,
// one check, the two leaves redone exactly from zero on a miss) for the FP32
// and BF16 accumulators. Measured at 8192^3 on one B200: FP32 pairwise +8%.
// Not for FP16, whose normal range starts at 2^-14: on N(0,1) x lognormal
// data about 0.1% of products fall below it, so a thread's tile misses about
// 3.7% of the time, and a warp redoes the tile when any of its 32 lanes
// misses, 70% of warp-tiles (2.5x slower). Nor for the sequential and blocked
// orders, which lost 4-5% with a tile-start copy of the accumulators in
// shared memory to restart from.
template <int ACC, int ORDER>
constexpr bool tile_validated() {
    return ORDER == DRIFT_PAIRWISE && (ACC == DRIFT_ACC_FP32 || ACC == DRIFT_ACC_BF16);
}
constexpr int kMaxPairwiseDepth = 30;  // stack depth; enough for any int32 K
// Unroll of the k-pair loop of a full tile, chosen by measurement on B200:
// the narrow accumulators' rounding makes a long tile body fall out of the
// instruction cache, so they unroll less (pairwise least, as its per-tile
// merge code is the largest); FP64/FP32 bodies are small and unroll fully.
// (With FastForm's shorter step, FP16/BF16 sequential gained 3% going from
// 2 to 4.)
template <int ACC, int ORDER>
constexpr int kp_unroll() {
    return ORDER == DRIFT_PAIRWISE ? 1 : (ACC == DRIFT_ACC_FP64 || ACC == DRIFT_ACC_FP32) ? 8 : 4;
}

enum SegMode { SEG_NONE = 0, SEG_TILE = 1, SEG_SCHED = 2 };

// The proven FP32/BF16 builds round a thread's four output columns on three
// pipes: the last column on the conversion pipe (cvt to float / bf16 and
// back, step_cvt), the int_cols columns before it on the integer pipes
// (step_int), the rest on the FP64 pipe (step). Splitting the rounding lifts
// the FP64 pipe's share below four operations per MAC. Measured at 8192^3 on
// one B200 against every column on the FP64 pipe:
//   conversion column + one integer column: FP32 sequential +8.6%, pairwise
//     +5.3%, blocked +7.7%; BF16 sequential +7.9%, pairwise +5.2%, blocked
//     +5.7%;
//   + a second integer column: FP32 sequential and blocked another +1.9% and
//     +1.0%, FP32 pairwise -1.0%, BF16 sequential and blocked -2.6% and
//     -3.4% (so FP32 sequential and blocked only);
//   integer columns alone, one / two: FP32 sequential +5.1% / +6.3%, BF16
//     sequential +2.5% / +5.0%;
//   two conversion columns saturate that pipe: FP32 sequential +0.6%.
template <int ACC, int RM, bool PROVEN>
constexpr bool cvt_col() {
    return PROVEN && RM == DRIFT_NEAREST_EVEN && (ACC == DRIFT_ACC_FP32 || ACC == DRIFT_ACC_BF16);
}
template <int ACC, int ORDER, int RM, bool PROVEN>
constexpr int int_cols() {
    if (!cvt_col<ACC, RM, PROVEN>()) return 0;
    return ACC == DRIFT_ACC_FP32 && ORDER != DRIFT_PAIRWISE ? 2 : 1;
}

// The accumulator rounding of a contraction. PROVEN: an operand scan showed
// that every sum of this call stays inside the fast form's exact range (see
// range_proven below), so no sum is checked and no group is ever redone.
template <int ACC, int RM, bool PROVEN>
struct GemmRound : AccRound<ACC, RM> {
    __device__ static bool valid(unsigned run) { return PROVEN || AccRound<ACC, RM>::valid(run); }
};

struct GemmArgs {
    int64_t M, N, K;
    const double *A;
    int64_t a_rs, a_ks;
    const double *B;
    int64_t b_rs, b_ks;
    const double *bias;
    double *C;
    int64_t c_rs;
    int64_t acc_block;
    const uint8_t *leaf_len;     // SEG_SCHED PAIRWISE: length of each leaf, in k order
    const uint8_t *leaf_merges;  // SEG_SCHED PAIRWISE: combines after each leaf
    int a_tma, b_tma;            // operand has a TMA map
    int *err;                    // context error word (timeouts)
    // Batched launches (blockIdx.z): element strides between the problems,
    // and for a TMA operand the same stride in rows of its map.
    int64_t a_bs, b_bs, c_bs;
    int64_t a_brows, b_brows;
    // When set, the kernel leaves at once if the word reads nonzero: the FP32
    // path (gemm32.cu) took the call.
    const int *skip;
    // When set, the operand scan's words (range_scan_kernel): the PROVEN
    // build runs if they prove the call's range, the checked build otherwise,
    // and the other leaves at once. range_limit bounds the sum of the two
    // operands' top exponents (range_limit_for).
    const unsigned *range;
    int range_limit;
    int *route;  // receives DRIFT_ROUTE_PROVEN from the PROVEN build when it runs
};

// Offset, in doubles, of element (row, k) of a staged operand tile.
__device__ __forceinline__ int tile_off(int row, int k) { return row * LDK + k; }

// The fast rounding is validated for a group of a thread's outputs at a time:
// one branch per group, and a miss recomputes that group exactly. Groups of
// two rows (eight sums) keep the temporaries small where the kernel is
// register-tight (pairwise, blocked). The sequential orders validate all
// sixteen sums of a k step at once: at 8192^3 on one B200 that measured 4.1%
// faster for FP16/BF16 and 0.8% for FP32, while it cost BF16 pairwise 5.7%.
constexpr int GROUP_ROWS = 2;

template <int ORDER>
constexpr int mac_group() {
    return ORDER == DRIFT_SEQUENTIAL || ORDER == DRIFT_REVERSED ? TM : GROUP_ROWS;
}

// One k step for the thread's 16 outputs: acc = round(acc + a_i * b_j), the
// rounded value written straight into the accumulator. Each group of G rows
// folds its sums' range words into one word, checked once: a miss (zero, the
// accumulator's subnormal range, its top binade, Inf, NaN) recomputes that
// group's sums exactly from the kept sums.
// FIRST starts a fresh sum: acc = round(0.0 + a_i * b_j), whatever acc held
// (0.0 + p is not p when p is -0.0, so the add stays).
template <int ACC, int RM, int G = GROUP_ROWS, bool FIRST = false, bool PV = false, int NI = 0>
__device__ __forceinline__ void mac16(double (&acc)[TM][TN], const double (&a)[TM],
                                      const double (&b)[TN]) {
    using R = GemmRound<ACC, RM, PV>;
    constexpr int CV = cvt_col<ACC, RM, PV>() ? 1 : 0;
    if constexpr (ACC == DRIFT_ACC_FP64) {
#pragma unroll
        for (int i = 0; i < TM; i++)
#pragma unroll
            for (int j = 0; j < TN; j++)
                acc[i][j] = __dadd_rn(FIRST ? 0.0 : acc[i][j], __dmul_rn(a[i], b[j]));
    } else {
#pragma unroll
        for (int i0 = 0; i0 < TM; i0 += G) {
            double t[G][TN];       // the sums, kept until the group is validated
            unsigned run = 0, u[G][TN];
#pragma unroll
            for (int i = 0; i < G; i++)
#pragma unroll
                for (int j = 0; j < TN; j++) {
                    t[i][j] = __dadd_rn(FIRST ? 0.0 : acc[i0 + i][j], __dmul_rn(a[i0 + i], b[j]));
                    if constexpr (CV == 1) {
                        if (j == TN - 1) {
                            acc[i0 + i][j] = R::step_cvt(t[i][j]);
                            u[i][j] = 0;
                            continue;
                        }
                    }
                    acc[i0 + i][j] =
                        j >= TN - CV - NI
                            ? R::step_int(t[i][j], u[i][j])
                            : R::step(t[i][j], FIRST ? 0 : __double2loint(acc[i0 + i][j]), u[i][j]);
                }
#pragma unroll
            for (int i = 0; i < G; i++)
#pragma unroll
                for (int j = 0; j < TN; j += 2) run = R::fold2(run, u[i][j], u[i][j + 1]);
            if (!R::valid(run)) {  // rare: round these sums exactly
#pragma unroll
                for (int i = 0; i < G; i++)
#pragma unroll
                    for (int j = 0; j < TN; j++) acc[i0 + i][j] = R::exact(t[i][j]);
            }
        }
    }
}

// One k step of a full tile: as mac16, but the sums' range words are folded
// into `run`, which the caller checks once for the whole tile. No sum is kept
// for a recompute: a tile that misses is redone from its start (redo_*).
template <int ACC, int RM, bool FIRST = false, bool PV = false, int NI = 0>
__device__ __forceinline__ void mac16_run(double (&acc)[TM][TN], const double (&a)[TM],
                                          const double (&b)[TN], unsigned &run) {
    using R = GemmRound<ACC, RM, PV>;
    constexpr int CV = cvt_col<ACC, RM, PV>() ? 1 : 0;
#pragma unroll
    for (int i = 0; i < TM; i++) {
        unsigned u[TN];
#pragma unroll
        for (int j = 0; j < TN; j++) {
            const double t = __dadd_rn(FIRST ? 0.0 : acc[i][j], __dmul_rn(a[i], b[j]));
            if constexpr (CV == 1) {
                if (j == TN - 1) {
                    acc[i][j] = R::step_cvt(t);
                    u[j] = 0;
                    continue;
                }
            }
            acc[i][j] = j >= TN - CV - NI ? R::step_int(t, u[j])
                                          : R::step(t, FIRST ? 0 : __double2loint(acc[i][j]), u[j]);
        }
#pragma unroll
        for (int j = 0; j < TN; j += 2) run = R::fold2(run, u[j], u[j + 1]);
    }
}

// A tile's k steps [k0, k1) (in reverse when REV) with the exact rounding,
// into acc (Dot.java:50-68): the rare path of a tile whose fast steps left the
// accumulator's normal range. The tile is still in shared memory.
template <int ACC, int RM, bool REV>
__device__ __forceinline__ void redo_steps(const double *sA, const double *sB, int ty, int tx,
                                           int k0, int k1, double (&acc)[TM][TN]) {
    using R = AccRound<ACC, RM>;
#pragma unroll 1
    for (int q = k0; q < k1; q++) {
        const int kk = REV ? k1 - 1 - (q - k0) : q;
        double a[TM], b[TN];
#pragma unroll
        for (int i = 0; i < TM; i++) a[i] = sA[tile_off(ty + 16 * i, kk)];
#pragma unroll
        for (int j = 0; j < TN; j++) b[j] = sB[tile_off(tx + 16 * j, kk)];
#pragma unroll
        for (int i = 0; i < TM; i++)
#pragma unroll
            for (int j = 0; j < TN; j++)
                acc[i][j] = R::exact(__dadd_rn(acc[i][j], __dmul_rn(a[i], b[j])));
    }
}

// Fold of a BLOCKED chunk into the running total (Dot.java:104-121): the
// total is a float for every accumulator but FP64.
template <int ACC>
__device__ __forceinline__ void blocked_fold(double (&tot)[TM][TN], double (&acc)[TM][TN]) {
#pragma unroll
    for (int i = 0; i < TM; i++)
#pragma unroll
        for (int j = 0; j < TN; j++) {
            const double t = __dadd_rn(tot[i][j], acc[i][j]);
            tot[i][j] = ACC == DRIFT_ACC_FP64 ? t : (double)__double2float_rn(t);
            acc[i][j] = 0.0;
        }
}

// Pairwise combine of the stack top with the current node (Dot.java:97-101):
// right = round(left + right), validated in groups of GROUP_ROWS rows.
template <int ACC, int RM, bool PV = false>
__device__ __forceinline__ void combine(const double (&left)[TM][TN], double (&right)[TM][TN]) {
    using R = GemmRound<ACC, RM, PV>;
    constexpr int CV = cvt_col<ACC, RM, PV>() ? 1 : 0;
    constexpr int NI = int_cols<ACC, DRIFT_PAIRWISE, RM, PV>();
#pragma unroll
    for (int i0 = 0; i0 < TM; i0 += GROUP_ROWS) {
        double t[GROUP_ROWS][TN];
        unsigned run = 0, u[GROUP_ROWS][TN];
#pragma unroll
        for (int i = 0; i < GROUP_ROWS; i++)
#pragma unroll
            for (int j = 0; j < TN; j++) {
                t[i][j] = __dadd_rn(left[i0 + i][j], right[i0 + i][j]);
                if constexpr (CV == 1) {
                    if (j == TN - 1) {
                        right[i0 + i][j] = R::step_cvt(t[i][j]);
                        u[i][j] = 0;
                        continue;
                    }
                }
                right[i0 + i][j] = j >= TN - CV - NI
                                       ? R::step_int(t[i][j], u[i][j])
                                       : R::step(t[i][j], __double2loint(right[i0 + i][j]), u[i][j]);
            }
#pragma unroll
        for (int i = 0; i < GROUP_ROWS; i++)
#pragma unroll
            for (int j = 0; j < TN; j += 2) run = R::fold2(run, u[i][j], u[i][j + 1]);
        if (!R::valid(run)) {
#pragma unroll
            for (int i = 0; i < GROUP_ROWS; i++)
#pragma unroll
                for (int j = 0; j < TN; j++) right[i0 + i][j] = R::exact(t[i][j]);
        }
    }
}

// ------------------------------------------------------------------ range proof
//
// The fast rounding (FastForm) is exact for every sum t with 2^-126 <= |t| <
// 2^127, the FP32 and BF16 accumulators' normal range below their top binade;
// the checks exist for the sums outside it. For FP32 and BF16 the operands
// alone can prove that no sum of a call leaves that range:
//
//  - Low side. If every nonzero |a| >= 2^la and |b| >= 2^lb with la + lb >=
//    -74, every product is zero or at least 2^-74 in magnitude, and its double
//    is then a multiple of its ulp, at least 2^-126. The sums start at +0, and
//    a sum or a rounding of multiples of 2^-126 is again one: a double sum
//    rounds to a coarser grid or is exact, and a value below 2^-103 (FP32) or
//    2^-119 (BF16) that is a multiple of 2^-126 has at most 24 (8) significant
//    bits, so the accumulator holds it as is. So a nonzero sum is at least
//    2^-126. A zero sum is +0: it is x + (-x), or +0 plus a zero, as no
//    chain value is ever -0 (a nonzero sum never rounds to zero).
//  - High side. With |a| < 2^(ta+1) and |b| < 2^(tb+1), every product's
//    double is at most 2^(ta+tb+2), and a sum over k of them, each step rounded
//    to double and to the accumulator (relative error at most d each), is at
//    most k * 2^(ta+tb+2) * (1+d)^k. Pairwise nodes and blocked chunks sum
//    subsets with fewer roundings. range_limit_for bounds ta + tb + 2 so that
//    this stays at or below 2^126.
//
// One scan of each operand gives la, ta and whether it holds Inf, NaN or a
// subnormal; each contraction build reads the words and either runs or
// leaves, so the decision never waits on the host.

constexpr int kRangeWords = 4;  // per operand: top exponent field, 2047 - lowest, bad, unused
// Below this many multiply-accumulates the scan's launch costs more than the
// checks it removes.
constexpr double kRangeMinMacs = 134217728.0;  // 2^27

// Folds one element into the scan maxima: [0] largest biased exponent,
// [1] 2047 - smallest biased exponent of a nonzero element, [2] Inf, NaN or a
// subnormal seen. Zeros are skipped; an operand of zeros leaves [0] == 0.
__device__ __forceinline__ void range_fold(double x, unsigned &top, unsigned &low, unsigned &bad) {
    const unsigned hi = (unsigned)__double2hiint(x) & 0x7FFFFFFFu;
    const unsigned ef = hi >> 20;
    if (ef == 0x7FF || (ef == 0 && (hi | (unsigned)__double2loint(x)) != 0)) bad = 1;
    if (ef != 0 && ef != 0x7FF) {
        top = max(top, ef);
        low = max(low, 2047u - ef);
    }
}

// Scans operand blockIdx.y (0: A with rows_a rows, 1: B with rows_b) into
// words[4 * y ..]. Rows are K long, element (r, k) at X[r*rs + k*ks].
// Contiguous operands are read 16 bytes at a time.
__global__ void __launch_bounds__(256) range_scan_kernel(const double *A, int64_t rows_a,
                                                         int64_t a_rs, int64_t a_ks,
                                                         const double *B, int64_t rows_b,
                                                         int64_t b_rs, int64_t b_ks, int64_t K,
                                                         unsigned *words) {
    const bool second = blockIdx.y == 1;
    const double *X = second ? B : A;
    const int64_t rows = second ? rows_b : rows_a, rs = second ? b_rs : a_rs;
    const int64_t ks = second ? b_ks : a_ks;
    unsigned top = 0, low = 0, bad = 0;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t first = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (ks == 1 && (rs == K || rows == 1)) {  // one contiguous span
        const int64_t n = rows * K;
        const bool aligned = ((uintptr_t)X & 15) == 0;
        const int64_t n2 = aligned ? n / 2 : 0;
        const double2 *X2 = reinterpret_cast<const double2 *>(X);
        for (int64_t i = first; i < n2; i += stride) {
            const double2 v = X2[i];
            range_fold(v.x, top, low, bad);
            range_fold(v.y, top, low, bad);
        }
        for (int64_t i = 2 * n2 + first; i < n; i += stride) range_fold(X[i], top, low, bad);
    } else {  // any strides: walk the unit-stride axis innermost
        const bool kfast = ks == 1 || rs != 1;
        const int64_t inner = kfast ? K : rows, outer = kfast ? rows : K;
        const int64_t si = kfast ? ks : rs, so = kfast ? rs : ks;
        for (int64_t o = blockIdx.x; o < outer; o += gridDim.x)
            for (int64_t i = threadIdx.x; i < inner; i += blockDim.x)
                range_fold(X[o * so + i * si], top, low, bad);
    }
    top = __reduce_max_sync(0xFFFFFFFFu, top);
    low = __reduce_max_sync(0xFFFFFFFFu, low);
    bad = __reduce_max_sync(0xFFFFFFFFu, bad);
    if ((threadIdx.x & 31) == 0) {
        unsigned *w = words + (second ? kRangeWords : 0);
        if (top) atomicMax(&w[0], top);
        if (low) atomicMax(&w[1], low);
        if (bad) atomicMax(&w[2], bad);
    }
}

// Whether the scan words prove the call's range (see above).
__device__ __forceinline__ bool range_proven(const unsigned *w, int limit) {
    const unsigned *a = w, *b = w + kRangeWords;
    if (a[2] | b[2]) return false;           // Inf, NaN or a subnormal
    if (a[0] == 0 || b[0] == 0) return true;  // an operand of zeros: every sum is +0
    const int ta = (int)a[0] - 1023, tb = (int)b[0] - 1023;
    const int la = 2047 - (int)a[1] - 1023, lb = 2047 - (int)b[1] - 1023;
    return la + lb >= -74 && ta + tb + 2 <= limit;
}

// The bound on ta + tb + 2 for K terms: 126 - ceil(log2 K) - ceil(log2 of
// (1+d)^(K+1)), d the relative error of a double add followed by the
// accumulator's rounding. Negative when K is too long for any proof.
static int range_limit_for(int acc, int64_t K) {
    const double u = acc == DRIFT_ACC_FP32 ? std::ldexp(1.0, -24) : std::ldexp(1.0, -8);
    const double d = u + std::ldexp(1.0, -53) + u * std::ldexp(1.0, -53);
    const double growth = (double)(K + 1) * std::log1p(d) / std::log(2.0);
    if (!(growth < 256.0)) return -1024;
    int lg = 0;
    while (lg < 63 && (int64_t(1) << lg) < K) lg++;
    return 126 - lg - (int)std::ceil(growth + 1e-9);
}

// One 18 x 64 box of doubles (k0 .. k0+17 of rows r0 .. r0+63) into a tile.
__device__ __forceinline__ void tma_load_box(double *dst, const CUtensorMap *map, int k0, int r0,
                                             uint64_t *bar) {
    tma_load_2d(dst, map, k0, r0, bar);
}

// The register loader: rows [r0, r0+64) x k [k0, k0+16) of any-strided X into
// the padded layout, coalescing along whichever axis has unit stride.
__device__ __forceinline__ void stage_generic(double *s, const double *X, int64_t rows, int64_t r0,
                                              int64_t rs, int64_t ks, int64_t k0, int64_t K,
                                              int tid) {
    const bool kfast = ks == 1 || rs != 1;
#pragma unroll
    for (int e = tid; e < BM * BK; e += GEMM_THREADS) {
        const int kk = kfast ? (e & 15) : (e >> 6);
        const int rr = kfast ? (e >> 4) : (e & 63);
        const int64_t r = r0 + rr, k = k0 + kk;
        s[tile_off(rr, kk)] = (r < rows && k < K) ? X[r * rs + k * ks] : 0.0;
    }
}

// BATCH instantiations read the problem index from blockIdx.z; the others are
// compiled for one problem, with every batch offset folded away.
template <int ACC, int ORDER, int RM, int SEG, bool BATCH, bool PV>
__global__ void __launch_bounds__(GEMM_THREADS, 2)
    gemm_kernel(const GemmArgs g, const __grid_constant__ CUtensorMap tmA,
                const __grid_constant__ CUtensorMap tmB) {
    extern __shared__ __align__(128) double smem[];
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + STAGES * STAGE_DOUBLES);
    constexpr bool REV = ORDER == DRIFT_REVERSED;
    constexpr bool PAIR = ORDER == DRIFT_PAIRWISE;
    constexpr bool BLOCK = ORDER == DRIFT_BLOCKED;

    if (g.skip && *g.skip) return;
    const int tid = threadIdx.x;
    if (g.range) {  // the scan decides which build runs; the other leaves
        if (range_proven(g.range, g.range_limit) != PV) return;
        if (PV && g.route && tid == 0 && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0)
            *g.route = DRIFT_ROUTE_PROVEN;
    }
    const int tx = tid & 15, ty = tid >> 4;
    const int64_t m0 = (int64_t)blockIdx.y * BM;
    const int64_t n0 = (int64_t)blockIdx.x * BN;
    const int64_t K = g.K;
    const int64_t T = (K + BK - 1) / BK;
    // The problem of a batched launch and its operands (all offsets fold to
    // zero in a one-problem build).
    const int64_t z = BATCH ? (int64_t)blockIdx.z : 0;
    const double *Az = g.A + z * g.a_bs;
    const double *Bz = g.B + z * g.b_bs;
    double *Cz = g.C + z * g.c_bs;

    double acc[TM][TN], tot[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; i++)
#pragma unroll
        for (int j = 0; j < TN; j++) acc[i][j] = tot[i][j] = 0.0;
    double stk[PAIR ? kMaxPairwiseDepth : 1][TM][TN];
    int sp = 0;

    constexpr int NI = int_cols<ACC, ORDER, RM, PV>();
    const bool a_fast = g.a_tma, b_fast = g.b_tma;
    const bool any_tma = a_fast || b_fast;
    const unsigned tx_bytes = (g.a_tma ? TILE_BYTES : 0) + (g.b_tma ? TILE_BYTES : 0);
    // TMA writes need 128-byte-aligned destinations; every stage and tile
    // offset is a multiple of 128 bytes, so only the base is checked.
    if (any_tma && (smem_addr(smem) & 127u) != 0) {
        if (tid == 0) atomicOr(g.err, DEV_ERR_TIMEOUT);
        return;
    }
    if (any_tma && tid == 0) {
        for (int st = 0; st < STAGES; st++) mbar_init(&bars[st], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    auto issue = [&](int64_t it) {
        if (it < T) {
            const int64_t t = REV ? T - 1 - it : it;
            const int st = (int)(it % STAGES);
            double *s = smem + st * STAGE_DOUBLES;
            if (any_tma && tid == 0) {
                mbar_expect_tx(&bars[st], tx_bytes);
                if (a_fast)
                    tma_load_box(s, &tmA, (int)(t * BK), (int)(m0 + z * g.a_brows), &bars[st]);
                if (b_fast)
                    tma_load_box(s + BM * LDK, &tmB, (int)(t * BK), (int)(n0 + z * g.b_brows),
                                 &bars[st]);
            }
            if (!a_fast) stage_generic(s, Az, g.M, m0, g.a_rs, g.a_ks, t * BK, K, tid);
            if (!b_fast) stage_generic(s + BM * LDK, Bz, g.N, n0, g.b_rs, g.b_ks, t * BK, K, tid);
        }
    };

    // `fresh`: the next leaf starts with a FIRST step, so acc need not be zeroed.
    auto push = [&](int merges, bool fresh = false) {
        for (; merges > 0; merges--) {
            sp--;
            combine<ACC, RM, PV>(stk[sp], acc);
        }
#pragma unroll
        for (int i = 0; i < TM; i++)
#pragma unroll
            for (int j = 0; j < TN; j++) {
                stk[sp][i][j] = acc[i][j];
                if (!fresh) acc[i][j] = 0.0;
            }
        sp++;
    };

    // SEG_SCHED bookkeeping: the open chunk / leaf and how much of it is left.
    int64_t seg_left = 0, leaf = 0;
    if (SEG == SEG_SCHED) seg_left = PAIR ? g.leaf_len[0] : g.acc_block;
    auto after_k = [&]() {
        if (SEG != SEG_SCHED || !(PAIR || BLOCK)) return;
        if (--seg_left != 0) return;
        if (BLOCK) {
            blocked_fold<ACC>(tot, acc);
            seg_left = g.acc_block;
        } else {
            push(g.leaf_merges[leaf]);
            leaf++;
            seg_left = g.leaf_len[leaf];  // the schedule carries a sentinel entry
        }
    };

    for (int s = 0; s < STAGES - 1; s++) issue(s);
    for (int64_t it = 0; it < T; it++) {
        const int st = (int)(it % STAGES);
        // One warp watches the stage's barrier; the CTA barrier then orders
        // the landed tile (and any register-loaded one) before every thread's
        // reads, tells every thread that all have finished the previous tile
        // (so its stage may be refilled), and makes the whole CTA leave
        // together if a stage timed out.
        bool lost = false;
        if (any_tma && tid < 32) lost = !mbar_wait(&bars[st], (unsigned)((it / STAGES) & 1));
        if (__syncthreads_or(lost)) {
            if (tid == 0) {
                atomicOr(g.err, DEV_ERR_TIMEOUT);
                // Give the copies this CTA still has in flight a bounded
                // chance to land before its shared memory goes away.
                for (int64_t j = it; j < T && j < it + STAGES - 1; j++)
                    mbar_wait(&bars[j % STAGES], (unsigned)((j / STAGES) & 1));
            }
            return;
        }
        issue(it + STAGES - 1);
        const int64_t t = REV ? T - 1 - it : it;
        const double *sA = smem + st * STAGE_DOUBLES;
        const double *sB = sA + BM * LDK;
        const int kn = (int)(K - t * BK < BK ? K - t * BK : BK);

        if (SEG != SEG_SCHED && kn == BK) {
            // A full tile, no per-k segment work: two k per 16-byte read.
            // Tile-validated kernels fold the range words of the whole tile
            // into `run` and check it once (a miss redoes the leaves exactly);
            // the others validate each k step's groups (mac16).
            using R = GemmRound<ACC, RM, PV>;
            constexpr bool TV = tile_validated<ACC, ORDER>();
            constexpr int G = mac_group<ORDER>();
            unsigned run = 0;
            auto kpair = [&](int q, double(&dst)[TM][TN], auto first) {
                const int kp = REV ? BK / 2 - 1 - q : q;
                double2 a2[TM], b2[TN];
#pragma unroll
                for (int i = 0; i < TM; i++)
                    a2[i] = *reinterpret_cast<const double2 *>(sA + tile_off(ty + 16 * i, 2 * kp));
#pragma unroll
                for (int j = 0; j < TN; j++)
                    b2[j] = *reinterpret_cast<const double2 *>(sB + tile_off(tx + 16 * j, 2 * kp));
                const double ax[TM] = {a2[0].x, a2[1].x, a2[2].x, a2[3].x};
                const double ay[TM] = {a2[0].y, a2[1].y, a2[2].y, a2[3].y};
                const double bx[TN] = {b2[0].x, b2[1].x, b2[2].x, b2[3].x};
                const double by[TN] = {b2[0].y, b2[1].y, b2[2].y, b2[3].y};
                constexpr bool F = decltype(first)::value;
                if constexpr (TV) {
                    mac16_run<ACC, RM, F, PV, NI>(dst, ax, bx, run);
                    mac16_run<ACC, RM, false, PV, NI>(dst, ay, by, run);
                } else if (REV) {
                    mac16<ACC, RM, G, F, PV, NI>(dst, ay, by);
                    mac16<ACC, RM, G, false, PV, NI>(dst, ax, bx);
                } else {
                    mac16<ACC, RM, G, F, PV, NI>(dst, ax, bx);
                    mac16<ACC, RM, G, false, PV, NI>(dst, ay, by);
                }
            };
            // The tile's two pairwise leaves of 8 from zero, exactly.
            auto redo_leaves = [&](double(&l0)[TM][TN], double(&l1)[TM][TN]) {
#pragma unroll
                for (int i = 0; i < TM; i++)
#pragma unroll
                    for (int j = 0; j < TN; j++) l0[i][j] = l1[i][j] = 0.0;
                redo_steps<ACC, RM, false>(sA, sB, ty, tx, 0, BK / 2, l0);
                redo_steps<ACC, RM, false>(sA, sB, ty, tx, BK / 2, BK, l1);
            };
            using Fresh = std::integral_constant<bool, true>;
            using Cont = std::integral_constant<bool, false>;
            if constexpr (PAIR && SEG == SEG_TILE &&
                          (ACC <= DRIFT_ACC_FP32 || ACC == DRIFT_ACC_BF16)) {
                // The tile is two leaves of 8 (Dot.java:86-102): each starts a
                // fresh sum, then they combine into the tile's level-1 node.
                // (FP64, FP32 and tile-validated BF16: BF16 gained 3.8% at
                // 8192^3 on one B200. For FP16, validated per group, four copies
                // of the step code measured 9% slower than one loop that copies
                // and zeroes between the leaves.)
                // The proven FP32 build unrolls the leaves' k pairs: +3.4% at
                // 8192^3 (BF16 unchanged, so it keeps the shorter body).
                double leaf0[TM][TN];
                constexpr int kLeafUnroll = PV && ACC == DRIFT_ACC_FP32 ? 3 : 1;
                kpair(0, leaf0, Fresh{});
#pragma unroll kLeafUnroll
                for (int q = 1; q < BK / 4; q++) kpair(q, leaf0, Cont{});
                kpair(BK / 4, acc, Fresh{});
#pragma unroll kLeafUnroll
                for (int q = BK / 4 + 1; q < BK / 2; q++) kpair(q, acc, Cont{});
                if (TV && !R::valid(run)) redo_leaves(leaf0, acc);
                combine<ACC, RM, PV>(leaf0, acc);
                push(__ffsll(t + 1) - 1, true);    // ctz(t+1) merges in a perfect tree
            } else {
                double leaf0[PAIR ? TM : 1][PAIR ? TN : 1];
                constexpr int kUnroll = kp_unroll<ACC, ORDER>();
#pragma unroll kUnroll
                for (int q = 0; q < BK / 2; q++) {
                    kpair(q, acc, Cont{});
                    if constexpr (PAIR && SEG == SEG_TILE) {
                        if (q == BK / 4 - 1) {  // end of the tile's first leaf of 8
#pragma unroll
                            for (int i = 0; i < TM; i++)
#pragma unroll
                                for (int j = 0; j < TN; j++) {
                                    leaf0[i][j] = acc[i][j];
                                    acc[i][j] = 0.0;
                                }
                        }
                    }
                }
                if constexpr (TV && PAIR && SEG == SEG_TILE) {
                    if (!R::valid(run)) redo_leaves(leaf0, acc);  // rare
                }
                if constexpr (PAIR && SEG == SEG_TILE) {
                    combine<ACC, RM, PV>(leaf0, acc);   // the tile's level-1 node
                    push(__ffsll(t + 1) - 1);       // ctz(t+1) merges in a perfect tree
                } else if constexpr (SEG == SEG_TILE && BLOCK) {
                    if (((t + 1) * BK) % g.acc_block == 0) blocked_fold<ACC>(tot, acc);
                }
            }
        } else {
            // Partial tile, or per-k segment bookkeeping.
#pragma unroll 1
            for (int q = 0; q < kn; q++) {
                const int kk = REV ? kn - 1 - q : q;
                double a[TM], b[TN];
#pragma unroll
                for (int i = 0; i < TM; i++) a[i] = sA[tile_off(ty + 16 * i, kk)];
#pragma unroll
                for (int j = 0; j < TN; j++) b[j] = sB[tile_off(tx + 16 * j, kk)];
                mac16<ACC, RM, mac_group<ORDER>(), false, PV, NI>(acc, a, b);
                after_k();
            }
        }
    }
    // A BLOCKED chunk still open at the end is folded like the others.
    if (BLOCK) {
        const bool open = SEG == SEG_SCHED ? seg_left != g.acc_block : (K % g.acc_block) != 0;
        if (open) blocked_fold<ACC>(tot, acc);
    }

#pragma unroll
    for (int i = 0; i < TM; i++) {
        const int64_t m = m0 + ty + 16 * i;
        if (m >= g.M) continue;
#pragma unroll
        for (int j = 0; j < TN; j++) {
            const int64_t n = n0 + tx + 16 * j;
            if (n >= g.N) continue;
            double v;
            if (BLOCK) v = tot[i][j];
            else if (PAIR) v = K > 0 ? stk[0][i][j] : 0.0;
            else v = acc[i][j];
            if (g.bias) v = __dadd_rn(v, g.bias[n]);  // Pass.java:202
            Cz[m * g.c_rs + n] = v;
        }
    }
}

// ------------------------------------------------------------------ schedule

// Leaf lengths and post-leaf merge counts of Dot.pairwise over `count` terms
// (Dot.java:86-102), in k order.
static void pairwise_walk(int64_t count, std::vector<uint8_t> &len, std::vector<uint8_t> &merges) {
    if (count <= 8) {
        len.push_back((uint8_t)count);
        merges.push_back(0);
        return;
    }
    const int64_t half = (int64_t)((uint64_t)count >> 1);
    pairwise_walk(half, len, merges);
    pairwise_walk(count - half, len, merges);
    merges.back()++;  // this node combines right after its last leaf
}

int pairwise_schedule(int64_t K, std::vector<uint8_t> &sched, int *depth) {
    std::vector<uint8_t> len, merges;
    pairwise_walk(K, len, merges);
    int sp = 0, deepest = 0;
    for (size_t j = 0; j < len.size(); j++) {
        sp = sp - merges[j] + 1;  // pops, then the push
        deepest = std::max(deepest, sp);
    }
    *depth = deepest;
    if (deepest > kMaxPairwiseDepth) return DRIFT_EUNSUPPORTED;
    // Layout: lengths, a sentinel length, then merges.
    sched.clear();
    sched.insert(sched.end(), len.begin(), len.end());
    sched.push_back(0);
    sched.insert(sched.end(), merges.begin(), merges.end());
    return DRIFT_OK;
}

// ------------------------------------------------------------------ launcher

template <int ACC, int ORDER, int RM, int SEG, bool BATCH, bool PV>
static int launch_one(const GemmArgs &g, const CUtensorMap &ma, const CUtensorMap &mb, dim3 grid,
                      cudaStream_t st) {
    // The shared-memory opt-in is per device; setting it is a cheap host call.
    if (cudaFuncSetAttribute(gemm_kernel<ACC, ORDER, RM, SEG, BATCH, PV>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, GEMM_SMEM) != cudaSuccess)
        return DRIFT_ECUDA;
    gemm_kernel<ACC, ORDER, RM, SEG, BATCH, PV><<<grid, GEMM_THREADS, GEMM_SMEM, st>>>(g, ma, mb);
    return DRIFT_OK;
}

template <int ACC, int RM, bool PV = false>
static int launch_order(int order, int seg, const GemmArgs &g, const CUtensorMap &ma,
                        const CUtensorMap &mb, dim3 grid, cudaStream_t st) {
    // Pairwise and blocked run the BATCH build for one problem too: at 8192^3
    // on one B200 it measured 1.1% (fp16) and 1.8% (bf16) faster for pairwise
    // and the same for blocked, while the sequential orders lose about 2% in
    // it and so keep a one-problem build.
    // The PROVEN builds serve one-problem calls only (launch_gemm).
    const bool batch = grid.z > 1 && !PV;
    switch (order) {
        case DRIFT_SEQUENTIAL:
            return batch ? launch_one<ACC, DRIFT_SEQUENTIAL, RM, SEG_NONE, !PV, PV>(g, ma, mb, grid, st)
                         : launch_one<ACC, DRIFT_SEQUENTIAL, RM, SEG_NONE, false, PV>(g, ma, mb, grid, st);
        case DRIFT_REVERSED:
            return batch ? launch_one<ACC, DRIFT_REVERSED, RM, SEG_NONE, !PV, PV>(g, ma, mb, grid, st)
                         : launch_one<ACC, DRIFT_REVERSED, RM, SEG_NONE, false, PV>(g, ma, mb, grid, st);
        case DRIFT_PAIRWISE:
            return seg == SEG_TILE
                       ? launch_one<ACC, DRIFT_PAIRWISE, RM, SEG_TILE, true, PV>(g, ma, mb, grid, st)
                       : launch_one<ACC, DRIFT_PAIRWISE, RM, SEG_SCHED, true, PV>(g, ma, mb, grid, st);
        case DRIFT_BLOCKED:
            return seg == SEG_TILE
                       ? launch_one<ACC, DRIFT_BLOCKED, RM, SEG_TILE, true, PV>(g, ma, mb, grid, st)
                       : launch_one<ACC, DRIFT_BLOCKED, RM, SEG_SCHED, true, PV>(g, ma, mb, grid, st);
        default: return DRIFT_EINVAL;
    }
}

// A TMA map of a K-contiguous operand: dims {K, rows}, row stride rs doubles,
// 18 x 64 boxes (a padded tile), zero fill outside. TMA needs a 16-byte
// aligned base and a row stride that is a multiple of 16 bytes; every box
// starts at a k that is a multiple of 16 (128 bytes), so the innermost
// coordinate is always aligned.
static bool make_map(CUtensorMap *map, const double *X, int64_t rows, int64_t rs, int64_t ks,
                     int64_t K) {
    if (ks != 1 || (rs % 2) != 0 || ((uintptr_t)X % 16) != 0 || K <= 0 || rows <= 0) return false;
    if (K > 0x7fffffffLL || rows > 0x7fffffffLL || rs * 8 >= (1LL << 40)) return false;
    if (rows > 1 && rs < K) return false;  // overlapping rows: the register loader handles those
    EncodeTiledFn fn = encode_tiled();
    if (!fn) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)(rows > 1 ? rs : K + (K & 1)) * 8};
    const cuuint32_t box[2] = {LDK, BM};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT64, 2, const_cast<double *>(X), dims, strides, box,
              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static int gemm_batched(ScheduleCache &cache, const drift_policy *p, int64_t batch, int64_t M,
                        int64_t N, int64_t K, const double *A, int64_t a_rs, int64_t a_ks,
                        int64_t a_bs, const double *B, int64_t b_rs, int64_t b_ks, int64_t b_bs,
                        const double *bias, double *C, int64_t c_rs, int64_t c_bs, int *d_err,
                        const int *skip, cudaStream_t st, const unsigned *range = nullptr,
                        int *route = nullptr, int *n_launched = nullptr);

int launch_gemm(Workspace &ws, ScheduleCache &cache, const drift_policy *p, int64_t M, int64_t N,
                int64_t K, const double *A, int64_t a_rs, int64_t a_ks, const double *B,
                int64_t b_rs, int64_t b_ks, const double *bias, double *C, int64_t c_rs,
                int64_t thin_tiles, int *d_err, int *d_route, cudaStream_t st, unsigned *d_scan,
                int *n_launched) {
    if (n_launched) *n_launched = 0;
    if (M < 0 || N < 0 || K < 0 || a_rs < 0 || a_ks < 0 || b_rs < 0 || b_ks < 0 || c_rs < 0 ||
        p->acc < 0 || p->acc > 3 || p->order < 0 || p->order > 3)
        return DRIFT_EINVAL;
    if (M == 0 || N == 0) return DRIFT_OK;
    // FP32 accumulation over narrow products may go to the FP32 pipe; the
    // decision is made on the device, and the launch below stands down if taken.
    const int *skip = nullptr;
    int rc = launch_gemm_f32(ws, p, M, N, K, A, a_rs, a_ks, B, b_rs, b_ks, bias, C, c_rs, d_err,
                             d_route, st, &skip);
    if (rc) return rc;
    if (skip && n_launched) *n_launched += 4;  // two scans, the decision, the FP32 contraction
    // Too few 64 x 64 tiles to occupy the GPU: one output per thread instead,
    // so that every SM has chains to run. A batch-64 linear layer of 2048
    // outputs is 32 tiles, which left 116 of 148 SMs idle while each busy
    // thread ran sixteen chains. The default limit depends on the policy
    // (staged_tile_limit, measured); an explicit one applies to every call.
    const int64_t tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
    const bool thin = tiles < (thin_tiles < 0 ? staged_tile_limit(p) : thin_tiles);
    const bool staged = thin && (M + 15) / 16 <= 65535;
    if (!skip && !staged && d_route && cudaMemsetAsync(d_route, 0, sizeof(int), st) != cudaSuccess)
        return DRIFT_ECUDA;  // DRIFT_ROUTE_DOUBLE
    if (staged) {
        ContractDesc d{};
        d.op.batch = 1;
        d.op.rows = M;
        d.op.cols = N;
        d.op.depth = K;
        d.op.a_row = a_rs;
        d.op.a_k = a_ks;
        d.op.b_col = b_rs;
        d.op.b_k = b_ks;
        d.op.c_row = c_rs;
        d.op.c_col = 1;
        d.op.alpha = 1.0;
        d.op.window = DRIFT_WINDOW_FULL;
        d.a = A;
        d.b = B;
        d.c = C;
        d.bias = bias;
        if (n_launched) *n_launched += 1;
        return launch_contract_staged(p, d, skip, skip ? nullptr : d_route, st);
    }
    // FP32 and BF16 accumulators: scan both operands for the range proof
    // (range_proven), on the device, ahead of the two contraction builds.
    const bool narrow_rm = p->acc != DRIFT_ACC_BF16 || p->acc_rounding == DRIFT_NEAREST_EVEN ||
                           p->acc_rounding == DRIFT_TRUNCATE;
    const bool prove = d_scan && (p->acc == DRIFT_ACC_FP32 || p->acc == DRIFT_ACC_BF16) &&
                       narrow_rm && K > 0 && (double)M * (double)N * (double)K >= kRangeMinMacs &&
                       range_limit_for(p->acc, K) > -1024;
    if (prove) {
        if (cudaMemsetAsync(d_scan, 0, 2 * kRangeWords * sizeof(unsigned), st) != cudaSuccess)
            return DRIFT_ECUDA;
        const dim3 sgrid((unsigned)(sm_count() * 4), 2);
        range_scan_kernel<<<sgrid, 256, 0, st>>>(A, M, a_rs, a_ks, B, N, b_rs, b_ks, K, d_scan);
        if (n_launched) *n_launched += 1;
    }
    return gemm_batched(cache, p, 1, M, N, K, A, a_rs, a_ks, 0, B, b_rs, b_ks, 0, bias, C, c_rs, 0,
                        d_err, skip, st, prove ? d_scan : nullptr, d_route, n_launched);
}

int launch_gemm_batched(Workspace &ws, ScheduleCache &cache, const drift_policy *p, int64_t batch,
                        int64_t M, int64_t N, int64_t K, const double *A, int64_t a_rs,
                        int64_t a_ks, int64_t a_bs, const double *B, int64_t b_rs, int64_t b_ks,
                        int64_t b_bs, const double *bias, double *C, int64_t c_rs, int64_t c_bs,
                        int *d_err, cudaStream_t st) {
    (void)ws;
    return gemm_batched(cache, p, batch, M, N, K, A, a_rs, a_ks, a_bs, B, b_rs, b_ks, b_bs, bias, C,
                        c_rs, c_bs, d_err, nullptr, st);
}

static int gemm_batched(ScheduleCache &cache, const drift_policy *p, int64_t batch, int64_t M,
                        int64_t N, int64_t K, const double *A, int64_t a_rs, int64_t a_ks,
                        int64_t a_bs, const double *B, int64_t b_rs, int64_t b_ks, int64_t b_bs,
                        const double *bias, double *C, int64_t c_rs, int64_t c_bs, int *d_err,
                        const int *skip, cudaStream_t st, const unsigned *range, int *route,
                        int *n_launched) {
    if (M < 0 || N < 0 || K < 0 || a_rs < 0 || a_ks < 0 || b_rs < 0 || b_ks < 0 || c_rs < 0)
        return DRIFT_EINVAL;
    if (batch < 0 || a_bs < 0 || b_bs < 0 || c_bs < 0 || batch > 65535) return DRIFT_EINVAL;
    if (batch == 0) return DRIFT_OK;
    if (p->acc < 0 || p->acc > 3 || p->order < 0 || p->order > 3) return DRIFT_EINVAL;
    const bool narrow = p->acc == DRIFT_ACC_FP16 || p->acc == DRIFT_ACC_BF16;
    if (narrow && (p->acc_rounding < 0 || p->acc_rounding > 2)) return DRIFT_EINVAL;
    if (narrow && p->acc_rounding == DRIFT_STOCHASTIC) return DRIFT_EINVAL;  // contract.cu
    if (M == 0 || N == 0) return DRIFT_OK;
    const int64_t gx = (N + BN - 1) / BN, gy = (M + BM - 1) / BM;
    if (gx > 0x7fffffffLL || gy > 65535) return DRIFT_EINVAL;

    GemmArgs g{};
    g.M = M;
    g.N = N;
    g.K = K;
    g.A = A;
    g.a_rs = a_rs;
    g.a_ks = a_ks;
    g.B = B;
    g.b_rs = b_rs;
    g.b_ks = b_ks;
    g.bias = bias;
    g.C = C;
    g.c_rs = c_rs;
    g.acc_block = std::max<int64_t>(1, p->acc_block);  // Dot.java:105
    g.err = d_err;
    g.skip = skip;
    CUtensorMap ma, mb;
    memset(&ma, 0, sizeof(ma));
    memset(&mb, 0, sizeof(mb));
    g.a_bs = a_bs;
    g.b_bs = b_bs;
    g.c_bs = c_bs;
    // A TMA map spans every problem of the batch when they sit a whole number
    // of rows apart; rows past a problem's end are read but never stored.
    if (batch == 1 || (a_rs > 0 && a_bs % a_rs == 0)) {
        g.a_brows = batch == 1 ? 0 : a_bs / a_rs;
        g.a_tma = make_map(&ma, A, (batch - 1) * g.a_brows + M, a_rs, a_ks, K);
    }
    if (batch == 1 || (b_rs > 0 && b_bs % b_rs == 0)) {
        g.b_brows = batch == 1 ? 0 : b_bs / b_rs;
        g.b_tma = make_map(&mb, B, (batch - 1) * g.b_brows + N, b_rs, b_ks, K);
    }
    int seg = SEG_NONE;
    if (p->order == DRIFT_BLOCKED) seg = (g.acc_block % BK == 0) ? SEG_TILE : SEG_SCHED;
    if (p->order == DRIFT_PAIRWISE) {
        seg = (K >= 16 && (K & (K - 1)) == 0) ? SEG_TILE : SEG_SCHED;
        if (seg == SEG_SCHED) {
            const uint8_t *d = cache.get(K, st);
            if (!d) return cache.last_status();
            g.leaf_len = d;
            g.leaf_merges = d + cache.leaves(K) + 1;
        }
    }
    const dim3 grid((unsigned)gx, (unsigned)gy, (unsigned)batch);
    // With scan words, both builds are queued and the scan picks one; the
    // proof covers FP32 and BF16 accumulators of one problem.
    const bool prove = range && batch == 1 &&
                       (p->acc == DRIFT_ACC_FP32 || p->acc == DRIFT_ACC_BF16);
    if (prove) {
        g.range = range;
        g.range_limit = range_limit_for(p->acc, K);
        g.route = route;
    }
    int rc;
    const bool trunc = p->acc_rounding == DRIFT_TRUNCATE;
    switch (p->acc) {
        case DRIFT_ACC_FP64:
            rc = launch_order<DRIFT_ACC_FP64, DRIFT_NEAREST_EVEN>(p->order, seg, g, ma, mb, grid, st);
            break;
        case DRIFT_ACC_FP32:
            rc = launch_order<DRIFT_ACC_FP32, DRIFT_NEAREST_EVEN>(p->order, seg, g, ma, mb, grid, st);
            if (!rc && prove)
                rc = launch_order<DRIFT_ACC_FP32, DRIFT_NEAREST_EVEN, true>(p->order, seg, g, ma, mb,
                                                                            grid, st);
            break;
        case DRIFT_ACC_FP16:
            rc = trunc ? launch_order<DRIFT_ACC_FP16, DRIFT_TRUNCATE>(p->order, seg, g, ma, mb, grid, st)
                       : launch_order<DRIFT_ACC_FP16, DRIFT_NEAREST_EVEN>(p->order, seg, g, ma, mb, grid, st);
            break;
        default:
            rc = trunc ? launch_order<DRIFT_ACC_BF16, DRIFT_TRUNCATE>(p->order, seg, g, ma, mb, grid, st)
                       : launch_order<DRIFT_ACC_BF16, DRIFT_NEAREST_EVEN>(p->order, seg, g, ma, mb, grid, st);
            if (!rc && prove)
                rc = trunc ? launch_order<DRIFT_ACC_BF16, DRIFT_TRUNCATE, true>(p->order, seg, g, ma,
                                                                                mb, grid, st)
                           : launch_order<DRIFT_ACC_BF16, DRIFT_NEAREST_EVEN, true>(p->order, seg, g,
                                                                                    ma, mb, grid, st);
    }
    if (rc) return rc;
    if (n_launched) *n_launched += prove ? 2 : 1;
    return cudaGetLastError() == cudaSuccess ? DRIFT_OK : DRIFT_ECUDA;
}

}  // namespace drift
