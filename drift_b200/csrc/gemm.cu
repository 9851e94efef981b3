// gemm.cu — the emulated contraction: C[i,o] = Dot.dot(A row i, B row o, K).
//
// Device form of the (i, o) loops of java/src/main/java/io/drift/train/
// Pass.java:200-232 over Dot.dot (java/src/main/java/io/drift/kernel/
// Dot.java:26-121). Tensor cores are not used: the order of the additions is
// the quantity under study, so every output runs its own scalar chain in
// exactly the Java order, and parallelism comes only from independent outputs.
//
// Per multiply-accumulate: one DMUL and one DADD (never fused: Java rounds the
// product to double before the add, Dot.java:46/:54/:63) and, for narrow
// accumulators, the fast rounding of codec.cuh, validated for eight of a
// thread's sixteen outputs at a time.
//
// Tiling. A CTA of 256 threads owns a 64x64 output tile; thread (ty, tx) owns
// rows ty + 16i and columns tx + 16j (i, j < 4), so the sixteen threads that
// share a row read sixteen consecutive B rows. K advances in tiles of 16
// through a 3-stage shared-memory ring laid out [row][k] with a 2-double pad
// (row stride 144 B), which makes the 16-byte (k, k+1) reads conflict-free.
// K-contiguous operands with 16-byte-aligned rows are staged with cp.async
// (LDGSTS, 16 bytes per instruction, zero-filled past the edges); any other
// strides (the dgrad / wgrad operands, Pass.java:224, :230) go through a
// register loader into the same layout. The summation order never depends on
// the staging.
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
#include <vector>

#include "codec.cuh"
#include "internal.h"

namespace drift {

constexpr int BM = 64, BN = 64, BK = 16, TM = 4, TN = 4, GEMM_THREADS = 256;
constexpr int LDK = BK + 2;  // padded row length of a staged tile, in doubles
constexpr int STAGES = 3;
constexpr int STAGE_DOUBLES = (BM + BN) * LDK;
constexpr int GEMM_SMEM = STAGES * STAGE_DOUBLES * (int)sizeof(double);
constexpr int kMaxPairwiseDepth = 30;  // stack depth; enough for any int32 K
// Unroll of the k-pair loop of a full tile, chosen by measurement on B200:
// the narrow accumulators' rounding makes a long tile body fall out of the
// instruction cache, so they unroll less (pairwise least, as its per-tile
// merge code is the largest); FP64/FP32 bodies are small and unroll fully.
template <int ACC, int ORDER>
constexpr int kp_unroll() {
    return ORDER == DRIFT_PAIRWISE ? 1 : (ACC == DRIFT_ACC_FP64 || ACC == DRIFT_ACC_FP32) ? 8 : 2;
}

enum SegMode { SEG_NONE = 0, SEG_TILE = 1, SEG_SCHED = 2 };

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
    int a_async, b_async;        // operand staged by cp.async
};

// The fast rounding is validated for half of a thread's outputs (two rows of
// four) at a time: one branch per eight sums keeps the temporaries to eight
// doubles, and a miss recomputes those eight exactly.
constexpr int GROUP_ROWS = 2;

// Rounds sixteen sums in place as the accumulator does (Dot.java:54, :63,
// :99, :224). The rounded value overwrites the sum and the sum is kept aside
// only until its group is validated, so no copy is needed on the fast path.
template <int ACC, int RM>
__device__ __forceinline__ void round16(double (&t)[TM][TN]) {
    using R = AccRound<ACC, RM>;
    if constexpr (ACC != DRIFT_ACC_FP64) {
#pragma unroll
        for (int i0 = 0; i0 < TM; i0 += GROUP_ROWS) {
            double keep[GROUP_ROWS][TN];
            bool ok = true;
#pragma unroll
            for (int i = 0; i < GROUP_ROWS; i++)
#pragma unroll
                for (int j = 0; j < TN; j++) {
                    keep[i][j] = t[i0 + i][j];
                    t[i0 + i][j] = R::fast(keep[i][j]);
                    ok = ok & R::ok(t[i0 + i][j]);
                }
            if (!ok) {
#pragma unroll
                for (int i = 0; i < GROUP_ROWS; i++)
#pragma unroll
                    for (int j = 0; j < TN; j++) t[i0 + i][j] = R::exact(keep[i][j]);
            }
        }
    }
}

// One k step for the thread's 16 outputs: acc = round(acc + a_i * b_j), the
// rounded value written straight into the accumulator.
template <int ACC, int RM>
__device__ __forceinline__ void mac16(double (&acc)[TM][TN], const double (&a)[TM],
                                      const double (&b)[TN]) {
    using R = AccRound<ACC, RM>;
    if constexpr (ACC == DRIFT_ACC_FP64) {
#pragma unroll
        for (int i = 0; i < TM; i++)
#pragma unroll
            for (int j = 0; j < TN; j++) acc[i][j] = __dadd_rn(acc[i][j], __dmul_rn(a[i], b[j]));
    } else {
#pragma unroll
        for (int i0 = 0; i0 < TM; i0 += GROUP_ROWS) {
            double t[GROUP_ROWS][TN];
            bool ok = true;
#pragma unroll
            for (int i = 0; i < GROUP_ROWS; i++)
#pragma unroll
                for (int j = 0; j < TN; j++) {
                    t[i][j] = __dadd_rn(acc[i0 + i][j], __dmul_rn(a[i0 + i], b[j]));
                    acc[i0 + i][j] = R::fast(t[i][j]);
                    ok = ok & R::ok(acc[i0 + i][j]);
                }
            if (!ok) {  // rare: round these eight sums exactly
#pragma unroll
                for (int i = 0; i < GROUP_ROWS; i++)
#pragma unroll
                    for (int j = 0; j < TN; j++) acc[i0 + i][j] = R::exact(t[i][j]);
            }
        }
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

// Pairwise combine of the stack top with the current node (Dot.java:97-101).
template <int ACC, int RM>
__device__ __forceinline__ void combine(const double (&left)[TM][TN], double (&right)[TM][TN]) {
#pragma unroll
    for (int i = 0; i < TM; i++)
#pragma unroll
        for (int j = 0; j < TN; j++) right[i][j] = __dadd_rn(left[i][j], right[i][j]);
    round16<ACC, RM>(right);
}

__device__ __forceinline__ void cp_async16(double *dst, const double *src, int bytes) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(src), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// Stages rows [r0, r0+64) x k [k0, k0+16) of an operand into s[row][k].
__device__ __forceinline__ void stage_operand(double *s, const double *X, int64_t rows,
                                              int64_t r0, int64_t rs, int64_t ks, int64_t k0,
                                              int64_t K, bool async, int tid) {
    if (async) {
        // 64 rows x 8 chunks of 16 bytes; two chunks per thread.
#pragma unroll
        for (int c = tid; c < 512; c += GEMM_THREADS) {
            const int row = c >> 3, ch = c & 7;
            const int64_t r = r0 + row, k = k0 + 2 * ch;
            int bytes = 0;
            if (r < rows && k < K) bytes = (K - k >= 2) ? 16 : 8;
            const double *src = bytes ? X + r * rs + k : X;
            cp_async16(s + row * LDK + 2 * ch, src, bytes);
        }
    } else {
        const bool kfast = ks == 1 || rs != 1;  // coalesce along the unit stride
#pragma unroll
        for (int e = tid; e < BM * BK; e += GEMM_THREADS) {
            const int kk = kfast ? (e & 15) : (e >> 6);
            const int rr = kfast ? (e >> 4) : (e & 63);
            const int64_t r = r0 + rr, k = k0 + kk;
            s[rr * LDK + kk] = (r < rows && k < K) ? X[r * rs + k * ks] : 0.0;
        }
    }
}

template <int ACC, int ORDER, int RM, int SEG>
__global__ void __launch_bounds__(GEMM_THREADS, 2) gemm_kernel(const GemmArgs g) {
    extern __shared__ __align__(16) double smem[];
    constexpr bool REV = ORDER == DRIFT_REVERSED;
    constexpr bool PAIR = ORDER == DRIFT_PAIRWISE;
    constexpr bool BLOCK = ORDER == DRIFT_BLOCKED;

    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const int64_t m0 = (int64_t)blockIdx.y * BM;
    const int64_t n0 = (int64_t)blockIdx.x * BN;
    const int64_t K = g.K;
    const int64_t T = (K + BK - 1) / BK;

    double acc[TM][TN], tot[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; i++)
#pragma unroll
        for (int j = 0; j < TN; j++) acc[i][j] = tot[i][j] = 0.0;
    double stk[PAIR ? kMaxPairwiseDepth : 1][TM][TN];
    int sp = 0;

    auto issue = [&](int64_t it) {
        if (it < T) {
            const int64_t t = REV ? T - 1 - it : it;
            double *s = smem + (int)(it % STAGES) * STAGE_DOUBLES;
            stage_operand(s, g.A, g.M, m0, g.a_rs, g.a_ks, t * BK, K, g.a_async, tid);
            stage_operand(s + BM * LDK, g.B, g.N, n0, g.b_rs, g.b_ks, t * BK, K, g.b_async, tid);
        }
        cp_async_commit();
    };

    auto push = [&](int merges) {
        for (; merges > 0; merges--) {
            sp--;
            combine<ACC, RM>(stk[sp], acc);
        }
#pragma unroll
        for (int i = 0; i < TM; i++)
#pragma unroll
            for (int j = 0; j < TN; j++) {
                stk[sp][i][j] = acc[i][j];
                acc[i][j] = 0.0;
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
        cp_async_wait<STAGES - 2>();
        __syncthreads();
        issue(it + STAGES - 1);
        const int64_t t = REV ? T - 1 - it : it;
        const double *sA = smem + (int)(it % STAGES) * STAGE_DOUBLES;
        const double *sB = sA + BM * LDK;
        const int kn = (int)(K - t * BK < BK ? K - t * BK : BK);

        if (SEG != SEG_SCHED && kn == BK) {
            // A full tile, no per-k segment work: two k per 16-byte read.
            double leaf0[PAIR ? TM : 1][PAIR ? TN : 1];
            constexpr int kUnroll = kp_unroll<ACC, ORDER>();
#pragma unroll kUnroll
            for (int q = 0; q < BK / 2; q++) {
                const int kp = REV ? BK / 2 - 1 - q : q;
                double2 a2[TM], b2[TN];
#pragma unroll
                for (int i = 0; i < TM; i++)
                    a2[i] = *reinterpret_cast<const double2 *>(sA + (ty + 16 * i) * LDK + 2 * kp);
#pragma unroll
                for (int j = 0; j < TN; j++)
                    b2[j] = *reinterpret_cast<const double2 *>(sB + (tx + 16 * j) * LDK + 2 * kp);
                const double ax[TM] = {a2[0].x, a2[1].x, a2[2].x, a2[3].x};
                const double ay[TM] = {a2[0].y, a2[1].y, a2[2].y, a2[3].y};
                const double bx[TN] = {b2[0].x, b2[1].x, b2[2].x, b2[3].x};
                const double by[TN] = {b2[0].y, b2[1].y, b2[2].y, b2[3].y};
                if (REV) {
                    mac16<ACC, RM>(acc, ay, by);
                    mac16<ACC, RM>(acc, ax, bx);
                } else {
                    mac16<ACC, RM>(acc, ax, bx);
                    mac16<ACC, RM>(acc, ay, by);
                }
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
            if constexpr (SEG == SEG_TILE && PAIR) {
                combine<ACC, RM>(leaf0, acc);      // the tile's level-1 node
                push(__ffsll(t + 1) - 1);          // ctz(t+1) merges in a perfect tree
            } else if constexpr (SEG == SEG_TILE && BLOCK) {
                if (((t + 1) * BK) % g.acc_block == 0) blocked_fold<ACC>(tot, acc);
            }
        } else {
            // Partial tile, or per-k segment bookkeeping.
#pragma unroll 1
            for (int q = 0; q < kn; q++) {
                const int kk = REV ? kn - 1 - q : q;
                double a[TM], b[TN];
#pragma unroll
                for (int i = 0; i < TM; i++) a[i] = sA[(ty + 16 * i) * LDK + kk];
#pragma unroll
                for (int j = 0; j < TN; j++) b[j] = sB[(tx + 16 * j) * LDK + kk];
                mac16<ACC, RM>(acc, a, b);
                after_k();
            }
        }
    }
    cp_async_wait<0>();

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
            g.C[m * g.c_rs + n] = v;
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

template <int ACC, int ORDER, int RM, int SEG>
static int launch_one(const GemmArgs &g, dim3 grid, cudaStream_t st) {
    // The shared-memory opt-in is per device; setting it is a cheap host call.
    if (cudaFuncSetAttribute(gemm_kernel<ACC, ORDER, RM, SEG>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, GEMM_SMEM) != cudaSuccess)
        return DRIFT_ECUDA;
    gemm_kernel<ACC, ORDER, RM, SEG><<<grid, GEMM_THREADS, GEMM_SMEM, st>>>(g);
    return DRIFT_OK;
}

template <int ACC, int RM>
static int launch_order(int order, int seg, const GemmArgs &g, dim3 grid, cudaStream_t st) {
    switch (order) {
        case DRIFT_SEQUENTIAL: return launch_one<ACC, DRIFT_SEQUENTIAL, RM, SEG_NONE>(g, grid, st);
        case DRIFT_REVERSED: return launch_one<ACC, DRIFT_REVERSED, RM, SEG_NONE>(g, grid, st);
        case DRIFT_PAIRWISE:
            return seg == SEG_TILE ? launch_one<ACC, DRIFT_PAIRWISE, RM, SEG_TILE>(g, grid, st)
                                   : launch_one<ACC, DRIFT_PAIRWISE, RM, SEG_SCHED>(g, grid, st);
        case DRIFT_BLOCKED:
            return seg == SEG_TILE ? launch_one<ACC, DRIFT_BLOCKED, RM, SEG_TILE>(g, grid, st)
                                   : launch_one<ACC, DRIFT_BLOCKED, RM, SEG_SCHED>(g, grid, st);
        default: return DRIFT_EINVAL;
    }
}

static bool async_ok(const double *X, int64_t rs, int64_t ks) {
    return ks == 1 && (rs % 2) == 0 && ((uintptr_t)X % 16) == 0;
}

int launch_gemm(Workspace &ws, ScheduleCache &cache, const drift_policy *p, int64_t M, int64_t N,
                int64_t K, const double *A, int64_t a_rs, int64_t a_ks, const double *B,
                int64_t b_rs, int64_t b_ks, const double *bias, double *C, int64_t c_rs,
                cudaStream_t st) {
    (void)ws;
    if (M < 0 || N < 0 || K < 0 || a_rs < 0 || a_ks < 0 || b_rs < 0 || b_ks < 0 || c_rs < 0)
        return DRIFT_EINVAL;
    if (p->acc < 0 || p->acc > 3 || p->order < 0 || p->order > 3) return DRIFT_EINVAL;
    const bool narrow = p->acc == DRIFT_ACC_FP16 || p->acc == DRIFT_ACC_BF16;
    if (narrow && (p->acc_rounding < 0 || p->acc_rounding > 2)) return DRIFT_EINVAL;
    if (narrow && p->acc_rounding == DRIFT_STOCHASTIC) return DRIFT_EUNSUPPORTED;
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
    g.a_async = async_ok(A, a_rs, a_ks);
    g.b_async = async_ok(B, b_rs, b_ks);
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
    const dim3 grid((unsigned)gx, (unsigned)gy);
    int rc;
    switch (p->acc) {
        case DRIFT_ACC_FP64:
            rc = launch_order<DRIFT_ACC_FP64, DRIFT_NEAREST_EVEN>(p->order, seg, g, grid, st);
            break;
        case DRIFT_ACC_FP32:
            rc = launch_order<DRIFT_ACC_FP32, DRIFT_NEAREST_EVEN>(p->order, seg, g, grid, st);
            break;
        case DRIFT_ACC_FP16:
            rc = p->acc_rounding == DRIFT_TRUNCATE
                     ? launch_order<DRIFT_ACC_FP16, DRIFT_TRUNCATE>(p->order, seg, g, grid, st)
                     : launch_order<DRIFT_ACC_FP16, DRIFT_NEAREST_EVEN>(p->order, seg, g, grid, st);
            break;
        default:
            rc = p->acc_rounding == DRIFT_TRUNCATE
                     ? launch_order<DRIFT_ACC_BF16, DRIFT_TRUNCATE>(p->order, seg, g, grid, st)
                     : launch_order<DRIFT_ACC_BF16, DRIFT_NEAREST_EVEN>(p->order, seg, g, grid, st);
    }
    if (rc) return rc;
    return cudaGetLastError() == cudaSuccess ? DRIFT_OK : DRIFT_ECUDA;
}

}  // namespace drift
