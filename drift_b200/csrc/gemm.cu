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
// accumulators, the integer rounding of codec.cuh.
//
// Tiling. A CTA of 256 threads owns a 64x64 output tile; each thread owns a
// 4x4 block (four rows of A, four rows of B). K advances in steps of 16
// through a double-buffered shared-memory stage: global loads for step t+1
// are issued into registers before step t is computed. The loader coalesces
// along whichever operand axis has unit stride, so the strided dgrad/wgrad
// operands (Pass.java:224, :230) are staged as they lie and the summation
// order never changes.
//
// Orders. SEQUENTIAL and REVERSED walk k up or down. BLOCKED folds each
// acc_block chunk into an FP32 (FP64 for FP64 accumulation) total
// (Dot.java:104-121). PAIRWISE follows a leaf schedule built on the host from
// the same recursion as Dot.pairwise (half = count >>> 1, leaves of at most 8,
// Dot.java:86-102): after leaf j the kernel pops and combines merges[j]
// partial sums from a per-thread stack. The schedule is the same for every
// output, so the control flow is uniform across the CTA.
#include <algorithm>
#include <vector>

#include "codec.cuh"
#include "internal.h"

namespace drift {

constexpr int BM = 64, BN = 64, BK = 16, TM = 4, TN = 4, GEMM_THREADS = 256;
constexpr int kMaxPairwiseDepth = 30;  // stack depth; enough for any int32 K

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
    const uint8_t *leaf_len;     // PAIRWISE: length of each leaf, in k order
    const uint8_t *leaf_merges;  // PAIRWISE: combines after each leaf
    int a_kfast, b_kfast;        // loader coalescing direction
};

// s + p rounded as the accumulator does (Dot.java:46, :54, :63).
template <int ACC, int RM>
__device__ __forceinline__ double acc_add(double s, double p) {
    const double t = __dadd_rn(s, p);
    if constexpr (ACC == DRIFT_ACC_FP64) return t;
    else if constexpr (ACC == DRIFT_ACC_FP32) return round_to_f32(t);
    else return round_acc_fast<ACC, RM>(t);
}

template <int ACC, int RM>
__device__ __forceinline__ double mac(double s, double a, double b) {
    return acc_add<ACC, RM>(s, __dmul_rn(a, b));
}

// Fold of a BLOCKED chunk into the running total (Dot.java:104-121).
template <int ACC>
__device__ __forceinline__ double blocked_fold(double total, double partial) {
    const double t = __dadd_rn(total, partial);
    return ACC == DRIFT_ACC_FP64 ? t : round_to_f32(t);
}

template <int ACC, int ORDER, int RM>
__global__ void __launch_bounds__(GEMM_THREADS) gemm_kernel(const GemmArgs g) {
    __shared__ __align__(16) double As[2][BK][BM];
    __shared__ __align__(16) double Bs[2][BK][BN];

    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const int64_t m0 = (int64_t)blockIdx.y * BM;
    const int64_t n0 = (int64_t)blockIdx.x * BN;
    const int64_t K = g.K;

    double acc[TM][TN];
    double tot[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; i++)
#pragma unroll
        for (int j = 0; j < TN; j++) acc[i][j] = tot[i][j] = 0.0;

    double stk[ORDER == DRIFT_PAIRWISE ? kMaxPairwiseDepth : 1][TM][TN];
    int sp = 0;

    const int64_t T = (K + BK - 1) / BK;
    double ra[4], rb[4];

    auto load_tile = [&](int64_t t) {
        const int64_t k0 = t * BK;
#pragma unroll
        for (int r = 0; r < 4; r++) {
            const int e = tid + GEMM_THREADS * r;
            int kk = g.a_kfast ? (e & 15) : (e >> 6);
            int mm = g.a_kfast ? (e >> 4) : (e & 63);
            int64_t m = m0 + mm, k = k0 + kk;
            ra[r] = (m < g.M && k < K) ? g.A[m * g.a_rs + k * g.a_ks] : 0.0;
            kk = g.b_kfast ? (e & 15) : (e >> 6);
            mm = g.b_kfast ? (e >> 4) : (e & 63);
            m = n0 + mm;
            k = k0 + kk;
            rb[r] = (m < g.N && k < K) ? g.B[m * g.b_rs + k * g.b_ks] : 0.0;
        }
    };
    auto store_tile = [&](int buf) {
#pragma unroll
        for (int r = 0; r < 4; r++) {
            const int e = tid + GEMM_THREADS * r;
            As[buf][g.a_kfast ? (e & 15) : (e >> 6)][g.a_kfast ? (e >> 4) : (e & 63)] = ra[r];
            Bs[buf][g.b_kfast ? (e & 15) : (e >> 6)][g.b_kfast ? (e >> 4) : (e & 63)] = rb[r];
        }
    };

    // Segment bookkeeping for BLOCKED chunks and PAIRWISE leaves.
    int64_t seg_left = 0;
    int64_t leaf = 0;
    if (ORDER == DRIFT_BLOCKED) seg_left = g.acc_block;
    if (ORDER == DRIFT_PAIRWISE) seg_left = g.leaf_len[0];

    auto end_segment = [&]() {
        if (ORDER == DRIFT_BLOCKED) {
#pragma unroll
            for (int i = 0; i < TM; i++)
#pragma unroll
                for (int j = 0; j < TN; j++) {
                    tot[i][j] = blocked_fold<ACC>(tot[i][j], acc[i][j]);
                    acc[i][j] = 0.0;
                }
            seg_left = g.acc_block;
        } else if (ORDER == DRIFT_PAIRWISE) {
            int merges = g.leaf_merges[leaf];
            for (; merges > 0; merges--) {
                sp--;
#pragma unroll
                for (int i = 0; i < TM; i++)
#pragma unroll
                    for (int j = 0; j < TN; j++) acc[i][j] = acc_add<ACC, RM>(stk[sp][i][j], acc[i][j]);
            }
#pragma unroll
            for (int i = 0; i < TM; i++)
#pragma unroll
                for (int j = 0; j < TN; j++) {
                    stk[sp][i][j] = acc[i][j];
                    acc[i][j] = 0.0;
                }
            sp++;
            leaf++;
            seg_left = g.leaf_len[leaf];  // the schedule carries a sentinel entry
        }
    };

    auto step = [&](int buf, int kk) {
        const double2 a01 = *reinterpret_cast<const double2 *>(&As[buf][kk][ty * TM]);
        const double2 a23 = *reinterpret_cast<const double2 *>(&As[buf][kk][ty * TM + 2]);
        const double2 b01 = *reinterpret_cast<const double2 *>(&Bs[buf][kk][tx * TN]);
        const double2 b23 = *reinterpret_cast<const double2 *>(&Bs[buf][kk][tx * TN + 2]);
        const double a[4] = {a01.x, a01.y, a23.x, a23.y};
        const double b[4] = {b01.x, b01.y, b23.x, b23.y};
#pragma unroll
        for (int i = 0; i < TM; i++)
#pragma unroll
            for (int j = 0; j < TN; j++) acc[i][j] = mac<ACC, RM>(acc[i][j], a[i], b[j]);
        if (ORDER == DRIFT_BLOCKED || ORDER == DRIFT_PAIRWISE) {
            if (--seg_left == 0) end_segment();
        }
    };

    if (T > 0) {
        load_tile(ORDER == DRIFT_REVERSED ? T - 1 : 0);
        store_tile(0);
        __syncthreads();
    }
    for (int64_t it = 0; it < T; it++) {
        const int64_t t = ORDER == DRIFT_REVERSED ? T - 1 - it : it;
        const int buf = (int)(it & 1);
        if (it + 1 < T) load_tile(ORDER == DRIFT_REVERSED ? t - 1 : t + 1);
        const int kn = (int)(K - t * BK < BK ? K - t * BK : BK);
        if (ORDER == DRIFT_REVERSED) {
            if (kn == BK) {
#pragma unroll
                for (int kk = BK - 1; kk >= 0; kk--) step(buf, kk);
            } else {
                for (int kk = kn - 1; kk >= 0; kk--) step(buf, kk);
            }
        } else {
            if (kn == BK) {
#pragma unroll
                for (int kk = 0; kk < BK; kk++) step(buf, kk);
            } else {
                for (int kk = 0; kk < kn; kk++) step(buf, kk);
            }
        }
        if (it + 1 < T) {
            store_tile(buf ^ 1);
            __syncthreads();
        }
    }

    // A BLOCKED chunk still open at the end is folded like the others.
    if (ORDER == DRIFT_BLOCKED && seg_left != g.acc_block) end_segment();

#pragma unroll
    for (int i = 0; i < TM; i++) {
        const int64_t m = m0 + ty * TM + i;
        if (m >= g.M) continue;
#pragma unroll
        for (int j = 0; j < TN; j++) {
            const int64_t n = n0 + tx * TN + j;
            if (n >= g.N) continue;
            double v;
            if (ORDER == DRIFT_BLOCKED) v = tot[i][j];
            else if (ORDER == DRIFT_PAIRWISE) v = K > 0 ? stk[0][i][j] : 0.0;
            else v = acc[i][j];
            if (g.bias) v = __dadd_rn(v, g.bias[n]);  // Pass.java:202
            g.C[m * g.c_rs + n] = v;
        }
    }
}

// ------------------------------------------------------------------ schedule

// Leaf lengths and post-leaf merge counts of Dot.pairwise over `count` terms
// (Dot.java:86-102), in k order, plus the stack depth the walk reaches.
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

template <int ACC, int ORDER, int RM>
static void launch_one(const GemmArgs &g, dim3 grid, cudaStream_t st) {
    gemm_kernel<ACC, ORDER, RM><<<grid, GEMM_THREADS, 0, st>>>(g);
}

template <int ACC, int RM>
static int launch_order(int order, const GemmArgs &g, dim3 grid, cudaStream_t st) {
    switch (order) {
        case DRIFT_SEQUENTIAL: launch_one<ACC, DRIFT_SEQUENTIAL, RM>(g, grid, st); break;
        case DRIFT_REVERSED: launch_one<ACC, DRIFT_REVERSED, RM>(g, grid, st); break;
        case DRIFT_PAIRWISE: launch_one<ACC, DRIFT_PAIRWISE, RM>(g, grid, st); break;
        case DRIFT_BLOCKED: launch_one<ACC, DRIFT_BLOCKED, RM>(g, grid, st); break;
        default: return DRIFT_EINVAL;
    }
    return DRIFT_OK;
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
    // Coalesce along k when k has unit stride or rows do not.
    g.a_kfast = (a_ks == 1 || a_rs != 1) ? 1 : 0;
    g.b_kfast = (b_ks == 1 || b_rs != 1) ? 1 : 0;
    if (p->order == DRIFT_PAIRWISE) {
        const uint8_t *d = cache.get(K, st);
        if (!d) return cache.last_status();
        g.leaf_len = d;
        g.leaf_merges = d + cache.leaves(K) + 1;
    }
    const dim3 grid((unsigned)gx, (unsigned)gy);
    int rc;
    switch (p->acc) {
        case DRIFT_ACC_FP64: rc = launch_order<DRIFT_ACC_FP64, DRIFT_NEAREST_EVEN>(p->order, g, grid, st); break;
        case DRIFT_ACC_FP32: rc = launch_order<DRIFT_ACC_FP32, DRIFT_NEAREST_EVEN>(p->order, g, grid, st); break;
        case DRIFT_ACC_FP16:
            rc = p->acc_rounding == DRIFT_TRUNCATE
                     ? launch_order<DRIFT_ACC_FP16, DRIFT_TRUNCATE>(p->order, g, grid, st)
                     : launch_order<DRIFT_ACC_FP16, DRIFT_NEAREST_EVEN>(p->order, g, grid, st);
            break;
        default:
            rc = p->acc_rounding == DRIFT_TRUNCATE
                     ? launch_order<DRIFT_ACC_BF16, DRIFT_TRUNCATE>(p->order, g, grid, st)
                     : launch_order<DRIFT_ACC_BF16, DRIFT_NEAREST_EVEN>(p->order, g, grid, st);
    }
    if (rc) return rc;
    return cudaGetLastError() == cudaSuccess ? DRIFT_OK : DRIFT_ECUDA;
}

}  // namespace drift
