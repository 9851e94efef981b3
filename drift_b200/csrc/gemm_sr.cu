// gemm_sr.cu — the contraction with a stochastically rounded accumulator.
//
// Dot.round with STOCHASTIC (java/src/main/java/io/drift/kernel/Dot.java:171-175)
// draws from the Rng shared by the whole GEMM, in the order the dots run
// ((i, o) loops of Pass.java:200-232) and, inside a dot, in its evaluation
// order, and only when the sum is not exactly representable. So dot j starts
// drawing at D_j = (draws of dots 0..j-1), which the earlier dots' data
// decide.
//
// The engine finds the D_j by a fixed point: it predicts every dot's count,
// scans the predictions into offsets, computes all dots in parallel from
// those offsets (splitmix64 is counter-based, so any draw is available
// directly), and records each dot's true count. If the scan of the true
// counts gives back the offsets that were used, every dot started at the
// right draw (by induction from D_0 = 0) and the result is the sequential
// one. Otherwise the new offsets are used and the pass repeats. The first
// prediction — one draw per rounding the order performs — is exact unless
// some sum is exactly representable, so one pass usually settles it. After a
// bounded number of passes the dots are walked in order by one thread, which
// is correct for any data. Nothing spins: each pass is a separate launch and
// the host reads a flag between them.
//
// One output per thread; each thread reads its row of A and of B through the
// read-only cache with any strides.
#include <algorithm>
#include <vector>

#include "codec.cuh"
#include "internal.h"

namespace drift {

struct GemmSrArgs {
    int64_t M, N, K;
    const double *A;
    int64_t a_rs, a_ks;
    const double *B;
    int64_t b_rs, b_ks;
    const double *bias;
    double *C;
    int64_t c_rs;
    int64_t acc_block;
    int order;
    const uint8_t *leaf_len;     // PAIRWISE schedule (lengths, sentinel, merges)
    const uint8_t *leaf_merges;
    const uint64_t *state;       // Rng state before the GEMM's first draw
    const int64_t *offsets;      // first draw index of each dot, (i, o) order
    uint32_t *counts;            // draws each dot made
};

// Dot.round(x, acc, STOCHASTIC, rng) (Dot.java:141-182), drawing the
// (idx + cnt)-th number of the stream only when the fraction is non-zero.
template <int ACC>
__device__ __forceinline__ double sr_round(double x, uint64_t state, uint64_t idx, uint32_t &cnt) {
    using F = AccFmt<ACC>;
    if (x == 0.0 || isnan(x)) return x;
    const double ax = fabs(x);
    if (isinf(ax)) return copysign(F::max(), x);
    int e = java_get_exponent(ax);
    if (e < F::min_exp) e = F::min_exp;
    const int q = e - F::mant;
    const double scaled = __dmul_rn(ax, pow2(-q));  // exact
    const double fl = floor(scaled);
    const double frac = __dsub_rn(scaled, fl);
    double m = fl;
    if (frac != 0.0) {
        const uint64_t u = draw_u53(state, idx + cnt);
        cnt++;
        if (__dmul_rn((double)u, 0x1p-53) < frac) m = fl + 1.0;
    }
    double r = __dmul_rn(m, pow2(q));
    if (r > F::max()) r = F::max();
    return copysign(r, x);
}

template <int ACC>
__device__ double sr_dot(const GemmSrArgs &g, const double *a, const double *b, uint64_t state,
                         uint64_t idx, uint32_t &cnt) {
    const int64_t K = g.K;
    auto term = [&](int64_t k) { return __dmul_rn(a[k * g.a_ks], b[k * g.b_ks]); };
    auto fwd = [&](int64_t from, int64_t count) {  // Dot.forward (Dot.java:37-68)
        double s = 0.0;
        for (int64_t k = from; k < from + count; k++)
            s = sr_round<ACC>(__dadd_rn(s, term(k)), state, idx, cnt);
        return s;
    };
    if (g.order == DRIFT_SEQUENTIAL) return fwd(0, K);
    if (g.order == DRIFT_REVERSED) {  // Dot.backward (Dot.java:70-84)
        double s = 0.0;
        for (int64_t k = K - 1; k >= 0; k--)
            s = sr_round<ACC>(__dadd_rn(s, term(k)), state, idx, cnt);
        return s;
    }
    if (g.order == DRIFT_BLOCKED) {  // Dot.blocked (Dot.java:104-121): FP32 totals, no draws
        double total = 0.0;
        for (int64_t start = 0; start < K; start += g.acc_block) {
            const double partial = fwd(start, min(g.acc_block, K - start));
            total = (double)__double2float_rn(__dadd_rn(total, partial));
        }
        return total;
    }
    // Dot.pairwise (Dot.java:86-102): leaves in order, each node's combine
    // right after its last leaf, every combine a stochastic rounding.
    double stk[32];
    int sp = 0;
    int64_t k = 0;
    for (int64_t leaf = 0;; leaf++) {
        const int len = g.leaf_len[leaf];
        if (len == 0) break;  // the sentinel
        double v = fwd(k, len);
        k += len;
        for (int mg = g.leaf_merges[leaf]; mg > 0; mg--) {
            sp--;
            v = sr_round<ACC>(__dadd_rn(stk[sp], v), state, idx, cnt);
        }
        stk[sp++] = v;
    }
    return K > 0 ? stk[0] : 0.0;
}

template <int ACC>
__global__ void __launch_bounds__(128) gemm_sr_kernel(const GemmSrArgs g) {
    const int64_t out = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (out >= g.M * g.N) return;
    const int64_t i = out / g.N, o = out % g.N;
    uint32_t cnt = 0;
    double v = sr_dot<ACC>(g, g.A + i * g.a_rs, g.B + o * g.b_rs, *g.state,
                           (uint64_t)g.offsets[out], cnt);
    if (g.bias) v = __dadd_rn(v, g.bias[o]);  // Pass.java:202
    g.C[i * g.c_rs + o] = v;
    g.counts[out] = cnt;
}

// The dots in order, one thread: the fallback that is correct for any data.
template <int ACC>
__global__ void gemm_sr_serial_kernel(const GemmSrArgs g, uint64_t *total) {
    if (blockIdx.x != 0 || threadIdx.x != 0) return;
    uint64_t idx = 0;
    for (int64_t out = 0; out < g.M * g.N; out++) {
        const int64_t i = out / g.N, o = out % g.N;
        uint32_t cnt = 0;
        double v = sr_dot<ACC>(g, g.A + i * g.a_rs, g.B + o * g.b_rs, *g.state, idx, cnt);
        if (g.bias) v = __dadd_rn(v, g.bias[o]);
        g.C[i * g.c_rs + o] = v;
        idx += cnt;
    }
    *total = idx;
}

// ------------------------------------------------------------------ offsets

constexpr int kScanThreads = 1024;

// Per-block sums of n uint32 counts (block b covers [b*chunk, (b+1)*chunk)).
__global__ void __launch_bounds__(kScanThreads) block_sums_kernel(const uint32_t *counts, int64_t n,
                                                                  int64_t chunk, uint64_t *sums) {
    __shared__ uint64_t s_part[kScanThreads / 32];
    const int64_t lo = blockIdx.x * chunk, hi = min(n, lo + chunk);
    uint64_t acc = 0;
    for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) acc += counts[i];
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint64_t t = 0;
        for (int w = 0; w < kScanThreads / 32; w++) t += s_part[w];
        sums[blockIdx.x] = t;
    }
}

// Exclusive scan of the block sums in place (one CTA; a few thousand values);
// also writes the grand total to sums[nb].
__global__ void scan_sums_kernel(uint64_t *sums, int64_t nb) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    uint64_t run = 0;
    for (int64_t b = 0; b < nb; b++) {
        const uint64_t v = sums[b];
        sums[b] = run;
        run += v;
    }
    sums[nb] = run;
}

// offsets[i] = exclusive prefix of counts, block by block; raises *mismatch
// if it differs from the offsets already there (the ones the pass used).
__global__ void __launch_bounds__(kScanThreads) apply_offsets_kernel(const uint32_t *counts,
                                                                     int64_t n, int64_t chunk,
                                                                     const uint64_t *sums,
                                                                     int64_t *offsets,
                                                                     int *mismatch) {
    __shared__ uint64_t s_warp[kScanThreads / 32];
    __shared__ uint64_t s_carry;
    const int64_t lo = blockIdx.x * chunk, hi = min(n, lo + chunk);
    if (threadIdx.x == 0) s_carry = sums[blockIdx.x];
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    bool differ = false;
    for (int64_t base = lo; base < hi; base += blockDim.x) {
        const int64_t i = base + threadIdx.x;
        const uint64_t v = i < hi ? counts[i] : 0;
        uint64_t incl = v;
        for (int o = 1; o < 32; o <<= 1) {
            const uint64_t t = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += t;
        }
        if (lane == 31) s_warp[warp] = incl;
        __syncthreads();
        if (warp == 0) {
            const uint64_t w = s_warp[lane];
            uint64_t wi = w;
            for (int o = 1; o < 32; o <<= 1) {
                const uint64_t t = __shfl_up_sync(0xffffffffu, wi, o);
                if (lane >= o) wi += t;
            }
            s_warp[lane] = wi - w;
        }
        __syncthreads();
        const uint64_t carry = s_carry;
        if (i < hi) {
            const int64_t off = (int64_t)(carry + s_warp[warp] + incl - v);
            if (offsets[i] != off) differ = true;
            offsets[i] = off;
        }
        __syncthreads();
        if (threadIdx.x == blockDim.x - 1) s_carry = carry + s_warp[warp] + incl;
        __syncthreads();
    }
    if (differ) atomicOr(mismatch, 1);
}

__global__ void fill_counts_kernel(uint32_t *counts, int64_t n, uint32_t v) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        counts[i] = v;
}

__global__ void advance_state_kernel(uint64_t *state, const uint64_t *total) {
    *state += *total * kGolden;
}

// ------------------------------------------------------------------ launcher

constexpr int kMaxSrPasses = 8;

int launch_gemm_sr(Workspace &ws, ScheduleCache &cache, const drift_policy *p, int64_t M,
                   int64_t N, int64_t K, const double *A, int64_t a_rs, int64_t a_ks,
                   const double *B, int64_t b_rs, int64_t b_ks, const double *bias, double *C,
                   int64_t c_rs, uint64_t *d_state, cudaStream_t st) {
    if (p->acc != DRIFT_ACC_FP16 && p->acc != DRIFT_ACC_BF16) return DRIFT_EINVAL;
    if (!d_state) return DRIFT_EINVAL;  // Java: NullPointerException on the first draw
    const int64_t n = M * N;
    if (n == 0) return DRIFT_OK;
    GemmSrArgs g{};
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
    g.acc_block = std::max<int64_t>(1, p->acc_block);
    g.order = p->order;
    int64_t roundings = K;  // draws a dot makes when every sum is inexact
    if (p->order == DRIFT_PAIRWISE) {
        const uint8_t *d = cache.get(K, st);
        if (!d) return cache.last_status();
        g.leaf_len = d;
        g.leaf_merges = d + cache.leaves(K) + 1;
        roundings = K + std::max<int64_t>(0, cache.leaves(K) - 1);
    }
    if (roundings > 0xffffffffLL) return DRIFT_EUNSUPPORTED;

    const int64_t chunk = 64 * kScanThreads;
    const int64_t nb = (n + chunk - 1) / chunk;
    const size_t bytes = n * sizeof(int64_t) + n * sizeof(uint32_t) + (nb + 1) * sizeof(uint64_t) +
                         2 * sizeof(uint64_t) + 64;
    char *w = (char *)ws.get(bytes, st);
    if (!w) return DRIFT_ENOMEM;
    int64_t *offsets = (int64_t *)w;
    uint32_t *counts = (uint32_t *)(w + n * sizeof(int64_t));
    uint64_t *sums = (uint64_t *)(w + n * sizeof(int64_t) + ((n * sizeof(uint32_t) + 7) & ~7ULL));
    int *mismatch = (int *)(sums + nb + 2);
    g.state = d_state;
    g.offsets = offsets;
    g.counts = counts;

    auto launch_pass = [&]() {
        if (p->acc == DRIFT_ACC_FP16)
            gemm_sr_kernel<DRIFT_ACC_FP16><<<(unsigned)((n + 127) / 128), 128, 0, st>>>(g);
        else
            gemm_sr_kernel<DRIFT_ACC_BF16><<<(unsigned)((n + 127) / 128), 128, 0, st>>>(g);
    };
    auto scan = [&]() {
        cudaMemsetAsync(mismatch, 0, sizeof(int), st);
        block_sums_kernel<<<(unsigned)nb, kScanThreads, 0, st>>>(counts, n, chunk, sums);
        scan_sums_kernel<<<1, 32, 0, st>>>(sums, nb);
        apply_offsets_kernel<<<(unsigned)nb, kScanThreads, 0, st>>>(counts, n, chunk, sums, offsets,
                                                                    mismatch);
    };
    if ((n + 127) / 128 > 0x7fffffffLL) return DRIFT_EINVAL;

    // The first prediction: every rounding draws.
    fill_counts_kernel<<<148 * 8, 256, 0, st>>>(counts, n, (uint32_t)roundings);
    cudaMemsetAsync(offsets, 0xff, n * sizeof(int64_t), st);  // differs from any real offset
    scan();
    bool settled = false;
    for (int pass = 0; pass < kMaxSrPasses && !settled; pass++) {
        launch_pass();
        scan();
        int flag = 1;
        if (cudaMemcpyAsync(&flag, mismatch, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
            cudaStreamSynchronize(st) != cudaSuccess)
            return DRIFT_ECUDA;
        settled = flag == 0;
    }
    uint64_t *total = sums + nb;
    if (!settled) {
        if (p->acc == DRIFT_ACC_FP16)
            gemm_sr_serial_kernel<DRIFT_ACC_FP16><<<1, 1, 0, st>>>(g, total);
        else
            gemm_sr_serial_kernel<DRIFT_ACC_BF16><<<1, 1, 0, st>>>(g, total);
    }
    advance_state_kernel<<<1, 1, 0, st>>>(d_state, total);
    return cudaGetLastError() == cudaSuccess ? DRIFT_OK : DRIFT_ECUDA;
}

}  // namespace drift
