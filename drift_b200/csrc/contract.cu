// contract.cu — batched, ragged and causal contractions, and every
// contraction with a stochastically rounded accumulator.
//
// Output (t, i, o) of a contraction is Dot.dot over the window k in
// [lo(i), lo(i) + n(i)) of A[t, i, k] * B[t, o, k], the term at k = lo(i)
// first (Dot.dot's index 0). The windows are AttnPass's
// (java/src/main/java/io/drift/train/AttnPass.java): the whole depth for the
// score and dProb matmuls (:245-255, :373-381), the prefix [0, i] for the
// context and dq matmuls (:283-288, :412-417), the suffix [i, depth) for dv
// and dk (:382-388, :419-424). Causal contractions write 0.0 for o > i
// without a dot, as those loops do. The result is dot * alpha (the score
// scale, :248) when alpha is not 1, plus bias[o] for a linear, added into C
// for an accumulating dInput (:478-484).
//
// One output per thread, operands through the read-only cache with any
// strides: the attention shapes are small and ragged, and every order needs
// its own per-row tree.
//
// Stochastic accumulation. Dot.round with STOCHASTIC (Dot.java:171-175)
// draws from the Rng the caller shares across dots, in the order the dots run
// ((t, i, o) loops) and, inside a dot, in its evaluation order, and only when
// the sum is not exactly representable. So dot j starts drawing at D_j = the
// draws of dots 0..j-1, which the earlier dots' data decide. The engine finds
// the D_j by a fixed point: it predicts every dot's count, scans the
// predictions into offsets, computes all dots in parallel from those offsets
// (splitmix64 is counter-based, so any draw is available directly), and
// records each dot's true count. If the scan of the true counts gives back
// the offsets that were used, every dot started at the right draw (by
// induction from D_0 = 0) and the result is the sequential one. Otherwise the
// new offsets are used and the pass repeats. The first prediction — one draw
// per rounding the order performs — is exact unless some sum is exactly
// representable, so one pass usually settles it. After a bounded number of
// passes the dots are walked in order by one thread, which is correct for any
// data. Nothing spins: each pass is a separate launch and the host reads a
// flag between them.
#include <algorithm>
#include <type_traits>

#include "codec.cuh"
#include "internal.h"

namespace drift {

struct ContractArgs {
    int64_t batch, rows, cols, depth;
    const double *A;
    int64_t a_batch, a_row, a_k;
    const double *B;
    int64_t b_batch, b_col, b_k;
    double *C;
    int64_t c_batch, c_row, c_col;
    const double *bias;
    double alpha;
    int window, causal, accumulate, order;
    int64_t acc_block;
    const uint64_t *state;   // Rng state before the first draw (stochastic only)
    const int64_t *offsets;  // first draw index of each dot, (t, i, o) order
    uint32_t *counts;        // draws each dot made
    const int *skip;         // staged kernel: leave at once if this word is nonzero
    int *route;              // staged kernel: receives DRIFT_ROUTE_STAGED when given
};

__device__ __forceinline__ void window_of(const ContractArgs &g, int64_t i, int64_t &lo,
                                          int64_t &n) {
    if (g.window == DRIFT_WINDOW_PREFIX) {
        lo = 0;
        n = i + 1;
    } else if (g.window == DRIFT_WINDOW_SUFFIX) {
        lo = i;
        n = g.depth - i;
    } else {
        lo = 0;
        n = g.depth;
    }
}

// Dot.round(x, acc, STOCHASTIC, rng) (Dot.java:141-182), drawing the
// (idx + cnt)-th number of the stream only when the fraction is non-zero.
// `z` is the splitmix64 counter of the next draw, state + (idx + cnt + 1) *
// golden; a dot's draws are consecutive, so it advances by golden per draw.
//
// A sum in the accumulator's normal range below its top binade (every sum of
// ordinary data) is rounded on its bit pattern with integer operations only:
// its S = 52 - mant low significand bits are the fraction, scaled by 2^S;
// Java draws when they are non-zero, rounds up when nextDouble() < frac,
// that is when (mix >> 11) * 2^-53 < dropped * 2^-S, which for integers is
// (mix >> (64 - S)) < dropped; and rounding up adds 1 at bit S (a carry into
// the exponent is the next binade's value). No saturation can occur below the
// top binade. The other sums take the general form below.
template <int ACC>
__device__ __forceinline__ double sr_round(double x, uint64_t &z, uint32_t &cnt) {
    using F = AccFmt<ACC>;
    constexpr int S = 52 - F::mant;
    const uint64_t bits = (uint64_t)__double_as_longlong(x);
    const unsigned ex = (unsigned)(bits >> 52) & 0x7FFu;
    if (ex - (unsigned)(1023 + F::min_exp) <= (unsigned)(F::max_exp - 1 - F::min_exp)) {
        const uint64_t dropped = bits & ((1ULL << S) - 1);
        uint64_t r = bits - dropped;
        if (dropped != 0) {
            const uint64_t mix = splitmix_mix(z);
            z += kGolden;
            cnt++;
            if ((mix >> (64 - S)) < dropped) r += 1ULL << S;
        }
        return __longlong_as_double((long long)r);
    }
    if (x == 0.0 || isnan(x)) return x;
    const double ax = fabs(x);
    if (isinf(ax)) return copysign(F::max(), x);
    int e = java_get_exponent(ax);
    if (e < F::min_exp) e = F::min_exp;
    const int q = e - F::mant;
    const double scaled = __dmul_rn(ax, pow2(-q));  // exact
    const double fl = floor_small(scaled);  // scaled < 2^(mant+1)
    const double frac = __dsub_rn(scaled, fl);
    double m = fl;
    if (frac != 0.0) {
        const uint64_t u = splitmix_mix(z) >> 11;  // draw_u53(state, idx + cnt)
        z += kGolden;
        cnt++;
        if (__dmul_rn(u53_to_double(u), 0x1p-53) < frac) m = fl + 1.0;
    }
    double r = __dmul_rn(m, pow2(q));
    if (r > F::max()) r = F::max();
    return copysign(r, x);
}

// The accumulator's rounding after each add (Dot.java:43-63): identity for
// FP64, (float) for FP32, Dot.round for FP16/BF16.
template <int ACC, int RM> struct ExactRounder {
    __device__ double operator()(double t) {
        // The contraction kernel's fast rounding (FastForm), checked on the
        // sum's range word; the exact form only when the sum lies outside
        // the accumulator's normal range below its top binade. The low word
        // of the magic constant is zero here (any accumulator value's low
        // word keeps the rounding exact; zero is one).
        using R = AccRound<ACC, RM>;
        unsigned u;
        const double r = R::step(t, 0, u);
        return R::valid(R::fold2(0u, u, u)) ? r : R::exact(t);
    }
};

template <int ACC> struct SrRounder {
    uint64_t z;  // counter of the next draw: state + (first index + cnt + 1) * golden
    uint32_t cnt;
    __device__ SrRounder(uint64_t state, uint64_t idx) : z(state + (idx + 1) * kGolden), cnt(0) {}
    __device__ double operator()(double t) { return sr_round<ACC>(t, z, cnt); }
};

// Dot.dot (Dot.java:26-121) over n terms a[k*a_k] * b[k*b_k], any order.
// `term(k)` is the k-th product of the window (k from 0); it is called with
// the k of Dot.dot's evaluation order, so a caller may stage the operands.
template <int ACC, class T, class R>
__device__ double dot_terms(const ContractArgs &g, T term, int64_t n, R &rnd) {
    // The adds form one dependent chain; the products do not. With a rounding
    // accumulator the chain is long, so eight products are formed ahead of
    // their adds and their loads are in flight together. An FP64 chain is a
    // bare add: there, occupancy hides the loads and the extra registers cost
    // more than they save (19% at batch 64, t 256, d 64).
    constexpr int CH = ACC == DRIFT_ACC_FP64 ? 1 : 8;
    auto fwd = [&](int64_t from, int64_t count) {  // Dot.forward (:37-68)
        double s = 0.0;
        const int64_t end = from + count;
        int64_t k = from;
        for (; CH > 1 && k + 8 <= end; k += 8) {
            double p[8];
#pragma unroll
            for (int j = 0; j < 8; j++) p[j] = term(k + j);
#pragma unroll
            for (int j = 0; j < 8; j++) s = rnd(__dadd_rn(s, p[j]));
        }
        for (; k < end; k++) s = rnd(__dadd_rn(s, term(k)));
        return s;
    };
    if (g.order == DRIFT_SEQUENTIAL) return fwd(0, n);
    if (g.order == DRIFT_REVERSED) {  // Dot.backward (:70-84)
        double s = 0.0;
        int64_t k = n - 1;
        for (; CH > 1 && k >= 7; k -= 8) {
            double p[8];
#pragma unroll
            for (int j = 0; j < 8; j++) p[j] = term(k - j);
#pragma unroll
            for (int j = 0; j < 8; j++) s = rnd(__dadd_rn(s, p[j]));
        }
        for (; k >= 0; k--) s = rnd(__dadd_rn(s, term(k)));
        return s;
    }
    if (g.order == DRIFT_BLOCKED) {  // Dot.blocked (:104-121)
        double total = 0.0;
        for (int64_t start = 0; start < n; start += g.acc_block) {
            const double partial = fwd(start, min(g.acc_block, n - start));
            total = ACC == DRIFT_ACC_FP64 ? __dadd_rn(total, partial)
                                          : (double)__double2float_rn(__dadd_rn(total, partial));
        }
        return total;
    }
    // Dot.pairwise (:86-102): halves of count >>> 1, leaves of at most 8,
    // left subtree, right subtree, then the combine. An explicit stack of
    // pending nodes (count < 0 marks a combine) and of finished values; for
    // n < 2^31 the tree is at most 28 splits deep.
    if (n <= 8) return fwd(0, n);
    int64_t todo_off[60], todo_cnt[60];
    double vals[32];
    int tp = 1, vp = 0;
    todo_off[0] = 0;
    todo_cnt[0] = n;
    while (tp > 0) {
        tp--;
        const int64_t off = todo_off[tp], cnt = todo_cnt[tp];
        if (cnt < 0) {
            vp--;
            vals[vp - 1] = rnd(__dadd_rn(vals[vp - 1], vals[vp]));
        } else if (cnt <= 8) {
            vals[vp++] = fwd(off, cnt);
        } else {
            const int64_t half = cnt >> 1;
            todo_cnt[tp++] = -1;
            todo_off[tp] = off + half;
            todo_cnt[tp++] = cnt - half;
            todo_off[tp] = off;
            todo_cnt[tp++] = half;
        }
    }
    return vals[0];
}

template <int ACC, class R>
__device__ double dot_any(const ContractArgs &g, const double *a, const double *b, int64_t n,
                          R &rnd) {
    return dot_terms<ACC>(
        g, [&](int64_t k) { return __dmul_rn(__ldg(a + k * g.a_k), __ldg(b + k * g.b_k)); }, n,
        rnd);
}

// Leaves of Dot.pairwise's tree over n terms. Node sizes on one level differ
// by at most one, so two (size, count) slots carry a level.
__device__ __forceinline__ int64_t pairwise_leaves(int64_t n) {
    int64_t s0 = n, c0 = 1, c1 = 0, leaves = 0;  // sizes s0 and s0 + 1
    while (c0 + c1 > 0) {
        int64_t t0 = 0, t1 = 0;
        const int64_t ns0 = s0 >> 1;  // children of s0: ns0 and s0 - ns0
        auto add = [&](int64_t size, int64_t count) {
            if (count == 0) return;
            if (size == ns0) t0 += count;
            else t1 += count;  // size == ns0 + 1
        };
        int64_t sz[2] = {s0, s0 + 1}, ct[2] = {c0, c1};
        for (int j = 0; j < 2; j++) {
            if (ct[j] == 0) continue;
            if (sz[j] <= 8) {
                leaves += ct[j];
            } else {
                add(sz[j] >> 1, ct[j]);
                add(sz[j] - (sz[j] >> 1), ct[j]);
            }
        }
        s0 = ns0;
        c0 = t0;
        c1 = t1;
    }
    return leaves;
}

// Draws a dot of n terms makes when every sum is inexact: one per rounding.
__device__ __forceinline__ int64_t predicted_draws(int order, int64_t n) {
    if (n <= 0) return 0;
    return order == DRIFT_PAIRWISE ? n + pairwise_leaves(n) - 1 : n;
}

__device__ __forceinline__ void store(const ContractArgs &g, double *c, int64_t o, double v) {
    if (g.alpha != 1.0) v = __dmul_rn(v, g.alpha);
    if (g.bias) v = __dadd_rn(v, g.bias[o]);
    if (g.accumulate) v = __dadd_rn(*c, v);
    *c = v;
}

template <int ACC, int RM>
__global__ void __launch_bounds__(128) contract_kernel(const ContractArgs g) {
    const int64_t total = g.batch * g.rows * g.cols;
    for (int64_t out = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; out < total;
         out += (int64_t)gridDim.x * blockDim.x) {
        const int64_t o = out % g.cols, ti = out / g.cols;
        const int64_t i = ti % g.rows, t = ti / g.rows;
        double *c = g.C + t * g.c_batch + i * g.c_row + o * g.c_col;
        if (g.causal && o > i) {
            *c = 0.0;
            continue;
        }
        int64_t lo, n;
        window_of(g, i, lo, n);
        ExactRounder<ACC, RM> rnd;
        const double v = dot_any<ACC>(g, g.A + t * g.a_batch + i * g.a_row + lo * g.a_k,
                                      g.B + t * g.b_batch + o * g.b_col + lo * g.b_k, n, rnd);
        store(g, c, o, v);
    }
}

// The value of output `out` before it meets C (dot * alpha + bias), drawing
// from index idx on; 0.0 and no draws for a masked causal output.
template <int ACC>
__device__ __forceinline__ double sr_output(const ContractArgs &g, int64_t out, uint64_t idx,
                                            uint32_t &cnt) {
    const int64_t o = out % g.cols, i = (out / g.cols) % g.rows, t = out / g.cols / g.rows;
    cnt = 0;
    if (g.causal && o > i) return 0.0;
    int64_t lo, n;
    window_of(g, i, lo, n);
    SrRounder<ACC> rnd(*g.state, idx);
    double v = dot_any<ACC>(g, g.A + t * g.a_batch + i * g.a_row + lo * g.a_k,
                            g.B + t * g.b_batch + o * g.b_col + lo * g.b_k, n, rnd);
    cnt = rnd.cnt;
    if (g.alpha != 1.0) v = __dmul_rn(v, g.alpha);
    if (g.bias) v = __dadd_rn(v, g.bias[o]);
    return v;
}

// One speculative pass: every dot from its offset into the scratch values,
// its true count recorded. C is written once, after the offsets settle.
template <int ACC>
__global__ void __launch_bounds__(128) contract_sr_kernel(const ContractArgs g, double *vals) {
    const int64_t total = g.batch * g.rows * g.cols;
    for (int64_t out = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; out < total;
         out += (int64_t)gridDim.x * blockDim.x) {
        uint32_t cnt;
        vals[out] = sr_output<ACC>(g, out, (uint64_t)g.offsets[out], cnt);
        g.counts[out] = cnt;
    }
}

// ------------------------------------------------------------ staged stochastic pass
//
// With a FULL window every dot has the same length and order, so every thread
// of a CTA asks for the same terms in the same sequence (for pairwise, the
// same tree). A CTA of 16 x 16 outputs of one problem stages its operands in
// shared memory KC terms at a time: when a thread needs a k outside the staged
// chunk, every thread does, and they refill it together between two
// barriers. The products then come from shared memory instead of a pair of
// global loads per term. Threads past the matrix edge take part in every
// refill and store nothing, so the CTA's control flow stays uniform.
constexpr int kStageSide = 16;
constexpr int kStageK = 32;

template <int ACC>
__global__ void __launch_bounds__(kStageSide *kStageSide)
    contract_sr_staged_kernel(const ContractArgs g, double *vals) {
    __shared__ double sA[kStageSide][kStageK + 1], sB[kStageSide][kStageK + 1];
    const int tx = threadIdx.x % kStageSide, ty = threadIdx.x / kStageSide;
    const int64_t t = blockIdx.z;
    const int64_t i0 = (int64_t)blockIdx.y * kStageSide, o0 = (int64_t)blockIdx.x * kStageSide;
    const int64_t i = i0 + ty, o = o0 + tx;
    const bool live = i < g.rows && o < g.cols;
    const double *At = g.A + t * g.a_batch, *Bt = g.B + t * g.b_batch;
    int64_t k0 = -kStageK;  // start of the staged chunk (none yet)
    auto stage = [&](int64_t base) {
        __syncthreads();  // every thread has finished with the previous chunk
        for (int e = threadIdx.x; e < kStageSide * kStageK; e += kStageSide * kStageSide) {
            const int r = e / kStageK, c = e % kStageK;  // consecutive threads walk k
            const int64_t k = base + c;
            const bool kin = k < g.depth;
            sA[r][c] = (kin && i0 + r < g.rows) ? __ldg(At + (i0 + r) * g.a_row + k * g.a_k) : 0.0;
            sB[r][c] = (kin && o0 + r < g.cols) ? __ldg(Bt + (o0 + r) * g.b_col + k * g.b_k) : 0.0;
        }
        __syncthreads();
        k0 = base;
    };
    auto term = [&](int64_t k) {
        if (k < k0 || k >= k0 + kStageK) stage(k - k % kStageK);  // the same k in every thread
        return __dmul_rn(sA[ty][k - k0], sB[tx][k - k0]);
    };
    const int64_t out = (t * g.rows + i) * g.cols + o;
    SrRounder<ACC> rnd(*g.state, live ? (uint64_t)g.offsets[out] : 0);
    double v = dot_terms<ACC>(g, term, g.depth, rnd);
    if (!live) return;
    if (g.alpha != 1.0) v = __dmul_rn(v, g.alpha);
    if (g.bias) v = __dadd_rn(v, g.bias[o]);
    vals[out] = v;
    g.counts[out] = rnd.cnt;
}

// Orders the staged kernel walks chunk by chunk with a fixed body: the
// sequential and reversed chains over any window, and blocked chains whose
// blocks end on 32-term chunk edges when every window starts at term 0.
__host__ __device__ inline bool staged_walk(int order, int64_t acc_block, int window) {
    return order == DRIFT_SEQUENTIAL || order == DRIFT_REVERSED ||
           (order == DRIFT_BLOCKED && acc_block % kStageK == 0 && window != DRIFT_WINDOW_SUFFIX);
}

// One output per thread with nearest or truncating accumulation, the
// operands staged CTA-wide in 32-term chunks as above. Two routes use it:
// FULL-window contractions whose outputs are too few to fill the GPU with the
// tiled kernel's 64 x 64 tiles (a batch-64 linear layer gives 32 of them, so
// 32 SMs each ran sixteen 2048-long chains per thread while the rest idled),
// and the ragged PREFIX / SUFFIX windows of the attention matmuls in the
// orders it walks chunk by chunk (staged_walk).
// Four CTAs per SM (64 registers a thread): a batch-64 linear layer's 512
// CTAs then fit the GPU in one wave.
template <int ACC, int RM>
__global__ void __launch_bounds__(kStageSide *kStageSide, 4)
    contract_staged_kernel(const ContractArgs g) {
    if (g.skip && *g.skip) return;  // the FP32 pipe (gemm32.cu) took the call
    if (g.route && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && threadIdx.x == 0)
        *g.route = DRIFT_ROUTE_STAGED;
    // Two buffers: the chunk walk fills one while it reads the other. Rows are
    // padded to an even length so each starts 16-byte aligned and the fixed
    // body reads two terms per load.
    constexpr int kRow = kStageK + 2;
    __shared__ __align__(16) double sA[2][kStageSide][kRow], sB[2][kStageSide][kRow];
    const int tx = threadIdx.x % kStageSide, ty = threadIdx.x / kStageSide;
    const int64_t t = blockIdx.z;
    const int64_t i0 = (int64_t)blockIdx.y * kStageSide, o0 = (int64_t)blockIdx.x * kStageSide;
    const int64_t i = i0 + ty, o = o0 + tx;
    const bool live = i < g.rows && o < g.cols;
    const double *At = g.A + t * g.a_batch, *Bt = g.B + t * g.b_batch;
    int64_t k0 = -kStageK;
    // Consecutive threads walk whichever axis of an operand has unit stride
    // (k for a row-major operand, rows for one read down its columns, as
    // AttnPass's dv reads the probabilities), so each warp's loads coalesce.
    const bool a_kfast = g.a_k == 1 || g.a_row != 1, b_kfast = g.b_k == 1 || g.b_col != 1;
    constexpr int kPer = kStageSide * kStageK / (kStageSide * kStageSide);  // elements per thread
    double fa[kPer], fb[kPer];
    auto fetch = [&](int64_t base) {  // this thread's share of a chunk, into registers
#pragma unroll
        for (int j = 0; j < kPer; j++) {
            const int e = threadIdx.x + j * kStageSide * kStageSide;
            int r = a_kfast ? e / kStageK : e % kStageSide;
            int c = a_kfast ? e % kStageK : e / kStageSide;
            int64_t k = base + c;
            fa[j] = (k < g.depth && i0 + r < g.rows) ? __ldg(At + (i0 + r) * g.a_row + k * g.a_k)
                                                     : 0.0;
            r = b_kfast ? e / kStageK : e % kStageSide;
            c = b_kfast ? e % kStageK : e / kStageSide;
            k = base + c;
            fb[j] = (k < g.depth && o0 + r < g.cols) ? __ldg(Bt + (o0 + r) * g.b_col + k * g.b_k)
                                                     : 0.0;
        }
    };
    auto put = [&](int buf) {
#pragma unroll
        for (int j = 0; j < kPer; j++) {
            const int e = threadIdx.x + j * kStageSide * kStageSide;
            sA[buf][a_kfast ? e / kStageK : e % kStageSide][a_kfast ? e % kStageK : e / kStageSide] =
                fa[j];
            sB[buf][b_kfast ? e / kStageK : e % kStageSide][b_kfast ? e % kStageK : e / kStageSide] =
                fb[j];
        }
    };
    auto stage = [&](int64_t base) {  // the general walk: one buffer, staged on demand
        __syncthreads();
        fetch(base);
        put(0);
        __syncthreads();
        k0 = base;
    };
    ExactRounder<ACC, RM> rnd;
    auto step = [&](double acc, double a, double b) {  // Dot.forward's add (:46, :54, :63)
        const double t = __dadd_rn(acc, __dmul_rn(a, b));
        return ACC == DRIFT_ACC_FP64 ? t : rnd(t);
    };
    double v;
    if (staged_walk(g.order, g.acc_block, g.window)) {
        // One staged chunk at a time with a fixed 32-term body: the chunk
        // walk of Dot.forward / backward, and of Dot.blocked when its chunks
        // end on chunk edges. (The per-term window check of the general walk
        // below cost 34 instructions per multiply-accumulate.) Chunks sit at
        // absolute multiples of 32 and cover the union of the tile's windows;
        // each thread takes the part inside its own window (AttnPass's PREFIX
        // and SUFFIX rows differ by at most 16 terms within a tile), the fixed
        // body where that is the whole chunk. The next chunk's loads are in
        // flight while this one is summed.
        const bool rev = g.order == DRIFT_REVERSED, blk = g.order == DRIFT_BLOCKED;
        int64_t lo, n;
        window_of(g, i, lo, n);  // rows past the end are clamped into range
        lo = lo < g.depth ? lo : g.depth;
        const int64_t hi = lo + (n < 0 ? 0 : (n < g.depth - lo ? n : g.depth - lo));
        const int64_t last = (i0 + kStageSide < g.rows ? i0 + kStageSide : g.rows) - 1;
        int64_t u_lo = 0, u_hi = g.depth;  // the tile's union of windows
        if (g.window == DRIFT_WINDOW_PREFIX) u_hi = last + 1 < g.depth ? last + 1 : g.depth;
        if (g.window == DRIFT_WINDOW_SUFFIX) u_lo = i0 < g.depth ? i0 : g.depth;
        const int64_t ch_lo = u_lo / kStageK, ch_hi = (u_hi + kStageK - 1) / kStageK;
        const int64_t nc = ch_hi - ch_lo;
        auto chunk_of = [&](int64_t c) { return rev ? ch_hi - 1 - c : ch_lo + c; };
        double acc = 0.0, total = 0.0;
        // A whole chunk, eight steps at a time on the fast rounding with one
        // range check for the eight; a miss redoes them exactly from the sum
        // before them (as the tiled kernel's groups do across outputs): every
        // fast result that passes is the exact one. REV walks it downwards.
        auto whole = [&](const double *ra, const double *rb, auto rev_c) {
            constexpr bool REV = decltype(rev_c)::value;
#pragma unroll 2
            for (int q0 = 0; q0 < kStageK; q0 += 8) {
                // Terms q0 .. q0+7 of the walk, read as four aligned pairs
                // (reversed: pairs from the top of the chunk down).
                const double *pa = REV ? ra + (kStageK - 2 - q0) : ra + q0;
                const double *pb = REV ? rb + (kStageK - 2 - q0) : rb + q0;
                double pr[8];
#pragma unroll
                for (int jj = 0; jj < 4; jj++) {
                    const int off = REV ? -2 * jj : 2 * jj;
                    const double2 xa = *reinterpret_cast<const double2 *>(pa + off);
                    const double2 xb = *reinterpret_cast<const double2 *>(pb + off);
                    pr[2 * jj] = __dmul_rn(REV ? xa.y : xa.x, REV ? xb.y : xb.x);
                    pr[2 * jj + 1] = __dmul_rn(REV ? xa.x : xa.y, REV ? xb.x : xb.y);
                }
                if constexpr (ACC == DRIFT_ACC_FP64) {
#pragma unroll
                    for (int j = 0; j < 8; j++) acc = __dadd_rn(acc, pr[j]);
                } else {
                    using R = AccRound<ACC, RM>;
                    const double s0 = acc;
                    unsigned run = 0, u[8];
#pragma unroll
                    for (int j = 0; j < 8; j++)
                        acc = R::step(__dadd_rn(acc, pr[j]), __double2loint(acc), u[j]);
#pragma unroll
                    for (int j = 0; j < 8; j += 2) run = R::fold2(run, u[j], u[j + 1]);
                    if (!R::valid(run)) {
                        acc = s0;
#pragma unroll
                        for (int j = 0; j < 8; j++) acc = R::exact(__dadd_rn(acc, pr[j]));
                    }
                }
            }
        };
        // FP64 chains (a bare add per step) fetch the next chunk while they
        // sum this one. The rounding chains fetch at the top of each chunk:
        // holding the next chunk in registers cost them more than the hidden
        // load latency gave back (measured on one B200). Either way a buffer
        // is written only after every thread has passed the barrier that
        // follows its last reading, so one barrier per chunk suffices.
        constexpr bool PF = ACC == DRIFT_ACC_FP64;
        if (PF && nc > 0) {
            fetch(chunk_of(0) * kStageK);
            put(0);
        }
        __syncthreads();
        for (int64_t c = 0; c < nc; c++) {
            const int64_t cc = chunk_of(c), c0 = cc * kStageK;
            if (!PF) {
                fetch(c0);
                put(c & 1);  // last read two chunks ago
                __syncthreads();
            } else if (c + 1 < nc) {
                fetch(chunk_of(c + 1) * kStageK);  // in flight during the sums
            }
            const double *ra = sA[c & 1][ty], *rb = sB[c & 1][tx];
            const int qa = (int)(lo > c0 ? (lo - c0 < kStageK ? lo - c0 : kStageK) : 0);
            const int qb = (int)(hi > c0 ? (hi - c0 < kStageK ? hi - c0 : kStageK) : 0);
            if (qa < qb) {
                if (qa == 0 && qb == kStageK) {
                    if (rev) whole(ra, rb, std::true_type{});
                    else whole(ra, rb, std::false_type{});
                } else if (!rev) {
                    for (int q = qa; q < qb; q++) acc = step(acc, ra[q], rb[q]);
                } else {
                    for (int q = qb - 1; q >= qa; q--) acc = step(acc, ra[q], rb[q]);
                }
                // Dot.blocked (:115-118): a chunk of acc_block from the
                // window's start (0 here) closes on a block edge or at the
                // window's end.
                if (blk && (((cc + 1) * kStageK) % g.acc_block == 0 || hi <= c0 + kStageK)) {
                    total = ACC == DRIFT_ACC_FP64
                                ? __dadd_rn(total, acc)
                                : (double)__double2float_rn(__dadd_rn(total, acc));
                    acc = 0.0;
                }
            }
            if (PF) {
                if (c + 1 < nc) put((c + 1) & 1);  // that buffer was last read before the barrier
                __syncthreads();
            }
        }
        v = blk ? total : acc;
    } else if (g.order == DRIFT_PAIRWISE && g.depth >= kStageK &&
               (g.depth & (g.depth - 1)) == 0) {
        // Dot.pairwise (:86-102) over a power-of-two depth: every split is
        // exact and every leaf is 8 long, so each aligned 32-term chunk is a
        // whole subtree ((leaf0 + leaf1) + (leaf2 + leaf3)), and the chunks
        // combine as a perfect binary tree: after chunk c, ctz(c + 1) merges
        // of the pending nodes (left operand first, as the recursion's
        // post-order gives). One staged chunk at a time, double-buffered as
        // in the walk above; a thread's pending nodes stay in its own stack.
        const int64_t nc = g.depth / kStageK;
        double stk[32];  // log2(nc) + 1 entries; depth < 2^36
        int sp = 0;
        __syncthreads();
        for (int64_t c = 0; c < nc; c++) {
            fetch(c * kStageK);
            put(c & 1);  // last read two chunks ago
            __syncthreads();
            const double *ra = sA[c & 1][ty], *rb = sB[c & 1][tx];
            double leaf[4];
#pragma unroll
            for (int l = 0; l < 4; l++) {
                double p[8];
#pragma unroll
                for (int j = 0; j < 8; j++) p[j] = __dmul_rn(ra[8 * l + j], rb[8 * l + j]);
                double sum = 0.0;
#pragma unroll
                for (int j = 0; j < 8; j++) sum = rnd(__dadd_rn(sum, p[j]));
                leaf[l] = sum;
            }
            double node = rnd(__dadd_rn(rnd(__dadd_rn(leaf[0], leaf[1])),
                                        rnd(__dadd_rn(leaf[2], leaf[3]))));
            for (int64_t m = c + 1; (m & 1) == 0; m >>= 1) node = rnd(__dadd_rn(stk[--sp], node));
            stk[sp++] = node;
        }
        v = stk[0];
    } else {
        // FULL windows only (the launcher sends no other window here).
        auto term = [&](int64_t k) {
            if (k < k0 || k >= k0 + kStageK) stage(k - k % kStageK);  // the same k in every thread
            return __dmul_rn(sA[0][ty][k - k0], sB[0][tx][k - k0]);
        };
        v = dot_terms<ACC>(g, term, g.depth, rnd);
    }
    if (!live) return;
    double *c = g.C + t * g.c_batch + i * g.c_row + o * g.c_col;
    if (g.causal && o > i) *c = 0.0;
    else store(g, c, o, v);
}

// The dots in order, one thread: the fallback that is correct for any data.
template <int ACC>
__global__ void contract_sr_serial_kernel(const ContractArgs g, double *vals,
                                          uint64_t *total_draws) {
    if (blockIdx.x != 0 || threadIdx.x != 0) return;
    uint64_t idx = 0;
    const int64_t total = g.batch * g.rows * g.cols;
    for (int64_t out = 0; out < total; out++) {
        uint32_t cnt;
        vals[out] = sr_output<ACC>(g, out, idx, cnt);
        idx += cnt;
    }
    *total_draws = idx;
}

// C from the settled values: 0.0 where the causal mask hides the output,
// else the value, added into C for an accumulating contraction.
__global__ void contract_apply_kernel(const ContractArgs g, const double *vals) {
    const int64_t total = g.batch * g.rows * g.cols;
    for (int64_t out = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; out < total;
         out += (int64_t)gridDim.x * blockDim.x) {
        const int64_t o = out % g.cols, i = (out / g.cols) % g.rows, t = out / g.cols / g.rows;
        double *c = g.C + t * g.c_batch + i * g.c_row + o * g.c_col;
        if (g.causal && o > i) *c = 0.0;
        else *c = g.accumulate ? __dadd_rn(*c, vals[out]) : vals[out];
    }
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

// Exclusive scan of the block sums in place (one thread; a few thousand
// values at most); also writes the grand total to sums[nb].
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

// The first prediction of every dot's draw count.
__global__ void predict_counts_kernel(const ContractArgs g, uint32_t *counts) {
    const int64_t total = g.batch * g.rows * g.cols;
    for (int64_t out = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; out < total;
         out += (int64_t)gridDim.x * blockDim.x) {
        const int64_t o = out % g.cols, i = (out / g.cols) % g.rows;
        int64_t lo, n;
        window_of(g, i, lo, n);
        counts[out] = (g.causal && o > i) ? 0u : (uint32_t)predicted_draws(g.order, n);
    }
}

__global__ void advance_state_kernel(uint64_t *state, const uint64_t *total) {
    *state += *total * kGolden;
}

// ------------------------------------------------------------------ launcher

constexpr int kMaxSrPasses = 8;

static unsigned grid_of(int64_t total) {
    const int64_t blocks = (total + 127) / 128;
    return (unsigned)std::max<int64_t>(1, std::min<int64_t>(blocks, 148 * 64));
}

static ContractArgs args_of(const drift_policy *p, const ContractDesc &d) {
    ContractArgs g{};
    g.batch = d.op.batch;
    g.rows = d.op.rows;
    g.cols = d.op.cols;
    g.depth = d.op.depth;
    g.A = d.a + d.op.a_off;
    g.a_batch = d.op.a_batch;
    g.a_row = d.op.a_row;
    g.a_k = d.op.a_k;
    g.B = d.b + d.op.b_off;
    g.b_batch = d.op.b_batch;
    g.b_col = d.op.b_col;
    g.b_k = d.op.b_k;
    g.C = d.c + d.op.c_off;
    g.c_batch = d.op.c_batch;
    g.c_row = d.op.c_row;
    g.c_col = d.op.c_col;
    g.bias = d.bias;
    g.alpha = d.op.alpha;
    g.window = d.op.window;
    g.causal = d.op.causal;
    g.accumulate = d.op.accumulate;
    g.order = p->order;
    g.acc_block = std::max<int64_t>(1, p->acc_block);
    return g;
}

int check_contraction(const drift_contraction &op) {
    if (op.batch < 0 || op.rows < 0 || op.cols < 0 || op.depth < 0) return DRIFT_EINVAL;
    if (op.depth > 0x7fffffffLL) return DRIFT_EUNSUPPORTED;
    if (op.window != DRIFT_WINDOW_FULL && op.window != DRIFT_WINDOW_PREFIX &&
        op.window != DRIFT_WINDOW_SUFFIX)
        return DRIFT_EINVAL;
    if (op.window != DRIFT_WINDOW_FULL && op.rows > op.depth) return DRIFT_EINVAL;
    if ((op.causal | op.accumulate) & ~1 || op.reserved != 0) return DRIFT_EINVAL;
    if (op.a_off < 0 || op.b_off < 0 || op.c_off < 0) return DRIFT_EINVAL;
    return DRIFT_OK;
}

static bool stochastic(const drift_policy *p) {
    return p->acc_rounding == DRIFT_STOCHASTIC &&
           (p->acc == DRIFT_ACC_FP16 || p->acc == DRIFT_ACC_BF16);
}

// The score scale and the causal mask over a contraction the tiled kernel
// computed whole: masked outputs become 0.0, the others dot * alpha.
__global__ void contract_epilogue_kernel(const ContractArgs g) {
    const int64_t total = g.batch * g.rows * g.cols;
    for (int64_t out = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; out < total;
         out += (int64_t)gridDim.x * blockDim.x) {
        const int64_t o = out % g.cols, i = (out / g.cols) % g.rows, t = out / g.cols / g.rows;
        double *c = g.C + t * g.c_batch + i * g.c_row + o * g.c_col;
        if (g.causal && o > i) *c = 0.0;
        else if (g.alpha != 1.0) *c = __dmul_rn(*c, g.alpha);
    }
}

// A FULL-window contraction that writes (not adds) rows of C with unit
// column stride is a batch of plain contractions: the tiled TMA kernel of
// gemm.cu takes it, the causal upper triangle included (each output's dot is
// the same computation either way), and the epilogue then clears the masked
// outputs and applies the scale.
static bool tiled_route(const ContractDesc &d) {
    const drift_contraction &op = d.op;
    return op.window == DRIFT_WINDOW_FULL && !op.accumulate && op.c_col == 1 && !d.bias &&
           op.batch <= 65535 && (op.rows + 63) / 64 <= 65535 && op.c_row >= op.cols &&
           op.a_batch >= 0 && op.a_row >= 0 && op.a_k >= 0 && op.b_batch >= 0 && op.b_col >= 0 &&
           op.b_k >= 0 && op.c_batch >= 0;
}

static bool staged_fits(const drift_contraction &op) {
    return op.batch <= 65535 && (op.rows + kStageSide - 1) / kStageSide <= 65535 &&
           (op.cols + kStageSide - 1) / kStageSide <= 0x7fffffffLL;
}

int64_t staged_tile_limit(const drift_policy *p) {
    // Measured on one B200 (tiled time / staged time, K = 512-2048): at 32
    // tiles of 64 x 64 the staged kernel won everywhere (FP64 1.29, pairwise
    // 1.27, the chunk walks with a rounding accumulator 2.0-2.6); at 64 tiles
    // only the chunk walks still won (1.24-1.5; FP64 0.8, pairwise 0.7); at
    // 128 none did (0.4-0.86).
    const bool chunk_walk = p->order == DRIFT_SEQUENTIAL || p->order == DRIFT_REVERSED ||
                            (p->order == DRIFT_BLOCKED && std::max<int64_t>(1, p->acc_block) %
                                                             kStageK == 0);
    const int64_t sms = sm_count();
    return chunk_walk && p->acc != DRIFT_ACC_FP64 ? 2 * sms / 3 : sms / 3;
}

int launch_contract_staged(const drift_policy *p, const ContractDesc &d, const int *skip,
                           int *route, cudaStream_t st) {
    const drift_contraction &op = d.op;
    const int64_t blk = std::max<int64_t>(1, p->acc_block);
    if ((op.window != DRIFT_WINDOW_FULL && !staged_walk(p->order, blk, op.window)) ||
        stochastic(p) || !staged_fits(op))
        return DRIFT_EINVAL;
    if (op.batch * op.rows * op.cols == 0) return DRIFT_OK;
    ContractArgs g = args_of(p, d);
    g.skip = skip;
    g.route = route;
    const dim3 grid((unsigned)((op.cols + kStageSide - 1) / kStageSide),
                    (unsigned)((op.rows + kStageSide - 1) / kStageSide), (unsigned)op.batch);
    const unsigned threads = kStageSide * kStageSide;
    const bool tr = p->acc_rounding == DRIFT_TRUNCATE;
    switch (p->acc) {
        case DRIFT_ACC_FP64:
            contract_staged_kernel<DRIFT_ACC_FP64, DRIFT_NEAREST_EVEN><<<grid, threads, 0, st>>>(g);
            break;
        case DRIFT_ACC_FP32:
            contract_staged_kernel<DRIFT_ACC_FP32, DRIFT_NEAREST_EVEN><<<grid, threads, 0, st>>>(g);
            break;
        case DRIFT_ACC_FP16:
            if (tr) contract_staged_kernel<DRIFT_ACC_FP16, DRIFT_TRUNCATE><<<grid, threads, 0, st>>>(g);
            else contract_staged_kernel<DRIFT_ACC_FP16, DRIFT_NEAREST_EVEN><<<grid, threads, 0, st>>>(g);
            break;
        default:
            if (tr) contract_staged_kernel<DRIFT_ACC_BF16, DRIFT_TRUNCATE><<<grid, threads, 0, st>>>(g);
            else contract_staged_kernel<DRIFT_ACC_BF16, DRIFT_NEAREST_EVEN><<<grid, threads, 0, st>>>(g);
    }
    return cudaGetLastError() == cudaSuccess ? DRIFT_OK : DRIFT_ECUDA;
}

int launch_contract(Workspace &ws, ScheduleCache &cache, const drift_policy *p,
                    const ContractDesc &d, uint64_t *d_state, int *d_err, cudaStream_t st) {
    int rc = check_contraction(d.op);
    if (rc) return rc;
    const int64_t total = d.op.batch * d.op.rows * d.op.cols;
    if (total == 0) return DRIFT_OK;
    if (p->acc < DRIFT_ACC_FP64 || p->acc > DRIFT_ACC_BF16 || p->order < DRIFT_SEQUENTIAL ||
        p->order > DRIFT_BLOCKED)
        return DRIFT_EINVAL;
    ContractArgs g = args_of(p, d);
    const unsigned grid = grid_of(total);
    // Problems of fewer outputs than one staged CTA (a batch of single dots,
    // as the dot sweep runs them) go to the one-output-per-thread kernel: on
    // the tiled or staged kernels each such problem held a whole CTA that
    // walked all of K for a handful of live outputs (the dot sweep's 200-dot
    // batches ran 20x slower there).
    const bool tiny = d.op.rows * d.op.cols < (int64_t)kStageSide * kStageSide;

    if (!stochastic(p) && !tiny && tiled_route(d)) {
        const drift_contraction &op = d.op;
        rc = launch_gemm_batched(ws, cache, p, op.batch, op.rows, op.cols, op.depth, g.A, op.a_row,
                                 op.a_k, op.a_batch, g.B, op.b_col, op.b_k, op.b_batch, nullptr,
                                 g.C, op.c_row, op.c_batch, d_err, st);
        if (rc) return rc;
        if (op.causal || op.alpha != 1.0) contract_epilogue_kernel<<<grid, 128, 0, st>>>(g);
        return cudaGetLastError() == cudaSuccess ? DRIFT_OK : DRIFT_ECUDA;
    }
    // Ragged windows (and FULL ones the tiles do not take) in the orders the
    // staged kernel walks chunk by chunk: one output per thread with the
    // operands staged per 16 x 16 tile. Pairwise (a tree per row) and blocked
    // chunks off the chunk edges stay on the per-thread kernel below.
    if (!stochastic(p) && !tiny && staged_walk(p->order, g.acc_block, d.op.window) &&
        staged_fits(d.op))
        return launch_contract_staged(p, d, nullptr, nullptr, st);
    if (!stochastic(p)) {
        const bool tr = p->acc_rounding == DRIFT_TRUNCATE;
        switch (p->acc) {
            case DRIFT_ACC_FP64:
                contract_kernel<DRIFT_ACC_FP64, DRIFT_NEAREST_EVEN><<<grid, 128, 0, st>>>(g);
                break;
            case DRIFT_ACC_FP32:
                contract_kernel<DRIFT_ACC_FP32, DRIFT_NEAREST_EVEN><<<grid, 128, 0, st>>>(g);
                break;
            case DRIFT_ACC_FP16:
                if (tr) contract_kernel<DRIFT_ACC_FP16, DRIFT_TRUNCATE><<<grid, 128, 0, st>>>(g);
                else contract_kernel<DRIFT_ACC_FP16, DRIFT_NEAREST_EVEN><<<grid, 128, 0, st>>>(g);
                break;
            default:
                if (tr) contract_kernel<DRIFT_ACC_BF16, DRIFT_TRUNCATE><<<grid, 128, 0, st>>>(g);
                else contract_kernel<DRIFT_ACC_BF16, DRIFT_NEAREST_EVEN><<<grid, 128, 0, st>>>(g);
        }
        return cudaGetLastError() == cudaSuccess ? DRIFT_OK : DRIFT_ECUDA;
    }

    if (!d_state) return DRIFT_EINVAL;  // Java: NullPointerException on the first draw
    const int64_t chunk = 64 * kScanThreads;
    const int64_t nb = (total + chunk - 1) / chunk;
    const size_t count_bytes = (total * sizeof(uint32_t) + 7) & ~7ULL;
    const size_t bytes = total * sizeof(int64_t) + total * sizeof(double) + count_bytes +
                         (nb + 2) * sizeof(uint64_t) + 64;
    char *w = (char *)ws.get(bytes, st);
    if (!w) return DRIFT_ENOMEM;
    int64_t *offsets = (int64_t *)w;
    double *vals = (double *)(w + total * sizeof(int64_t));
    uint32_t *counts = (uint32_t *)(w + total * (sizeof(int64_t) + sizeof(double)));
    uint64_t *sums = (uint64_t *)((char *)counts + count_bytes);
    int *mismatch = (int *)(sums + nb + 2);
    uint64_t *total_draws = sums + nb;
    g.state = d_state;
    g.offsets = offsets;
    g.counts = counts;
    const bool fp16 = p->acc == DRIFT_ACC_FP16;
    // FULL windows without a mask take the staged pass (every dot the same shape).
    const int64_t sx = (d.op.cols + kStageSide - 1) / kStageSide;
    const int64_t sy = (d.op.rows + kStageSide - 1) / kStageSide;
    const bool staged = d.op.window == DRIFT_WINDOW_FULL && !d.op.causal && d.op.depth > 0 &&
                        sx <= 0x7fffffffLL && sy <= 65535 && d.op.batch <= 65535;
    const dim3 sgrid((unsigned)sx, (unsigned)sy, (unsigned)d.op.batch);

    auto scan = [&]() {
        if (cudaMemsetAsync(mismatch, 0, sizeof(int), st) != cudaSuccess) return false;
        block_sums_kernel<<<(unsigned)nb, kScanThreads, 0, st>>>(counts, total, chunk, sums);
        scan_sums_kernel<<<1, 32, 0, st>>>(sums, nb);
        apply_offsets_kernel<<<(unsigned)nb, kScanThreads, 0, st>>>(counts, total, chunk, sums,
                                                                    offsets, mismatch);
        return cudaGetLastError() == cudaSuccess;
    };
    predict_counts_kernel<<<grid, 128, 0, st>>>(g, counts);
    // Offsets that differ from any real one, so the first scan reports a change.
    if (cudaMemsetAsync(offsets, 0xff, total * sizeof(int64_t), st) != cudaSuccess || !scan())
        return DRIFT_ECUDA;
    bool settled = false;
    for (int pass = 0; pass < kMaxSrPasses && !settled; pass++) {
        if (staged) {
            if (fp16) contract_sr_staged_kernel<DRIFT_ACC_FP16><<<sgrid, kStageSide * kStageSide, 0, st>>>(g, vals);
            else contract_sr_staged_kernel<DRIFT_ACC_BF16><<<sgrid, kStageSide * kStageSide, 0, st>>>(g, vals);
        } else {
            if (fp16) contract_sr_kernel<DRIFT_ACC_FP16><<<grid, 128, 0, st>>>(g, vals);
            else contract_sr_kernel<DRIFT_ACC_BF16><<<grid, 128, 0, st>>>(g, vals);
        }
        if (!scan()) return DRIFT_ECUDA;
        int flag = 1;
        if (cudaMemcpyAsync(&flag, mismatch, sizeof(int), cudaMemcpyDeviceToHost, st) !=
                cudaSuccess ||
            cudaStreamSynchronize(st) != cudaSuccess)
            return DRIFT_ECUDA;
        settled = flag == 0;
    }
    if (!settled) {
        if (fp16) contract_sr_serial_kernel<DRIFT_ACC_FP16><<<1, 1, 0, st>>>(g, vals, total_draws);
        else contract_sr_serial_kernel<DRIFT_ACC_BF16><<<1, 1, 0, st>>>(g, vals, total_draws);
    }
    contract_apply_kernel<<<grid, 128, 0, st>>>(g, vals);
    advance_state_kernel<<<1, 1, 0, st>>>(d_state, total_draws);
    return cudaGetLastError() == cudaSuccess ? DRIFT_OK : DRIFT_ECUDA;
}

}  // namespace drift
