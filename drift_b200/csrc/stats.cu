// stats.cu — error statistics of an emulated GEMM against its exact twin.
//
// RealDotSweep reports, per policy, the RMS of (got - exact) over the RMS of
// exact (java/src/main/java/io/drift/tools/RealDotSweep.java:130-142, :149-155).
// One pass reads both outputs once (16 bytes per output element) and adds
// sum((got-exact)^2) and sum(exact^2) into two device doubles. The sums are
// reductions of squares, reported with a relative tolerance; the emulated
// outputs themselves are compared bit for bit elsewhere.
#include "common.cuh"
#include "internal.h"

namespace drift {

__global__ void __launch_bounds__(256) error_sums_kernel(const double *got, const double *exact,
                                                         int64_t n, double *sums) {
    double se = 0.0, sx = 0.0;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const double x = exact[i];
        const double e = got[i] - x;
        se += e * e;
        sx += x * x;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        se += __shfl_xor_sync(0xffffffffu, se, o);
        sx += __shfl_xor_sync(0xffffffffu, sx, o);
    }
    __shared__ double s_e[8], s_x[8];
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) {
        s_e[w] = se;
        s_x[w] = sx;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int k = 1; k < 8; k++) {
            se += s_e[k];
            sx += s_x[k];
        }
        atomicAdd(&sums[0], se);
        atomicAdd(&sums[1], sx);
    }
}

int launch_error_sums(const double *got, const double *exact, int64_t n, double *sums,
                      cudaStream_t st) {
    if (n <= 0) return DRIFT_OK;
    const int sms = sm_count();
    int64_t blocks = (n + 255) / 256;
    if (blocks > sms * 8) blocks = sms * 8;
    error_sums_kernel<<<(unsigned)blocks, 256, 0, st>>>(got, exact, n, sums);
    return cudaGetLastError() == cudaSuccess ? DRIFT_OK : DRIFT_ECUDA;
}

// ------------------------------------------------------------------ exact order statistics
//
// The k-th smallest relative error |got - exact| / |exact| (the median of
// DotSweep.java:152-153 and RealDotSweep.java:140-141) over all outputs, found
// by radix selection on the double's bit pattern: for non-negative doubles
// the bits order like the values, and NaN (0/0) is mapped above +Inf, where
// Java's sort puts it. Six passes of 11, 11, 11, 11, 11 and 9 bits each read
// both outputs once, histogram the next digit of the elements that match the
// digits chosen so far, and a one-CTA kernel picks the digit holding rank k.
// Between the passes the histograms of several ranks can be summed (NCCL), so
// the selection is over the union of every rank's outputs.

constexpr int kRadixBits = 11;
constexpr int kRadixBins = 1 << kRadixBits;
constexpr int kRadixPasses = 6;

__device__ __forceinline__ uint64_t rel_error_key(double got, double exact) {
    const double rel = fabs(__dsub_rn(got, exact)) / fabs(exact);  // IEEE division
    return isnan(rel) ? ~0ULL : dbits(rel);
}

__host__ __device__ inline int radix_shift(int pass) {
    const int s = 64 - kRadixBits * (pass + 1);
    return s < 0 ? 0 : s;
}

// The first passes' digits are the top bits of the errors' bit patterns,
// which most elements share (errors of one policy span a few binades), so the
// lanes of a warp that hold the same digit add it once (match_any); the later
// passes count the few elements still matching the prefix, spread over many
// bins, directly. The loop is warp-uniform so that every lane takes part.
__global__ void __launch_bounds__(256) radix_hist_kernel(const double *got, const double *exact,
                                                         int64_t n, int pass,
                                                         const unsigned long long *state,
                                                         unsigned long long *hist) {
    __shared__ unsigned int s_hist[kRadixBins];
    for (int i = threadIdx.x; i < kRadixBins; i += blockDim.x) s_hist[i] = 0;
    __syncthreads();
    const int shift = radix_shift(pass);
    const int top = 64 - kRadixBits * pass;  // bits >= top are already chosen
    const uint64_t prefix = state[0];
    const uint64_t mask = (uint64_t)((1u << (top - shift)) - 1u);
    const bool aggregate = pass < 2;
    const int lane = threadIdx.x & 31;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t base = (int64_t)blockIdx.x * blockDim.x; base < n; base += stride) {
        const int64_t i = base + threadIdx.x;
        unsigned bin = 0xFFFFFFFFu;  // not counted
        if (i < n) {
            const uint64_t key = rel_error_key(got[i], exact[i]);
            if (top == 64 || (key >> top) == (prefix >> top)) bin = (unsigned)((key >> shift) & mask);
        }
        if (aggregate) {
            const unsigned peers = __match_any_sync(0xFFFFFFFFu, bin);
            if (bin != 0xFFFFFFFFu && lane == __ffs(peers) - 1)
                atomicAdd(&s_hist[bin], (unsigned)__popc(peers));
        } else if (bin != 0xFFFFFFFFu) {
            atomicAdd(&s_hist[bin], 1u);
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < kRadixBins; i += blockDim.x)
        if (s_hist[i]) atomicAdd(&hist[i], (unsigned long long)s_hist[i]);
}

// state[0] = digits chosen so far, state[1] = rank still sought among the
// elements that match them. One CTA of 256 threads: thread t sums bins
// [8t, 8t+8), a block-wide exclusive scan of those sums finds the thread
// whose bins hold rank k, and that thread picks the bin.
constexpr int kSelectThreads = 256;
__global__ void __launch_bounds__(kSelectThreads) radix_select_kernel(int pass,
                                                                      const unsigned long long *hist,
                                                                      unsigned long long *state) {
    constexpr int kPer = kRadixBins / kSelectThreads;
    __shared__ unsigned long long warp_sum[kSelectThreads / 32];
    const int shift = radix_shift(pass);
    const int bins = 1 << (64 - kRadixBits * pass - shift);
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const unsigned long long k = state[1];
    unsigned long long h[kPer], mine = 0;
#pragma unroll
    for (int j = 0; j < kPer; j++) {
        const int b = t * kPer + j;
        h[j] = b < bins ? hist[b] : 0ULL;
        mine += h[j];
    }
    // Inclusive scan of the per-thread sums within the warp, then across warps.
    unsigned long long incl = mine;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const unsigned long long v = __shfl_up_sync(0xFFFFFFFFu, incl, d);
        if (lane >= d) incl += v;
    }
    if (lane == 31) warp_sum[warp] = incl;
    __syncthreads();
    unsigned long long before = incl - mine;
    for (int w = 0; w < warp; w++) before += warp_sum[w];
    unsigned long long total = 0;
    for (int w = 0; w < kSelectThreads / 32; w++) total += warp_sum[w];
    __syncthreads();
    // The thread whose range holds rank k picks the bin; if k is out of
    // range (never, for a valid k), the last thread stays at the top bin.
    const bool holds = k >= before && k < before + mine;
    const bool last = t == kSelectThreads - 1 && k >= total;
    if (holds || last) {
        unsigned long long r = k - before;
        int j = 0;
        for (; j < kPer; j++) {
            if (r < h[j]) break;
            r -= h[j];
        }
        int bin = t * kPer + (j < kPer ? j : kPer - 1);
        if (bin >= bins) bin = bins - 1;
        state[0] |= (unsigned long long)bin << shift;
        state[1] = r;
    }
}

int launch_radix_pass(const double *got, const double *exact, int64_t n, int pass,
                      unsigned long long *state, unsigned long long *hist, cudaStream_t st) {
    if (pass < 0 || pass >= kRadixPasses) return DRIFT_EINVAL;
    if (cudaMemsetAsync(hist, 0, kRadixBins * sizeof(unsigned long long), st) != cudaSuccess)
        return DRIFT_ECUDA;
    if (n > 0) {
        const int sms = sm_count();
        int64_t blocks = (n + 255) / 256;
        if (blocks > sms * 4) blocks = sms * 4;
        radix_hist_kernel<<<(unsigned)blocks, 256, 0, st>>>(got, exact, n, pass, state, hist);
    }
    return cudaGetLastError() == cudaSuccess ? DRIFT_OK : DRIFT_ECUDA;
}

int launch_radix_select(int pass, const unsigned long long *hist, unsigned long long *state,
                        cudaStream_t st) {
    if (pass < 0 || pass >= kRadixPasses) return DRIFT_EINVAL;
    radix_select_kernel<<<1, kSelectThreads, 0, st>>>(pass, hist, state);
    return cudaGetLastError() == cudaSuccess ? DRIFT_OK : DRIFT_ECUDA;
}

// ------------------------------------------------------------------ per-group order statistics
//
// The dot sweep reports, per (policy, length), the upper median of a few
// hundred relative errors (DotSweep.java:152-153). Here every group is one
// CTA: its keys (the relative errors' bit patterns, NaN above +Inf, as in
// radix selection) are sorted in shared memory by a bitonic network padded
// to a power of two with the largest key, and element k is written out as a
// double. Groups of up to kGroupMax elements.

constexpr int kGroupMax = 4096;

__global__ void __launch_bounds__(1024) group_kth_kernel(const double *got, const double *exact,
                                                         int64_t n, int64_t k, double *out) {
    __shared__ uint64_t keys[kGroupMax];
    const int64_t g = blockIdx.x;
    int m = 1;
    while (m < n) m <<= 1;
    for (int i = threadIdx.x; i < m; i += blockDim.x)
        keys[i] = i < n ? rel_error_key(got[g * n + i], exact[g * n + i]) : ~0ULL;
    __syncthreads();
    for (int size = 2; size <= m; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < m; i += blockDim.x) {
                const int j = i ^ stride;
                if (j > i) {
                    const bool up = (i & size) == 0;
                    const uint64_t a = keys[i], b = keys[j];
                    if ((a > b) == up) {
                        keys[i] = b;
                        keys[j] = a;
                    }
                }
            }
            __syncthreads();
        }
    }
    if (threadIdx.x == 0) out[g] = bitsd(keys[k]);
}

int launch_group_kth(const double *got, const double *exact, int64_t groups, int64_t n,
                     int64_t k, double *out, cudaStream_t st) {
    if (groups < 0 || n <= 0 || n > kGroupMax || k < 0 || k >= n || groups > 0x7fffffffLL)
        return DRIFT_EINVAL;
    if (groups == 0) return DRIFT_OK;
    group_kth_kernel<<<(unsigned)groups, 1024, 0, st>>>(got, exact, n, k, out);
    return cudaGetLastError() == cudaSuccess ? DRIFT_OK : DRIFT_ECUDA;
}

}  // namespace drift
