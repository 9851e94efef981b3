// train.cu — the training step's own arithmetic, resident on the device.
//
// What Pass (java/src/main/java/io/drift/train/Pass.java) and Trainer
// (Trainer.java) do around the casts and contractions, as device kernels, so
// that weights, casts, gradients and the Adam moments stay in HBM across
// steps: the embedding lookup and its ordered gradient, bias gradients,
// tanh's derivative, delayed scaling's amax history, and the Adam update.
// Each keeps the Java evaluation order (and -fmad=false keeps every multiply
// and add separately rounded), so results equal the host loops bit for bit.
#include "common.cuh"
#include "internal.h"

namespace drift {

// Pass.forward's lookup (Pass.java:122-126): row r of out is row tokens[r] of
// the table. A token outside [0, vocab) raises DEV_ERR_INDEX and copies
// nothing (Java throws ArrayIndexOutOfBoundsException).
__global__ void embed_gather_kernel(const int32_t *tokens, int64_t n_tok, const double *table,
                                    int64_t vocab, int64_t width, double *out, int *err) {
    const int64_t total = n_tok * width;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / width, e = i % width;
        const int32_t tok = tokens[r];
        if (tok < 0 || tok >= vocab) {
            atomicOr(err, DEV_ERR_INDEX);
            continue;
        }
        out[i] = table[(int64_t)tok * width + e];
    }
}

// Pass.backward's embedding gradient (Pass.java:168-179): for each table row
// v, grad[v] += rows[r] over the positions r holding token v, in increasing
// r, the order of the (i, c) loop. One CTA per table row: the CTA collects
// the matching positions of each chunk of 256 tokens in order (warp ballots
// and a prefix over the warps), then every thread adds them to its columns.
constexpr int kEmbThreads = 256;

__global__ void __launch_bounds__(kEmbThreads) embed_grad_kernel(const int32_t *tokens,
                                                                 int64_t n_tok,
                                                                 const double *rows,
                                                                 int64_t width, double *grad) {
    __shared__ int32_t s_pos[kEmbThreads];
    __shared__ int s_warp[kEmbThreads / 32];
    const int64_t v = blockIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int64_t e0 = 0; e0 < width; e0 += kEmbThreads) {
        const int64_t e = e0 + threadIdx.x;
        double acc = e < width ? grad[v * width + e] : 0.0;
        for (int64_t base = 0; base < n_tok; base += kEmbThreads) {
            const int64_t r = base + threadIdx.x;
            const bool hit = r < n_tok && tokens[r] == v;
            const unsigned ballot = __ballot_sync(0xffffffffu, hit);
            if (lane == 0) s_warp[warp] = __popc(ballot);
            __syncthreads();
            int before = 0, count = 0;
            for (int w = 0; w < kEmbThreads / 32; w++) {
                if (w < warp) before += s_warp[w];
                count += s_warp[w];
            }
            if (hit) s_pos[before + __popc(ballot & ((1u << lane) - 1))] = (int32_t)(r - base);
            __syncthreads();
            if (e < width)
                for (int j = 0; j < count; j++)
                    acc = __dadd_rn(acc, rows[(base + s_pos[j]) * width + e]);
            __syncthreads();
        }
        if (e < width) grad[v * width + e] = acc;
    }
}

// Pass.linearBackward's bias gradient (Pass.java:234-240): db[o] is the sum
// of dy[i*cols + o] over i in increasing order, from 0.0.
__global__ void bias_grad_kernel(const double *dy, int64_t rows, int64_t cols, double *db) {
    for (int64_t o = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; o < cols;
         o += (int64_t)gridDim.x * blockDim.x) {
        double s = 0.0;
        for (int64_t i = 0; i < rows; i++) s = __dadd_rn(s, dy[i * cols + o]);
        db[o] = s;
    }
}

// Pass.tanhBackward (Pass.java:279-283): grad[i] *= 1.0 - out[i] * out[i].
__global__ void tanh_backward_kernel(const double *out, double *grad, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        grad[i] = __dmul_rn(grad[i], __dsub_rn(1.0, __dmul_rn(out[i], out[i])));
}

// Pass.scaleFor's delayed branch (Pass.java:249-271): the largest amax of
// the previous min(count, len) steps (this one's for the first), then this
// step's amax recorded at count % len, then Quant.perTensorScale
// (Quant.java:37-42).
__global__ void scale_for_kernel(double max_finite, const double *amax_now, double *hist,
                                 int32_t len, int64_t *count, double *scale) {
    const double now = *amax_now;
    const int64_t c = *count;
    double use;
    if (c == 0) {
        use = now;
    } else {
        use = 0.0;
        const int64_t m = c < len ? c : len;
        for (int64_t i = 0; i < m; i++) use = hist[i] > use ? hist[i] : use;  // Math.max, no NaN
    }
    hist[c % len] = now;
    *count = c + 1;
    *scale = (use == 0.0 || !isfinite(use)) ? 1.0 : __ddiv_rn(max_finite, use);
}

// Trainer.adam (Trainer.java:246-269) for one tensor. c1 = 1 - B1^step and
// c2 = 1 - B2^step come from the host (Math.pow); FP32 masters store the
// weight and both moments as floats.
__global__ void adam_kernel(double *p, const double *g, double *m, double *v, int64_t n, double c1,
                            double c2, double lr, int fp32) {
    constexpr double B1 = 0.9, B2 = 0.999, EPS = 1e-8;
    constexpr double OB1 = 1 - B1, OB2 = 1 - B2;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const double gi = g[i];
        double mi = __dadd_rn(__dmul_rn(B1, m[i]), __dmul_rn(OB1, gi));
        double vi = __dadd_rn(__dmul_rn(B2, v[i]), __dmul_rn(__dmul_rn(OB2, gi), gi));
        const double step = __ddiv_rn(__dmul_rn(lr, __ddiv_rn(mi, c1)),
                                      __dadd_rn(__dsqrt_rn(__ddiv_rn(vi, c2)), EPS));
        double pi = __dsub_rn(p[i], step);
        if (fp32) {
            mi = (double)__double2float_rn(mi);
            vi = (double)__double2float_rn(vi);
            pi = (double)__double2float_rn(pi);
        }
        m[i] = mi;
        v[i] = vi;
        p[i] = pi;
    }
}

static unsigned grid_for(int64_t n, int threads) {
    const int64_t b = (n + threads - 1) / threads;
    return (unsigned)(b < 1 ? 1 : (b > 148 * 16 ? 148 * 16 : b));
}

static int launched() { return cudaGetLastError() == cudaSuccess ? DRIFT_OK : DRIFT_ECUDA; }

int launch_embed_gather(const int32_t *tokens, int64_t n_tok, const double *table, int64_t vocab,
                        int64_t width, double *out, int *err, cudaStream_t st) {
    if (n_tok <= 0 || width <= 0) return DRIFT_OK;
    embed_gather_kernel<<<grid_for(n_tok * width, 256), 256, 0, st>>>(tokens, n_tok, table, vocab,
                                                                     width, out, err);
    return launched();
}

int launch_embed_grad(const int32_t *tokens, int64_t n_tok, const double *rows, int64_t width,
                      double *grad, int64_t vocab, cudaStream_t st) {
    if (n_tok <= 0 || width <= 0 || vocab <= 0) return DRIFT_OK;
    if (vocab > 0x7fffffffLL || n_tok > 0x7fffffffLL) return DRIFT_EINVAL;
    embed_grad_kernel<<<(unsigned)vocab, kEmbThreads, 0, st>>>(tokens, n_tok, rows, width, grad);
    return launched();
}

int launch_bias_grad(const double *dy, int64_t rows, int64_t cols, double *db, cudaStream_t st) {
    if (cols <= 0) return DRIFT_OK;
    bias_grad_kernel<<<grid_for(cols, 128), 128, 0, st>>>(dy, rows, cols, db);
    return launched();
}

int launch_tanh_backward(const double *out, double *grad, int64_t n, cudaStream_t st) {
    if (n <= 0) return DRIFT_OK;
    tanh_backward_kernel<<<grid_for(n, 256), 256, 0, st>>>(out, grad, n);
    return launched();
}

int launch_scale_for(int fmt, const double *amax_now, double *hist, int32_t len, int64_t *count,
                     double *scale, cudaStream_t st) {
    FmtDesc f;
    if (!fmt_desc(fmt, &f) || len <= 0) return DRIFT_EINVAL;
    scale_for_kernel<<<1, 1, 0, st>>>(f.max_finite, amax_now, hist, len, count, scale);
    return launched();
}

int launch_adam(double *p, const double *g, double *m, double *v, int64_t n, double c1, double c2,
                double lr, int fp32, cudaStream_t st) {
    if (n <= 0) return DRIFT_OK;
    adam_kernel<<<grid_for(n, 256), 256, 0, st>>>(p, g, m, v, n, c1, c2, lr, fp32);
    return launched();
}

}  // namespace drift
