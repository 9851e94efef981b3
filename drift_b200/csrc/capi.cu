// capi.cu — the C ABI (include/drift_b200.h): contexts, host-buffer entry
// points that stage through device memory, and device-resident entry points.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "common.cuh"
#include "internal.h"

using namespace drift;

// ------------------------------------------------------------------ errors

static thread_local std::string g_last_error;

static int fail(int status, const char *what) {
    g_last_error = what;
    return status;
}

static int cuda_fail(cudaError_t e, const char *what) {
    g_last_error = std::string(what) + ": " + cudaGetErrorString(e);
    return DRIFT_ECUDA;
}

#define CUDA_TRY(call, what)                       \
    do {                                           \
        cudaError_t e_ = (call);                   \
        if (e_ != cudaSuccess) return cuda_fail(e_, what); \
    } while (0)

// ------------------------------------------------------------------ formats

namespace drift {

// Formats.java:20-45 through the MiniFloat constructor (MiniFloat.java:70-107).
bool fmt_desc(int id, FmtDesc *out) {
    static const int table[DRIFT_NUM_FORMATS][4] = {
        {4, 3, 7, SP_FN},       {5, 2, 15, SP_IEEE}, {2, 1, 1, SP_FINITE},
        {3, 2, 3, SP_FINITE},   {2, 3, 1, SP_FINITE}, {5, 10, 15, SP_IEEE},
        {8, 7, 127, SP_IEEE},
    };
    if (id < 0 || id >= DRIFT_NUM_FORMATS) return false;
    const int e = table[id][0], m = table[id][1], bias = table[id][2], sp = table[id][3];
    FmtDesc f;
    f.mant_bits = m;
    f.bias = bias;
    f.specials = sp;
    f.max_exp_field = (1 << e) - 1;
    f.mant_mask = (1 << m) - 1;
    f.exp_mask = f.max_exp_field << m;
    f.sign_bit = 1 << (e + m);
    f.code_mask = (1 << (1 + e + m)) - 1;
    f.min_normal_exp = 1 - bias;
    int top_exp, top_mant;
    if (sp == SP_IEEE) {
        top_exp = f.max_exp_field - 1;
        top_mant = f.mant_mask;
        f.nan_bits = f.exp_mask | 1;
    } else if (sp == SP_FN) {
        top_exp = f.max_exp_field;
        top_mant = f.mant_mask - 1;
        f.nan_bits = f.exp_mask | f.mant_mask;
    } else {
        top_exp = f.max_exp_field;
        top_mant = f.mant_mask;
        f.nan_bits = 0;
    }
    f.max_finite_bits = (top_exp << m) | top_mant;
    f.max_finite = std::ldexp(1.0 + (double)top_mant / (1 << m), top_exp - bias);
    f.emax = java_get_exponent(f.max_finite);
    *out = f;
    return true;
}

void *Workspace::get(size_t bytes, cudaStream_t st) {
    if (bytes <= cap_ && ptr_) return ptr_;
    if (ptr_) cudaFreeAsync(ptr_, st);
    ptr_ = nullptr;
    cap_ = 0;
    size_t want = bytes < 4096 ? 4096 : bytes;
    if (cudaMallocAsync(&ptr_, want, st) != cudaSuccess) {
        ptr_ = nullptr;
        return nullptr;
    }
    cap_ = want;
    return ptr_;
}

void Workspace::release(cudaStream_t st) {
    if (ptr_) cudaFreeAsync(ptr_, st);
    ptr_ = nullptr;
    cap_ = 0;
}

const uint8_t *ScheduleCache::get(int64_t K, cudaStream_t st) {
    (void)st;
    auto it = entries_.find(K);
    if (it != entries_.end()) return it->second.d;
    std::vector<uint8_t> sched;
    int depth = 0;
    status_ = pairwise_schedule(K, sched, &depth);
    if (status_ != DRIFT_OK) return nullptr;
    uint8_t *d = nullptr;
    if (cudaMalloc(&d, sched.size()) != cudaSuccess) {
        status_ = DRIFT_ENOMEM;
        return nullptr;
    }
    if (cudaMemcpy(d, sched.data(), sched.size(), cudaMemcpyHostToDevice) != cudaSuccess) {
        cudaFree(d);
        status_ = DRIFT_ECUDA;
        return nullptr;
    }
    const int64_t leaves = (int64_t)(sched.size() - 1) / 2;
    entries_[K] = Entry{d, leaves};
    return d;
}

int64_t ScheduleCache::leaves(int64_t K) const {
    auto it = entries_.find(K);
    return it == entries_.end() ? 0 : it->second.leaves;
}

void ScheduleCache::clear() {
    for (auto &kv : entries_) cudaFree(kv.second.d);
    entries_.clear();
}

}  // namespace drift

// ------------------------------------------------------------------ context

constexpr int kPipeChunks = 8;  // host-buffer calls copy and compute in up to 8 chunks

struct drift_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    // Copy streams and events of the pipelined host-buffer calls: chunk c
    // goes in on `h2d`, is computed on `stream`, and comes back on `d2h`.
    cudaStream_t h2d = nullptr, d2h = nullptr;
    cudaEvent_t ev_in[kPipeChunks] = {}, ev_done[kPipeChunks] = {};
    cudaEvent_t ev_b[kPipeChunks] = {};  // drift_gemm: B's column blocks landed
    cudaEvent_t ev_start = nullptr;
    Workspace ws;       // kernel scratch
    Workspace io;       // staging for host-buffer calls
    ScheduleCache sched;
    // Small device words: [0] error flags (int), [8] rng state, [16] clamp
    // counter, [24] scalar result, [32] the last GEMM's route (int), [64] the
    // range proof's eight operand-scan words.
    char *d_small = nullptr;
    int *d_err() { return (int *)d_small; }
    uint64_t *d_state() { return (uint64_t *)(d_small + 8); }
    unsigned long long *d_clamped() { return (unsigned long long *)(d_small + 16); }
    double *d_scalar() { return (double *)(d_small + 24); }
    int *d_route() { return (int *)(d_small + 32); }
    unsigned *d_scan() { return (unsigned *)(d_small + 64); }
    int last_launches = 0;  // kernels the last GEMM queued (drift_gemm_launches)
    int64_t thin_tiles = -1;  // drift_set_thin_tiles; negative: two per SM
};

static int enter(drift_ctx *ctx) {
    if (!ctx) return fail(DRIFT_EINVAL, "null context");
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    return DRIFT_OK;
}

// Device entry points run on the caller's stream exactly as given; NULL is
// the CUDA default stream, as everywhere in the CUDA runtime.
static cudaStream_t pick(drift_ctx *ctx, void *stream) {
    (void)ctx;
    return (cudaStream_t)stream;
}

// Reads and clears the device error word; maps it to a status.
static int take_device_error(drift_ctx *ctx, cudaStream_t st) {
    int flags = 0;
    CUDA_TRY(cudaMemcpyAsync(&flags, ctx->d_err(), sizeof(int), cudaMemcpyDeviceToHost, st),
             "read error word");
    CUDA_TRY(cudaMemsetAsync(ctx->d_err(), 0, sizeof(int), st), "clear error word");
    CUDA_TRY(cudaStreamSynchronize(st), "synchronize");
    if (flags & DEV_ERR_NAN_FINITE) return fail(DRIFT_ENAN_FINITE, "NaN cast into a format without NaN");
    if (flags & DEV_ERR_NO_RNG) return fail(DRIFT_EINVAL, "stochastic rounding needs an Rng");
    if (flags & DEV_ERR_TIMEOUT) return fail(DRIFT_ETIMEOUT, "device wait gave up");
    if (flags & DEV_ERR_INDEX) return fail(DRIFT_EINVAL, "token outside the embedding table");
    return DRIFT_OK;
}

// ------------------------------------------------------------------ pipelines
//
// A host-buffer call moves its operands over PCIe at about 55 GB/s each way.
// Large calls split into up to kPipeChunks chunks: chunk c is copied in on
// ctx->h2d, computed on ctx->stream once its copy has landed, and copied out
// on ctx->d2h once computed, so the copies of one chunk overlap the compute
// of its neighbours. Every pipelined call waits for both copy streams before
// it returns, on every path, so the staging buffer is never reused early.

// The copy streams start after everything already queued on ctx->stream
// (the staging buffer's stream-ordered allocation included).
static int pipe_begin(drift_ctx *ctx) {
    CUDA_TRY(cudaEventRecord(ctx->ev_start, ctx->stream), "record");
    CUDA_TRY(cudaStreamWaitEvent(ctx->h2d, ctx->ev_start, 0), "wait");
    CUDA_TRY(cudaStreamWaitEvent(ctx->d2h, ctx->ev_start, 0), "wait");
    return DRIFT_OK;
}

// Waits for both copy streams; returns `rc` unless waiting itself failed.
static int pipe_end(drift_ctx *ctx, int rc) {
    const cudaError_t a = cudaStreamSynchronize(ctx->h2d);
    const cudaError_t b = cudaStreamSynchronize(ctx->d2h);
    if (rc) return rc;
    if (a != cudaSuccess) return cuda_fail(a, "synchronize");
    if (b != cudaSuccess) return cuda_fail(b, "synchronize");
    return DRIFT_OK;
}

// Chunk length in units of `unit` elements (or rows) for a call of n of
// them; 0 when the call is too small to gain from a pipeline.
static int64_t pipe_chunk(int64_t n, int64_t min_total, int64_t unit) {
    if (n < min_total) return 0;
    int64_t c = (n + kPipeChunks - 1) / kPipeChunks;
    return (c + unit - 1) / unit * unit;
}

extern "C" {

const char *drift_last_error(void) { return g_last_error.c_str(); }

const char *drift_version(void) { return "drift_b200 0.1 (sm_100a)"; }

int drift_open(int device, drift_ctx **out) {
    if (!out) return fail(DRIFT_EINVAL, "null out");
    *out = nullptr;
    int count = 0;
    CUDA_TRY(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
    if (device < 0 || device >= count) return fail(DRIFT_EINVAL, "no such device");
    CUDA_TRY(cudaSetDevice(device), "cudaSetDevice");
    drift_ctx *ctx = new drift_ctx();
    ctx->device = device;
    cudaError_t e = cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&ctx->h2d, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&ctx->d2h, cudaStreamNonBlocking);
    for (int c = 0; c < kPipeChunks && e == cudaSuccess; c++) {
        e = cudaEventCreateWithFlags(&ctx->ev_in[c], cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->ev_done[c], cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->ev_b[c], cudaEventDisableTiming);
    }
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->ev_start, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaMalloc(&ctx->d_small, 128);
    if (e == cudaSuccess) e = cudaMemset(ctx->d_small, 0, 128);
    if (e != cudaSuccess) {
        for (int c = 0; c < kPipeChunks; c++) {
            if (ctx->ev_in[c]) cudaEventDestroy(ctx->ev_in[c]);
            if (ctx->ev_done[c]) cudaEventDestroy(ctx->ev_done[c]);
            if (ctx->ev_b[c]) cudaEventDestroy(ctx->ev_b[c]);
        }
        if (ctx->ev_start) cudaEventDestroy(ctx->ev_start);
        if (ctx->h2d) cudaStreamDestroy(ctx->h2d);
        if (ctx->d2h) cudaStreamDestroy(ctx->d2h);
        if (ctx->stream) cudaStreamDestroy(ctx->stream);
        delete ctx;
        return cuda_fail(e, "drift_open");
    }
    *out = ctx;
    return DRIFT_OK;
}

int drift_close(drift_ctx *ctx) {
    if (!ctx) return DRIFT_OK;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    ctx->ws.release(ctx->stream);
    ctx->io.release(ctx->stream);
    cudaStreamSynchronize(ctx->stream);
    ctx->sched.clear();
    cudaFree(ctx->d_small);
    for (int c = 0; c < kPipeChunks; c++) {
        cudaEventDestroy(ctx->ev_in[c]);
        cudaEventDestroy(ctx->ev_done[c]);
        cudaEventDestroy(ctx->ev_b[c]);
    }
    cudaEventDestroy(ctx->ev_start);
    cudaStreamDestroy(ctx->h2d);
    cudaStreamDestroy(ctx->d2h);
    cudaStreamDestroy(ctx->stream);
    delete ctx;
    return DRIFT_OK;
}

int drift_format_info(int fmt, double *max_finite, double *min_normal, double *min_subnormal,
                      int32_t *width) {
    FmtDesc f;
    if (!fmt_desc(fmt, &f)) return fail(DRIFT_EINVAL, "bad format id");
    if (max_finite) *max_finite = f.max_finite;
    if (min_normal) *min_normal = std::ldexp(1.0, f.min_normal_exp);
    if (min_subnormal) *min_subnormal = std::ldexp(1.0, f.min_normal_exp - f.mant_bits);
    if (width) *width = __builtin_popcount((unsigned)f.code_mask);
    return DRIFT_OK;
}

int drift_per_tensor_scale(int fmt, double amax, double *scale_out) {
    FmtDesc f;
    if (!fmt_desc(fmt, &f) || !scale_out) return fail(DRIFT_EINVAL, "bad format id");
    *scale_out = (amax == 0.0 || !std::isfinite(amax)) ? 1.0 : f.max_finite / amax;
    return DRIFT_OK;
}

// ------------------------------------------------------------------ host-buffer calls

int drift_encode(drift_ctx *ctx, int fmt, int rounding, const double *v, int32_t *codes,
                 int64_t n, uint64_t *rng_state) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (n < 0 || (n > 0 && (!v || !codes))) return fail(DRIFT_EINVAL, "bad arguments");
    if (n == 0) return DRIFT_OK;
    cudaStream_t st = ctx->stream;
    char *buf = (char *)ctx->io.get((size_t)n * 12 + 256, st);
    if (!buf) return fail(DRIFT_ENOMEM, "staging");
    double *d_v = (double *)buf;
    int32_t *d_c = (int32_t *)(buf + n * 8);
    CUDA_TRY(cudaMemcpyAsync(d_v, v, n * 8, cudaMemcpyHostToDevice, st), "copy in");
    if (rng_state)
        CUDA_TRY(cudaMemcpyAsync(ctx->d_state(), rng_state, 8, cudaMemcpyHostToDevice, st), "rng in");
    rc = launch_encode(ctx->ws, fmt, rounding, d_v, d_c, n, rng_state ? ctx->d_state() : nullptr,
                       ctx->d_err(), st);
    if (rc) return fail(rc, "encode launch");
    uint64_t state = 0;
    CUDA_TRY(cudaMemcpyAsync(codes, d_c, n * 4, cudaMemcpyDeviceToHost, st), "copy out");
    if (rng_state)
        CUDA_TRY(cudaMemcpyAsync(&state, ctx->d_state(), 8, cudaMemcpyDeviceToHost, st), "rng out");
    rc = take_device_error(ctx, st);
    if (rc) return rc;
    if (rng_state) *rng_state = state;
    return DRIFT_OK;
}

int drift_decode(drift_ctx *ctx, int fmt, const int32_t *codes, double *v, int64_t n) {
    int rc = enter(ctx);
    if (rc) return rc;
    FmtDesc f;
    if (!fmt_desc(fmt, &f)) return fail(DRIFT_EINVAL, "bad format id");
    if (n < 0 || (n > 0 && (!v || !codes))) return fail(DRIFT_EINVAL, "bad arguments");
    for (int64_t i = 0; i < n; i++)  // MiniFloat.java:118-120
        if (codes[i] & ~f.code_mask) return fail(DRIFT_EINVAL, "bits outside format width");
    if (n == 0) return DRIFT_OK;
    cudaStream_t st = ctx->stream;
    char *buf = (char *)ctx->io.get((size_t)n * 12 + 256, st);
    if (!buf) return fail(DRIFT_ENOMEM, "staging");
    double *d_v = (double *)buf;
    int32_t *d_c = (int32_t *)(buf + n * 8);
    CUDA_TRY(cudaMemcpyAsync(d_c, codes, n * 4, cudaMemcpyHostToDevice, st), "copy in");
    rc = launch_decode(fmt, d_c, d_v, n, st);
    if (rc) return fail(rc, "decode launch");
    CUDA_TRY(cudaMemcpyAsync(v, d_v, n * 8, cudaMemcpyDeviceToHost, st), "copy out");
    CUDA_TRY(cudaStreamSynchronize(st), "synchronize");
    return DRIFT_OK;
}

int drift_value_table_dev(drift_ctx *ctx, int fmt, uint64_t *d_bits, void *stream) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (!d_bits) return fail(DRIFT_EINVAL, "null pointer");
    rc = launch_value_table(fmt, d_bits, pick(ctx, stream));
    return rc ? fail(rc, "value table") : DRIFT_OK;
}

int drift_pair_table_dev(drift_ctx *ctx, int fmt, int mode, uint64_t seed, int64_t first,
                         int64_t n, int32_t *d_a, int32_t *d_b, int32_t *d_prod, int32_t *d_sum,
                         void *stream) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (n > 0 && (!d_prod || !d_sum)) return fail(DRIFT_EINVAL, "null pointer");
    rc = launch_pair_table(fmt, mode, seed, first, n, d_a, d_b, d_prod, d_sum, pick(ctx, stream));
    return rc ? fail(rc, "pair table") : DRIFT_OK;
}

int drift_value_table(drift_ctx *ctx, int fmt, uint64_t *bits) {
    int rc = enter(ctx);
    if (rc) return rc;
    FmtDesc f;
    if (!fmt_desc(fmt, &f)) return fail(DRIFT_EINVAL, "bad format id");
    if (!bits) return fail(DRIFT_EINVAL, "null pointer");
    const int64_t codes = (int64_t)f.code_mask + 1;
    cudaStream_t st = ctx->stream;
    uint64_t *d_bits = (uint64_t *)ctx->io.get((size_t)codes * 8, st);
    if (!d_bits) return fail(DRIFT_ENOMEM, "staging");
    rc = launch_value_table(fmt, d_bits, st);
    if (rc) return fail(rc, "value table");
    CUDA_TRY(cudaMemcpyAsync(bits, d_bits, codes * 8, cudaMemcpyDeviceToHost, st), "copy out");
    CUDA_TRY(cudaStreamSynchronize(st), "synchronize");
    return DRIFT_OK;
}

int drift_pair_table(drift_ctx *ctx, int fmt, int mode, uint64_t seed, int64_t first, int64_t n,
                     int32_t *a, int32_t *b, int32_t *prod, int32_t *sum) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (n < 0 || (n > 0 && (!prod || !sum))) return fail(DRIFT_EINVAL, "bad arguments");
    if (n == 0) return launch_pair_table(fmt, mode, seed, first, 0, 0, 0, 0, 0, ctx->stream)
                          ? fail(DRIFT_EINVAL, "bad arguments") : DRIFT_OK;
    cudaStream_t st = ctx->stream;
    int32_t *buf = (int32_t *)ctx->io.get((size_t)n * 16, st);
    if (!buf) return fail(DRIFT_ENOMEM, "staging");
    rc = launch_pair_table(fmt, mode, seed, first, n, buf, buf + n, buf + 2 * n, buf + 3 * n, st);
    if (rc) return fail(rc, "pair table");
    int32_t *outs[4] = {a, b, prod, sum};
    for (int j = 0; j < 4; j++)
        if (outs[j])
            CUDA_TRY(cudaMemcpyAsync(outs[j], buf + j * n, n * 4, cudaMemcpyDeviceToHost, st),
                     "copy out");
    CUDA_TRY(cudaStreamSynchronize(st), "synchronize");
    return DRIFT_OK;
}

int drift_acc_round(drift_ctx *ctx, int acc, int rounding, const double *x, double *y, int64_t n,
                    uint64_t *rng_state) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (n < 0 || (n > 0 && (!x || !y))) return fail(DRIFT_EINVAL, "bad arguments");
    if (n == 0) return DRIFT_OK;
    cudaStream_t st = ctx->stream;
    char *buf = (char *)ctx->io.get((size_t)n * 16 + 256, st);
    if (!buf) return fail(DRIFT_ENOMEM, "staging");
    double *d_x = (double *)buf;
    double *d_y = (double *)(buf + n * 8);
    CUDA_TRY(cudaMemcpyAsync(d_x, x, n * 8, cudaMemcpyHostToDevice, st), "copy in");
    if (rng_state)
        CUDA_TRY(cudaMemcpyAsync(ctx->d_state(), rng_state, 8, cudaMemcpyHostToDevice, st), "rng in");
    rc = launch_acc_round(ctx->ws, acc, rounding, d_x, d_y, n,
                          rng_state ? ctx->d_state() : nullptr, ctx->d_err(), st);
    if (rc) return fail(rc, "acc_round launch");
    uint64_t state = 0;
    CUDA_TRY(cudaMemcpyAsync(y, d_y, n * 8, cudaMemcpyDeviceToHost, st), "copy out");
    if (rng_state)
        CUDA_TRY(cudaMemcpyAsync(&state, ctx->d_state(), 8, cudaMemcpyDeviceToHost, st), "rng out");
    rc = take_device_error(ctx, st);
    if (rc) return rc;
    if (rng_state) *rng_state = state;
    return DRIFT_OK;
}

int drift_amax(drift_ctx *ctx, const double *x, int64_t n, double *amax_out) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (n < 0 || !amax_out || (n > 0 && !x)) return fail(DRIFT_EINVAL, "bad arguments");
    cudaStream_t st = ctx->stream;
    double *d_x = nullptr;
    if (n > 0) {
        d_x = (double *)ctx->io.get((size_t)n * 8, st);
        if (!d_x) return fail(DRIFT_ENOMEM, "staging");
        CUDA_TRY(cudaMemcpyAsync(d_x, x, n * 8, cudaMemcpyHostToDevice, st), "copy in");
    }
    rc = launch_amax(d_x, n, ctx->d_scalar(), st);
    if (rc) return fail(rc, "amax launch");
    CUDA_TRY(cudaMemcpyAsync(amax_out, ctx->d_scalar(), 8, cudaMemcpyDeviceToHost, st), "copy out");
    CUDA_TRY(cudaStreamSynchronize(st), "synchronize");
    return DRIFT_OK;
}

int drift_quantize(drift_ctx *ctx, const drift_policy *p, int fmt, int rounding, const double *src,
                   double *dst, int64_t n, double scale, uint64_t *rng_state,
                   int64_t *clamped_out) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (!p || n < 0 || (n > 0 && (!src || !dst))) return fail(DRIFT_EINVAL, "bad arguments");
    if (clamped_out) *clamped_out = 0;
    if (n == 0) return DRIFT_OK;
    cudaStream_t st = ctx->stream;
    char *buf = (char *)ctx->io.get((size_t)n * 16 + 256, st);
    if (!buf) return fail(DRIFT_ENOMEM, "staging");
    double *d_src = (double *)buf;
    double *d_dst = (double *)(buf + n * 8);
    CUDA_TRY(cudaMemsetAsync(ctx->d_clamped(), 0, 8, st), "clear clamps");
    // Without stochastic rounding the elements (and MX blocks, which follow
    // the flat index from 0) are independent, so the cast travels in chunks
    // whose copies overlap: in on one copy engine, out on the other.
    const int64_t unit = (p->scaling == DRIFT_MX_BLOCK && p->scale_block > 0 ? p->scale_block : 1) * 256;
    const int64_t chunk = rounding != DRIFT_STOCHASTIC ? pipe_chunk(n, (int64_t)1 << 22, unit) : 0;
    if (chunk > 0) {
        rc = pipe_begin(ctx);
        int c = 0;
        for (int64_t e0 = 0; e0 < n && !rc; e0 += chunk, c++) {
            const int64_t len = n - e0 < chunk ? n - e0 : chunk;
            if (cudaMemcpyAsync(d_src + e0, src + e0, len * 8, cudaMemcpyHostToDevice, ctx->h2d) !=
                    cudaSuccess ||
                cudaEventRecord(ctx->ev_in[c], ctx->h2d) != cudaSuccess ||
                cudaStreamWaitEvent(st, ctx->ev_in[c], 0) != cudaSuccess) {
                rc = fail(DRIFT_ECUDA, "copy in");
                break;
            }
            rc = launch_quantize(ctx->ws, p, fmt, rounding, d_src + e0, d_dst + e0, len, nullptr,
                                 scale, nullptr, ctx->d_clamped(), ctx->d_err(), st);
            if (rc) {
                rc = fail(rc, "quantize launch");
                break;
            }
            if (cudaEventRecord(ctx->ev_done[c], st) != cudaSuccess ||
                cudaStreamWaitEvent(ctx->d2h, ctx->ev_done[c], 0) != cudaSuccess ||
                cudaMemcpyAsync(dst + e0, d_dst + e0, len * 8, cudaMemcpyDeviceToHost, ctx->d2h) !=
                    cudaSuccess)
                rc = fail(DRIFT_ECUDA, "copy out");
        }
        unsigned long long clamped = 0;
        if (!rc && cudaMemcpyAsync(&clamped, ctx->d_clamped(), 8, cudaMemcpyDeviceToHost, st) !=
                       cudaSuccess)
            rc = fail(DRIFT_ECUDA, "clamps out");
        rc = pipe_end(ctx, rc);
        if (rc) return rc;
        rc = take_device_error(ctx, st);
        if (rc) return rc;
        if (clamped_out) *clamped_out = (int64_t)clamped;
        return DRIFT_OK;
    }
    CUDA_TRY(cudaMemcpyAsync(d_src, src, n * 8, cudaMemcpyHostToDevice, st), "copy in");
    if (rng_state)
        CUDA_TRY(cudaMemcpyAsync(ctx->d_state(), rng_state, 8, cudaMemcpyHostToDevice, st), "rng in");
    rc = launch_quantize(ctx->ws, p, fmt, rounding, d_src, d_dst, n, nullptr, scale,
                         rng_state ? ctx->d_state() : nullptr, ctx->d_clamped(), ctx->d_err(), st);
    if (rc) return fail(rc, "quantize launch");
    uint64_t state = 0;
    unsigned long long clamped = 0;
    CUDA_TRY(cudaMemcpyAsync(dst, d_dst, n * 8, cudaMemcpyDeviceToHost, st), "copy out");
    CUDA_TRY(cudaMemcpyAsync(&clamped, ctx->d_clamped(), 8, cudaMemcpyDeviceToHost, st), "clamps out");
    if (rng_state)
        CUDA_TRY(cudaMemcpyAsync(&state, ctx->d_state(), 8, cudaMemcpyDeviceToHost, st), "rng out");
    rc = take_device_error(ctx, st);
    if (rc) return rc;
    if (rng_state) *rng_state = state;
    if (clamped_out) *clamped_out = (int64_t)clamped;
    return DRIFT_OK;
}

// Number of elements an operand with these strides spans from its offset.
static int64_t span_of(int64_t rows, int64_t rs, int64_t K, int64_t ks) {
    if (rows <= 0 || K <= 0) return 0;
    return (rows - 1) * rs + (K - 1) * ks + 1;
}

static bool stochastic_acc(const drift_policy *p) {
    return (p->acc == DRIFT_ACC_FP16 || p->acc == DRIFT_ACC_BF16) &&
           p->acc_rounding == DRIFT_STOCHASTIC;
}

// drift_gemm's C[i*c_rs + o] = dot(A row i, B row o) + bias[o] as a
// one-batch contraction over the full depth.
static ContractDesc gemm_as_contraction(int64_t M, int64_t N, int64_t K, const double *A,
                                        int64_t a_rs, int64_t a_ks, const double *B, int64_t b_rs,
                                        int64_t b_ks, const double *bias, double *C, int64_t c_rs) {
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
    return d;
}

int drift_gemm(drift_ctx *ctx, const drift_policy *p, int64_t M, int64_t N, int64_t K,
               const double *A, int64_t a_off, int64_t a_row_stride, int64_t a_k_stride,
               const double *B, int64_t b_off, int64_t b_row_stride, int64_t b_k_stride,
               const double *bias, double *C, int64_t c_row_stride, uint64_t *rng_state) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (!p || M < 0 || N < 0 || K < 0 || a_off < 0 || b_off < 0 || a_row_stride < 0 ||
        a_k_stride < 0 || b_row_stride < 0 || b_k_stride < 0 || c_row_stride < N)
        return fail(DRIFT_EINVAL, "bad shape or stride");
    if (M == 0 || N == 0) return DRIFT_OK;
    if (!C || (K > 0 && (!A || !B))) return fail(DRIFT_EINVAL, "null buffer");
    cudaStream_t st = ctx->stream;
    const int64_t sa = span_of(M, a_row_stride, K, a_k_stride);
    const int64_t sb = span_of(N, b_row_stride, K, b_k_stride);
    const int64_t sc = M * N;
    const int64_t total = sa + sb + sc + (bias ? N : 0) + 8;
    char *buf = (char *)ctx->io.get((size_t)total * 8 + 512, st);
    if (!buf) return fail(DRIFT_ENOMEM, "staging");
    double *d_a = (double *)buf;
    double *d_b = d_a + ((sa + 1) & ~1LL);
    double *d_c = d_b + ((sb + 1) & ~1LL);
    double *d_bias = bias ? d_c + ((sc + 1) & ~1LL) : nullptr;
    const bool sr = stochastic_acc(p);
    // Rows of a row-major A own disjoint spans, so A can travel in row chunks
    // (multiples of the 64-row tile) that overlap the contraction.
    const int64_t chunk = (!sr && K > 0 && a_k_stride == 1 && a_row_stride >= K)
                              ? pipe_chunk(M, 1024, 64) : 0;
    // When B's rows own disjoint K-contiguous spans too, B travels in
    // kBBlocks column blocks behind A's first row chunk, and that chunk is
    // contracted block by block as they land: the first sums start after one
    // A chunk and one B block instead of the whole of B (at 8192^3, 3.5 ms of
    // copies instead of 10.5).
    constexpr int64_t kBBlocks = 4;
    int64_t bcols = 0;
    if (chunk > 0 && b_k_stride == 1 && b_row_stride >= K && N >= 1024) {
        bcols = (N + kBBlocks - 1) / kBBlocks;
        bcols = (bcols + 63) / 64 * 64;
    }
    if (sb && !bcols)
        CUDA_TRY(cudaMemcpyAsync(d_b, B + b_off, sb * 8, cudaMemcpyHostToDevice, st), "copy B");
    if (bias) CUDA_TRY(cudaMemcpyAsync(d_bias, bias, N * 8, cudaMemcpyHostToDevice, st), "copy bias");
    if (chunk > 0) {
        rc = pipe_begin(ctx);
        int c = 0;
        for (int64_t r0 = 0; r0 < M && !rc; r0 += chunk, c++) {
            const int64_t rows = M - r0 < chunk ? M - r0 : chunk;
            const int64_t off = r0 * a_row_stride;
            if (cudaMemcpyAsync(d_a + off, A + a_off + off, span_of(rows, a_row_stride, K, 1) * 8,
                                cudaMemcpyHostToDevice, ctx->h2d) != cudaSuccess ||
                cudaEventRecord(ctx->ev_in[c], ctx->h2d) != cudaSuccess ||
                cudaStreamWaitEvent(st, ctx->ev_in[c], 0) != cudaSuccess) {
                rc = fail(DRIFT_ECUDA, "copy A");
                break;
            }
            if (c == 0 && bcols > 0) {
                int jb = 0;
                for (int64_t j0 = 0; j0 < N && !rc; j0 += bcols, jb++) {
                    const int64_t cols = N - j0 < bcols ? N - j0 : bcols;
                    const int64_t boff = j0 * b_row_stride;
                    if (cudaMemcpyAsync(d_b + boff, B + b_off + boff,
                                        span_of(cols, b_row_stride, K, 1) * 8,
                                        cudaMemcpyHostToDevice, ctx->h2d) != cudaSuccess ||
                        cudaEventRecord(ctx->ev_b[jb], ctx->h2d) != cudaSuccess)
                        rc = fail(DRIFT_ECUDA, "copy B");
                }
                jb = 0;
                for (int64_t j0 = 0; j0 < N && !rc; j0 += bcols, jb++) {
                    const int64_t cols = N - j0 < bcols ? N - j0 : bcols;
                    if (cudaStreamWaitEvent(st, ctx->ev_b[jb], 0) != cudaSuccess) {
                        rc = fail(DRIFT_ECUDA, "wait B");
                        break;
                    }
                    rc = launch_gemm(ctx->ws, ctx->sched, p, rows, cols, K, d_a + off, a_row_stride,
                                     1, d_b + j0 * b_row_stride, b_row_stride, 1,
                                     d_bias ? d_bias + j0 : nullptr, d_c + r0 * N + j0, N,
                                     ctx->thin_tiles, ctx->d_err(), ctx->d_route(), st,
                                     ctx->d_scan(), &ctx->last_launches);
                    if (rc) rc = fail(rc, "gemm launch");
                }
                if (rc) break;
            } else {
                rc = launch_gemm(ctx->ws, ctx->sched, p, rows, N, K, d_a + off, a_row_stride, 1,
                                 d_b, b_row_stride, b_k_stride, d_bias, d_c + r0 * N, N,
                                 ctx->thin_tiles, ctx->d_err(), ctx->d_route(), st,
                                 ctx->d_scan(), &ctx->last_launches);
                if (rc) {
                    rc = fail(rc, "gemm launch");
                    break;
                }
            }
            if (cudaEventRecord(ctx->ev_done[c], st) != cudaSuccess ||
                cudaStreamWaitEvent(ctx->d2h, ctx->ev_done[c], 0) != cudaSuccess ||
                cudaMemcpy2DAsync(C + r0 * c_row_stride, c_row_stride * 8, d_c + r0 * N, N * 8,
                                  N * 8, rows, cudaMemcpyDeviceToHost, ctx->d2h) != cudaSuccess)
                rc = fail(DRIFT_ECUDA, "copy C");
        }
        rc = pipe_end(ctx, rc);
        if (rc) return rc;
        return take_device_error(ctx, st);
    }
    if (sa) CUDA_TRY(cudaMemcpyAsync(d_a, A + a_off, sa * 8, cudaMemcpyHostToDevice, st), "copy A");
    if (sr) {
        // The Rng state travels on the device; without one, start from zero
        // and fail afterwards if any draw was taken (Java fails on the first).
        const uint64_t s0 = rng_state ? *rng_state : 0;
        CUDA_TRY(cudaMemcpyAsync(ctx->d_state(), &s0, 8, cudaMemcpyHostToDevice, st), "rng in");
        rc = launch_contract(ctx->ws, ctx->sched, p,
                             gemm_as_contraction(M, N, K, d_a, a_row_stride, a_k_stride, d_b,
                                                 b_row_stride, b_k_stride, d_bias, d_c, N),
                             ctx->d_state(), ctx->d_err(), st);
    } else {
        rc = launch_gemm(ctx->ws, ctx->sched, p, M, N, K, d_a, a_row_stride, a_k_stride, d_b,
                         b_row_stride, b_k_stride, d_bias, d_c, N, ctx->thin_tiles, ctx->d_err(),
                         ctx->d_route(), st, ctx->d_scan(), &ctx->last_launches);
    }
    if (rc) return fail(rc, "gemm launch");
    CUDA_TRY(cudaMemcpy2DAsync(C, c_row_stride * 8, d_c, N * 8, N * 8, M, cudaMemcpyDeviceToHost, st),
             "copy C");
    uint64_t s1 = 0;
    if (sr) CUDA_TRY(cudaMemcpyAsync(&s1, ctx->d_state(), 8, cudaMemcpyDeviceToHost, st), "rng out");
    rc = take_device_error(ctx, st);
    if (rc) return rc;
    if (sr) {
        if (!rng_state && s1 != 0) return fail(DRIFT_EINVAL, "stochastic rounding needs an Rng");
        if (rng_state) *rng_state = s1;
    }
    return DRIFT_OK;
}

// ------------------------------------------------------------------ RealDotSweep in one call
//
// RealDotSweep's per-policy loop (RealDotSweep.java:119-142) over one pair of
// host tensors: X and W cross once, and everything else stays on the device
// until the statistics come back. Per policy, in Java's order: a fresh Rng,
// the whole-tensor per-tensor scales, X's cast then W's, the contraction,
// then the true median of the relative errors (two radix selections) and the
// RMS sums against the exact FP64 contraction.
int drift_real_dot_sweep(drift_ctx *ctx, const drift_policy *policies, int n_policies,
                         int64_t M, int64_t N, int64_t K, const double *X, const double *W,
                         uint64_t rng_seed, double *stats_out) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (!policies || n_policies < 0 || M <= 0 || N <= 0 || K <= 0 || !X || !W ||
        (n_policies > 0 && !stats_out))
        return fail(DRIFT_EINVAL, "bad arguments");
    if (n_policies == 0) return DRIFT_OK;
    cudaStream_t st = ctx->stream;
    const int64_t nx = M * K, nw = N * K, nc = M * N, P = n_policies;
    // Device layout: X, W, their casts, C, the exact C, then per policy two
    // sums, two clamp counts, two radix states of two words, and scratch.
    const size_t words = (size_t)(2 * nx + 2 * nw + 2 * nc) + (size_t)P * 8 + DRIFT_RADIX_BINS + 8;
    double *d_x = (double *)ctx->io.get(words * 8 + 512, st);
    if (!d_x) return fail(DRIFT_ENOMEM, "staging");
    double *d_w = d_x + nx, *d_qx = d_w + nw, *d_qw = d_qx + nx, *d_c = d_qw + nw;
    double *d_exact = d_c + nc;
    double *d_sums = d_exact + nc;                                          // P x 2
    unsigned long long *d_cl = (unsigned long long *)(d_sums + 2 * P);     // P x 2
    unsigned long long *d_med = d_cl + 2 * P;                              // P x 2 x 2
    unsigned long long *d_hist = d_med + 4 * P;                            // radix bins
    double *d_scal = (double *)(d_hist + DRIFT_RADIX_BINS);                  // amax, scale
    uint64_t *d_state = (uint64_t *)(d_scal + 4);
    // Radix states start at (0, k) for k = total/2 - 1 and total/2.
    std::vector<unsigned long long> med0((size_t)P * 4);
    for (int64_t p = 0; p < P; p++) {
        med0[4 * p + 0] = 0;
        med0[4 * p + 1] = (unsigned long long)(nc / 2 - 1);
        med0[4 * p + 2] = 0;
        med0[4 * p + 3] = (unsigned long long)(nc / 2);
    }
    CUDA_TRY(cudaMemcpyAsync(d_x, X, nx * 8, cudaMemcpyHostToDevice, st), "copy X");
    CUDA_TRY(cudaMemcpyAsync(d_w, W, nw * 8, cudaMemcpyHostToDevice, st), "copy W");
    CUDA_TRY(cudaMemsetAsync(d_sums, 0, (size_t)P * 4 * 8, st), "clear sums");
    CUDA_TRY(cudaMemcpyAsync(d_med, med0.data(), med0.size() * 8, cudaMemcpyHostToDevice, st),
             "radix states");
    drift_policy exact{};
    exact.input_format = exact.grad_format = DRIFT_FMT_NONE;
    exact.grad_rounding = DRIFT_ROUND_INHERIT;
    exact.scale_block = exact.acc_block = 32;
    exact.acc = DRIFT_ACC_FP64;
    exact.order = DRIFT_SEQUENTIAL;
    rc = launch_gemm(ctx->ws, ctx->sched, &exact, M, N, K, d_x, K, 1, d_w, K, 1, nullptr, d_exact,
                     N, ctx->thin_tiles, ctx->d_err(), ctx->d_route(), st,
                     ctx->d_scan(), &ctx->last_launches);
    if (rc) return fail(rc, "exact contraction");
    for (int64_t k = 0; k < P; k++) {
        const drift_policy *p = &policies[k];
        CUDA_TRY(cudaMemcpyAsync(d_state, &rng_seed, 8, cudaMemcpyHostToDevice, st), "rng in");
        const double *a = d_x, *b = d_w;
        if (p->input_format != DRIFT_FMT_NONE) {
            const double *src[2] = {d_x, d_w};
            double *dst[2] = {d_qx, d_qw};
            const int64_t n[2] = {nx, nw};
            // Quant.quantize reads the per-tensor factor only under PER_TENSOR
            // scaling (Quant.java:63-80), so the amax pass runs only there.
            const bool per_tensor = p->scaling == DRIFT_PER_TENSOR;
            for (int t = 0; t < 2; t++) {
                rc = DRIFT_OK;
                if (per_tensor) {
                    rc = launch_amax(src[t], n[t], d_scal, st);
                    if (!rc) rc = launch_per_tensor_scale(p->input_format, d_scal, d_scal + 1, st);
                }
                if (!rc)
                    rc = launch_quantize(ctx->ws, p, p->input_format, p->input_rounding, src[t],
                                         dst[t], n[t], per_tensor ? d_scal + 1 : nullptr, 1.0,
                                         d_state, d_cl + 2 * k + t, ctx->d_err(), st);
                if (rc) return fail(rc, "cast");
            }
            a = d_qx;
            b = d_qw;
        }
        if (stochastic_acc(p))
            rc = launch_contract(ctx->ws, ctx->sched, p,
                                 gemm_as_contraction(M, N, K, a, K, 1, b, K, 1, nullptr, d_c, N),
                                 d_state, ctx->d_err(), st);
        else
            rc = launch_gemm(ctx->ws, ctx->sched, p, M, N, K, a, K, 1, b, K, 1, nullptr, d_c, N,
                             ctx->thin_tiles, ctx->d_err(), ctx->d_route(), st,
                             ctx->d_scan(), &ctx->last_launches);
        if (rc) return fail(rc, "contraction");
        rc = launch_error_sums(d_c, d_exact, nc, d_sums + 2 * k, st);
        for (int m = 0; m < 2 && !rc; m++)
            for (int pass = 0; pass < DRIFT_RADIX_PASSES && !rc; pass++) {
                rc = launch_radix_pass(d_c, d_exact, nc, pass, d_med + 4 * k + 2 * m, d_hist, st);
                if (!rc) rc = launch_radix_select(pass, d_hist, d_med + 4 * k + 2 * m, st);
            }
        if (rc) return fail(rc, "statistics");
    }
    std::vector<double> sums((size_t)P * 2);
    std::vector<unsigned long long> cl((size_t)P * 2), med((size_t)P * 4);
    CUDA_TRY(cudaMemcpyAsync(sums.data(), d_sums, sums.size() * 8, cudaMemcpyDeviceToHost, st),
             "read sums");
    CUDA_TRY(cudaMemcpyAsync(cl.data(), d_cl, cl.size() * 8, cudaMemcpyDeviceToHost, st),
             "read clamps");
    CUDA_TRY(cudaMemcpyAsync(med.data(), d_med, med.size() * 8, cudaMemcpyDeviceToHost, st),
             "read medians");
    rc = take_device_error(ctx, st);
    if (rc) return rc;
    for (int64_t k = 0; k < P; k++) {
        const double lo = bitsd(med[4 * k]), hi = bitsd(med[4 * k + 2]);
        stats_out[4 * k + 0] = 0.5 * (lo + hi);
        stats_out[4 * k + 1] = std::sqrt(sums[2 * k] / sums[2 * k + 1]);
        stats_out[4 * k + 2] = (double)cl[2 * k];
        stats_out[4 * k + 3] = (double)cl[2 * k + 1];
    }
    return DRIFT_OK;
}

// ------------------------------------------------------------------ device-resident calls

int drift_amax_dev(drift_ctx *ctx, const double *d_x, int64_t n, double *d_amax, void *stream) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (n < 0 || !d_amax || (n > 0 && !d_x)) return fail(DRIFT_EINVAL, "bad arguments");
    rc = launch_amax(d_x, n, d_amax, pick(ctx, stream));
    return rc ? fail(rc, "amax launch") : DRIFT_OK;
}

int drift_quantize_dev(drift_ctx *ctx, const drift_policy *p, int fmt, int rounding,
                       const double *d_src, double *d_dst, int64_t n, const double *d_scale,
                       double scale, uint64_t *d_rng_state, int64_t *d_clamped, void *stream) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (!p || n < 0 || (n > 0 && (!d_src || !d_dst))) return fail(DRIFT_EINVAL, "bad arguments");
    rc = launch_quantize(ctx->ws, p, fmt, rounding, d_src, d_dst, n, d_scale, scale, d_rng_state,
                         (unsigned long long *)d_clamped, ctx->d_err(), pick(ctx, stream));
    return rc ? fail(rc, "quantize launch") : DRIFT_OK;
}

int drift_quantize_rows_dev(drift_ctx *ctx, const drift_policy *p, int fmt, int rounding,
                            const double *d_src, double *d_dst, int64_t rows, int64_t len,
                            int64_t *d_clamped, void *stream) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (!p || rows < 0 || len < 0 || (rows * len > 0 && (!d_src || !d_dst)))
        return fail(DRIFT_EINVAL, "bad arguments");
    rc = launch_quantize_rows(p, fmt, rounding, d_src, d_dst, rows, len,
                              (unsigned long long *)d_clamped, ctx->d_err(), pick(ctx, stream));
    return rc ? fail(rc, "row-wise cast (stochastic rounding and MX scaling are per tensor)")
              : DRIFT_OK;
}

int drift_quantize_draws_dev(drift_ctx *ctx, const drift_policy *p, int fmt, int rounding,
                             const double *d_src, int64_t n, const double *d_scale, double scale,
                             int64_t *d_draws, void *stream) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (!p || n < 0 || !d_draws || (n > 0 && !d_src)) return fail(DRIFT_EINVAL, "bad arguments");
    rc = launch_quantize_draws(ctx->ws, p, fmt, rounding, d_src, n, d_scale, scale,
                               (uint64_t *)d_draws, ctx->d_err(), pick(ctx, stream));
    return rc ? fail(rc, "draw count launch") : DRIFT_OK;
}

int drift_per_tensor_scale_dev(drift_ctx *ctx, int fmt, const double *d_amax, double *d_scale,
                               void *stream) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (!d_amax || !d_scale) return fail(DRIFT_EINVAL, "null pointer");
    rc = launch_per_tensor_scale(fmt, d_amax, d_scale, pick(ctx, stream));
    return rc ? fail(rc, "per-tensor scale") : DRIFT_OK;
}

int drift_error_sums_dev(drift_ctx *ctx, const double *d_got, const double *d_exact, int64_t n,
                         double *d_sums, void *stream) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (n < 0 || !d_sums || (n > 0 && (!d_got || !d_exact))) return fail(DRIFT_EINVAL, "bad arguments");
    rc = launch_error_sums(d_got, d_exact, n, d_sums, pick(ctx, stream));
    return rc ? fail(rc, "error sums") : DRIFT_OK;
}

int drift_gemm_dev(drift_ctx *ctx, const drift_policy *p, int64_t M, int64_t N, int64_t K,
                   const double *d_A, int64_t a_row_stride, int64_t a_k_stride, const double *d_B,
                   int64_t b_row_stride, int64_t b_k_stride, const double *d_bias, double *d_C,
                   int64_t c_row_stride, uint64_t *d_rng_state, void *stream) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (!p || c_row_stride < N || M < 0 || N < 0 || K < 0) return fail(DRIFT_EINVAL, "bad shape or stride");
    if (M > 0 && N > 0 && (!d_C || (K > 0 && (!d_A || !d_B)))) return fail(DRIFT_EINVAL, "null buffer");
    if (stochastic_acc(p)) {
        if (!d_rng_state) return fail(DRIFT_EINVAL, "stochastic accumulation needs d_rng_state");
        rc = launch_contract(ctx->ws, ctx->sched, p,
                             gemm_as_contraction(M, N, K, d_A, a_row_stride, a_k_stride, d_B,
                                                 b_row_stride, b_k_stride, d_bias, d_C,
                                                 c_row_stride),
                             d_rng_state, ctx->d_err(), pick(ctx, stream));
    } else {
        rc = launch_gemm(ctx->ws, ctx->sched, p, M, N, K, d_A, a_row_stride, a_k_stride, d_B,
                         b_row_stride, b_k_stride, d_bias, d_C, c_row_stride, ctx->thin_tiles,
                         ctx->d_err(), ctx->d_route(), pick(ctx, stream), ctx->d_scan(),
                         &ctx->last_launches);
    }
    return rc ? fail(rc, "gemm launch") : DRIFT_OK;
}

int drift_set_thin_tiles(drift_ctx *ctx, int64_t tiles) {
    int rc = enter(ctx);
    if (rc) return rc;
    ctx->thin_tiles = tiles < 0 ? -1 : tiles;
    return DRIFT_OK;
}

int drift_gemm_launches(drift_ctx *ctx, int *launches) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (!launches) return fail(DRIFT_EINVAL, "null launches");
    *launches = ctx->last_launches;
    return DRIFT_OK;
}

int drift_gemm_route(drift_ctx *ctx, int *route, void *stream) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (!route) return fail(DRIFT_EINVAL, "null route");
    cudaStream_t st = pick(ctx, stream);
    int r = 0;
    CUDA_TRY(cudaMemcpyAsync(&r, ctx->d_route(), sizeof(int), cudaMemcpyDeviceToHost, st),
             "read route");
    CUDA_TRY(cudaStreamSynchronize(st), "synchronize");
    *route = r;
    return DRIFT_OK;
}

// Lowest and highest element index an affine access off + sum(coef_j * x_j),
// 0 <= x_j < ext_j, reaches over the box of its indices.
static void reach(int64_t off, const int64_t *coef, const int64_t *ext, int n, int64_t *lo,
                  int64_t *hi) {
    *lo = *hi = off;
    for (int j = 0; j < n; j++) {
        const int64_t span = coef[j] * (ext[j] - 1);
        if (span > 0) *hi += span;
        else *lo += span;
    }
}

// Whether every element the contraction reaches lies in [0, len) of each
// buffer. The box over (t, i, o, k) holds every window, so this is exact for
// FULL windows and conservative for the others.
static bool contraction_fits(const drift_contraction &op, int64_t a_len, int64_t b_len,
                             int64_t c_len) {
    const int64_t total = op.batch * op.rows * op.cols;
    if (total == 0) return true;
    int64_t lo, hi;
    const int64_t c_coef[3] = {op.c_batch, op.c_row, op.c_col};
    const int64_t c_ext[3] = {op.batch, op.rows, op.cols};
    reach(op.c_off, c_coef, c_ext, 3, &lo, &hi);
    if (lo < 0 || hi >= c_len) return false;
    if (op.depth == 0) return true;
    const int64_t a_coef[3] = {op.a_batch, op.a_row, op.a_k};
    const int64_t a_ext[3] = {op.batch, op.rows, op.depth};
    reach(op.a_off, a_coef, a_ext, 3, &lo, &hi);
    if (lo < 0 || hi >= a_len) return false;
    const int64_t b_coef[3] = {op.b_batch, op.b_col, op.b_k};
    const int64_t b_ext[3] = {op.batch, op.cols, op.depth};
    reach(op.b_off, b_coef, b_ext, 3, &lo, &hi);
    return lo >= 0 && hi < b_len;
}

int drift_contract(drift_ctx *ctx, const drift_policy *p, const drift_contraction *op,
                   const double *a, int64_t a_len, const double *b, int64_t b_len, double *c,
                   int64_t c_len, uint64_t *rng_state) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (!p || !op) return fail(DRIFT_EINVAL, "null argument");
    rc = check_contraction(*op);
    if (rc) return fail(rc, "bad contraction");
    if (a_len < 0 || b_len < 0 || c_len < 0 || !contraction_fits(*op, a_len, b_len, c_len))
        return fail(DRIFT_EINVAL, "contraction reaches outside its buffers");
    if (op->batch * op->rows * op->cols == 0) return DRIFT_OK;
    if (!c || (op->depth > 0 && (!a || !b))) return fail(DRIFT_EINVAL, "null buffer");
    cudaStream_t st = ctx->stream;
    const int64_t la = op->depth > 0 ? a_len : 0, lb = op->depth > 0 ? b_len : 0;
    char *buf = (char *)ctx->io.get((size_t)(la + lb + c_len + 6) * 8 + 512, st);
    if (!buf) return fail(DRIFT_ENOMEM, "staging");
    double *d_a = (double *)buf;
    double *d_b = d_a + ((la + 1) & ~1LL);
    double *d_c = d_b + ((lb + 1) & ~1LL);
    if (la) CUDA_TRY(cudaMemcpyAsync(d_a, a, la * 8, cudaMemcpyHostToDevice, st), "copy A");
    if (lb) CUDA_TRY(cudaMemcpyAsync(d_b, b, lb * 8, cudaMemcpyHostToDevice, st), "copy B");
    CUDA_TRY(cudaMemcpyAsync(d_c, c, c_len * 8, cudaMemcpyHostToDevice, st), "copy C");
    const bool sr = stochastic_acc(p);
    if (sr) {
        const uint64_t s0 = rng_state ? *rng_state : 0;
        CUDA_TRY(cudaMemcpyAsync(ctx->d_state(), &s0, 8, cudaMemcpyHostToDevice, st), "rng in");
    }
    ContractDesc d{*op, d_a, d_b, d_c, nullptr};
    rc = launch_contract(ctx->ws, ctx->sched, p, d, sr ? ctx->d_state() : nullptr, ctx->d_err(),
                         st);
    if (rc) return fail(rc, "contraction launch");
    CUDA_TRY(cudaMemcpyAsync(c, d_c, c_len * 8, cudaMemcpyDeviceToHost, st), "copy C");
    uint64_t s1 = 0;
    if (sr) CUDA_TRY(cudaMemcpyAsync(&s1, ctx->d_state(), 8, cudaMemcpyDeviceToHost, st), "rng out");
    rc = take_device_error(ctx, st);
    if (rc) return rc;
    if (sr) {
        if (!rng_state && s1 != 0) return fail(DRIFT_EINVAL, "stochastic rounding needs an Rng");
        if (rng_state) *rng_state = s1;
    }
    return DRIFT_OK;
}

int drift_contract_dev(drift_ctx *ctx, const drift_policy *p, const drift_contraction *op,
                       const double *d_a, const double *d_b, double *d_c, uint64_t *d_rng_state,
                       void *stream) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (!p || !op) return fail(DRIFT_EINVAL, "null argument");
    rc = check_contraction(*op);
    if (rc) return fail(rc, "bad contraction");
    if (op->batch * op->rows * op->cols == 0) return DRIFT_OK;
    if (!d_c || (op->depth > 0 && (!d_a || !d_b))) return fail(DRIFT_EINVAL, "null buffer");
    if (stochastic_acc(p) && !d_rng_state)
        return fail(DRIFT_EINVAL, "stochastic accumulation needs d_rng_state");
    ContractDesc d{*op, d_a, d_b, d_c, nullptr};
    rc = launch_contract(ctx->ws, ctx->sched, p, d, d_rng_state, ctx->d_err(), pick(ctx, stream));
    return rc ? fail(rc, "contraction launch") : DRIFT_OK;
}

int drift_radix_hist_dev(drift_ctx *ctx, const double *d_got, const double *d_exact, int64_t n,
                         int pass, const uint64_t *d_state, uint64_t *d_hist, void *stream) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (n < 0 || !d_state || !d_hist || (n > 0 && (!d_got || !d_exact)))
        return fail(DRIFT_EINVAL, "bad arguments");
    rc = launch_radix_pass(d_got, d_exact, n, pass, (unsigned long long *)d_state,
                           (unsigned long long *)d_hist, pick(ctx, stream));
    return rc ? fail(rc, "radix histogram") : DRIFT_OK;
}

int drift_radix_select_dev(drift_ctx *ctx, int pass, const uint64_t *d_hist, uint64_t *d_state,
                           void *stream) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (!d_state || !d_hist) return fail(DRIFT_EINVAL, "bad arguments");
    rc = launch_radix_select(pass, (const unsigned long long *)d_hist,
                             (unsigned long long *)d_state, pick(ctx, stream));
    return rc ? fail(rc, "radix select") : DRIFT_OK;
}

int drift_group_kth_rel_error_dev(drift_ctx *ctx, const double *d_got, const double *d_exact,
                                  int64_t groups, int64_t n, int64_t k, double *d_out,
                                  void *stream) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (groups < 0 || (groups > 0 && (!d_got || !d_exact || !d_out)))
        return fail(DRIFT_EINVAL, "bad arguments");
    rc = launch_group_kth(d_got, d_exact, groups, n, k, d_out, pick(ctx, stream));
    return rc ? fail(rc, "per-group order statistic (n <= DRIFT_GROUP_MAX, 0 <= k < n)")
              : DRIFT_OK;
}

int drift_probe_fp64(drift_ctx *ctx, double *ops_per_s) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (!ops_per_s) return fail(DRIFT_EINVAL, "null out");
    rc = launch_fp64_probe(ctx->stream, ops_per_s);
    return rc ? fail(rc, "fp64 probe") : DRIFT_OK;
}

int drift_probe_fp32(drift_ctx *ctx, double *fma_per_s) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (!fma_per_s) return fail(DRIFT_EINVAL, "null out");
    rc = launch_fp32_probe(ctx->stream, fma_per_s);
    return rc ? fail(rc, "fp32 probe") : DRIFT_OK;
}

int drift_quantize_dev_noalloc(const drift_policy *p, int fmt, int rounding, const double *d_src,
                               double *d_dst, int64_t n, const double *d_scale, double scale,
                               uint64_t *d_rng_state, int64_t *d_clamped, int *d_err,
                               void *stream) {
    if (!p || !d_err || n < 0 || (n > 0 && (!d_src || !d_dst)))
        return fail(DRIFT_EINVAL, "bad arguments");
    const int rc = launch_quantize_noalloc(p, fmt, rounding, d_src, d_dst, n, d_scale, scale,
                                           d_rng_state, (unsigned long long *)d_clamped, d_err,
                                           (cudaStream_t)stream);
    if (rc == DRIFT_ENOMEM)
        return fail(rc, "a stochastic cast of more items than the fixed scratch array holds (DRIFT_NOALLOC_MAX_ITEMS)");
    return rc ? fail(rc, "no-allocation quantize launch") : DRIFT_OK;
}

// ------------------------------------------------------------------ training step

int drift_embed_gather_dev(drift_ctx *ctx, const int32_t *d_tokens, int64_t n_tok,
                           const double *d_table, int64_t vocab, int64_t width, double *d_out,
                           void *stream) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (n_tok < 0 || vocab < 0 || width < 0 || (n_tok * width > 0 && (!d_tokens || !d_table || !d_out)))
        return fail(DRIFT_EINVAL, "bad arguments");
    rc = launch_embed_gather(d_tokens, n_tok, d_table, vocab, width, d_out, ctx->d_err(),
                             pick(ctx, stream));
    return rc ? fail(rc, "embedding gather") : DRIFT_OK;
}

int drift_embed_grad_dev(drift_ctx *ctx, const int32_t *d_tokens, int64_t n_tok,
                         const double *d_rows, int64_t width, double *d_table_grad, int64_t vocab,
                         void *stream) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (n_tok < 0 || vocab < 0 || width < 0 ||
        (n_tok * width * vocab > 0 && (!d_tokens || !d_rows || !d_table_grad)))
        return fail(DRIFT_EINVAL, "bad arguments");
    rc = launch_embed_grad(d_tokens, n_tok, d_rows, width, d_table_grad, vocab, pick(ctx, stream));
    return rc ? fail(rc, "embedding gradient") : DRIFT_OK;
}

int drift_bias_grad_dev(drift_ctx *ctx, const double *d_dy, int64_t rows, int64_t cols,
                        double *d_db, void *stream) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (rows < 0 || cols < 0 || (cols > 0 && (!d_db || (rows > 0 && !d_dy))))
        return fail(DRIFT_EINVAL, "bad arguments");
    rc = launch_bias_grad(d_dy, rows, cols, d_db, pick(ctx, stream));
    return rc ? fail(rc, "bias gradient") : DRIFT_OK;
}

int drift_tanh_backward_dev(drift_ctx *ctx, const double *d_out, double *d_grad, int64_t n,
                            void *stream) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (n < 0 || (n > 0 && (!d_out || !d_grad))) return fail(DRIFT_EINVAL, "bad arguments");
    rc = launch_tanh_backward(d_out, d_grad, n, pick(ctx, stream));
    return rc ? fail(rc, "tanh backward") : DRIFT_OK;
}

int drift_scale_for_dev(drift_ctx *ctx, int fmt, const double *d_amax_now, double *d_history,
                        int32_t history_len, int64_t *d_count, double *d_scale, void *stream) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (!d_amax_now || !d_history || !d_count || !d_scale || history_len <= 0)
        return fail(DRIFT_EINVAL, "bad arguments");
    rc = launch_scale_for(fmt, d_amax_now, d_history, history_len, d_count, d_scale,
                          pick(ctx, stream));
    return rc ? fail(rc, "delayed scale") : DRIFT_OK;
}

int drift_adam_dev(drift_ctx *ctx, double *d_param, const double *d_grad, double *d_m,
                   double *d_v, int64_t n, int32_t step, double lr, int32_t fp32_master,
                   void *stream) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (n < 0 || step < 1 || (n > 0 && (!d_param || !d_grad || !d_m || !d_v)))
        return fail(DRIFT_EINVAL, "bad arguments");
    // Trainer.java:248-249, Math.pow on the host.
    const double c1 = 1 - std::pow(0.9, (double)step);
    const double c2 = 1 - std::pow(0.999, (double)step);
    rc = launch_adam(d_param, d_grad, d_m, d_v, n, c1, c2, lr, fp32_master ? 1 : 0,
                     pick(ctx, stream));
    return rc ? fail(rc, "adam") : DRIFT_OK;
}

int drift_check_dev(drift_ctx *ctx, void *stream) {
    int rc = enter(ctx);
    if (rc) return rc;
    return take_device_error(ctx, pick(ctx, stream));
}

}  // extern "C"
