// quant.cu — the cast pass: amax, per-tensor / MX scaling, minifloat rounding.
//
// Device form of Quant (java/src/main/java/io/drift/kernel/Quant.java) and of
// the element-wise MiniFloat / Dot.round entry points.
//
// Work decomposition. Elements are grouped into "items": 32 consecutive
// elements for element-wise work, one scale block for MX (Quant.java:101-103,
// blocks follow the flattened span). One warp handles one item at a time,
// lane = element, so a warp reads 256 contiguous bytes; a CTA of 8 warps owns
// kItemsPerWarp * 8 consecutive items, visited j-major so the 8 warps stream
// one contiguous 2 KiB window per step.
//
// Stochastic rounding. Java draws from one splitmix64 stream in element
// order, and only for elements whose scaled value is inexact
// (MiniFloat.java:264-273). splitmix64 is counter-based, so an element's draw
// is fixed once its index among the drawing elements is known. A count pass
// stores the number of draws per item and per CTA, a one-CTA scan turns the
// CTA counts into offsets (and advances the stored Rng state by the total),
// and the apply pass recomputes each element's rank from the item counts and
// a warp ballot. No kernel waits on another CTA, so nothing can spin.
#include <algorithm>
#include <cstdio>
#include <mutex>

#include "codec.cuh"
#include "internal.h"

namespace drift {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kItemsPerWarp = 8;
constexpr int kItemsPerCta = kWarps * kItemsPerWarp;

__device__ __forceinline__ double canon_nan(double v) {
    return isnan(v) ? bitsd(kJavaNaNBits) : v;
}

__device__ __forceinline__ double warp_max(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// ------------------------------------------------------------------ ops
// An op maps one input element to one output element. begin_item runs once
// per item on the whole warp (MX computes its shared exponent there).

struct QuantOp {
    const double *src;
    double *dst;
    FmtDesc f;
    int rm;
    int scaling;
    int headroom;
    const double *d_scale;  // device-resident per-tensor scale, or null
    double scale;
    double inv;

    struct Item {
        double down, up;
        bool zero;
    };

    // Loads a device-resident scale once per thread (Quant.java:72).
    __device__ void prepare() {
        if (d_scale) {
            scale = *d_scale;
            inv = __ddiv_rn(1.0, scale);
        }
    }

    __device__ Item begin_item(int64_t lo, int64_t hi, int lane) const {
        Item it{1.0, 1.0, false};
        if (scaling != DRIFT_MX_BLOCK) return it;
        // Quant.amax over the block (Quant.java:25-34): NaN never wins.
        double m = 0.0;
        for (int64_t i = lo + lane; i < hi; i += 32) m = fmax(m, fabs(src[i]));
        m = warp_max(m);
        if (m == 0.0 || !isfinite(m)) {  // Quant.java:105-110
            it.zero = true;
            return it;
        }
        int shared = java_get_exponent(m) - f.emax + headroom;  // Quant.java:112-113
        shared = max(-127, min(127, shared));
        it.down = pow2(-shared);
        it.up = pow2(shared);
        return it;
    }
    __device__ double load(int64_t i) const { return src[i]; }
    __device__ double scaled(const Item &it, double x) const {
        if (scaling == DRIFT_PER_TENSOR) return __dmul_rn(x, scale);  // Quant.java:74
        if (scaling == DRIFT_MX_BLOCK) return __dmul_rn(x, it.down);  // scalb, Quant.java:116
        return x;
    }
    __device__ bool needs_draw(const Item &it, double x, int &err) const {
        if (it.zero) return false;
        bool drew;
        quantize_value(f, scaled(it, x), DRIFT_STOCHASTIC, 0, drew, err);
        return drew;
    }
    // The cast of one element: what Quant.quantize stores (Quant.java:56-123).
    __device__ double value(const Item &it, double x, uint64_t u53, bool &clamp, int &err) const {
        if (it.zero) return 0.0;
        const double s = scaled(it, x);
        clamp = fabs(s) > f.max_finite;  // counted before rounding (Quant.java:67, :75, :117)
        bool drew;
        double q = quantize_value(f, s, rm, u53, drew, err);
        if (scaling == DRIFT_PER_TENSOR) q = __dmul_rn(q, inv);  // Quant.java:76
        else if (scaling == DRIFT_MX_BLOCK) q = __dmul_rn(q, it.up);  // exact, Quant.java:119
        return canon_nan(q);
    }
    __device__ void apply(const Item &it, int64_t i, double x, uint64_t u53, bool &clamp,
                          int &err) const {
        dst[i] = value(it, x, u53, clamp, err);
    }
};

struct EncodeOp {  // MiniFloat.encode over an array
    const double *src;
    int32_t *dst;
    FmtDesc f;
    int rm;
    struct Item {};
    __device__ void prepare() {}
    __device__ Item begin_item(int64_t, int64_t, int) const { return Item{}; }
    __device__ double load(int64_t i) const { return src[i]; }
    __device__ bool needs_draw(const Item &, double x, int &err) const {
        bool drew;
        encode_value(f, x, DRIFT_STOCHASTIC, 0, drew, err);
        return drew;
    }
    __device__ void apply(const Item &, int64_t i, double x, uint64_t u53, bool &, int &err) const {
        bool drew;
        dst[i] = encode_value(f, x, rm, u53, drew, err);
    }
};

struct AccRoundOp {  // Dot.round over an array
    const double *src;
    double *dst;
    int acc;
    int rm;
    struct Item {};
    __device__ void prepare() {}
    __device__ Item begin_item(int64_t, int64_t, int) const { return Item{}; }
    __device__ double load(int64_t i) const { return src[i]; }
    __device__ bool needs_draw(const Item &, double x, int &) const {
        bool drew;
        acc_round_any(acc, x, DRIFT_STOCHASTIC, 0, drew);
        return drew;
    }
    __device__ void apply(const Item &, int64_t i, double x, uint64_t u53, bool &, int &) const {
        bool drew;
        dst[i] = acc_round_any(acc, x, rm, u53, drew);
    }
};

// ------------------------------------------------------------------ kernels

struct SrArgs {
    uint32_t *item_counts;        // draws per item (count pass writes, apply pass reads)
    uint64_t *cta_counts;         // draws per CTA, then exclusive offsets after the scan
    const uint64_t *state_before; // Rng state the draws are taken from
    unsigned long long *clamped;  // may be null
    int *err;
};

// PASS 0: single pass, no random draws. PASS 1: count draws. PASS 2: apply
// with draws.
template <class Op, int PASS>
__global__ void __launch_bounds__(kThreads) elem_kernel(Op op_in, int64_t n, int64_t item_len,
                                                         SrArgs sr) {
    Op op = op_in;
    op.prepare();
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t lt_mask = (1u << lane) - 1u;
    const int64_t cta = blockIdx.x;
    __shared__ uint64_t s_base[kItemsPerCta];
    __shared__ uint64_t s_total[kWarps];

    uint64_t state = 0;
    if (PASS == 2) {
        // Exclusive scan of this CTA's item counts, in item order.
        if (warp == 0) {
            uint64_t carry = sr.cta_counts[cta];
            for (int c = 0; c < kItemsPerCta; c += 32) {
                const int64_t item = cta * kItemsPerCta + c + lane;
                uint64_t v = sr.item_counts[item];
                uint64_t incl = v;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    uint64_t t = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= o) incl += t;
                }
                s_base[c + lane] = carry + incl - v;
                carry += __shfl_sync(0xffffffffu, incl, 31);
            }
        }
        __syncthreads();
        state = sr.state_before ? *sr.state_before : 0;
    }

    int err = 0;
    uint32_t clamps = 0;
    uint64_t warp_draws = 0;
    for (int j = 0; j < kItemsPerWarp; j++) {
        const int slot = j * kWarps + warp;
        const int64_t item = cta * kItemsPerCta + slot;
        const int64_t lo = item * item_len;
        if (lo >= n) {
            if (PASS == 1 && lane == 0) sr.item_counts[item] = 0;
            continue;
        }
        const int64_t hi = min(n, lo + item_len);
        const auto it = op.begin_item(lo, hi, lane);
        uint64_t rank = PASS == 2 ? s_base[slot] : 0;
        uint32_t count = 0;
        for (int64_t c = lo; c < hi; c += 32) {
            const int64_t i = c + lane;
            const bool valid = i < hi;
            const double x = valid ? op.load(i) : 0.0;
            if (PASS == 0) {
                if (valid) {
                    bool clamp = false;
                    op.apply(it, i, x, 0, clamp, err);
                    clamps += clamp;
                }
            } else {
                const bool need = valid && op.needs_draw(it, x, err);
                const uint32_t m = __ballot_sync(0xffffffffu, need);
                if (PASS == 1) {
                    count += __popc(m);
                } else {
                    const uint64_t idx = rank + __popc(m & lt_mask);
                    rank += __popc(m);
                    if (valid) {
                        bool clamp = false;
                        op.apply(it, i, x, need ? draw_u53(state, idx) : 0, clamp, err);
                        clamps += clamp;
                    }
                }
            }
        }
        if (PASS == 1 && lane == 0) {
            sr.item_counts[item] = count;
            warp_draws += count;
        }
    }

    if (PASS == 1) {
        if (lane == 0) s_total[warp] = warp_draws;
        __syncthreads();
        if (threadIdx.x == 0) {
            uint64_t t = 0;
            for (int w = 0; w < kWarps; w++) t += s_total[w];
            sr.cta_counts[cta] = t;
        }
    }
    if (PASS != 1 && sr.clamped) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) clamps += __shfl_xor_sync(0xffffffffu, clamps, o);
        if (lane == 0 && clamps) atomicAdd(sr.clamped, (unsigned long long)clamps);
    }
    if (err) atomicOr(sr.err, err);
}

// The single pass of a nearest-even or truncating cast when both arrays are
// 16-byte aligned and items are 32 elements (no scaling, per-tensor, or MX
// blocks of 32). A warp takes 128 consecutive elements per step as two
// coalesced 512-byte loads (lane l holds elements 2l, 2l+1 and 64+2l,
// 65+2l), so sixteen lanes hold one 32-element MX block and its amax is four
// shuffles. The grid strides over the array; the clamp count is reduced once
// per warp at the end.
template <int SCALING>
__global__ void __launch_bounds__(kThreads) cast_vec_kernel(QuantOp op_in, int64_t n,
                                                            unsigned long long *clamped,
                                                            int *err_out) {
    QuantOp op = op_in;
    op.prepare();
    const int lane = threadIdx.x & 31;
    const int64_t warp0 = ((int64_t)blockIdx.x * kThreads + threadIdx.x - lane) * 4;
    const int64_t step = (int64_t)gridDim.x * kThreads * 4;
    int err = 0;
    unsigned clamps = 0;
    for (int64_t base = warp0; base < n; base += step) {
        double x[4];
        int64_t at[2];
#pragma unroll
        for (int h = 0; h < 2; h++) {
            at[h] = base + 64 * h + 2 * lane;
            if (at[h] + 1 < n) {
                const double2 v = __ldcs(reinterpret_cast<const double2 *>(op.src + at[h]));
                x[2 * h] = v.x;
                x[2 * h + 1] = v.y;
            } else {
                x[2 * h] = at[h] < n ? __ldcs(op.src + at[h]) : 0.0;
                x[2 * h + 1] = 0.0;
            }
        }
#pragma unroll
        for (int h = 0; h < 2; h++) {
            QuantOp::Item it{1.0, 1.0, false};
            if (SCALING == DRIFT_MX_BLOCK) {
                // Quant.amax over the block (Quant.java:25-34): NaN never wins,
                // and lanes past the end hold 0.
                double m = fmax(fabs(x[2 * h]), fabs(x[2 * h + 1]));
#pragma unroll
                for (int o = 1; o < 16; o <<= 1) m = fmax(m, __shfl_xor_sync(0xffffffffu, m, o));
                if (m == 0.0 || !isfinite(m)) {  // Quant.java:105-110
                    it.zero = true;
                } else {
                    const int sh = max(-127, min(127, java_get_exponent(m) - op.f.emax + op.headroom));
                    it.down = pow2(-sh);
                    it.up = pow2(sh);
                }
            }
            bool c0 = false, c1 = false;
            const double q0 = op.value(it, x[2 * h], 0, c0, err);
            const double q1 = op.value(it, x[2 * h + 1], 0, c1, err);
            if (at[h] + 1 < n) {
                *reinterpret_cast<double2 *>(op.dst + at[h]) = make_double2(q0, q1);
                clamps += c0 + c1;
            } else if (at[h] < n) {
                op.dst[at[h]] = q0;
                clamps += c0;
            }
        }
    }
    if (clamped) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) clamps += __shfl_xor_sync(0xffffffffu, clamps, o);
        if (lane == 0 && clamps) atomicAdd(clamped, (unsigned long long)clamps);
    }
    if (err) atomicOr(err_out, err);
}

// Launches cast_vec_kernel when the call fits it; false leaves it to elem_kernel.
static bool launch_cast_vec(const QuantOp &op, int64_t n, int64_t item_len,
                            unsigned long long *d_clamped, int *d_err, cudaStream_t st) {
    if (op.rm == DRIFT_STOCHASTIC || item_len != 32) return false;
    if (((uintptr_t)op.src | (uintptr_t)op.dst) % 16 != 0) return false;
    if (n <= 0) return true;
    // One wave: the CTAs every SM holds at once, or fewer for small casts.
    const int64_t need = (n + kThreads * 4 - 1) / (kThreads * 4);
    auto launch = [&](auto kernel) {
        int dev = 0, sms = 148, per_sm = 1;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, 0);
        const int64_t wave = (int64_t)std::max(1, sms) * std::max(1, per_sm);
        kernel<<<(unsigned)std::min(need, wave), kThreads, 0, st>>>(op, n, d_clamped, d_err);
    };
    switch (op.scaling) {
        case DRIFT_PER_TENSOR: launch(cast_vec_kernel<DRIFT_PER_TENSOR>); break;
        case DRIFT_MX_BLOCK: launch(cast_vec_kernel<DRIFT_MX_BLOCK>); break;
        default: launch(cast_vec_kernel<DRIFT_SCALE_NONE>);
    }
    return true;
}

// One CTA turns per-CTA draw counts into exclusive offsets and advances the
// Rng state by the total number of draws (the state Java holds afterwards).
__global__ void __launch_bounds__(1024) sr_scan_kernel(uint64_t *cta_counts, int64_t n_ctas,
                                                       uint64_t *state, uint64_t *state_before,
                                                       int *err) {
    __shared__ uint64_t s_warp[32];
    const int t = threadIdx.x;
    const int64_t per = (n_ctas + 1023) / 1024;
    const int64_t lo = min(n_ctas, (int64_t)t * per);
    const int64_t hi = min(n_ctas, lo + per);
    uint64_t sum = 0;
    for (int64_t i = lo; i < hi; i++) sum += cta_counts[i];
    // Block-wide exclusive scan of the per-thread sums.
    const int lane = t & 31, warp = t >> 5;
    uint64_t incl = sum;
    for (int o = 1; o < 32; o <<= 1) {
        uint64_t v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    if (lane == 31) s_warp[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        uint64_t w = s_warp[lane];
        uint64_t wi = w;
        for (int o = 1; o < 32; o <<= 1) {
            uint64_t v = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= o) wi += v;
        }
        s_warp[lane] = wi - w;  // exclusive warp offsets
    }
    __syncthreads();
    uint64_t run = s_warp[warp] + incl - sum;
    for (int64_t i = lo; i < hi; i++) {
        const uint64_t c = cta_counts[i];
        cta_counts[i] = run;
        run += c;
    }
    if (t == 1023) {
        const uint64_t total = run;  // thread 1023 ends at the grand total
        if (state) {
            *state_before = *state;
            *state = *state + total * kGolden;
        } else if (total) {
            atomicOr(err, DEV_ERR_NO_RNG);
        }
    }
}

__global__ void amax_kernel(const double *x, int64_t n, unsigned long long *out) {
    double m = 0.0;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        m = fmax(m, fabs(x[i]));
    m = warp_max(m);
    // Non-negative doubles order like their bit patterns.
    if ((threadIdx.x & 31) == 0 && m > 0.0) atomicMax(out, (unsigned long long)dbits(m));
}

__global__ void decode_kernel(FmtDesc f, const int32_t *codes, double *out, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        out[i] = decode_value(f, codes[i]);
}

// ------------------------------------------------------------------ launchers

template <class Op>
static int run_elem(Workspace &ws, const Op &op, int64_t n, int64_t item_len, bool stochastic,
                    uint64_t *d_state, unsigned long long *d_clamped, int *d_err,
                    cudaStream_t st) {
    if (n <= 0) return DRIFT_OK;
    const int64_t items_needed = (n + item_len - 1) / item_len;
    const int64_t grid = (items_needed + kItemsPerCta - 1) / kItemsPerCta;
    if (grid > 0x7fffffffLL) return DRIFT_EINVAL;
    SrArgs sr{nullptr, nullptr, nullptr, d_clamped, d_err};
    if (!stochastic) {
        elem_kernel<Op, 0><<<(unsigned)grid, kThreads, 0, st>>>(op, n, item_len, sr);
        return cudaGetLastError() == cudaSuccess ? DRIFT_OK : DRIFT_ECUDA;
    }
    const size_t items = (size_t)grid * kItemsPerCta;
    const size_t bytes = items * sizeof(uint32_t) + (size_t)grid * sizeof(uint64_t) + 256;
    char *base = (char *)ws.get(bytes, st);
    if (!base) return DRIFT_ENOMEM;
    sr.cta_counts = (uint64_t *)base;
    uint64_t *state_before = (uint64_t *)(base + (size_t)grid * sizeof(uint64_t));
    sr.item_counts = (uint32_t *)(base + (size_t)grid * sizeof(uint64_t) + 256);
    sr.state_before = state_before;
    elem_kernel<Op, 1><<<(unsigned)grid, kThreads, 0, st>>>(op, n, item_len, sr);
    sr_scan_kernel<<<1, 1024, 0, st>>>(sr.cta_counts, grid, d_state, state_before, d_err);
    elem_kernel<Op, 2><<<(unsigned)grid, kThreads, 0, st>>>(op, n, item_len, sr);
    return cudaGetLastError() == cudaSuccess ? DRIFT_OK : DRIFT_ECUDA;
}

int launch_amax(const double *d_x, int64_t n, double *d_amax, cudaStream_t st) {
    if (cudaMemsetAsync(d_amax, 0, sizeof(double), st) != cudaSuccess) return DRIFT_ECUDA;
    if (n <= 0) return DRIFT_OK;
    int64_t blocks = (n + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    amax_kernel<<<(unsigned)blocks, 256, 0, st>>>(d_x, n, (unsigned long long *)d_amax);
    return cudaGetLastError() == cudaSuccess ? DRIFT_OK : DRIFT_ECUDA;
}

// Quant.perTensorScale on the device (Quant.java:37-42).
__global__ void per_tensor_scale_kernel(const double *amax, double max_finite, double *scale) {
    const double a = *amax;
    *scale = (a == 0.0 || !isfinite(a)) ? 1.0 : __ddiv_rn(max_finite, a);
}

int launch_per_tensor_scale(int fmt, const double *d_amax, double *d_scale, cudaStream_t st) {
    FmtDesc f;
    if (!fmt_desc(fmt, &f)) return DRIFT_EINVAL;
    per_tensor_scale_kernel<<<1, 1, 0, st>>>(d_amax, f.max_finite, d_scale);
    return cudaGetLastError() == cudaSuccess ? DRIFT_OK : DRIFT_ECUDA;
}

// The cast operator of Quant.quantize for one call (Quant.java:50-123), or
// an error status.
static int make_quant_op(const drift_policy *p, int fmt, int rm, const double *d_src,
                         double *d_dst, const double *d_scale, double scale, QuantOp *op,
                         int64_t *item_len) {
    if (!fmt_desc(fmt, &op->f)) return DRIFT_EINVAL;
    if (rm < 0 || rm > 2) return DRIFT_EINVAL;
    if (p->scaling < 0 || p->scaling > 2) return DRIFT_EINVAL;
    if (p->scaling == DRIFT_MX_BLOCK && p->scale_block <= 0) return DRIFT_EINVAL;
    op->src = d_src;
    op->dst = d_dst;
    op->rm = rm;
    op->scaling = p->scaling;
    op->headroom = p->mx_headroom;
    op->d_scale = p->scaling == DRIFT_PER_TENSOR ? d_scale : nullptr;
    op->scale = scale;
    op->inv = 1.0 / scale;  // host IEEE division, round to nearest (Quant.java:72)
    *item_len = p->scaling == DRIFT_MX_BLOCK ? p->scale_block : 32;
    return DRIFT_OK;
}

int launch_quantize(Workspace &ws, const drift_policy *p, int fmt, int rm, const double *d_src,
                    double *d_dst, int64_t n, const double *d_scale, double scale,
                    uint64_t *d_state, unsigned long long *d_clamped, int *d_err,
                    cudaStream_t st) {
    if (n < 0) return DRIFT_EINVAL;
    if (fmt == DRIFT_FMT_NONE) {  // Quant.java:58-61: a plain copy
        if (n && d_dst != d_src &&
            cudaMemcpyAsync(d_dst, d_src, n * sizeof(double), cudaMemcpyDeviceToDevice, st) !=
                cudaSuccess)
            return DRIFT_ECUDA;
        return DRIFT_OK;
    }
    QuantOp op;
    int64_t item_len = 0;
    const int rc = make_quant_op(p, fmt, rm, d_src, d_dst, d_scale, scale, &op, &item_len);
    if (rc) return rc;
    if (launch_cast_vec(op, n, item_len, d_clamped, d_err, st))
        return cudaGetLastError() == cudaSuccess ? DRIFT_OK : DRIFT_ECUDA;
    return run_elem(ws, op, n, item_len, rm == DRIFT_STOCHASTIC, d_state, d_clamped, d_err, st);
}

// ------------------------------------------------------------------ row-wise casts
//
// `rows` tensors of `len` elements each (row r at src + r*len), every one cast
// as Quant.quantize casts one tensor, with its own per-tensor scale
// (Quant.perTensorScale of its own amax): DotSweep.run casts each vector so
// (DotSweep.java:112-122). One CTA per row: the row's amax, its scale, then
// QuantOp's element cast, clamps counted per row.
constexpr int kRowThreads = 256;

__global__ void __launch_bounds__(kRowThreads) rows_cast_kernel(QuantOp op, int64_t len,
                                                                unsigned long long *clamped,
                                                                int *d_err) {
    __shared__ double s_max[kRowThreads / 32];
    __shared__ unsigned s_cl[kRowThreads / 32];
    const int64_t base = (int64_t)blockIdx.x * len;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (op.scaling == DRIFT_PER_TENSOR) {
        double m = 0.0;  // Quant.amax: NaN never wins
        for (int64_t i = threadIdx.x; i < len; i += blockDim.x) m = fmax(m, fabs(op.src[base + i]));
        m = warp_max(m);
        if (lane == 0) s_max[warp] = m;
        __syncthreads();
        m = 0.0;
        for (int w = 0; w < kRowThreads / 32; w++) m = fmax(m, s_max[w]);
        op.scale = (m == 0.0 || !isfinite(m)) ? 1.0 : __ddiv_rn(op.f.max_finite, m);
        op.inv = __ddiv_rn(1.0, op.scale);  // Quant.java:37-42, :72
    }
    const QuantOp::Item it{1.0, 1.0, false};
    int err = 0;
    unsigned clamps = 0;
    for (int64_t i = threadIdx.x; i < len; i += blockDim.x) {
        bool clamp = false;
        op.apply(it, base + i, op.src[base + i], 0, clamp, err);
        clamps += clamp;
    }
    for (int o = 16; o > 0; o >>= 1) clamps += __shfl_xor_sync(0xffffffffu, clamps, o);
    if (lane == 0) s_cl[warp] = clamps;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long t = 0;
        for (int w = 0; w < kRowThreads / 32; w++) t += s_cl[w];
        if (clamped) clamped[blockIdx.x] += t;
    }
    if (err) atomicOr(d_err, err);
}

int launch_quantize_rows(const drift_policy *p, int fmt, int rm, const double *d_src,
                         double *d_dst, int64_t rows, int64_t len,
                         unsigned long long *d_clamped, int *d_err, cudaStream_t st) {
    if (rows < 0 || len < 0 || rows > 0x7fffffffLL) return DRIFT_EINVAL;
    if (rm == DRIFT_STOCHASTIC || p->scaling == DRIFT_MX_BLOCK) return DRIFT_EINVAL;
    if (rows == 0 || len == 0) return DRIFT_OK;
    if (fmt == DRIFT_FMT_NONE)  // Quant.java:58-61: a plain copy
        return d_dst == d_src || cudaMemcpyAsync(d_dst, d_src, rows * len * sizeof(double),
                                                 cudaMemcpyDeviceToDevice, st) == cudaSuccess
                   ? DRIFT_OK
                   : DRIFT_ECUDA;
    QuantOp op;
    int64_t item_len = 0;
    const int rc = make_quant_op(p, fmt, rm, d_src, d_dst, nullptr, 1.0, &op, &item_len);
    if (rc) return rc;
    rows_cast_kernel<<<(unsigned)rows, kRowThreads, 0, st>>>(op, len, d_clamped, d_err);
    return cudaGetLastError() == cudaSuccess ? DRIFT_OK : DRIFT_ECUDA;
}

// Sum of the per-CTA draw counts of a count pass (one CTA).
__global__ void __launch_bounds__(1024) sum_counts_kernel(const uint64_t *cta_counts,
                                                          int64_t n_ctas, uint64_t *out) {
    __shared__ uint64_t s_part[32];
    uint64_t acc = 0;
    for (int64_t i = threadIdx.x; i < n_ctas; i += blockDim.x) acc += cta_counts[i];
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint64_t t = 0;
        for (int w = 0; w < (int)(blockDim.x >> 5); w++) t += s_part[w];
        *out = t;
    }
}

int launch_quantize_draws(Workspace &ws, const drift_policy *p, int fmt, int rm,
                          const double *d_src, int64_t n, const double *d_scale, double scale,
                          uint64_t *d_draws, int *d_err, cudaStream_t st) {
    if (!d_err || !d_draws) return DRIFT_EINVAL;
    if (n < 0) return DRIFT_EINVAL;
    if (fmt == DRIFT_FMT_NONE || rm != DRIFT_STOCHASTIC || n == 0)
        return cudaMemsetAsync(d_draws, 0, sizeof(uint64_t), st) == cudaSuccess ? DRIFT_OK
                                                                               : DRIFT_ECUDA;
    QuantOp op;
    int64_t item_len = 0;
    int rc = make_quant_op(p, fmt, rm, d_src, nullptr, d_scale, scale, &op, &item_len);
    if (rc) return rc;
    const int64_t items_needed = (n + item_len - 1) / item_len;
    const int64_t grid = (items_needed + kItemsPerCta - 1) / kItemsPerCta;
    if (grid > 0x7fffffffLL) return DRIFT_EINVAL;
    const size_t items = (size_t)grid * kItemsPerCta;
    char *base = (char *)ws.get(items * sizeof(uint32_t) + (size_t)grid * sizeof(uint64_t) + 256, st);
    if (!base) return DRIFT_ENOMEM;
    SrArgs sr{nullptr, nullptr, nullptr, nullptr, nullptr};
    sr.cta_counts = (uint64_t *)base;
    sr.item_counts = (uint32_t *)(base + (size_t)grid * sizeof(uint64_t) + 256);
    sr.err = d_err;  // a NaN into a format without NaN is reported here already
    elem_kernel<QuantOp, 1><<<(unsigned)grid, kThreads, 0, st>>>(op, n, item_len, sr);
    sum_counts_kernel<<<1, 1024, 0, st>>>(sr.cta_counts, grid, d_draws);
    return cudaGetLastError() == cudaSuccess ? DRIFT_OK : DRIFT_ECUDA;
}

int launch_encode(Workspace &ws, int fmt, int rm, const double *d_v, int32_t *d_codes, int64_t n,
                  uint64_t *d_state, int *d_err, cudaStream_t st) {
    EncodeOp op;
    if (!fmt_desc(fmt, &op.f) || rm < 0 || rm > 2) return DRIFT_EINVAL;
    op.src = d_v;
    op.dst = d_codes;
    op.rm = rm;
    return run_elem(ws, op, n, 32, rm == DRIFT_STOCHASTIC, d_state, nullptr, d_err, st);
}

int launch_decode(int fmt, const int32_t *d_codes, double *d_v, int64_t n, cudaStream_t st) {
    FmtDesc f;
    if (!fmt_desc(fmt, &f)) return DRIFT_EINVAL;
    if (n <= 0) return DRIFT_OK;
    int64_t blocks = (n + 255) / 256;
    if (blocks > 148 * 32) blocks = 148 * 32;
    decode_kernel<<<(unsigned)blocks, 256, 0, st>>>(f, d_codes, d_v, n);
    return cudaGetLastError() == cudaSuccess ? DRIFT_OK : DRIFT_ECUDA;
}

int launch_acc_round(Workspace &ws, int acc, int rm, const double *d_x, double *d_y, int64_t n,
                     uint64_t *d_state, int *d_err, cudaStream_t st) {
    if ((acc != DRIFT_ACC_FP16 && acc != DRIFT_ACC_BF16) || rm < 0 || rm > 2) return DRIFT_EINVAL;
    AccRoundOp op{d_x, d_y, acc, rm};
    return run_elem(ws, op, n, 32, rm == DRIFT_STOCHASTIC, d_state, nullptr, d_err, st);
}

// ------------------------------------------------------------------ no-allocation cast
//
// A second entry to the same cast passes for callers that must not allocate
// device memory while they run. The stochastic passes need scratch (draw
// counts per item and per CTA, and the Rng state before the call); here it
// lives in one fixed array in this file instead of a growable workspace, so a
// call never allocates or frees anything. The array is a device symbol: host
// code may not use its name as an address, so on the first call on each
// device (with that device current) its device address is looked up with
// cudaGetSymbolAddress and cached.
//
// Every call on a device shares the array and it keeps the last call's
// contents; the count pass writes every entry the apply pass reads, so nothing
// needs clearing between calls. Two calls that overlap on the GPU (different
// streams, or different host threads on one device) race on it.

constexpr int64_t kNoAllocCtas = (DRIFT_NOALLOC_MAX_ITEMS + kItemsPerCta - 1) / kItemsPerCta;
constexpr size_t kNoAllocBytes =
    (size_t)kNoAllocCtas * sizeof(uint64_t) + 256 + (size_t)kNoAllocCtas * kItemsPerCta * sizeof(uint32_t);

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

static constexpr int kNoAllocMaxDevices = 64;
static void *g_noalloc_addr[kNoAllocMaxDevices];
static std::mutex g_noalloc_mutex;

// Device address of this device's copy of the scratch array (looked up once).
static int noalloc_scratch(char **out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return DRIFT_ECUDA;
    if (dev < 0 || dev >= kNoAllocMaxDevices) return DRIFT_EUNSUPPORTED;
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (!g_noalloc_addr[dev]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return DRIFT_ECUDA;
        g_noalloc_addr[dev] = p;
    }
    *out = (char *)g_noalloc_addr[dev];
    return DRIFT_OK;
}

int launch_quantize_noalloc(const drift_policy *p, int fmt, int rm, const double *d_src,
                            double *d_dst, int64_t n, const double *d_scale, double scale,
                            uint64_t *d_state, unsigned long long *d_clamped, int *d_err,
                            cudaStream_t st) {
    if (n < 0) return DRIFT_EINVAL;
    if (fmt == DRIFT_FMT_NONE) {  // Quant.java:58-61: a plain copy
        if (n && d_dst != d_src &&
            cudaMemcpyAsync(d_dst, d_src, n * sizeof(double), cudaMemcpyDeviceToDevice, st) !=
                cudaSuccess)
            return DRIFT_ECUDA;
        return DRIFT_OK;
    }
    QuantOp op;
    int64_t item_len = 0;
    int rc = make_quant_op(p, fmt, rm, d_src, d_dst, d_scale, scale, &op, &item_len);
    if (rc) return rc;
    // The array's address is looked up on the first call that casts, whatever
    // its rounding or size, so that a first call made before a stream capture
    // leaves nothing to look up inside it.
    char *base = nullptr;
    rc = noalloc_scratch(&base);
    if (rc) return rc;
    const int64_t items = (n + item_len - 1) / item_len;
    const int64_t grid = (items + kItemsPerCta - 1) / kItemsPerCta;
    if (grid > 0x7fffffffLL) return DRIFT_EINVAL;
    // Only stochastic rounding uses the array; the other casts take one pass
    // and have no size limit beyond the launch's.
    if (rm == DRIFT_STOCHASTIC && items > DRIFT_NOALLOC_MAX_ITEMS) return DRIFT_ENOMEM;
    if (n == 0) return DRIFT_OK;
    SrArgs sr{nullptr, nullptr, nullptr, d_clamped, d_err};
    if (rm != DRIFT_STOCHASTIC) {
        elem_kernel<QuantOp, 0><<<(unsigned)grid, kThreads, 0, st>>>(op, n, item_len, sr);
        return cudaGetLastError() == cudaSuccess ? DRIFT_OK : DRIFT_ECUDA;
    }
    sr.cta_counts = (uint64_t *)base;
    uint64_t *state_before = (uint64_t *)(base + (size_t)kNoAllocCtas * sizeof(uint64_t));
    sr.item_counts = (uint32_t *)(base + (size_t)kNoAllocCtas * sizeof(uint64_t) + 256);
    sr.state_before = state_before;
    elem_kernel<QuantOp, 1><<<(unsigned)grid, kThreads, 0, st>>>(op, n, item_len, sr);
    sr_scan_kernel<<<1, 1024, 0, st>>>(sr.cta_counts, grid, d_state, state_before, d_err);
    elem_kernel<QuantOp, 2><<<(unsigned)grid, kThreads, 0, st>>>(op, n, item_len, sr);
    return cudaGetLastError() == cudaSuccess ? DRIFT_OK : DRIFT_ECUDA;
}

}  // namespace drift
