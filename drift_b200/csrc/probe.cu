// probe.cu — measured denominators for the contraction rooflines.
//
// Every emulated multiply-accumulate of the double-precision contraction costs
// at least one DMUL and one DADD on the FP64 pipe (the product and the sum are
// rounded to double separately). fp64_probe_kernel issues nothing but
// independent DMUL/DADD pairs, so its rate is the FP64 pipe's peak on this
// part, the ceiling that contraction is held to. The FP32-pipe contraction
// (gemm32.cu) costs one FFMA per multiply-accumulate; fp32_probe_kernel issues
// nothing but independent FFMAs for its ceiling.
#include "common.cuh"
#include "internal.h"

namespace drift {

constexpr int kProbeChains = 8;

__global__ void __launch_bounds__(256) fp64_probe_kernel(double seed, int iters, double *sink) {
    double x[kProbeChains], y[kProbeChains];
#pragma unroll
    for (int c = 0; c < kProbeChains; c++) {
        x[c] = seed + threadIdx.x * 1e-9 + c;
        y[c] = 1.0 + c * 1e-12;
    }
    for (int i = 0; i < iters; i++) {
#pragma unroll
        for (int c = 0; c < kProbeChains; c++) {
            x[c] = __dadd_rn(__dmul_rn(x[c], y[c]), 1e-300);  // one DMUL + one DADD
        }
    }
    double s = 0.0;
#pragma unroll
    for (int c = 0; c < kProbeChains; c++) s += x[c];
    if (s == 12345.678) *sink = s;  // keeps the chains live
}

constexpr int kFmaChains = 16;

__global__ void __launch_bounds__(256) fp32_probe_kernel(float seed, int iters, float *sink) {
    float x[kFmaChains];
#pragma unroll
    for (int c = 0; c < kFmaChains; c++) x[c] = seed + threadIdx.x * 1e-6f + c;
    for (int i = 0; i < iters; i++) {
#pragma unroll
        for (int c = 0; c < kFmaChains; c++) x[c] = __fmaf_rn(x[c], 0.999999f, 1e-7f);
    }
    float s = 0.0f;
#pragma unroll
    for (int c = 0; c < kFmaChains; c++) s += x[c];
    if (s == 12345.678f) *sink = s;  // keeps the chains live
}

// Times `launch(iters)` (after a short warm-up launch) on `st`; ms of the timed launch.
template <class Launch>
static int time_probe(cudaStream_t st, int iters, Launch launch, float *ms) {
    cudaEvent_t a = nullptr, b = nullptr;
    bool ok = cudaEventCreate(&a) == cudaSuccess && cudaEventCreate(&b) == cudaSuccess;
    if (ok) {
        launch(256);  // warm-up
        ok = cudaEventRecord(a, st) == cudaSuccess;
        launch(iters);
        ok = ok && cudaEventRecord(b, st) == cudaSuccess && cudaEventSynchronize(b) == cudaSuccess &&
             cudaEventElapsedTime(ms, a, b) == cudaSuccess && *ms > 0.f;
    }
    if (a) cudaEventDestroy(a);
    if (b) cudaEventDestroy(b);
    return ok ? DRIFT_OK : DRIFT_ECUDA;
}

int launch_fp64_probe(cudaStream_t st, double *ops_per_s) {
    const int blocks = sm_count() * 8, iters = 1 << 14;
    double *sink = nullptr;
    if (cudaMallocAsync(&sink, 8, st) != cudaSuccess) return DRIFT_ENOMEM;
    float ms = 0.f;
    int rc = time_probe(st, iters, [&](int n) {
        fp64_probe_kernel<<<blocks, 256, 0, st>>>(1.0, n, sink);
    }, &ms);
    cudaFreeAsync(sink, st);
    if (cudaStreamSynchronize(st) != cudaSuccess || cudaGetLastError() != cudaSuccess) rc = DRIFT_ECUDA;
    if (rc) return rc;
    *ops_per_s = (double)blocks * 256 * iters * kProbeChains * 2 / (ms * 1e-3);
    return DRIFT_OK;
}

int launch_fp32_probe(cudaStream_t st, double *fma_per_s) {
    const int blocks = sm_count() * 8, iters = 1 << 15;
    float *sink = nullptr;
    if (cudaMallocAsync(&sink, 8, st) != cudaSuccess) return DRIFT_ENOMEM;
    float ms = 0.f;
    int rc = time_probe(st, iters, [&](int n) {
        fp32_probe_kernel<<<blocks, 256, 0, st>>>(1.0f, n, sink);
    }, &ms);
    cudaFreeAsync(sink, st);
    if (cudaStreamSynchronize(st) != cudaSuccess || cudaGetLastError() != cudaSuccess) rc = DRIFT_ECUDA;
    if (rc) return rc;
    *fma_per_s = (double)blocks * 256 * iters * kFmaChains / (ms * 1e-3);
    return DRIFT_OK;
}

}  // namespace drift
