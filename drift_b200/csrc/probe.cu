// probe.cu — measured denominators for the contraction roofline.
//
// Every emulated multiply-accumulate costs at least one DMUL and one DADD on
// the FP64 pipe (the product and the sum are rounded to double separately).
// This kernel issues nothing but independent DMUL/DADD pairs, so its rate is
// the FP64 pipe's peak on this part, the ceiling the contraction is held to.
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

int launch_fp64_probe(cudaStream_t st, double *ops_per_s) {
    const int blocks = sm_count() * 8, iters = 1 << 14;
    double *sink = nullptr;
    if (cudaMallocAsync(&sink, 8, st) != cudaSuccess) return DRIFT_ENOMEM;
    cudaEvent_t a = nullptr, b = nullptr;
    bool ok = cudaEventCreate(&a) == cudaSuccess && cudaEventCreate(&b) == cudaSuccess;
    float ms = 0.f;
    if (ok) {
        fp64_probe_kernel<<<blocks, 256, 0, st>>>(1.0, 256, sink);  // warm-up
        ok = cudaEventRecord(a, st) == cudaSuccess;
        fp64_probe_kernel<<<blocks, 256, 0, st>>>(1.0, iters, sink);
        ok = ok && cudaEventRecord(b, st) == cudaSuccess && cudaEventSynchronize(b) == cudaSuccess &&
             cudaEventElapsedTime(&ms, a, b) == cudaSuccess && ms > 0.f;
    }
    if (a) cudaEventDestroy(a);
    if (b) cudaEventDestroy(b);
    cudaFreeAsync(sink, st);
    ok = cudaStreamSynchronize(st) == cudaSuccess && ok;
    if (!ok || cudaGetLastError() != cudaSuccess) return DRIFT_ECUDA;
    *ops_per_s = (double)blocks * 256 * iters * kProbeChains * 2 / (ms * 1e-3);
    return DRIFT_OK;
}

}  // namespace drift
