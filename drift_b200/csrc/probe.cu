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
    int sms = 0, dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    double *sink = nullptr;
    if (cudaMallocAsync(&sink, 8, st) != cudaSuccess) return DRIFT_ENOMEM;
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    const int blocks = sms * 8, iters = 1 << 14;
    fp64_probe_kernel<<<blocks, 256, 0, st>>>(1.0, 256, sink);  // warm-up
    cudaEventRecord(a, st);
    fp64_probe_kernel<<<blocks, 256, 0, st>>>(1.0, iters, sink);
    cudaEventRecord(b, st);
    cudaEventSynchronize(b);
    float ms = 0.f;
    cudaEventElapsedTime(&ms, a, b);
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    cudaFreeAsync(sink, st);
    cudaStreamSynchronize(st);
    if (cudaGetLastError() != cudaSuccess) return DRIFT_ECUDA;
    *ops_per_s = (double)blocks * 256 * iters * kProbeChains * 2 / (ms * 1e-3);
    return DRIFT_OK;
}

}  // namespace drift
