// stats.cu — error statistics of an emulated GEMM against its exact twin.
//
// RealDotSweep reports, per policy, the RMS of (got - exact) over the RMS of
// exact (java/src/main/java/io/drift/tools/RealDotSweep.java:245-257, :264-270).
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
    int sms = 148, dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    int64_t blocks = (n + 255) / 256;
    if (blocks > sms * 8) blocks = sms * 8;
    error_sums_kernel<<<(unsigned)blocks, 256, 0, st>>>(got, exact, n, sums);
    return cudaGetLastError() == cudaSuccess ? DRIFT_OK : DRIFT_ECUDA;
}

}  // namespace drift
