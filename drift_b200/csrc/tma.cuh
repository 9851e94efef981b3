// tma.cuh — Tensor Memory Accelerator staging shared by the tiled contractions:
// shared-memory mbarriers with bounded waits, one 2-D tiled bulk copy per
// operand tile, and the driver's tensor-map encoder found through the runtime.
#pragma once

#include <cstdint>

#include <cuda.h>
#include <cuda_runtime.h>

namespace drift {

constexpr long long kWaitLimit = 1LL << 22;  // try_wait rounds before giving up

__device__ __forceinline__ unsigned smem_addr(const void *p) {
    return (unsigned)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

// Bounded wait for the barrier's phase `parity` to complete; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, unsigned parity) {
    const unsigned a = smem_addr(bar);
    for (long long i = 0; i < kWaitLimit; i++) {
        unsigned done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
            " selp.u32 %0, 1, 0, p;\n}"
            : "=r"(done)
            : "r"(a), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}

// One box of a 2-D tensor map, starting at element (x, y), into shared memory;
// completion is counted on `bar`. x times the element size must be a multiple
// of 16 bytes, which every caller guarantees by starting boxes on tile edges.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

// cuTensorMapEncodeTiled, found through the runtime (no libcuda link).
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn lookup_encode_tiled() {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
        return reinterpret_cast<EncodeTiledFn>(p);
    return nullptr;
}

// Host threads with their own contexts make their first contraction at the
// same time; a function-local static is initialised exactly once (C++11),
// and the others wait for it, so the lookup needs no lock of its own.
inline EncodeTiledFn encode_tiled() {
    static const EncodeTiledFn fn = lookup_encode_tiled();
    return fn;
}

}  // namespace drift
