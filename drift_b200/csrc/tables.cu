// tables.cu — the format tables of DumpTables, written by the device codec.
//
// DumpTables (java/src/main/java/io/drift/tools/DumpTables.java:61-124)
// writes what the formats believe so an independent exact-rational
// verification can recompute it: the value of every code, and the nearest-even code of
// the product and of the sum of code pairs, every ordered pair for formats
// up to 8 bits and a fixed Rng sample for the 16-bit ones. These kernels
// produce the same rows from the same device encode/decode the casts use, so
// that verification covers the engine's codec directly.
#include "codec.cuh"
#include "internal.h"

namespace drift {

// values_<fmt>.csv (DumpTables.java:61-79): the raw bits of decode(c).
__global__ void value_table_kernel(FmtDesc f, int64_t codes, uint64_t *bits) {
    for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < codes;
         c += (int64_t)gridDim.x * blockDim.x)
        bits[c] = dbits(decode_value(f, (int)c));
}

// pairs_<fmt>.csv rows first .. first+n-1. Exhaustive: row p is the pair
// (p / codes, p % codes), the nested loops of DumpTables.java:91-98.
// Sampled: row p takes the Rng draws 2p and 2p+1 of a stream seeded `seed`,
// each mapped to (int)((nextLong() >>> 1) % codes) (:110-113). The product
// and the sum of two representable values are exact in double for widths up
// to 26 bits (:117-123), so the encode is the only rounding, as in Java.
__global__ void pair_table_kernel(FmtDesc f, int64_t codes, int mode, uint64_t seed, int64_t first,
                                  int64_t n, int32_t *a_out, int32_t *b_out, int32_t *prod,
                                  int32_t *sum) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t p = first + i;
        int a, b;
        if (mode == DRIFT_PAIRS_EXHAUSTIVE) {
            a = (int)(p / codes);
            b = (int)(p % codes);
        } else {
            const uint64_t ua = splitmix_mix(seed + (uint64_t)(2 * p + 1) * kGolden);
            const uint64_t ub = splitmix_mix(seed + (uint64_t)(2 * p + 2) * kGolden);
            a = (int)((ua >> 1) % (uint64_t)codes);
            b = (int)((ub >> 1) % (uint64_t)codes);
        }
        const double av = decode_value(f, a);
        const double bv = decode_value(f, b);
        bool drew;
        int err = 0;
        if (a_out) a_out[i] = a;
        if (b_out) b_out[i] = b;
        prod[i] = encode_value(f, __dmul_rn(av, bv), DRIFT_NEAREST_EVEN, 0, drew, err);
        sum[i] = encode_value(f, __dadd_rn(av, bv), DRIFT_NEAREST_EVEN, 0, drew, err);
    }
}

static unsigned grid_for(int64_t n) {
    int64_t blocks = (n + 255) / 256;
    return (unsigned)(blocks < 148 * 16 ? (blocks > 0 ? blocks : 1) : 148 * 16);
}

int launch_value_table(int fmt, uint64_t *d_bits, cudaStream_t st) {
    FmtDesc f;
    if (!fmt_desc(fmt, &f)) return DRIFT_EINVAL;
    const int64_t codes = (int64_t)f.code_mask + 1;
    value_table_kernel<<<grid_for(codes), 256, 0, st>>>(f, codes, d_bits);
    return cudaGetLastError() == cudaSuccess ? DRIFT_OK : DRIFT_ECUDA;
}

int launch_pair_table(int fmt, int mode, uint64_t seed, int64_t first, int64_t n, int32_t *d_a,
                      int32_t *d_b, int32_t *d_prod, int32_t *d_sum, cudaStream_t st) {
    FmtDesc f;
    if (!fmt_desc(fmt, &f)) return DRIFT_EINVAL;
    const int64_t codes = (int64_t)f.code_mask + 1;
    if (mode != DRIFT_PAIRS_EXHAUSTIVE && mode != DRIFT_PAIRS_SAMPLED) return DRIFT_EINVAL;
    if (first < 0 || n < 0) return DRIFT_EINVAL;
    if (mode == DRIFT_PAIRS_EXHAUSTIVE && (first > codes * codes || n > codes * codes - first))
        return DRIFT_EINVAL;
    if (mode == DRIFT_PAIRS_SAMPLED && (first > ((int64_t)1 << 61) || n > ((int64_t)1 << 61)))
        return DRIFT_EINVAL;
    if (n == 0) return DRIFT_OK;
    pair_table_kernel<<<grid_for(n), 256, 0, st>>>(f, codes, mode, seed, first, n, d_a, d_b,
                                                   d_prod, d_sum);
    return cudaGetLastError() == cudaSuccess ? DRIFT_OK : DRIFT_ECUDA;
}

}  // namespace drift
