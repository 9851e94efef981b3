// common.cuh — shared definitions of the B200 emulated-matmul engine.
//
// Formats, Java-exact helpers (Math.getExponent, exact powers of two) and the
// counter form of splitmix64 that lets every element find its own random draw.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/drift_b200.h"

namespace drift {

// What the all-ones exponent means (MiniFloat.Specials,
// java/src/main/java/io/drift/fmt/MiniFloat.java:22-33).
enum Specials : int { SP_IEEE = 0, SP_FN = 1, SP_FINITE = 2 };

// A minifloat format as the kernels need it: every derived constant of the
// MiniFloat constructor (MiniFloat.java:70-107) precomputed on the host.
struct FmtDesc {
    int mant_bits;
    int bias;
    int specials;
    int max_exp_field;
    int mant_mask;
    int exp_mask;
    int sign_bit;
    int code_mask;
    int min_normal_exp;
    int nan_bits;         // MiniFloat.nanBits (:231-237); unused for FINITE
    int max_finite_bits;  // MiniFloat.maxFiniteBits (:250-256) == overflowBits
    int emax;             // Math.getExponent(maxFinite), the MX emax_elem
    double max_finite;
};

// Host: descriptor of format `id` (Formats.java:20-45). Returns false for a
// bad id.
bool fmt_desc(int id, FmtDesc *out);

// Java's canonical NaN (Double.NaN), 0x7ff8000000000000.
constexpr uint64_t kJavaNaNBits = 0x7ff8000000000000ULL;
constexpr uint64_t kGolden = 0x9E3779B97F4A7C15ULL;

__host__ __device__ inline uint64_t dbits(double d) {
#ifdef __CUDA_ARCH__
    return (uint64_t)__double_as_longlong(d);
#else
    uint64_t b;
    __builtin_memcpy(&b, &d, 8);
    return b;
#endif
}

__host__ __device__ inline double bitsd(uint64_t b) {
#ifdef __CUDA_ARCH__
    return __longlong_as_double((long long)b);
#else
    double d;
    __builtin_memcpy(&d, &b, 8);
    return d;
#endif
}

// Math.getExponent(double): unbiased exponent field; -1023 for zero and
// subnormals, 1024 for Inf and NaN.
__host__ __device__ inline int java_get_exponent(double d) {
    return (int)((dbits(d) >> 52) & 0x7FF) - 1023;
}

// Exactly 2^k as a double, for -1074 <= k <= 1023 (subnormal powers included).
__host__ __device__ inline double pow2(int k) {
    if (k >= -1022) return bitsd((uint64_t)(k + 1023) << 52);
    return bitsd(1ULL << (k + 1074));
}

// splitmix64's output for one counter value: the k-th Rng.nextLong() of a
// stream whose state is s is mix(s + (k+1)*golden)
// (java/src/main/java/io/drift/fmt/Rng.java:17-22).
__host__ __device__ inline uint64_t splitmix_mix(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

// The 53 random bits of the k-th Rng.nextDouble() (Rng.java:25-27) after
// state s; nextDouble() == u53 * 2^-53 exactly.
__host__ __device__ inline uint64_t draw_u53(uint64_t state, uint64_t k) {
    return splitmix_mix(state + (k + 1) * kGolden) >> 11;
}

// Device error flags, OR-ed into a context word and read by drift_check_dev.
enum DevErr : int {
    DEV_ERR_NAN_FINITE = 1,
    DEV_ERR_NO_RNG = 2,
    DEV_ERR_TIMEOUT = 4,
    DEV_ERR_INDEX = 8,  // a token outside the embedding table
};

}  // namespace drift
