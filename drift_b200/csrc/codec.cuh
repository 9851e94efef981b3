// codec.cuh — device minifloat codec and accumulator rounding.
//
// Bit-exact device forms of MiniFloat.encode/decode
// (java/src/main/java/io/drift/fmt/MiniFloat.java:117-211) and Dot.round
// (java/src/main/java/io/drift/kernel/Dot.java:141-182). Stochastic rounding
// is split in two so a kernel can first learn whether an element needs a
// random draw, then fetch exactly that draw from the counter-based stream.
#pragma once

#include "common.cuh"

namespace drift {

// Rounds the exact, non-negative `scaled` to an integer under `rm`
// (MiniFloat.roundToIntegral, MiniFloat.java:258-278). For STOCHASTIC, `drew`
// reports whether the fraction was non-zero, i.e. whether Java would have
// consumed a draw; u53 holds that draw's 53 random bits.
__device__ __forceinline__ double round_integral(double scaled, int rm, uint64_t u53,
                                                 bool &drew) {
    if (rm == DRIFT_NEAREST_EVEN) return rint(scaled);
    double fl = floor(scaled);
    if (rm == DRIFT_TRUNCATE) return fl;
    double frac = __dsub_rn(scaled, fl);  // exact
    if (frac == 0.0) return fl;
    drew = true;
    return __dmul_rn((double)u53, 0x1p-53) < frac ? fl + 1.0 : fl;
}

// MiniFloat.encode(v, rm, rng) (MiniFloat.java:156-211). Sets `drew` when a
// stochastic draw was used, ORs DEV_ERR_NAN_FINITE into `err` for a NaN cast
// into a format without NaN.
__device__ __forceinline__ int encode_value(const FmtDesc &f, double v, int rm, uint64_t u53,
                                            bool &drew, int &err) {
    drew = false;
    if (isnan(v)) {
        if (f.specials == SP_FINITE) {
            err |= DEV_ERR_NAN_FINITE;
            return 0;
        }
        return f.nan_bits;
    }
    const int sign = (dbits(v) >> 63) ? f.sign_bit : 0;
    const double a = fabs(v);
    if (a == 0.0) return sign;
    if (isinf(a)) return sign | f.max_finite_bits;

    int e = java_get_exponent(a);
    if (e < f.min_normal_exp) e = f.min_normal_exp;  // also catches -1023
    // scalb(a, -(e - mant)): a multiply by an exact power of two whose result
    // lies in [0, 2^(mant+1)), so it is exact.
    const double scaled = __dmul_rn(a, pow2(f.mant_bits - e));
    long long m = (long long)round_integral(scaled, rm, u53, drew);

    const long long normal_base = 1LL << f.mant_bits;
    if (m < normal_base) return sign | (int)m;
    if (m >= (normal_base << 1)) {
        m >>= 1;
        e += 1;
    }
    const int exp_field = e + f.bias;
    const int mant_field = (int)(m - normal_base);
    bool overflow = exp_field > f.max_exp_field;
    if (exp_field == f.max_exp_field) {
        // MiniFloat.topBinadeAllows (MiniFloat.java:223-229).
        if (f.specials == SP_IEEE) overflow = true;
        else if (f.specials == SP_FN && mant_field >= f.mant_mask) overflow = true;
    }
    if (overflow) return sign | f.max_finite_bits;
    return sign | (exp_field << f.mant_bits) | mant_field;
}

// MiniFloat.decode(bits) (MiniFloat.java:117-142). Every value is an integer
// times an exact power of two, so it is built without rounding.
__device__ __forceinline__ double decode_value(const FmtDesc &f, int bits) {
    const int exp_field = (bits & f.exp_mask) >> f.mant_bits;
    const int mant = bits & f.mant_mask;
    const bool neg = (bits & f.sign_bit) != 0;
    if (exp_field == f.max_exp_field) {
        if (f.specials == SP_IEEE) {
            if (mant != 0) return bitsd(kJavaNaNBits);
            return neg ? -bitsd(0x7ff0000000000000ULL) : bitsd(0x7ff0000000000000ULL);
        }
        if (f.specials == SP_FN && mant == f.mant_mask) return bitsd(kJavaNaNBits);
    }
    double mag;
    if (exp_field == 0) {
        mag = __dmul_rn((double)mant, pow2(f.min_normal_exp - f.mant_bits));
    } else {
        mag = __dmul_rn((double)((1 << f.mant_bits) + mant),
                        pow2(exp_field - f.bias - f.mant_bits));
    }
    return neg ? -mag : mag;
}

// Accumulator format constants of Dot.round (Dot.java:125-131).
template <int ACC> struct AccFmt;
template <> struct AccFmt<DRIFT_ACC_FP16> {
    static constexpr int mant = 10;
    static constexpr int min_exp = -14;
    static constexpr int max_exp = 15;
    __device__ static double max() { return 65504.0; }
};
template <> struct AccFmt<DRIFT_ACC_BF16> {
    static constexpr int mant = 7;
    static constexpr int min_exp = -126;
    static constexpr int max_exp = 127;
    __device__ static double max() { return 0x1.FEp127; }  // 255 * 2^120
};

// Dot.round(x, acc, rm, rng), the general form (Dot.java:141-182). The
// contraction kernel reaches it only when its integer fast path cannot
// decide (zero, subnormal range, saturation, Inf/NaN).
template <int ACC>
__device__ __noinline__ double acc_round_general(double x, int rm, uint64_t u53, bool &drew) {
    using F = AccFmt<ACC>;
    drew = false;
    if (x == 0.0 || isnan(x)) return x;
    const double ax = fabs(x);
    if (isinf(ax)) return copysign(F::max(), x);
    int e = java_get_exponent(ax);
    if (e < F::min_exp) e = F::min_exp;
    const int q = e - F::mant;
    const double scaled = __dmul_rn(ax, pow2(-q));  // exact
    const double m = round_integral(scaled, rm, u53, drew);
    double r = q >= -1022 ? __dmul_rn(m, pow2(q)) : m * 0.0;  // q >= -133 always
    if (r > F::max()) r = F::max();
    return copysign(r, x);
}

// Runtime-dispatched Dot.round for the element-wise kernel.
__device__ __forceinline__ double acc_round_any(int acc, double x, int rm, uint64_t u53,
                                                bool &drew) {
    return acc == DRIFT_ACC_FP16 ? acc_round_general<DRIFT_ACC_FP16>(x, rm, u53, drew)
                                 : acc_round_general<DRIFT_ACC_BF16>(x, rm, u53, drew);
}

// ------------------------------------------------------- fast accumulator rounding
//
// The contraction rounds once per multiply-accumulate, so it rounds on the
// double's bit pattern: for a result that stays a normal number of the target
// format, rounding to p significant bits is an integer add of (half-ulp - 1 +
// lsb) followed by clearing the low bits; a carry out of the mantissa bumps
// the exponent, which is the correct round-up. The result's exponent is then
// range-checked in two integer ops; anything outside (zero, a subnormal of the
// target format, overflow, Inf, NaN) is recomputed by the general path.
// A value below the normal range that the fine rounding lifts to exactly the
// smallest normal is also right: the coarser subnormal quantum rounds it there
// too, so the check on the result alone suffices.

// (float) of a double, returned as the double holding that float
// (Dot.java:54, :61, :99, :118): round to nearest even at 24 bits.
__device__ __forceinline__ double round_to_f32(double t) {
    const uint64_t u = dbits(t);
    const uint64_t r = (u + 0x0FFFFFFFULL + ((u >> 29) & 1ULL)) & ~0x1FFFFFFFULL;
    const uint32_t hi2 = (uint32_t)(r >> 32) << 1;  // exponent in bits 21..31
    if (hi2 - (897u << 21) < (254u << 21)) return bitsd(r);
    return (double)__double2float_rn(t);
}

// Dot.round for FP16/BF16 with NEAREST_EVEN or TRUNCATE.
template <int ACC, int RM>
__device__ __forceinline__ double round_acc_fast(double t) {
    using F = AccFmt<ACC>;
    constexpr int P = 52 - F::mant;  // bits below the kept significand
    constexpr uint64_t low = (1ULL << P) - 1;
    const uint64_t u = dbits(t);
    uint64_t r;
    if (RM == DRIFT_NEAREST_EVEN) {
        r = (u + (low >> 1) + ((u >> P) & 1ULL)) & ~low;
    } else {
        r = u & ~low;
    }
    constexpr uint32_t lo_e = (uint32_t)(1023 + F::min_exp) << 21;
    constexpr uint32_t span = (uint32_t)(F::max_exp - F::min_exp + 1) << 21;
    const uint32_t hi2 = (uint32_t)(r >> 32) << 1;
    if (hi2 - lo_e < span) return bitsd(r);
    bool drew;
    return acc_round_general<ACC>(t, RM, 0, drew);
}

}  // namespace drift
