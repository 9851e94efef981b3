// codec.cuh — device minifloat codec and accumulator rounding.
//
// Bit-exact device forms of MiniFloat.encode/decode
// (java/src/main/java/io/drift/fmt/MiniFloat.java:117-211) and Dot.round
// (java/src/main/java/io/drift/kernel/Dot.java:141-182). Stochastic rounding
// is split in two so a kernel can first learn whether an element needs a
// random draw, then fetch exactly that draw from the counter-based stream.
#pragma once

#include <cuda_bf16.h>

#include "common.cuh"

namespace drift {

// Integer parts of a non-negative x < 2^52 on the FP64 pipe: with 2^52 added,
// the unit in the last place is 1, so the add itself rounds x to an integer
// (to nearest even, or toward zero), and subtracting 2^52 again is exact.
__device__ __forceinline__ double rint_small(double x) {
    return __dsub_rn(__dadd_rn(x, 0x1p52), 0x1p52);
}
__device__ __forceinline__ double floor_small(double x) {
    return __dsub_rn(__dadd_rz(x, 0x1p52), 0x1p52);
}

// A draw's 53 random bits as a double, exactly: the low 52 bits under the
// exponent of 2^52, less 2^52, plus the top bit's 2^52 (no integer
// conversion instruction).
__device__ __forceinline__ double u53_to_double(uint64_t u) {
    const double lo = __dsub_rn(
        __longlong_as_double((long long)(0x4330000000000000ULL | (u & 0xFFFFFFFFFFFFFULL))),
        0x1p52);
    return (u >> 52) ? __dadd_rn(lo, 0x1p52) : lo;
}

// Rounds the exact, non-negative `scaled` to an integer under `rm`
// (MiniFloat.roundToIntegral, MiniFloat.java:258-278). For STOCHASTIC, `drew`
// reports whether the fraction was non-zero, i.e. whether Java would have
// consumed a draw; u53 holds that draw's 53 random bits.
__device__ __forceinline__ double round_integral(double scaled, int rm, uint64_t u53,
                                                 bool &drew) {
    // `scaled` is below 2^(mant+1) <= 2^11 for every format.
    if (rm == DRIFT_NEAREST_EVEN) return rint_small(scaled);
    double fl = floor_small(scaled);
    if (rm == DRIFT_TRUNCATE) return fl;
    double frac = __dsub_rn(scaled, fl);  // exact
    if (frac == 0.0) return fl;
    drew = true;
    return __dmul_rn(u53_to_double(u53), 0x1p-53) < frac ? fl + 1.0 : fl;
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

// 2^k for -1022 <= k <= 1023, without a branch.
__device__ __forceinline__ double pow2_normal(int k) {
    return __longlong_as_double((long long)(k + 1023) << 52);
}

// decode(encode(s, rm, rng)), the value a cast writes (MiniFloat.java:156-221
// through Quant.java:56-123), computed on the value instead of the code. With
// e = max(getExponent(|s|), minNormalExp), the significand m = round(|s| *
// 2^(mant - e)) and the value m * 2^(e - mant) cover the normal and subnormal
// codes alike, and a carry into the next binade (m = 2^(mant+1)) is the same
// value as its code. Every format saturates, and its overflow rule
// (MiniFloat.java:197-205, :223-229) keeps exactly the values up to
// maxFinite, so overflow is one min. Infinity keeps e at 1023 and rounds to
// infinity, which the min turns into maxFinite, as encode does; it and NaN
// take no draw, zero takes none either (its fraction is 0). NaN gives Java's
// NaN, or, for a format without NaN, sets DEV_ERR_NAN_FINITE and gives +0.0
// (the decode of the code 0 that encode's caller then sees). Same drew/u53
// contract as round_integral.
__device__ __forceinline__ double quantize_value(const FmtDesc &f, double s, int rm, uint64_t u53,
                                                 bool &drew, int &err) {
    drew = false;
    const double a = fabs(s);
    const int e = min(max(java_get_exponent(a), f.min_normal_exp), 1023);
    const double sc = __dmul_rn(a, pow2_normal(f.mant_bits - e));  // exact, < 2^(mant+1)
    double m;
    if (rm == DRIFT_NEAREST_EVEN) {
        m = rint_small(sc);
    } else {
        m = floor_small(sc);
        if (rm == DRIFT_STOCHASTIC) {
            const double frac = __dsub_rn(sc, m);  // exact
            drew = frac != 0.0 && a < __longlong_as_double(0x7ff0000000000000LL);
            if (drew && __dmul_rn(u53_to_double(u53), 0x1p-53) < frac) m = __dadd_rn(m, 1.0);
        }
    }
    const double q = copysign(fmin(__dmul_rn(m, pow2_normal(e - f.mant_bits)), f.max_finite), s);
    if (isnan(s)) {
        if (f.specials == SP_FINITE) {
            err |= DEV_ERR_NAN_FINITE;
            return 0.0;
        }
        return bitsd(kJavaNaNBits);
    }
    return q;
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
// contraction kernel reaches it only when its fast path cannot decide (zero,
// subnormal range, saturation, Inf/NaN).
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
    double r = __dmul_rn(m, pow2(q));  // exact below the top binade; q >= -133
    if (r > F::max()) r = F::max();
    return copysign(r, x);
}

// Runtime-dispatched Dot.round for the element-wise kernel.
__device__ __forceinline__ double acc_round_any(int acc, double x, int rm, uint64_t u53,
                                                bool &drew) {
    return acc == DRIFT_ACC_FP16 ? acc_round_general<DRIFT_ACC_FP16>(x, rm, u53, drew)
                                 : acc_round_general<DRIFT_ACC_BF16>(x, rm, u53, drew);
}

// ------------------------------------------------------- magic-constant rounding
//
// For a sum t whose rounded value is a normal number of the accumulator
// format, rounding to nearest even at a fixed number of significand bits is
// (t + C) - C with C = 1.5 * 2^(e + SHIFT), e the binade of t and SHIFT = 52 -
// kept fraction bits: the ulp of C is exactly the target quantum, C is an
// even multiple of it (so ties go to even), and the subtraction is exact.
// Truncation clears the low bits. The exact FP16/BF16 rounding uses these for
// its normal range (narrow_exact); the contraction's fast form below builds
// the same constant more cheaply.

template <int SHIFT>
__device__ __forceinline__ double rne_shift(double t) {
    const int hi = __double2hiint(t);
    const int chi = ((hi & 0x7FF00000) | 0x00080000) + (SHIFT << 20);
    const double c = __hiloint2double(chi, 0);
    return __dsub_rn(__dadd_rn(t, c), c);
}

template <int SHIFT>
__device__ __forceinline__ double trunc_shift(double t) {
    if constexpr (SHIFT >= 32) {
        return __hiloint2double(__double2hiint(t) & ~((1 << (SHIFT - 32)) - 1), 0);
    } else {
        return __hiloint2double(__double2hiint(t), __double2loint(t) & ~((1 << SHIFT) - 1));
    }
}

// ------------------------------------------------- fast rounding (FastForm)
//
// Every contraction rounds every sum, so this form is the cheapest in issued
// instructions: one LOP3, two FP64-pipe ops, and a range word per sum that
// the caller folds into one word per group (a 3-input max takes two sums at
// a time) and checks once. The tiled kernel checks groups of a thread's
// outputs; the one-output-per-thread kernels check eight steps of a chain, or
// each step.
//
// With e the binade of t and D = 1.5 * 2^e, C = D * 2^SHIFT is the magic
// constant of rne_shift, and fma(D, 2^SHIFT, t) = RN(t + C); fma(D, -2^SHIFT,
// r1) = r1 - C is exact. D's high word is t's with the sign cleared and the
// fraction's top bit set (one LOP3). Its low word is reused from the
// previous accumulator value instead of being zeroed: every value an FP16 or
// BF16 accumulator holds has a zero low word (at most 11 significant bits),
// and every float has its low 29 bits zero, so the low word is 0 or a
// multiple of 2^29. C then stays an even multiple of the target quantum
// (C / q = 1.5 * 2^52 + lo, lo a multiple of 2^29), so ties still go to even,
// and C + t stays in C's binade for SHIFT >= 3.
//
// Validation looks at t's binade, not the rounded value's: the range word
// dh - ((LO_E << 20) | 2^19), read unsigned, is (E - LO_E) << 20 for a biased
// exponent E >= LO_E and wraps far above the limit below it (zero and the
// subnormal range), so one running max over a group checks both ends. HI_E
// stops one binade below the accumulator's top one, where a sum can round up
// past the largest finite value (Inf for FP32, saturation for FP16/BF16);
// those sums, and Inf/NaN (E = 2047), take the exact path.
//
// Measured at 8192^3 on one B200 against the earlier form (rne_shift and two
// float compares of the rounded value): +8% sequential, +10% pairwise and
// blocked. Folding with an add-then-max per sum, or a separate 3-input min
// and max of the unshifted words, or two float compares of the range word,
// each measured slower than this.
template <int SHIFT, int LO_E, int HI_E>
struct FastForm {
    static constexpr unsigned kBase = ((unsigned)LO_E << 20) | 0x00080000u;
    static constexpr unsigned kLimit = (unsigned)(HI_E - LO_E) << 20;
    static constexpr double kScale = (double)(1ULL << SHIFT);

    __device__ static __forceinline__ unsigned exp_word(double t) {
        return ((unsigned)__double2hiint(t) & 0x7FF00000u) | 0x00080000u;
    }
    // Round to nearest even at the accumulator's precision; `range` gets t's
    // range word.
    __device__ static __forceinline__ double rne(double t, int prev_lo, unsigned &range) {
        const unsigned dh = exp_word(t);
        range = dh - kBase;
        const double d = __hiloint2double((int)dh, prev_lo);
        return __fma_rn(d, -kScale, __fma_rn(d, kScale, t));
    }
    // Round toward zero (SHIFT >= 32: only the high word holds kept bits, and
    // the low word of the result is zero). The low word is written as a
    // constant rather than carried over from the accumulator register: with
    // the carried form, a blocked contraction on the schedule-driven path
    // returned sums that differ from Dot.round's on B200.
    __device__ static __forceinline__ double trunc(double t, int, unsigned &range) {
        range = exp_word(t) - kBase;
        return __hiloint2double(__double2hiint(t) & ~((1 << (SHIFT - 32)) - 1), 0);
    }
    // Round to nearest even on the integer pipes: add half a quantum less one
    // plus the kept part's lowest bit to t's bit pattern, then clear the
    // dropped bits (a carry out of the significand moves t into the next
    // binade, as rounding up should). Exact on the same range as rne. It
    // takes no FP64 instruction, so a contraction that rounds some of its
    // sums this way and the rest with rne keeps both pipes busy.
    __device__ static __forceinline__ double rne_int(double t, unsigned &range) {
        range = exp_word(t) - kBase;
        unsigned long long u = (unsigned long long)__double_as_longlong(t);
        u += ((1ULL << (SHIFT - 1)) - 1) + ((u >> SHIFT) & 1ULL);
        return __longlong_as_double((long long)(u & ~((1ULL << SHIFT) - 1)));
    }
    // Folds two range words into a group's running max.
    __device__ static __forceinline__ unsigned fold2(unsigned run, unsigned r0, unsigned r1) {
        return __vimax3_u32(run, r0, r1);
    }
    __device__ static __forceinline__ bool valid(unsigned run) { return run <= kLimit; }
};

// Per-accumulator rounding (Dot.java:54, :63 and Dot.round, :141-182):
//   step(t, prev_lo, r)    the fast form above (prev_lo: the low word of the
//                          accumulator value this sum replaces, or 0; r gets
//                          the sum's range word);
//   step_int(t, r)         the same rounding on the integer pipes;
//   fold2(run, r0, r1)     folds two range words into a group's word;
//   valid(run)             whether every step folded into run was exact;
//   exact(t)               any input.
template <int ACC, int RM> struct AccRound;

template <int RM> struct AccRound<DRIFT_ACC_FP64, RM> {
    __device__ static double step(double t, int, unsigned &) { return t; }
    __device__ static double step_int(double t, unsigned &) { return t; }
    __device__ static unsigned fold2(unsigned run, unsigned, unsigned) { return run; }
    __device__ static bool valid(unsigned) { return true; }
    __device__ static double exact(double t) { return t; }
};

// (float) of a double, held as the double of that float.
template <int RM> struct AccRound<DRIFT_ACC_FP32, RM> {
    using Fast = FastForm<29, 1023 - 126, 1023 + 126>;
    __device__ static double step(double t, int prev_lo, unsigned &run) {
        return Fast::rne(t, prev_lo, run);
    }
    __device__ static double step_int(double t, unsigned &run) { return Fast::rne_int(t, run); }
    // On the conversion pipe: cvt.rn.f32.f64 and back, (float) itself.
    __device__ static double step_cvt(double t) { return (double)__double2float_rn(t); }
    __device__ static unsigned fold2(unsigned run, unsigned r0, unsigned r1) {
        return Fast::fold2(run, r0, r1);
    }
    __device__ static bool valid(unsigned run) { return Fast::valid(run); }
    __device__ static double exact(double t) { return (double)__double2float_rn(t); }
};

// Dot.round for FP16/BF16 under NEAREST_EVEN or TRUNCATE, for any input,
// inline (no call on the contraction's rare path). Below 2^min_exp the
// quantum is fixed (2^(min_exp - mant)), so one magic constant serves; above
// it the binade's own quantum applies; 2^(max_exp+1) and beyond (Inf
// included) saturate to max; zero and NaN pass through with their sign.
template <int ACC, int RM>
__device__ __forceinline__ double narrow_exact(double t) {
    using F = AccFmt<ACC>;
    constexpr int S = 52 - F::mant;
    const double a = fabs(t);
    const double lo_bound = pow2(F::min_exp);
    double r;
    if (!(a >= lo_bound)) {  // below the normal range, or NaN
        const double c0 = 1.5 * pow2(F::min_exp - F::mant + 52);
        r = RM == DRIFT_TRUNCATE ? __dsub_rn(__dadd_rz(a, c0), c0) : __dsub_rn(__dadd_rn(a, c0), c0);
    } else {
        r = RM == DRIFT_TRUNCATE ? trunc_shift<S>(a) : rne_shift<S>(a);
        if (a >= pow2(F::max_exp + 1)) r = F::max();
    }
    if (r > F::max()) r = F::max();
    return copysign(r, t);
}

template <int RM> struct AccRound<DRIFT_ACC_FP16, RM> {
    using F = AccFmt<DRIFT_ACC_FP16>;
    using Fast = FastForm<52 - F::mant, 1023 + F::min_exp, 1023 + F::max_exp - 1>;
    __device__ static double step(double t, int prev_lo, unsigned &run) {
        return RM == DRIFT_TRUNCATE ? Fast::trunc(t, prev_lo, run) : Fast::rne(t, prev_lo, run);
    }
    __device__ static double step_int(double t, unsigned &run) {
        return RM == DRIFT_TRUNCATE ? Fast::trunc(t, 0, run) : Fast::rne_int(t, run);
    }
    __device__ static unsigned fold2(unsigned run, unsigned r0, unsigned r1) {
        return Fast::fold2(run, r0, r1);
    }
    __device__ static bool valid(unsigned run) { return Fast::valid(run); }
    __device__ static double exact(double t) { return narrow_exact<DRIFT_ACC_FP16, RM>(t); }
};

template <int RM> struct AccRound<DRIFT_ACC_BF16, RM> {
    using F = AccFmt<DRIFT_ACC_BF16>;
    using Fast = FastForm<52 - F::mant, 1023 + F::min_exp, 1023 + F::max_exp - 1>;
    __device__ static double step(double t, int prev_lo, unsigned &run) {
        return RM == DRIFT_TRUNCATE ? Fast::trunc(t, prev_lo, run) : Fast::rne(t, prev_lo, run);
    }
    __device__ static double step_int(double t, unsigned &run) {
        return RM == DRIFT_TRUNCATE ? Fast::trunc(t, 0, run) : Fast::rne_int(t, run);
    }
    // On the conversion pipe: cvt.rn.bf16.f64 and back. Nearest even with
    // subnormals, as Dot.round; it gives Inf where Dot.round saturates, so it
    // serves only sums proven to stay below the top binade.
    __device__ static double step_cvt(double t) {
        return (double)__bfloat162float(__double2bfloat16(t));
    }
    __device__ static unsigned fold2(unsigned run, unsigned r0, unsigned r1) {
        return Fast::fold2(run, r0, r1);
    }
    __device__ static bool valid(unsigned run) { return Fast::valid(run); }
    __device__ static double exact(double t) { return narrow_exact<DRIFT_ACC_BF16, RM>(t); }
};

}  // namespace drift
