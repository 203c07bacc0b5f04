#pragma once

// The nvcr.intconv.v1 arithmetic on sm_100a (reference contract:
// src/deterministic/program.hpp:1-44 and det_math.hpp). Every float operation
// is one IEEE binary32 operation rounded to nearest-even, written with the _rn
// intrinsics so the compiler can neither contract nor reorder it; the rest is
// exact integer or bit manipulation. The translation units that include this
// header are also built with -fmad=false and without -use_fast_math, and keep
// denormals (no -ftz).

#include <cstdint>

#if defined(__CUDACC__)
#define NV_HD __host__ __device__ __forceinline__
#else
#define NV_HD inline
#endif

namespace nvcr_sm100 {

NV_HD float bits_as_float(std::uint32_t bits) {
#if defined(__CUDA_ARCH__)
    return __uint_as_float(bits);
#else
    float f;
    __builtin_memcpy(&f, &bits, 4);
    return f;
#endif
}

NV_HD std::uint32_t float_as_bits(float value) {
#if defined(__CUDA_ARCH__)
    return __float_as_uint(value);
#else
    std::uint32_t b;
    __builtin_memcpy(&b, &value, 4);
    return b;
#endif
}

#if defined(__CUDACC__)

__device__ __forceinline__ float canonical_nan() { return __uint_as_float(0x7fc00000u); }

// A value is finite when it equals itself and x - x is zero (inf - inf and
// NaN - NaN are NaN): the reference's test (det_math.hpp:156-158).
__device__ __forceinline__ bool is_finite_value(float v) { return v == v && __fsub_rn(v, v) == 0.0f; }

// 2^n for n in [-126, 127], built from bits.
__device__ __forceinline__ float power_of_two(int n) {
    return __uint_as_float(static_cast<std::uint32_t>(n + 127) << 23);
}

// x * 2^n rounded once to nearest-even, for any n (ldexp). Multiplying by a
// normal power of two is exact unless the product is subnormal or overflows,
// and then the multiply itself is the single correct rounding; outside
// [-126, 127] the power is not a float, so the exponent is moved in the bits
// and a subnormal result is rounded explicitly.
static __device__ __noinline__ float ldexp_wide(float x, int n) {
    const std::uint32_t b = __float_as_uint(x);
    const std::uint32_t sign = b & 0x80000000u;
    std::uint32_t magnitude = b & 0x7fffffffu;
    if (magnitude == 0 || magnitude >= 0x7f800000u) return x;  // zero, inf, NaN
    int biased = static_cast<int>(magnitude >> 23);
    std::uint32_t significand = magnitude & 0x7fffffu;
    if (biased == 0) {  // subnormal input: normalise
        const int lead = __clz(significand) - 8;  // shift that brings bit 23 up
        significand <<= lead;
        biased = 1 - lead;
    }
    significand |= 0x800000u;  // x = significand * 2^(biased - 150)
    const long long result_biased = static_cast<long long>(biased) + n;
    if (result_biased >= 255) return __uint_as_float(sign | 0x7f800000u);
    if (result_biased >= 1) {
        return __uint_as_float(sign | (static_cast<std::uint32_t>(result_biased) << 23) |
                               (significand & 0x7fffffu));
    }
    const long long shift = 1 - result_biased;  // subnormal result: drop `shift` bits
    if (shift > 25) return __uint_as_float(sign);
    const std::uint32_t s = static_cast<std::uint32_t>(shift);
    std::uint32_t kept = significand >> s;
    const std::uint32_t dropped = significand & ((1u << s) - 1u);
    const std::uint32_t halfway = 1u << (s - 1u);
    if (dropped > halfway || (dropped == halfway && (kept & 1u) != 0)) ++kept;
    return __uint_as_float(sign | kept);
}

__device__ __forceinline__ float exact_ldexp(float x, int n) {
    if (n >= -126 && n <= 127) return __fmul_rn(x, power_of_two(n));
    return ldexp_wide(x, n);
}

// E with a = f * 2^E, 0.5 <= f < 1, for finite a > 0 (frexp's exponent).
__device__ __forceinline__ int frexp_exponent(float a) {
    const std::uint32_t b = __float_as_uint(a) & 0x7fffffffu;
    const int biased = static_cast<int>(b >> 23);
    if (biased == 0) return (32 - __clz(b)) - 149;  // subnormal: a = m * 2^-149
    return biased - 126;
}

// Activation exponent of a position whose largest magnitude is `maximum`
// (program.hpp:33-36): e = E - (bits - 1), and 0 for an all-zero position.
__device__ __forceinline__ int activation_exponent(float maximum, int bits) {
    return maximum > 0.0f ? frexp_exponent(maximum) - (bits - 1) : 0;
}

// q = clamp(rint(ldexp(x, -e)), +-L) with L = 127 or 32767.
template <int Bits>
__device__ __forceinline__ int quantize_value(float x, int exponent) {
    constexpr float limit = Bits == 16 ? 32767.0f : 127.0f;
    const float scaled = rintf(exact_ldexp(x, -exponent));
    return scaled > limit ? static_cast<int>(limit)
                          : (scaled < -limit ? -static_cast<int>(limit) : static_cast<int>(scaled));
}

// out = ((float(acc) * scale) * 2^e) + bias, each step rounded to nearest-even.
__device__ __forceinline__ float integer_output(long long accumulator, float scale, int exponent, float bias) {
    const float widened = __ll2float_rn(accumulator);
    return __fadd_rn(exact_ldexp(__fmul_rn(widened, scale), exponent), bias);
}

__device__ __forceinline__ float integer_output32(int accumulator, float scale, int exponent, float bias) {
    const float widened = __int2float_rn(accumulator);
    return __fadd_rn(exact_ldexp(__fmul_rn(widened, scale), exponent), bias);
}

// The profile's exp (reference det_math.hpp:92-112): x = k ln2 + r with the
// two-part Cody-Waite split of ln2 (0.693359375 and -2.12194440e-4, the split
// Cephes' expf uses), then exp(r) as the degree-7 Taylor polynomial in Horner
// form with float coefficients 1/n!, times 2^k built from bits. The constants
// and the operation order are part of the profile: any other evaluation gives
// other bits. NaN passes through, x >= 88 gives +inf, x < -87 gives 0.

// exp on [-87, 88): the profile's Cody-Waite reduction and Taylor polynomial.
// k = rint(x log2 e) by the round-to-nearest-even of adding 1.5 * 2^23 (exact
// for |x log2 e| < 2^22; here it is below 127), which leaves the integer k in
// the low bits of the sum: no conversion instruction for k or for 2^k.
__device__ __forceinline__ float profile_exp_inside(float x) {
    constexpr float magic = 12582912.0f;  // 1.5 * 2^23
    const float shifted = __fadd_rn(__fmul_rn(x, 1.44269502162933349609375f), magic);
    const float k = __fsub_rn(shifted, magic);
    const int k_int = static_cast<int>(__float_as_uint(shifted) - __float_as_uint(magic));
    float r = __fmaf_rn(-k, 0.693359375f, x);
    r = __fmaf_rn(-k, -2.12194440e-4f, r);
    float p = 1.98412698e-4f;
    p = __fmaf_rn(p, r, 1.38888889e-3f);
    p = __fmaf_rn(p, r, 8.33333377e-3f);
    p = __fmaf_rn(p, r, 4.16666679e-2f);
    p = __fmaf_rn(p, r, 1.66666672e-1f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    return __fmul_rn(p, __uint_as_float(static_cast<std::uint32_t>(k_int + 127) << 23));
}

// The polynomial runs on every argument (0 stands in outside [-87, 88)) and
// the special cases are selected afterwards: straight-line code, so several
// values' evaluations interleave; in-range arguments take the same operations.
__device__ __forceinline__ float profile_exp(float x) {
    const bool inside = x >= -87.0f && x < 88.0f;  // false for NaN
    const float y = profile_exp_inside(inside ? x : 0.0f);
    const float outside = x >= 88.0f ? __uint_as_float(0x7f800000u) : (x < -87.0f ? 0.0f : x);
    return inside ? y : outside;
}

// 1 / d rounded to nearest-even for d in [1, 2^126) (the sigmoid's denominator
// 1 + exp(-x) outside its rare extremes), as straight-line code: the hardware
// approximate reciprocal refined by two Newton-Raphson steps whose residuals
// 1 - d y come exact from a fused multiply-add (Markstein's method, IBM J. Res.
// Dev. 34(1), 1990). Checked against the IEEE division for every float in
// [1, 2^126) by nvcr_sm100_test_reciprocal.
__device__ __forceinline__ float sigmoid_reciprocal(float d) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(d));
    float e = __fmaf_rn(-d, y, 1.0f);
    y = __fmaf_rn(y, e, y);
    e = __fmaf_rn(-d, y, 1.0f);
    return __fmaf_rn(y, e, y);
}
constexpr float sigmoid_reciprocal_limit = 8.50705917302346158659e37f;  // 2^126

// sigmoid(x) = 1 / (1 + exp(-x)) with the IEEE division's bits: the refined
// reciprocal for denominators in [1, 2^126), the division itself beyond (a
// subnormal or zero quotient) and for NaN.
__device__ __forceinline__ float profile_sigmoid(float x) {
    const float d = __fadd_rn(1.0f, profile_exp(-x));
    return d < sigmoid_reciprocal_limit ? sigmoid_reciprocal(d) : __fdiv_rn(1.0f, d);
}

// WSiLU as the reference graph computes it: mul(sigmoid(mul(v, k)), v).
__device__ __forceinline__ float profile_wsilu(float v, float k) {
    return __fmul_rn(profile_sigmoid(__fmul_rn(v, k)), v);
}

#endif  // __CUDACC__

}  // namespace nvcr_sm100
