#pragma once

// DCVC-RT's inter-stage glue under an exact numerics profile, per output
// element: the exact scale-to-entropy-table index, the four- and two-way
// checkerboard masks and the restore of the masked latents (reference
// src/dcvcrt/host_ops.cpp:307-349, 412-472, 523-556 and scale_index.hpp).
// Tensors are FP16 bit patterns; every arithmetic step is one IEEE binary32
// operation rounded to nearest even, as the reference's host code does, and
// FP16 stores round to nearest even with NaN stored as 0x7e00 (sign kept).
// The kernels (k_glue.cu) are grid-stride loops over these functions, which
// are also compiled for the host so the same code can be checked on CPU.

#include <cstddef>
#include <cstdint>
#include <cstring>

#if defined(__CUDACC__)
#define GLUE_HD __host__ __device__ __forceinline__
#else
#define GLUE_HD inline
#endif

namespace nvcr_sm100::glue {

using Half = std::uint16_t;

GLUE_HD std::uint32_t float_bits(float value) {
#if defined(__CUDA_ARCH__)
    return __float_as_uint(value);
#else
    std::uint32_t bits;
    std::memcpy(&bits, &value, 4);
    return bits;
#endif
}

GLUE_HD float bits_float(std::uint32_t bits) {
#if defined(__CUDA_ARCH__)
    return __uint_as_float(bits);
#else
    float value;
    std::memcpy(&value, &bits, 4);
    return value;
#endif
}

// One binary32 operation each, never contracted into an FMA.
GLUE_HD float add(float a, float b) {
#if defined(__CUDA_ARCH__)
    return __fadd_rn(a, b);
#else
    return a + b;
#endif
}

GLUE_HD float mul(float a, float b) {
#if defined(__CUDA_ARCH__)
    return __fmul_rn(a, b);
#else
    return a * b;
#endif
}

GLUE_HD float div(float a, float b) {
#if defined(__CUDA_ARCH__)
    return __fdiv_rn(a, b);
#else
    return a / b;
#endif
}

GLUE_HD float sub(float a, float b) {
#if defined(__CUDA_ARCH__)
    return __fsub_rn(a, b);
#else
    return a - b;
#endif
}

// Round half away from zero (exact, as the reference's std::round).
GLUE_HD float round_away(float v) {
#if defined(__CUDA_ARCH__)
    return roundf(v);
#else
    return __builtin_roundf(v);
#endif
}

// Minimum and maximum as the reference's std::fmin / std::fmax give them on
// its x86-64 host (IEEE 754-2008 minNum / maxNum): a signaling NaN operand
// gives that NaN quieted, a quiet NaN operand is ignored, and of two operands
// that compare equal (+0 and -0) the second is returned. IEEE 754 leaves the
// sign of equal zeros open, so all of it is spelled out here rather than left
// to a library or an instruction. (FP16 signaling NaNs such as 0x7c01 widen to
// signaling float NaNs, so they do reach these.)
GLUE_HD bool is_nan(float v) { return v != v; }

GLUE_HD bool is_signaling(float v) {
    const std::uint32_t bits = float_bits(v);
    return (bits & 0x7fc00000u) == 0x7f800000u && (bits & 0x003fffffu) != 0u;
}

GLUE_HD float quieted(float v) { return bits_float(float_bits(v) | 0x00400000u); }

GLUE_HD float fmin_ieee(float a, float b) {
    if (is_signaling(a)) return quieted(a);
    if (is_signaling(b)) return quieted(b);
    if (is_nan(a)) return b;
    if (is_nan(b)) return a;
    return a < b ? a : b;
}

GLUE_HD float fmax_ieee(float a, float b) {
    if (is_signaling(a)) return quieted(a);
    if (is_signaling(b)) return quieted(b);
    if (is_nan(a)) return b;
    if (is_nan(b)) return a;
    return a > b ? a : b;
}

// binary16 -> binary32, exact.
GLUE_HD float to_float(Half h) {
    const std::uint32_t sign = static_cast<std::uint32_t>(h & 0x8000u) << 16;
    const std::uint32_t exponent = (h >> 10) & 0x1fu;
    std::uint32_t mantissa = h & 0x3ffu;
    if (exponent == 31u) return bits_float(sign | 0x7f800000u | (mantissa << 13));
    if (exponent != 0u) return bits_float(sign | ((exponent + 112u) << 23) | (mantissa << 13));
    if (mantissa == 0u) return bits_float(sign);
    // Subnormal: normalise the mantissa into an implicit-one float.
    int shift = 0;
    while ((mantissa & 0x400u) == 0u) {
        mantissa <<= 1;
        ++shift;
    }
    return bits_float(sign | (static_cast<std::uint32_t>(113 - shift) << 23) | ((mantissa & 0x3ffu) << 13));
}

// binary32 -> binary16, round to nearest even; overflow to infinity, NaN to 0x7e00.
GLUE_HD Half to_half(float value) {
    const std::uint32_t bits = float_bits(value);
    const std::uint32_t sign = (bits >> 16) & 0x8000u;
    const std::uint32_t magnitude = bits & 0x7fffffffu;
    if (magnitude > 0x7f800000u) return static_cast<Half>(sign | 0x7e00u);
    if (magnitude >= 0x477ff000u) return static_cast<Half>(sign | 0x7c00u);  // 65520 and up round to infinity
    if (magnitude < 0x38800000u) {                                          // below 2^-14: a subnormal half
        if (magnitude < 0x33000000u) return static_cast<Half>(sign);         // at most 2^-25: rounds to zero
        const std::uint32_t exponent = magnitude >> 23;                      // 102..112
        const std::uint32_t significand = (magnitude & 0x7fffffu) | 0x800000u;
        const std::uint32_t shift = 126u - exponent;                         // 14..24: units of 2^-24
        std::uint32_t q = significand >> shift;
        const std::uint32_t rest = significand & ((1u << shift) - 1u);
        const std::uint32_t half = 1u << (shift - 1u);
        if (rest > half || (rest == half && (q & 1u))) ++q;
        return static_cast<Half>(sign | q);
    }
    std::uint32_t q = ((magnitude >> 23) - 112u) << 10 | ((magnitude >> 13) & 0x3ffu);
    const std::uint32_t rest = magnitude & 0x1fffu;
    if (rest > 0x1000u || (rest == 0x1000u && (q & 1u))) ++q;  // a carry steps the exponent, as it should
    return static_cast<Half>(sign | q);
}

// The shapes the reference's host ops accept: positive extents, channels a
// multiple of `ways` (2 or 4).
GLUE_HD bool valid_shape(int batch, int channels, int height, int width, int ways) {
    return batch > 0 && channels > 0 && height > 0 && width > 0 && (ways == 2 || ways == 4) && channels % ways == 0;
}

inline constexpr float scale_min = 0.11f;
inline constexpr float scale_max = 16.0f;

// #{ i in 1..127 : clamp(scale) >= thresholds[i - 1] }; NaN maps to table 0.
GLUE_HD std::uint8_t exact_scale_index(float scale, const float* thresholds) {
    if (!(scale >= scale_min)) scale = scale_min;
    if (scale > scale_max) scale = scale_max;
    int low = 0;
    int high = 127;
    while (low < high) {
        const int middle = (low + high + 1) / 2;
        if (thresholds[middle - 1] <= scale) {
            low = middle;
        } else {
            high = middle - 1;
        }
    }
    return static_cast<std::uint8_t>(low);
}

// Decode indexes: the table of each scale, 0 where a positive force-zero
// threshold is not exceeded.
GLUE_HD void decode_index(const Half* scales, std::uint8_t* out, float force_zero, const float* thresholds,
                          std::size_t i) {
    const float scale = to_float(scales[i]);
    out[i] = force_zero > 0.0f && scale <= force_zero ? 0 : exact_scale_index(scale, thresholds);
}

// Encode indexes: symbol in the high byte, table in the low byte (0 where
// forced to zero). Symbols are integers in [-128, 127].
GLUE_HD void encode_index(const Half* symbols, const Half* scales, std::int16_t* out, float force_zero,
                          const float* thresholds, std::size_t i) {
    const float scale = to_float(scales[i]);
    if (force_zero > 0.0f && scale <= force_zero) {
        out[i] = 0;
        return;
    }
    const auto symbol = static_cast<std::int16_t>(static_cast<int>(to_float(symbols[i])));
    out[i] = static_cast<std::int16_t>(static_cast<std::uint16_t>(static_cast<std::uint16_t>(symbol) << 8) |
                                       exact_scale_index(scale, thresholds));
}

// Element i of a [batch][channels][height][width] mask: channel quarter q is
// selected where the pixel's parity (y & 1) * 2 + (x & 1) is pattern[stage][q],
// with the patterns {0,1,2,3}, {3,2,1,0}, {2,3,0,1}, {1,0,3,2} of the four
// stages, i.e. q ^ s with s = 0, 3, 2, 1 = (4 - stage) & 3.
GLUE_HD void four_way_mask(Half* mask, int channels, int height, int width, int stage, std::size_t i) {
    const std::size_t plane = static_cast<std::size_t>(height) * width;
    const int channel = static_cast<int>((i / plane) % channels);
    const int y = static_cast<int>((i % plane) / width);
    const int x = static_cast<int>(i % width);
    const int quarter = channel / (channels / 4);
    const int parity = (y & 1) * 2 + (x & 1);
    mask[i] = (quarter ^ ((4 - stage) & 3)) == parity ? 0x3c00u : 0x0000u;  // 1.0 or 0.0
}

// Two-way: the first channel half takes the diagonal pixels at stage 0 and the
// off-diagonal ones at stage 1; the second half the others.
GLUE_HD void two_way_mask(Half* mask, int channels, int height, int width, int stage, std::size_t i) {
    const std::size_t plane = static_cast<std::size_t>(height) * width;
    const int channel = static_cast<int>((i / plane) % channels);
    const int y = static_cast<int>((i % plane) / width);
    const int x = static_cast<int>(i % width);
    const bool first_half = channel < channels / 2;
    const bool diagonal = (y & 1) == (x & 1);
    const bool selected = stage == 0 ? first_half == diagonal : first_half != diagonal;
    mask[i] = selected ? 0x3c00u : 0x0000u;
}

// Restore: output[d] = (symbol[i] + mean[d]) * mask[d] for each of the `parts`
// (4 or 2) destinations d = i + part * part_size of symbol i.
GLUE_HD void restore(const Half* symbols, const Half* means, const Half* mask, Half* out, std::size_t part_size,
                     int parts, std::size_t i) {
    const float symbol = to_float(symbols[i]);
    for (int part = 0; part < parts; ++part) {
        const std::size_t d = i + static_cast<std::size_t>(part) * part_size;
        out[d] = to_half(mul(add(symbol, to_float(means[d])), to_float(mask[d])));
    }
}

// process_with_mask, element i: the masked scale, mean and residual, the
// symbol round(residual) (0 where a positive force-zero threshold is not
// exceeded) clamped to [-128, 127], and the reconstruction symbol + mean;
// `residual` may be null.
GLUE_HD void process_with_mask(const Half* values, const Half* scales, const Half* means, const Half* mask,
                               Half* residual, Half* symbols, Half* reconstructed, Half* masked_scales,
                               float force_zero, std::size_t i) {
    const float mask_value = to_float(mask[i]);
    const float scale = mul(to_float(scales[i]), mask_value);
    const float mean = mul(to_float(means[i]), mask_value);
    const float value_residual = mul(sub(to_float(values[i]), mean), mask_value);
    float symbol = round_away(value_residual);
    if (force_zero > 0.0f && scale <= force_zero) symbol = 0.0f;
    symbol = fmin_ieee(127.0f, fmax_ieee(-128.0f, symbol));
    if (residual != nullptr) residual[i] = to_half(value_residual);
    symbols[i] = to_half(symbol);
    reconstructed[i] = to_half(add(symbol, mean));
    masked_scales[i] = to_half(scale);
}

// Sum of the `parts` (4 or 2) channel slices at element i, each optionally
// multiplied by the mask first, added in slice order from 0 (quarters) or as
// first + second (halves), as the reference's reduce_* host ops do.
GLUE_HD void reduce_parts(const Half* input, const Half* mask, Half* output, std::size_t part_size, int parts,
                          std::size_t i) {
    if (parts == 2) {
        float first = to_float(input[i]);
        float second = to_float(input[i + part_size]);
        if (mask != nullptr) {
            first = mul(first, to_float(mask[i]));
            second = mul(second, to_float(mask[i + part_size]));
        }
        output[i] = to_half(add(first, second));
        return;
    }
    float value = 0.0f;
    for (int part = 0; part < parts; ++part) {
        const std::size_t source = i + static_cast<std::size_t>(part) * part_size;
        const float term = mask != nullptr ? mul(to_float(input[source]), to_float(mask[source])) : to_float(input[source]);
        value = add(value, term);
    }
    output[i] = to_half(value);
}

// The elementwise steps between stages (reference host_ops.cpp:101-167,
// 474-521), element i each.

// values[i] = round(values[i]) clamped to [-128, 127]; also stored as int8.
GLUE_HD void round_to_int8(Half* values, std::int8_t* quantized, std::size_t i) {
    const float value = fmin_ieee(127.0f, fmax_ieee(-128.0f, round_away(to_float(values[i]))));
    values[i] = to_half(value);
    quantized[i] = static_cast<std::int8_t>(static_cast<int>(value));
}

GLUE_HD void int8_to_half(const std::int8_t* values, Half* output, std::size_t i) {
    output[i] = to_half(static_cast<float>(values[i]));
}

GLUE_HD void clamp_min(Half* values, float minimum, std::size_t i) {
    values[i] = to_half(fmax_ieee(to_float(values[i]), minimum));
}

// quant[i] = max(quant[i], 0.5) in FP16; values[i] *= the FP16 reciprocal of it.
GLUE_HD void clamp_reciprocal_with_quant(Half* quant_step, Half* values, std::size_t i) {
    const Half quant = to_half(fmax_ieee(to_float(quant_step[i]), 0.5f));
    quant_step[i] = quant;
    const Half reciprocal = to_half(div(1.0f, to_float(quant)));
    values[i] = to_half(mul(to_float(values[i]), to_float(reciprocal)));
}

GLUE_HD void add_in_place(Half* first, const Half* second, std::size_t i) {
    first[i] = to_half(add(to_float(first[i]), to_float(second[i])));
}

// values[i] *= factors[i % spatial_count] (one factor plane for every channel).
GLUE_HD void multiply_broadcast(Half* values, const Half* factors, std::size_t spatial_count, std::size_t i) {
    values[i] = to_half(mul(to_float(values[i]), to_float(factors[i % spatial_count])));
}

// first[i] = FP16(first[i] + second[i]) * quant_step[i], rounded to FP16 after each step.
GLUE_HD void add_and_multiply(Half* first, const Half* second, const Half* quant_step, std::size_t i) {
    const Half sum = to_half(add(to_float(first[i]), to_float(second[i])));
    first[i] = to_half(mul(to_float(sum), to_float(quant_step[i])));
}

// Output element i of a (planes, out_h, out_w) tensor: the input pixel at the
// clamped coordinates (edge replication), or, with out_h <= height and
// out_w <= width, the crop from the origin.
GLUE_HD void replicate_or_crop(const Half* input, Half* output, int height, int width, int out_h, int out_w,
                               std::size_t i) {
    const std::size_t out_plane = static_cast<std::size_t>(out_h) * out_w;
    const std::size_t plane = i / out_plane;
    const int y = static_cast<int>((i % out_plane) / out_w);
    const int x = static_cast<int>(i % out_w);
    const int sy = y < height ? y : height - 1;
    const int sx = x < width ? x : width - 1;
    output[i] = input[(plane * height + sy) * width + sx];
}

// Colour conversion at the picture edges (reference host_ops.cpp:198-305), one
// output pixel each. The padded planes replicate the last row and column.
// BT.709 luma weights; every step is one binary32 operation in the reference's
// order.
GLUE_HD void rgb24_to_ycbcr(const std::uint8_t* input, int width, int height, Half* output, int out_h, int out_w,
                            std::size_t i) {
    const std::size_t plane = static_cast<std::size_t>(out_h) * out_w;
    const int y = static_cast<int>(i / out_w);
    const int x = static_cast<int>(i % out_w);
    const int sy = y < height ? y : height - 1;
    const int sx = x < width ? x : width - 1;
    const std::size_t source = (static_cast<std::size_t>(sy) * width + sx) * 3u;
    const float kr = 0.2126f;
    const float kg = 0.7152f;
    const float kb = 0.0722f;
    const float r = div(static_cast<float>(input[source]), 255.0f);
    const float g = div(static_cast<float>(input[source + 1]), 255.0f);
    const float b = div(static_cast<float>(input[source + 2]), 255.0f);
    const float luma = add(add(mul(kr, r), mul(kg, g)), mul(kb, b));
    const float cb = add(div(mul(0.5f, sub(b, luma)), sub(1.0f, kb)), 0.5f);
    const float cr = add(div(mul(0.5f, sub(r, luma)), sub(1.0f, kr)), 0.5f);
    output[i] = to_half(luma);
    output[plane + i] = to_half(cb);
    output[2 * plane + i] = to_half(cr);
}

// YUV 4:2:0 (8-bit planes Y, U, V; even width and height) to padded YCbCr.
GLUE_HD void yuv420p8_to_ycbcr(const std::uint8_t* input, int width, int height, Half* output, int out_h, int out_w,
                               std::size_t i) {
    const std::size_t plane = static_cast<std::size_t>(out_h) * out_w;
    const int y = static_cast<int>(i / out_w);
    const int x = static_cast<int>(i % out_w);
    const std::size_t sy = static_cast<std::size_t>(y < height ? y : height - 1);
    const std::size_t sx = static_cast<std::size_t>(x < width ? x : width - 1);
    const std::size_t y_size = static_cast<std::size_t>(width) * height;
    const std::size_t uv_width = static_cast<std::size_t>(width) / 2;
    const std::size_t uv_size = uv_width * (static_cast<std::size_t>(height) / 2);
    const std::size_t uv_index = (sy / 2) * uv_width + sx / 2;
    output[i] = to_half(div(static_cast<float>(input[sy * width + sx]), 255.0f));
    output[plane + i] = to_half(div(static_cast<float>(input[y_size + uv_index]), 255.0f));
    output[2 * plane + i] = to_half(div(static_cast<float>(input[y_size + uv_size + uv_index]), 255.0f));
}

// Padded YCbCr back to YUV 4:2:0: luma element i of the visible width x height
// picture (round(clamp(v, 0, 1) * 255)), or chroma element i (the mean of a
// 2x2 block, clamp(v * 255, 0, 255) truncated). `stride` is the padded width
// and `plane` the padded plane size.
GLUE_HD void ycbcr_luma_to_y(const Half* input, std::size_t stride, int width, std::uint8_t* output, std::size_t i) {
    const std::size_t y = i / width;
    const std::size_t x = i % width;
    const float v = fmin_ieee(1.0f, fmax_ieee(0.0f, to_float(input[y * stride + x])));
    output[i] = static_cast<std::uint8_t>(static_cast<int>(round_away(mul(v, 255.0f))));
}

GLUE_HD void ycbcr_chroma_to_uv(const Half* input, std::size_t plane, std::size_t stride, int width, int height,
                                std::uint8_t* output, std::size_t i) {
    const std::size_t uv_width = static_cast<std::size_t>(width) / 2;
    const std::size_t uv_size = uv_width * (static_cast<std::size_t>(height) / 2);
    const std::size_t uv_y = i / uv_width;
    const std::size_t uv_x = i % uv_width;
    float cb_sum = 0.0f;
    float cr_sum = 0.0f;
    for (int dy = 0; dy < 2; ++dy) {
        for (int dx = 0; dx < 2; ++dx) {
            const std::size_t spatial = (uv_y * 2 + dy) * stride + uv_x * 2 + dx;
            cb_sum = add(cb_sum, to_float(input[plane + spatial]));
            cr_sum = add(cr_sum, to_float(input[2 * plane + spatial]));
        }
    }
    const std::size_t y_size = static_cast<std::size_t>(width) * height;
    output[y_size + i] =
        static_cast<std::uint8_t>(static_cast<int>(fmin_ieee(255.0f, fmax_ieee(0.0f, mul(mul(cb_sum, 0.25f), 255.0f)))));
    output[y_size + uv_size + i] =
        static_cast<std::uint8_t>(static_cast<int>(fmin_ieee(255.0f, fmax_ieee(0.0f, mul(mul(cr_sum, 0.25f), 255.0f)))));
}

}  // namespace nvcr_sm100::glue
