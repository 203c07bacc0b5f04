/*
 * CPU oracle for nvcr.intconv.v1: a plain-C restatement of the reference CPU
 * executor. TEST INFRASTRUCTURE ONLY (see intconv_oracle.h): the product never
 * links or calls this file.
 *
 * Build flags matter: -O2 -ffp-contract=off -fno-fast-math, as the reference
 * builds its host executor (reference CMakeLists.txt:157-164), so that every
 * float operation below is one IEEE binary32 operation rounded to nearest-even.
 */
#include "intconv_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#if defined(__x86_64__)
#include <xmmintrin.h>
#endif

static float bits_to_float(uint32_t bits) {
    float value;
    memcpy(&value, &bits, sizeof(value));
    return value;
}

static uint32_t float_to_bits(float value) {
    uint32_t bits;
    memcpy(&bits, &value, sizeof(bits));
    return bits;
}

/* std::max(a, b) is (a < b) ? b : a: a NaN second operand is ignored. */
static float max_keep_first(float a, float b) { return a < b ? b : a; }

static int is_finite_value(float value) { return value == value && value - value == 0.0f; }

/* det_exp (det_math.hpp:92-112): Cody-Waite reduction by ln2 in two parts,
 * then a degree-7 Taylor polynomial in Horner form, scaled by 2^k built from
 * bits. Every step is a single exactly rounded operation. */
float or_exp(float x) {
    if (!(x == x)) return x;
    if (x >= 88.0f) return bits_to_float(0x7f800000u);
    if (x < -87.0f) return 0.0f;
    const float k = nearbyintf(x * 1.44269502162933349609375f);
    float r = fmaf(-k, 0.693359375f, x);
    r = fmaf(-k, -2.12194440e-4f, r);
    float p = 1.98412698e-4f;
    p = fmaf(p, r, 1.38888889e-3f);
    p = fmaf(p, r, 8.33333377e-3f);
    p = fmaf(p, r, 4.16666679e-2f);
    p = fmaf(p, r, 1.66666672e-1f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    const int32_t biased = (int32_t)k + 127;
    return p * bits_to_float((uint32_t)biased << 23);
}

/* det_sigmoid (det_math.hpp:114-116). */
float or_sigmoid(float x) { return 1.0f / (1.0f + or_exp(-x)); }

/* det_ldexp (det_math.hpp:119-131). */
float or_ldexp(float value, int exponent) {
    if (exponent >= -126 && exponent <= 127) {
        return value * bits_to_float((uint32_t)(exponent + 127) << 23);
    }
    return ldexpf(value, exponent);
}

/* det_frexp_exponent (det_math.hpp:134-142). */
int or_frexp_exponent(float value) {
    int exponent = 0;
    (void)frexpf(value, &exponent);
    return exponent;
}

/* det_int_exponent (det_math.hpp:161-163). */
int or_int_exponent(float maximum, int bits) {
    return maximum > 0.0f ? or_frexp_exponent(maximum) - (bits - 1) : 0;
}

/* det_int_quantize (det_math.hpp:165-170). */
int or_int_quantize(float value, int exponent, int bits) {
    const float limit = bits == 16 ? 32767.0f : 127.0f;
    const float scaled = nearbyintf(or_ldexp(value, -exponent));
    if (scaled > limit) return (int)limit;
    if (scaled < -limit) return -(int)limit;
    return (int)scaled;
}

/* det_int_output (det_math.hpp:172-174). */
float or_int_output(long long accumulator, float scale, int exponent, float bias) {
    return or_ldexp((float)accumulator * scale, exponent) + bias;
}

/* det_half_bits_to_float (det_math.hpp:177-198): exact widening. */
float or_half_to_float(uint16_t half) {
    const uint32_t sign = (uint32_t)(half & 0x8000u) << 16;
    uint32_t exponent = (half >> 10) & 0x1fu;
    uint32_t mantissa = half & 0x3ffu;
    if (exponent == 0x1fu) return bits_to_float(sign | 0x7f800000u | (mantissa << 13));
    if (exponent == 0) {
        if (mantissa == 0) return bits_to_float(sign);
        uint32_t shift = 0;
        while ((mantissa & 0x400u) == 0) {
            mantissa <<= 1;
            ++shift;
        }
        mantissa &= 0x3ffu;
        return bits_to_float(sign | ((113u - shift) << 23) | (mantissa << 13));
    }
    return bits_to_float(sign | ((exponent + 112u) << 23) | (mantissa << 13));
}

/* det_float_to_half_bits (det_math.hpp:203-229): round to nearest even. */
uint16_t or_float_to_half(float value) {
    const uint32_t bits = float_to_bits(value);
    const uint32_t sign = (bits >> 16) & 0x8000u;
    const uint32_t exponent = (bits >> 23) & 0xffu;
    uint32_t mantissa = bits & 0x7fffffu;
    if (exponent == 0xffu) return (uint16_t)(sign | 0x7c00u | (mantissa != 0 ? 0x200u : 0u));
    const int unbiased = (int)exponent - 127;
    if (unbiased > 15) return (uint16_t)(sign | 0x7c00u);
    if (unbiased >= -14) {
        uint32_t half = ((uint32_t)(unbiased + 15) << 10) | (mantissa >> 13);
        const uint32_t dropped = mantissa & 0x1fffu;
        if (dropped > 0x1000u || (dropped == 0x1000u && (half & 1u) != 0)) ++half;
        return (uint16_t)(sign | half);
    }
    if (unbiased < -25) return (uint16_t)sign;
    mantissa |= 0x800000u;
    const uint32_t shift = (uint32_t)(-unbiased - 14 + 13);
    uint32_t half = mantissa >> shift;
    const uint32_t remainder = mantissa & ((1u << shift) - 1u);
    const uint32_t halfway = 1u << (shift - 1u);
    if (remainder > halfway || (remainder == halfway && (half & 1u) != 0)) ++half;
    return (uint16_t)(sign | half);
}

/* quantize_weights (program.cpp:509-535): per output channel, in double. */
void or_quantize_weights(const float* weights, int32_t out_channels, int32_t in_channels,
                         int32_t weight_bits, int16_t* values, float* scales) {
    memset(values, 0, sizeof(int16_t) * (size_t)out_channels * (size_t)in_channels);
    for (int32_t row = 0; row < out_channels; ++row) {
        const float* w = weights + (size_t)row * (size_t)in_channels;
        float maximum = 0.0f;
        for (int32_t column = 0; column < in_channels; ++column) {
            maximum = max_keep_first(maximum, fabsf(w[column]));
        }
        if (maximum == 0.0f) {
            scales[row] = 1.0f;
            continue;
        }
        const double limit = weight_bits == 16 ? 32767.0 : 127.0;
        const double scale = (double)maximum / limit;
        scales[row] = (float)scale;
        for (int32_t column = 0; column < in_channels; ++column) {
            double q = nearbyint((double)w[column] / scale);
            /* std::clamp(q, -limit, limit) keeps a NaN, and the x86 conversion
             * of a NaN to int16 through int32 yields 0. */
            if (q < -limit) q = -limit;
            else if (limit < q) q = limit;
            values[(size_t)row * (size_t)in_channels + (size_t)column] = q == q ? (int16_t)q : 0;
        }
    }
}

static void set_error(char* error, size_t size, const char* message) {
    if (error != NULL && size > 0) snprintf(error, size, "%s", message);
}

static int is_integer_pointwise(const or_node* node) {
    return node->kind == OR_CONV && !node->depthwise && node->kernel_h == 1 && node->kernel_w == 1 &&
        node->stride_y == 1 && node->stride_x == 1 && node->pad_top == 0 && node->pad_left == 0 &&
        node->pad_bottom == 0 && node->pad_right == 0;
}

/* output_extent (program.cpp:628-700). extents holds (c, h, w) per input. */
int or_output_extent(const or_program* program, const or_node* node, const int32_t* extents,
                     int32_t* out, char* error, size_t error_size) {
    const int32_t c = extents[0], h = extents[1], w = extents[2];
    if (c != program->tensor_channels[node->input0] || h <= 0 || w <= 0) {
        set_error(error, error_size, "tensor has an unexpected shape");
        return -1;
    }
    const int32_t* second = extents + 3;
    switch (node->kind) {
    case OR_CONV:
    case OR_IM2COL: {
        if (node->kind == OR_CONV && c != node->in_channels) {
            set_error(error, error_size, "conv input channel mismatch");
            return -1;
        }
        const int32_t height = h + node->pad_top + node->pad_bottom - node->kernel_h;
        const int32_t width = w + node->pad_left + node->pad_right - node->kernel_w;
        if (height < 0 || width < 0) {
            set_error(error, error_size, "input is smaller than its kernel");
            return -1;
        }
        out[0] = node->kind == OR_CONV ? node->out_channels : c * node->kernel_h * node->kernel_w;
        out[1] = height / node->stride_y + 1;
        out[2] = width / node->stride_x + 1;
        return 0;
    }
    case OR_MUL:
    case OR_ADD:
        if (node->input_count != 2 || second[0] != c || second[1] != h || second[2] != w) {
            set_error(error, error_size, "elementwise inputs differ in shape");
            return -1;
        }
        break;
    case OR_SCALE_CHANNELS:
        if (node->input_count != 2 || second[0] != c || second[1] != 1 || second[2] != 1) {
            set_error(error, error_size, "scale_channels needs a [C, 1, 1] scale");
            return -1;
        }
        break;
    case OR_CONCAT:
        if (node->input_count != 2 || second[1] != h || second[2] != w ||
            second[0] != program->tensor_channels[node->input1]) {
            set_error(error, error_size, "concat inputs differ in spatial shape");
            return -1;
        }
        out[0] = c + second[0];
        out[1] = h;
        out[2] = w;
        return 0;
    case OR_CROP:
        if (node->input_count != 2 || (node->axis == 2 ? second[1] > h : second[2] > w)) {
            set_error(error, error_size, "crop reference is larger than its input");
            return -1;
        }
        out[0] = c;
        out[1] = node->axis == 2 ? second[1] : h;
        out[2] = node->axis == 2 ? w : second[2];
        return 0;
    case OR_SPACE_TO_DEPTH:
        if (h % node->block != 0 || w % node->block != 0) {
            set_error(error, error_size, "space_to_depth input is not a multiple of its block");
            return -1;
        }
        out[0] = c * node->block * node->block;
        out[1] = h / node->block;
        out[2] = w / node->block;
        return 0;
    case OR_SLICE_CHANNELS:
        if (node->begin < 0 || node->end <= node->begin || node->end > c) {
            set_error(error, error_size, "channel slice is out of range");
            return -1;
        }
        out[0] = node->end - node->begin;
        out[1] = h;
        out[2] = w;
        return 0;
    case OR_DEPTH_TO_SPACE:
        if (c % (node->block * node->block) != 0) {
            set_error(error, error_size, "depth_to_space channels are not divisible");
            return -1;
        }
        out[0] = c / (node->block * node->block);
        out[1] = h * node->block;
        out[2] = w * node->block;
        return 0;
    case OR_MUL_SCALAR:
    case OR_SIGMOID:
    case OR_CLAMP:
        break;
    default:
        set_error(error, error_size, "unknown op");
        return -1;
    }
    out[0] = c;
    out[1] = h;
    out[2] = w;
    return 0;
}

static size_t tensor_size(const or_tensor* t) {
    return (size_t)t->channels * (size_t)t->height * (size_t)t->width;
}

/* conv (program.cpp:361-404): FP32 fma from the bias over (channel, ky, kx),
 * padding taps contributing fma(w, 0, out). */
static void conv_fp32(const or_program* program, const or_node* node, const or_tensor* input,
                      or_tensor* output) {
    const float* weights = program->weights + node->weight_offset;
    const float* bias = program->weights + node->bias_offset;
    const int32_t group_inputs = node->depthwise ? 1 : node->in_channels;
    const size_t in_plane = (size_t)input->height * (size_t)input->width;
    const size_t out_plane = (size_t)output->height * (size_t)output->width;
    for (int32_t oc = 0; oc < node->out_channels; ++oc) {
        float* out = output->values + (size_t)oc * out_plane;
        for (size_t p = 0; p < out_plane; ++p) out[p] = bias[oc];
        for (int32_t local = 0; local < group_inputs; ++local) {
            const int32_t ic = node->depthwise ? oc : local;
            const float* in = input->values + (size_t)ic * in_plane;
            const float* kernel = weights +
                ((size_t)oc * (size_t)group_inputs + (size_t)local) * (size_t)node->kernel_h *
                    (size_t)node->kernel_w;
            for (int32_t ky = 0; ky < node->kernel_h; ++ky) {
                for (int32_t kx = 0; kx < node->kernel_w; ++kx) {
                    const float weight = kernel[ky * node->kernel_w + kx];
                    for (int32_t oy = 0; oy < output->height; ++oy) {
                        const int32_t iy = oy * node->stride_y - node->pad_top + ky;
                        for (int32_t ox = 0; ox < output->width; ++ox) {
                            const int32_t ix = ox * node->stride_x - node->pad_left + kx;
                            const float value = iy >= 0 && iy < input->height && ix >= 0 && ix < input->width
                                ? in[(size_t)iy * (size_t)input->width + (size_t)ix]
                                : 0.0f;
                            float* target = out + (size_t)oy * (size_t)output->width + (size_t)ox;
                            *target = fmaf(weight, value, *target);
                        }
                    }
                }
            }
        }
    }
}

/* integer_pointwise (program.cpp:407-449). */
static int integer_pointwise(const or_program* program, const or_node* node, const or_tensor* input,
                             or_tensor* output) {
    const size_t positions = (size_t)input->height * (size_t)input->width;
    const size_t channels = (size_t)node->in_channels;
    int16_t* wq = malloc(sizeof(int16_t) * (size_t)node->out_channels * channels + 2);
    float* scales = malloc(sizeof(float) * (size_t)node->out_channels + 4);
    int32_t* activations = malloc(sizeof(int32_t) * channels * positions + 4);
    int* exponents = malloc(sizeof(int) * positions + 4);
    unsigned char* finite = malloc(positions + 1);
    long long* accumulators = malloc(sizeof(long long) * positions + 8);
    if (!wq || !scales || !activations || !exponents || !finite || !accumulators) {
        free(wq); free(scales); free(activations); free(exponents); free(finite); free(accumulators);
        return -1;
    }
    or_quantize_weights(program->weights + node->weight_offset, node->out_channels, node->in_channels,
                        node->weight_bits, wq, scales);
    const float* bias = program->weights + node->bias_offset;
    for (size_t p = 0; p < positions; ++p) {
        float maximum = 0.0f;
        finite[p] = 1;
        for (size_t c = 0; c < channels; ++c) {
            const float value = input->values[c * positions + p];
            if (!is_finite_value(value)) finite[p] = 0;
            maximum = max_keep_first(maximum, fabsf(value));
        }
        exponents[p] = or_int_exponent(maximum, node->activation_bits);
        for (size_t c = 0; c < channels; ++c) {
            activations[c * positions + p] = finite[p]
                ? or_int_quantize(input->values[c * positions + p], exponents[p], node->activation_bits)
                : 0;
        }
    }
    for (int32_t row = 0; row < node->out_channels; ++row) {
        memset(accumulators, 0, sizeof(long long) * positions);
        for (size_t c = 0; c < channels; ++c) {
            const long long weight = wq[(size_t)row * channels + c];
            const int32_t* column = activations + c * positions;
            for (size_t p = 0; p < positions; ++p) accumulators[p] += weight * column[p];
        }
        float* out = output->values + (size_t)row * positions;
        for (size_t p = 0; p < positions; ++p) {
            out[p] = finite[p] ? or_int_output(accumulators[p], scales[row], exponents[p], bias[row])
                               : bits_to_float(0x7fc00000u);
        }
    }
    free(wq); free(scales); free(activations); free(exponents); free(finite); free(accumulators);
    return 0;
}

/* depth_to_space, CRD (program.cpp:451-463). */
static void depth_to_space(const or_node* node, const or_tensor* in, or_tensor* out) {
    const int32_t b = node->block;
    for (int32_t c = 0; c < out->channels; ++c)
        for (int32_t y = 0; y < out->height; ++y)
            for (int32_t x = 0; x < out->width; ++x) {
                const int32_t source = c * b * b + (y % b) * b + x % b;
                out->values[((size_t)c * out->height + y) * out->width + x] =
                    in->values[((size_t)source * in->height + y / b) * in->width + x / b];
            }
}

/* space_to_depth, PixelUnshuffle order (program.cpp:465-479). */
static void space_to_depth(const or_node* node, const or_tensor* in, or_tensor* out) {
    const int32_t b = node->block;
    for (int32_t c = 0; c < out->channels; ++c) {
        const int32_t source = c / (b * b);
        const int32_t oy = (c / b) % b;
        const int32_t ox = c % b;
        for (int32_t y = 0; y < out->height; ++y)
            for (int32_t x = 0; x < out->width; ++x)
                out->values[((size_t)c * out->height + y) * out->width + x] =
                    in->values[((size_t)source * in->height + y * b + oy) * in->width + x * b + ox];
    }
}

/* im2col (program.cpp:481-498). */
static void im2col(const or_node* node, const or_tensor* in, or_tensor* out) {
    const int32_t taps = node->kernel_h * node->kernel_w;
    for (int32_t c = 0; c < out->channels; ++c) {
        const int32_t source = c / taps;
        const int32_t ky = (c % taps) / node->kernel_w;
        const int32_t kx = c % node->kernel_w;
        for (int32_t y = 0; y < out->height; ++y) {
            const int32_t iy = y * node->stride_y - node->pad_top + ky;
            for (int32_t x = 0; x < out->width; ++x) {
                const int32_t ix = x * node->stride_x - node->pad_left + kx;
                out->values[((size_t)c * out->height + y) * out->width + x] =
                    iy >= 0 && iy < in->height && ix >= 0 && ix < in->width
                    ? in->values[((size_t)source * in->height + iy) * in->width + ix]
                    : 0.0f;
            }
        }
    }
}

void or_free(void* pointer) { free(pointer); }

int or_run(const or_program* program, const or_tensor* inputs, or_tensor* outputs, char* error,
           size_t error_size) {
#if defined(__x86_64__)
    /* Keep denormals, as the reference's DenormalGuard does (program.cpp:320-340). */
    const unsigned int saved_csr = _mm_getcsr();
    _mm_setcsr(saved_csr & ~0x8040u);
#endif
    int status = 0;
    const int32_t count = program->tensor_count;
    or_tensor* tensors = calloc((size_t)count, sizeof(or_tensor));
    int32_t* last_use = malloc(sizeof(int32_t) * (size_t)count);
    if (tensors == NULL || last_use == NULL) {
        free(tensors);
        free(last_use);
        set_error(error, error_size, "out of host memory");
        status = -1;
        goto done;
    }
    for (int32_t t = 0; t < count; ++t) last_use[t] = -1;
    for (int32_t n = 0; n < program->node_count; ++n) {
        last_use[program->nodes[n].input0] = n;
        if (program->nodes[n].input_count == 2) last_use[program->nodes[n].input1] = n;
    }
    for (int32_t o = 0; o < program->output_count; ++o) last_use[program->outputs[o]] = program->node_count;

    for (int32_t i = 0; i < program->input_count; ++i) {
        const int32_t id = program->inputs[i];
        if (inputs[i].channels != program->tensor_channels[id]) {
            set_error(error, error_size, "input has the wrong shape");
            status = -1;
            goto cleanup;
        }
        tensors[id] = inputs[i];
        const size_t bytes = sizeof(float) * tensor_size(&inputs[i]);
        tensors[id].values = malloc(bytes + 4);
        memcpy(tensors[id].values, inputs[i].values, bytes);
    }

    for (int32_t n = 0; n < program->node_count; ++n) {
        const or_node* node = &program->nodes[n];
        int32_t extents[6] = {0, 0, 0, 0, 0, 0};
        const or_tensor* first = &tensors[node->input0];
        const or_tensor* second = node->input_count == 2 ? &tensors[node->input1] : NULL;
        if (first->values == NULL || (second != NULL && second->values == NULL)) {
            set_error(error, error_size, "program reads a released tensor");
            status = -1;
            goto cleanup;
        }
        extents[0] = first->channels;
        extents[1] = first->height;
        extents[2] = first->width;
        if (second != NULL) {
            extents[3] = second->channels;
            extents[4] = second->height;
            extents[5] = second->width;
        }
        int32_t out_extent[3];
        if (or_output_extent(program, node, extents, out_extent, error, error_size) != 0) {
            status = -1;
            goto cleanup;
        }
        or_tensor output = {out_extent[0], out_extent[1], out_extent[2], NULL};
        const size_t size = tensor_size(&output);
        output.values = malloc(sizeof(float) * size + 4);
        switch (node->kind) {
        case OR_CONV:
            if (is_integer_pointwise(node)) {
                if (integer_pointwise(program, node, first, &output) != 0) {
                    set_error(error, error_size, "out of host memory");
                    free(output.values);
                    status = -1;
                    goto cleanup;
                }
            } else {
                conv_fp32(program, node, first, &output);
            }
            break;
        case OR_MUL:
            for (size_t i = 0; i < size; ++i) output.values[i] = first->values[i] * second->values[i];
            break;
        case OR_ADD:
            for (size_t i = 0; i < size; ++i) output.values[i] = first->values[i] + second->values[i];
            break;
        case OR_MUL_SCALAR:
            for (size_t i = 0; i < size; ++i) output.values[i] = first->values[i] * node->scalar;
            break;
        case OR_SIGMOID:
            for (size_t i = 0; i < size; ++i) output.values[i] = or_sigmoid(first->values[i]);
            break;
        case OR_SLICE_CHANNELS: {
            const size_t plane = (size_t)first->height * (size_t)first->width;
            memcpy(output.values, first->values + (size_t)node->begin * plane, sizeof(float) * size);
            break;
        }
        case OR_DEPTH_TO_SPACE:
            depth_to_space(node, first, &output);
            break;
        case OR_SCALE_CHANNELS: {
            const size_t plane = (size_t)first->height * (size_t)first->width;
            for (size_t i = 0; i < size; ++i) output.values[i] = first->values[i] * second->values[i / plane];
            break;
        }
        case OR_CLAMP:
            for (size_t i = 0; i < size; ++i) {
                const float v = first->values[i];
                output.values[i] = v < node->minimum ? node->minimum : (v > node->maximum ? node->maximum : v);
            }
            break;
        case OR_CONCAT: {
            const size_t head = tensor_size(first);
            memcpy(output.values, first->values, sizeof(float) * head);
            memcpy(output.values + head, second->values, sizeof(float) * tensor_size(second));
            break;
        }
        case OR_CROP:
            for (int32_t c = 0; c < output.channels; ++c)
                for (int32_t y = 0; y < output.height; ++y)
                    memcpy(output.values + ((size_t)c * output.height + y) * output.width,
                           first->values + ((size_t)c * first->height + y) * first->width,
                           sizeof(float) * (size_t)output.width);
            break;
        case OR_SPACE_TO_DEPTH:
            space_to_depth(node, first, &output);
            break;
        case OR_IM2COL:
            im2col(node, first, &output);
            break;
        default:
            break;
        }
        if (tensors[node->output].values != NULL) free(tensors[node->output].values);
        tensors[node->output] = output;
        if (last_use[node->input0] == n) {
            free(tensors[node->input0].values);
            tensors[node->input0].values = NULL;
        }
        if (node->input_count == 2 && node->input1 != node->input0 && last_use[node->input1] == n) {
            free(tensors[node->input1].values);
            tensors[node->input1].values = NULL;
        }
    }

    for (int32_t o = 0; o < program->output_count; ++o) {
        const or_tensor* t = &tensors[program->outputs[o]];
        if (t->values == NULL) {
            set_error(error, error_size, "program output was not produced");
            status = -1;
            for (int32_t p = 0; p < o; ++p) {
                free(outputs[p].values);
                outputs[p].values = NULL;
            }
            goto cleanup;
        }
        outputs[o] = *t;
        const size_t bytes = sizeof(float) * tensor_size(t);
        outputs[o].values = malloc(bytes + 4);
        memcpy(outputs[o].values, t->values, bytes);
    }

cleanup:
    for (int32_t t = 0; t < count; ++t) free(tensors[t].values);
    free(tensors);
    free(last_use);
done:
#if defined(__x86_64__)
    _mm_setcsr(saved_csr);
#endif
    return status;
}
