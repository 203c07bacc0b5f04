/*
 * CPU oracle for the nvcr.intconv.v1 exact-convolution path.
 *
 * TEST INFRASTRUCTURE ONLY. This is a plain-C restatement of the reference
 * CPU executor (0elghati/nvcr, src/deterministic/program.cpp `run_cpu` and
 * src/deterministic/det_math.hpp). Only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline leg may load it, and only as the checker. The
 * product (libnvcr_sm100.so) never links, loads or calls it.
 *
 * Parity pin: tests/test_oracle.py checks this oracle bit for bit against
 * the reference's own run_cpu compiled from its sources (oracle/_ref, built
 * by oracle/Makefile) and against the committed golden fixtures in
 * tests/golden/, which tests/golden/make_golden.py generated from that same
 * reference build.
 */
#ifndef NVCR_INTCONV_ORACLE_H
#define NVCR_INTCONV_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Op kinds, in the reference's OpKind order (program.hpp:57-71). */
enum or_op {
    OR_CONV = 0,
    OR_MUL,
    OR_ADD,
    OR_MUL_SCALAR,
    OR_SIGMOID,
    OR_SLICE_CHANNELS,
    OR_DEPTH_TO_SPACE,
    OR_SCALE_CHANNELS,
    OR_CLAMP,
    OR_CONCAT,
    OR_CROP,
    OR_SPACE_TO_DEPTH,
    OR_IM2COL
};

/* One program node (reference Node, program.hpp:73-103). */
typedef struct or_node {
    int32_t kind;
    int32_t input0, input1, input_count, output;
    int32_t in_channels, out_channels, depthwise;
    int32_t kernel_h, kernel_w, stride_y, stride_x;
    int32_t pad_top, pad_left, pad_bottom, pad_right;
    int64_t weight_offset, bias_offset;
    float scalar;
    int32_t begin, end, block, axis;
    float minimum, maximum;
    int32_t weight_bits, activation_bits;
} or_node;

typedef struct or_program {
    int32_t tensor_count;
    const int32_t* tensor_channels;
    int32_t input_count;
    const int32_t* inputs;
    int32_t output_count;
    const int32_t* outputs;
    int32_t node_count;
    const or_node* nodes;
    const float* weights;
    int64_t weight_count;
} or_program;

typedef struct or_tensor {
    int32_t channels, height, width;
    float* values; /* NCHW, batch 1 */
} or_tensor;

/* Scalar arithmetic of the profile (det_math.hpp). */
float or_exp(float x);
float or_sigmoid(float x);
float or_ldexp(float value, int exponent);
int or_frexp_exponent(float value);
float or_half_to_float(uint16_t half);
uint16_t or_float_to_half(float value);
int or_int_exponent(float maximum, int bits);
int or_int_quantize(float value, int exponent, int bits);
float or_int_output(long long accumulator, float scale, int exponent, float bias);

/* Per-output-channel weight quantisation (program.cpp:509-535).
 * values: out_channels * in_channels int16, scales: out_channels floats. */
void or_quantize_weights(const float* weights, int32_t out_channels, int32_t in_channels,
                         int32_t weight_bits, int16_t* values, float* scales);

/* Output extent of one node given its input extents (program.cpp:628-700).
 * Returns 0 on success, -1 with a message on an invalid shape. */
int or_output_extent(const or_program* program, const or_node* node, const int32_t* extents,
                     int32_t* out_extent, char* error, size_t error_size);

/* Runs the program (run_cpu, program.cpp:702-820). Outputs are allocated with
 * malloc in program.outputs order; free them with or_free. Returns 0 on success. */
int or_run(const or_program* program, const or_tensor* inputs, or_tensor* outputs,
           char* error, size_t error_size);

void or_free(void* pointer);

#ifdef __cplusplus
}
#endif

#endif
