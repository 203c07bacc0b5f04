#pragma once

// Launchers of the DCVC-RT inter-stage glue kernels (k_glue.cu). FP16 tensors
// are bit patterns in device memory, batch-first NCHW; every launcher enqueues
// on `stream` and returns the launch status (cudaErrorInvalidValue for the
// shapes and arguments the reference's host ops refuse,
// src/dcvcrt/host_ops.cpp:307-472, 523-556).

#include <cstddef>
#include <cstdint>

#include <cuda_runtime.h>

namespace nvcr_sm100::glue {

cudaError_t build_decode_indexes(const std::uint16_t* scales, std::uint8_t* out, std::size_t count,
                                 float force_zero, cudaStream_t stream);
cudaError_t build_encode_indexes(const std::uint16_t* symbols, const std::uint16_t* scales, std::int16_t* out,
                                 std::size_t count, float force_zero, cudaStream_t stream);
cudaError_t make_mask(std::uint16_t* mask, int batch, int channels, int height, int width, int ways, int stage,
                      cudaStream_t stream);
cudaError_t restore(const std::uint16_t* symbols, const std::uint16_t* means, const std::uint16_t* mask,
                    std::uint16_t* out, int batch, int channels, int height, int width, int ways,
                    cudaStream_t stream);

// `residual` may be null; every other tensor holds `count` values.
cudaError_t process_with_mask(const std::uint16_t* values, const std::uint16_t* scales, const std::uint16_t* means,
                              const std::uint16_t* mask, std::uint16_t* residual, std::uint16_t* symbols,
                              std::uint16_t* reconstructed, std::uint16_t* masked_scales, std::size_t count,
                              float force_zero, cudaStream_t stream);
// Channel quarters (ways 4) or halves (ways 2) of the input shape summed into
// one slice, each multiplied by the mask first unless it is null.
cudaError_t reduce(const std::uint16_t* input, const std::uint16_t* mask, std::uint16_t* output, int batch,
                   int channels, int height, int width, int ways, cudaStream_t stream);

// The elementwise steps between stages; which operands each reads is in
// glue_elements.cuh (a: the tensor updated or written; b: the second operand,
// which clamp_reciprocal_with_quant also updates (a is its quant step, b its
// values); c: the third operand; q: the int8 tensor of round_to_int8 /
// int8_to_half).
enum class PointwiseOp : int {
    round_to_int8,
    int8_to_half,
    clamp_min,
    clamp_reciprocal_with_quant,
    add_in_place,
    multiply_broadcast,
    add_and_multiply,
};
cudaError_t pointwise(PointwiseOp op, std::uint16_t* a, std::uint16_t* b, const std::uint16_t* c,
                      std::int8_t* q, std::size_t count, float scalar, std::size_t spatial_count, cudaStream_t stream);
cudaError_t replicate_pad(const std::uint16_t* input, std::uint16_t* output, int batch, int channels, int height,
                          int width, int padded_height, int padded_width, cudaStream_t stream);
cudaError_t crop_spatial(const std::uint16_t* input, std::uint16_t* output, int batch, int channels, int height,
                         int width, int out_height, int out_width, cudaStream_t stream);

// RGB24 (interleaved) or YUV 4:2:0 8-bit (planar, even size) to a padded
// 3-plane YCbCr FP16 picture, edges replicated.
cudaError_t to_ycbcr_padded(const std::uint8_t* input, int width, int height, std::uint16_t* output, int padded_height,
                            int padded_width, bool yuv420, cudaStream_t stream);
// A 1 x 3 x height x width YCbCr FP16 picture to the visible (even) YUV 4:2:0 8-bit planes.
cudaError_t ycbcr_padded_to_yuv420p8(const std::uint16_t* input, int batch, int channels, int height, int width,
                                     int visible_width, int visible_height, std::uint8_t* output, cudaStream_t stream);

}  // namespace nvcr_sm100::glue
