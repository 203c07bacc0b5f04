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

}  // namespace nvcr_sm100::glue
