// DCVC-RT inter-stage glue on the GPU (exact index build, checkerboard masks,
// restore): grid-stride kernels over glue_elements.cuh, on the caller's
// stream, so the masks and the restore between a decoder's spatial steps stay
// on the device (the reference's host backend runs them on the CPU,
// src/dcvcrt/host_ops.cpp; its TensorRT backend builds indexes on the GPU,
// src/dcvcrt/backend/tensorrt/cuda_ops.cu:421-476, 790-820). All are
// HBM-bound: each reads its inputs once and writes its output once.
#include "glue_elements.cuh"
#include "glue_kernels.hpp"

#include <algorithm>

namespace nvcr_sm100::glue {
namespace {

__constant__ float scale_thresholds[127] = {
#include "scale_thresholds.inc"
};

constexpr int threads = 256;

unsigned grid_for(std::size_t count) {
    return static_cast<unsigned>(std::max<std::size_t>(1, std::min<std::size_t>((count + threads - 1) / threads,
                                                                                  148 * 16)));
}

#define GLUE_GRID_STRIDE(i, count)                                                                   \
    for (std::size_t i = static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < (count); \
         i += static_cast<std::size_t>(gridDim.x) * blockDim.x)

__global__ void decode_index_kernel(const Half* __restrict__ scales, std::uint8_t* __restrict__ out,
                                    std::size_t count, float force_zero) {
    GLUE_GRID_STRIDE(i, count) decode_index(scales, out, force_zero, scale_thresholds, i);
}

__global__ void encode_index_kernel(const Half* __restrict__ symbols, const Half* __restrict__ scales,
                                    std::int16_t* __restrict__ out, std::size_t count, float force_zero) {
    GLUE_GRID_STRIDE(i, count) encode_index(symbols, scales, out, force_zero, scale_thresholds, i);
}

__global__ void mask_kernel(Half* __restrict__ mask, std::size_t count, int channels, int height, int width,
                            int ways, int stage) {
    GLUE_GRID_STRIDE(i, count) {
        if (ways == 4) {
            four_way_mask(mask, channels, height, width, stage, i);
        } else {
            two_way_mask(mask, channels, height, width, stage, i);
        }
    }
}

__global__ void restore_kernel(const Half* __restrict__ symbols, const Half* __restrict__ means,
                               const Half* __restrict__ mask, Half* __restrict__ out, std::size_t part_size,
                               int parts) {
    GLUE_GRID_STRIDE(i, part_size) restore(symbols, means, mask, out, part_size, parts, i);
}

__global__ void process_kernel(const Half* __restrict__ values, const Half* __restrict__ scales,
                               const Half* __restrict__ means, const Half* __restrict__ mask, Half* residual,
                               Half* __restrict__ symbols, Half* __restrict__ reconstructed,
                               Half* __restrict__ masked_scales, std::size_t count, float force_zero) {
    GLUE_GRID_STRIDE(i, count) {
        process_with_mask(values, scales, means, mask, residual, symbols, reconstructed, masked_scales, force_zero, i);
    }
}

__global__ void reduce_kernel(const Half* __restrict__ input, const Half* mask, Half* __restrict__ output,
                              std::size_t part_size, int parts) {
    GLUE_GRID_STRIDE(i, part_size) reduce_parts(input, mask, output, part_size, parts, i);
}

#undef GLUE_GRID_STRIDE

std::size_t volume(int batch, int channels, int height, int width) {
    return static_cast<std::size_t>(batch) * static_cast<std::size_t>(channels) * static_cast<std::size_t>(height) *
        static_cast<std::size_t>(width);
}

}  // namespace

cudaError_t build_decode_indexes(const Half* scales, std::uint8_t* out, std::size_t count, float force_zero,
                                 cudaStream_t stream) {
    if (count == 0 || scales == nullptr || out == nullptr) return cudaErrorInvalidValue;
    decode_index_kernel<<<grid_for(count), threads, 0, stream>>>(scales, out, count, force_zero);
    return cudaGetLastError();
}

cudaError_t build_encode_indexes(const Half* symbols, const Half* scales, std::int16_t* out, std::size_t count,
                                 float force_zero, cudaStream_t stream) {
    if (count == 0 || symbols == nullptr || scales == nullptr || out == nullptr) return cudaErrorInvalidValue;
    encode_index_kernel<<<grid_for(count), threads, 0, stream>>>(symbols, scales, out, count, force_zero);
    return cudaGetLastError();
}

cudaError_t make_mask(Half* mask, int batch, int channels, int height, int width, int ways, int stage,
                      cudaStream_t stream) {
    if (mask == nullptr || !valid_shape(batch, channels, height, width, ways) || stage < 0 || stage >= ways) {
        return cudaErrorInvalidValue;
    }
    const std::size_t count = volume(batch, channels, height, width);
    mask_kernel<<<grid_for(count), threads, 0, stream>>>(mask, count, channels, height, width, ways, stage);
    return cudaGetLastError();
}

cudaError_t restore(const Half* symbols, const Half* means, const Half* mask, Half* out, int batch, int channels,
                    int height, int width, int ways, cudaStream_t stream) {
    if (symbols == nullptr || means == nullptr || mask == nullptr || out == nullptr ||
        !valid_shape(batch, channels, height, width, ways)) {
        return cudaErrorInvalidValue;
    }
    const std::size_t part_size = volume(batch, channels, height, width) / static_cast<std::size_t>(ways);
    restore_kernel<<<grid_for(part_size), threads, 0, stream>>>(symbols, means, mask, out, part_size, ways);
    return cudaGetLastError();
}

cudaError_t process_with_mask(const Half* values, const Half* scales, const Half* means, const Half* mask,
                              Half* residual, Half* symbols, Half* reconstructed, Half* masked_scales,
                              std::size_t count, float force_zero, cudaStream_t stream) {
    if (count == 0 || values == nullptr || scales == nullptr || means == nullptr || mask == nullptr ||
        symbols == nullptr || reconstructed == nullptr || masked_scales == nullptr) {
        return cudaErrorInvalidValue;
    }
    process_kernel<<<grid_for(count), threads, 0, stream>>>(values, scales, means, mask, residual, symbols,
                                                            reconstructed, masked_scales, count, force_zero);
    return cudaGetLastError();
}

cudaError_t reduce(const Half* input, const Half* mask, Half* output, int batch, int channels, int height, int width,
                   int ways, cudaStream_t stream) {
    if (input == nullptr || output == nullptr || !valid_shape(batch, channels, height, width, ways)) {
        return cudaErrorInvalidValue;
    }
    const std::size_t part_size = volume(batch, channels, height, width) / static_cast<std::size_t>(ways);
    reduce_kernel<<<grid_for(part_size), threads, 0, stream>>>(input, mask, output, part_size, ways);
    return cudaGetLastError();
}

}  // namespace nvcr_sm100::glue
