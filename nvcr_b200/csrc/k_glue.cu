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

// The elementwise steps, one kernel for all (the op is uniform per launch).
__global__ void pointwise_kernel(PointwiseOp op, Half* a, Half* b, const Half* c, std::int8_t* q,
                                 std::size_t count, float scalar, std::size_t spatial_count) {
    GLUE_GRID_STRIDE(i, count) {
        switch (op) {
        case PointwiseOp::round_to_int8: round_to_int8(a, q, i); break;
        case PointwiseOp::int8_to_half: int8_to_half(q, a, i); break;
        case PointwiseOp::clamp_min: clamp_min(a, scalar, i); break;
        case PointwiseOp::clamp_reciprocal_with_quant: clamp_reciprocal_with_quant(a, b, i); break;
        case PointwiseOp::add_in_place: add_in_place(a, b, i); break;
        case PointwiseOp::multiply_broadcast: multiply_broadcast(a, b, spatial_count, i); break;
        case PointwiseOp::add_and_multiply: add_and_multiply(a, b, c, i); break;
        }
    }
}

__global__ void resize_kernel(const Half* __restrict__ input, Half* __restrict__ output, std::size_t count, int height,
                              int width, int out_h, int out_w) {
    GLUE_GRID_STRIDE(i, count) replicate_or_crop(input, output, height, width, out_h, out_w, i);
}

__global__ void to_ycbcr_kernel(const std::uint8_t* __restrict__ input, int width, int height, Half* __restrict__ output,
                                int out_h, int out_w, bool yuv) {
    GLUE_GRID_STRIDE(i, static_cast<std::size_t>(out_h) * out_w) {
        if (yuv) {
            yuv420p8_to_ycbcr(input, width, height, output, out_h, out_w, i);
        } else {
            rgb24_to_ycbcr(input, width, height, output, out_h, out_w, i);
        }
    }
}

__global__ void to_yuv_kernel(const Half* __restrict__ input, std::size_t plane, std::size_t stride, int width,
                              int height, std::uint8_t* __restrict__ output) {
    const std::size_t y_size = static_cast<std::size_t>(width) * height;
    GLUE_GRID_STRIDE(i, y_size + y_size / 4) {
        if (i < y_size) {
            ycbcr_luma_to_y(input, stride, width, output, i);
        } else {
            ycbcr_chroma_to_uv(input, plane, stride, width, height, output, i - y_size);
        }
    }
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

cudaError_t pointwise(PointwiseOp op, Half* a, Half* b, const Half* c, std::int8_t* q, std::size_t count,
                      float scalar, std::size_t spatial_count, cudaStream_t stream) {
    if (count == 0 || a == nullptr) return cudaErrorInvalidValue;
    const bool needs_b = op == PointwiseOp::clamp_reciprocal_with_quant || op == PointwiseOp::add_in_place ||
        op == PointwiseOp::multiply_broadcast || op == PointwiseOp::add_and_multiply;
    const bool needs_q = op == PointwiseOp::round_to_int8 || op == PointwiseOp::int8_to_half;
    if ((needs_b && b == nullptr) || (op == PointwiseOp::add_and_multiply && c == nullptr) || (needs_q && q == nullptr) ||
        (op == PointwiseOp::multiply_broadcast && spatial_count == 0)) {
        return cudaErrorInvalidValue;
    }
    pointwise_kernel<<<grid_for(count), threads, 0, stream>>>(op, a, b, c, q, count, scalar, spatial_count);
    return cudaGetLastError();
}

cudaError_t replicate_pad(const Half* input, Half* output, int batch, int channels, int height, int width,
                          int padded_height, int padded_width, cudaStream_t stream) {
    if (input == nullptr || output == nullptr || batch <= 0 || channels <= 0 || height <= 0 || width <= 0 ||
        padded_height < height || padded_width < width) {
        return cudaErrorInvalidValue;
    }
    const std::size_t count = static_cast<std::size_t>(batch) * channels * padded_height * padded_width;
    resize_kernel<<<grid_for(count), threads, 0, stream>>>(input, output, count, height, width, padded_height,
                                                           padded_width);
    return cudaGetLastError();
}

cudaError_t crop_spatial(const Half* input, Half* output, int batch, int channels, int height, int width,
                         int out_height, int out_width, cudaStream_t stream) {
    if (input == nullptr || output == nullptr || batch <= 0 || channels <= 0 || height <= 0 || width <= 0 ||
        out_height <= 0 || out_width <= 0 || out_height > height || out_width > width) {
        return cudaErrorInvalidValue;
    }
    const std::size_t count = static_cast<std::size_t>(batch) * channels * out_height * out_width;
    resize_kernel<<<grid_for(count), threads, 0, stream>>>(input, output, count, height, width, out_height, out_width);
    return cudaGetLastError();
}

cudaError_t to_ycbcr_padded(const std::uint8_t* input, int width, int height, Half* output, int padded_height,
                            int padded_width, bool yuv420, cudaStream_t stream) {
    if (input == nullptr || output == nullptr || width <= 0 || height <= 0 || padded_height < height ||
        padded_width < width || (yuv420 && ((width & 1) != 0 || (height & 1) != 0))) {
        return cudaErrorInvalidValue;
    }
    const std::size_t count = static_cast<std::size_t>(padded_height) * padded_width;
    to_ycbcr_kernel<<<grid_for(count), threads, 0, stream>>>(input, width, height, output, padded_height, padded_width,
                                                             yuv420);
    return cudaGetLastError();
}

cudaError_t ycbcr_padded_to_yuv420p8(const Half* input, int batch, int channels, int height, int width,
                                     int visible_width, int visible_height, std::uint8_t* output, cudaStream_t stream) {
    if (input == nullptr || output == nullptr || batch != 1 || channels != 3 || height <= 0 || width <= 0 ||
        visible_width <= 0 || visible_height <= 0 || (visible_width & 1) != 0 || (visible_height & 1) != 0 ||
        visible_width > width || visible_height > height) {
        return cudaErrorInvalidValue;
    }
    const std::size_t y_size = static_cast<std::size_t>(visible_width) * visible_height;
    to_yuv_kernel<<<grid_for(y_size + y_size / 4), threads, 0, stream>>>(
        input, static_cast<std::size_t>(height) * width, static_cast<std::size_t>(width), visible_width,
        visible_height, output);
    return cudaGetLastError();
}

}  // namespace nvcr_sm100::glue
