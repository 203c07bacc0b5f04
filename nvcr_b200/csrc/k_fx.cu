// nvcr.fx.v1 kernels: the profile's integer ops (docs/spec/numerics-fx-v1.md
// section 4; reference CPU arithmetic src/deterministic/fx.cpp) on batch-1
// NCHW int32 tensors. Every product fits int32 or is widened before it is
// formed, and every sum is int64, so the results are the reference's integers.
// The work per output value is in fx_elements.cuh; each kernel here is a
// grid-stride loop over it.
//
// All kernels are HBM-bound elementwise or gather work except the gemm, whose
// inner product this first version runs on the CUDA cores (a 32 x 32 -> 64-bit
// multiply-add per tap): each thread owns one pixel and four output groups,
// computes the rounded, saturated input digit once per input channel and
// reuses it for all 4 * group rows.
#include "fx_elements.cuh"
#include "fx_kernels.hpp"

#include <algorithm>

namespace nvcr_sm100::fx::kernels {
namespace {

namespace el = nvcr_sm100::fx::elements;

constexpr int threads = 256;
constexpr int gemm_pixels = 128;  // threads per gemm block, one pixel each

unsigned grid_for(std::size_t count) {
    return static_cast<unsigned>(std::max<std::size_t>(1, std::min<std::size_t>((count + threads - 1) / threads,
                                                                                  148 * 16)));
}

// Notes a stage failure in the run's failure word; the smallest key wins.
struct DeviceRecord {
    unsigned long long* failure;
    __device__ void operator()(unsigned long long key) const { atomicMin(failure, key); }
};

#define FX_GRID_STRIDE(i, count)                                                                 \
    for (std::size_t i = static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < (count); \
         i += static_cast<std::size_t>(gridDim.x) * blockDim.x)

__global__ void check_input_kernel(const std::int32_t* __restrict__ x, std::size_t count, unsigned long long base,
                                   unsigned long long* failure) {
    const DeviceRecord record{failure};
    FX_GRID_STRIDE(i, count) el::check_input(x, i, base, record);
}

template <int G>
__global__ void __launch_bounds__(gemm_pixels) gemm_kernel(GemmArgs a, unsigned long long node_key,
                                                           unsigned long long* failure) {
    const std::size_t p = static_cast<std::size_t>(blockIdx.x) * gemm_pixels + threadIdx.x;
    if (p >= a.pixels) return;
    const DeviceRecord record{failure};
    // Group tiles stride over gridDim.y (at most 65535), so any row count runs.
    for (int g0 = static_cast<int>(blockIdx.y) * el::gemm_groups; g0 < a.groups;
         g0 += static_cast<int>(gridDim.y) * el::gemm_groups) {
        el::gemm_tile<G>(a, p, g0, node_key, record);
    }
}

__global__ void depthwise3x3_kernel(const std::int32_t* __restrict__ x, int channels, int height, int width,
                                    const std::int32_t* __restrict__ weights, const std::int64_t* __restrict__ bias,
                                    const std::int32_t* __restrict__ shifts, std::int32_t* __restrict__ y,
                                    unsigned long long node_key, unsigned long long* failure) {
    const DeviceRecord record{failure};
    const std::size_t count = static_cast<std::size_t>(height) * width * channels;
    FX_GRID_STRIDE(i, count) el::depthwise3x3(x, height, width, weights, bias, shifts, y, i, node_key, record);
}

__global__ void mul_kernel(const std::int32_t* __restrict__ a, int channels, std::size_t plane,
                           const std::int32_t* __restrict__ b, int b_channels, std::size_t b_plane, int shift,
                           std::int32_t* __restrict__ y, unsigned long long node_key, unsigned long long* failure) {
    const DeviceRecord record{failure};
    FX_GRID_STRIDE(i, plane * channels) el::mul(a, plane, b, b_channels, b_plane, shift, y, i, node_key, record);
}

__global__ void affine_kernel(const std::int32_t* __restrict__ x, std::size_t count, std::int64_t alpha,
                              std::int64_t beta, int shift, std::int32_t* __restrict__ y, unsigned long long node_key,
                              unsigned long long* failure) {
    const DeviceRecord record{failure};
    FX_GRID_STRIDE(i, count) el::affine(x, alpha, beta, shift, y, i, node_key, record);
}

__global__ void add_kernel(const std::int32_t* __restrict__ a, const std::int32_t* __restrict__ b, std::size_t count,
                           std::int32_t* __restrict__ y, unsigned long long node_key, unsigned long long* failure) {
    const DeviceRecord record{failure};
    FX_GRID_STRIDE(i, count) el::add(a, b, y, i, node_key, record);
}

__global__ void sat_table_kernel(const std::int32_t* __restrict__ x, std::size_t count,
                                 const std::int32_t* __restrict__ table, std::int64_t n, std::int32_t top,
                                 std::int32_t* __restrict__ y) {
    FX_GRID_STRIDE(i, count) el::sat_table(x, table, n, top, y, i);
}

__global__ void delta_kernel(const std::int32_t* __restrict__ x, std::size_t count, Table table,
                             std::int32_t* __restrict__ y) {
    FX_GRID_STRIDE(i, count) el::delta(x, table, y, i);
}

__global__ void clamp_kernel(const std::int32_t* __restrict__ x, std::size_t count, std::int32_t lo, std::int32_t hi,
                             std::int32_t* __restrict__ y) {
    FX_GRID_STRIDE(i, count) el::clamp(x, lo, hi, y, i);
}

__global__ void shuffle_kernel(const std::int32_t* __restrict__ x, int deep_channels, int height, int width, int r,
                               bool up, std::int32_t* __restrict__ y) {
    FX_GRID_STRIDE(w, static_cast<std::size_t>(deep_channels) * height * width) el::shuffle(x, height, width, r, up, y, w);
}

__global__ void im2col_kernel(const std::int32_t* __restrict__ x, int channels, int height, int width, int k,
                              int stride, int out_h, int out_w, std::int32_t* __restrict__ y) {
    FX_GRID_STRIDE(i, static_cast<std::size_t>(channels) * k * k * out_h * out_w) {
        el::im2col(x, height, width, k, stride, out_h, out_w, y, i);
    }
}

__global__ void crop_kernel(const std::int32_t* __restrict__ x, int channels, int height, int width, int out_h,
                            int out_w, std::int32_t* __restrict__ y) {
    FX_GRID_STRIDE(i, static_cast<std::size_t>(out_h) * out_w * channels) el::crop(x, height, width, out_h, out_w, y, i);
}

__global__ void param_row_kernel(const std::int32_t* __restrict__ x, const std::int64_t* __restrict__ rows,
                                 int row_count, int channels, std::int32_t* __restrict__ y,
                                 unsigned long long node_key, unsigned long long* failure) {
    const DeviceRecord record{failure};
    for (int c = static_cast<int>(blockIdx.x * blockDim.x + threadIdx.x); c < channels;
         c += static_cast<int>(gridDim.x * blockDim.x)) {
        el::param_row(x, rows, row_count, channels, y, c, node_key, record);
    }
}

#undef FX_GRID_STRIDE

}  // namespace

cudaError_t check_input(const std::int32_t* x, std::size_t count, unsigned long long position_base,
                        unsigned long long* failure, cudaStream_t stream) {
    if (count == 0) return cudaSuccess;
    check_input_kernel<<<grid_for(count), threads, 0, stream>>>(x, count, position_base, failure);
    return cudaGetLastError();
}

cudaError_t gemm(const GemmArgs& args, unsigned long long node_key, unsigned long long* failure, cudaStream_t stream) {
    if (args.pixels == 0 || args.groups == 0) return cudaSuccess;
    if (args.in_channels < 1 || (args.group != 1 && args.group != 2 && args.group != 4)) return cudaErrorInvalidValue;
    const std::size_t pixel_tiles = (args.pixels + gemm_pixels - 1) / gemm_pixels;
    const int group_tiles = (args.groups + el::gemm_groups - 1) / el::gemm_groups;
    if (pixel_tiles > 0x7fffffffu) return cudaErrorInvalidValue;
    const dim3 grid(static_cast<unsigned>(pixel_tiles), static_cast<unsigned>(std::min(group_tiles, 65535)));
    switch (args.group) {
    case 1: gemm_kernel<1><<<grid, gemm_pixels, 0, stream>>>(args, node_key, failure); break;
    case 2: gemm_kernel<2><<<grid, gemm_pixels, 0, stream>>>(args, node_key, failure); break;
    default: gemm_kernel<4><<<grid, gemm_pixels, 0, stream>>>(args, node_key, failure); break;
    }
    return cudaGetLastError();
}

cudaError_t depthwise3x3(const std::int32_t* x, int channels, int height, int width, const std::int32_t* weights,
                         const std::int64_t* bias, const std::int32_t* shifts, std::int32_t* y,
                         unsigned long long node_key, unsigned long long* failure, cudaStream_t stream) {
    const std::size_t count = static_cast<std::size_t>(channels) * height * width;
    if (count == 0) return cudaSuccess;
    depthwise3x3_kernel<<<grid_for(count), threads, 0, stream>>>(x, channels, height, width, weights, bias, shifts, y,
                                                                  node_key, failure);
    return cudaGetLastError();
}

cudaError_t mul(const std::int32_t* a, int channels, std::size_t plane, const std::int32_t* b, int b_channels,
                std::size_t b_plane, int shift, std::int32_t* y, unsigned long long node_key,
                unsigned long long* failure, cudaStream_t stream) {
    const std::size_t count = plane * channels;
    if (count == 0) return cudaSuccess;
    mul_kernel<<<grid_for(count), threads, 0, stream>>>(a, channels, plane, b, b_channels, b_plane, shift, y, node_key,
                                                         failure);
    return cudaGetLastError();
}

cudaError_t affine(const std::int32_t* x, std::size_t count, std::int64_t alpha, std::int64_t beta, int shift,
                   std::int32_t* y, unsigned long long node_key, unsigned long long* failure, cudaStream_t stream) {
    if (count == 0) return cudaSuccess;
    affine_kernel<<<grid_for(count), threads, 0, stream>>>(x, count, alpha, beta, shift, y, node_key, failure);
    return cudaGetLastError();
}

cudaError_t add(const std::int32_t* a, const std::int32_t* b, std::size_t count, std::int32_t* y,
                unsigned long long node_key, unsigned long long* failure, cudaStream_t stream) {
    if (count == 0) return cudaSuccess;
    add_kernel<<<grid_for(count), threads, 0, stream>>>(a, b, count, y, node_key, failure);
    return cudaGetLastError();
}

cudaError_t sat_table(const std::int32_t* x, std::size_t count, const std::int32_t* table, std::int64_t n,
                      std::int32_t top, std::int32_t* y, cudaStream_t stream) {
    if (count == 0) return cudaSuccess;
    sat_table_kernel<<<grid_for(count), threads, 0, stream>>>(x, count, table, n, top, y);
    return cudaGetLastError();
}

cudaError_t delta(const std::int32_t* x, std::size_t count, Table table, std::int32_t* y, cudaStream_t stream) {
    if (count == 0) return cudaSuccess;
    if (table.dc == nullptr) return cudaErrorInvalidValue;
    delta_kernel<<<grid_for(count), threads, 0, stream>>>(x, count, table, y);
    return cudaGetLastError();
}

cudaError_t clamp(const std::int32_t* x, std::size_t count, std::int32_t lo, std::int32_t hi, std::int32_t* y,
                  cudaStream_t stream) {
    if (count == 0) return cudaSuccess;
    clamp_kernel<<<grid_for(count), threads, 0, stream>>>(x, count, lo, hi, y);
    return cudaGetLastError();
}

cudaError_t shuffle(const std::int32_t* x, int channels, int height, int width, int factor, bool up, std::int32_t* y,
                    cudaStream_t stream) {
    // The kernel walks the deep tensor's extents: for up the input is deep, for
    // pixel_unshuffle the output is (channels * r^2 at size / r).
    const int r = factor;
    const int deep_channels = up ? channels : channels * r * r;
    const int deep_h = up ? height : height / r;
    const int deep_w = up ? width : width / r;
    const std::size_t count = static_cast<std::size_t>(deep_channels) * deep_h * deep_w;
    if (count == 0) return cudaSuccess;
    shuffle_kernel<<<grid_for(count), threads, 0, stream>>>(x, deep_channels, deep_h, deep_w, r, up, y);
    return cudaGetLastError();
}

cudaError_t im2col(const std::int32_t* x, int channels, int height, int width, int kernel, int stride, int out_h,
                   int out_w, std::int32_t* y, cudaStream_t stream) {
    const std::size_t count = static_cast<std::size_t>(channels) * kernel * kernel * out_h * out_w;
    if (count == 0) return cudaSuccess;
    im2col_kernel<<<grid_for(count), threads, 0, stream>>>(x, channels, height, width, kernel, stride, out_h, out_w, y);
    return cudaGetLastError();
}

cudaError_t crop(const std::int32_t* x, int channels, int height, int width, int out_h, int out_w, std::int32_t* y,
                 cudaStream_t stream) {
    const std::size_t count = static_cast<std::size_t>(channels) * out_h * out_w;
    if (count == 0) return cudaSuccess;
    if (out_h > height || out_w > width) return cudaErrorInvalidValue;
    crop_kernel<<<grid_for(count), threads, 0, stream>>>(x, channels, height, width, out_h, out_w, y);
    return cudaGetLastError();
}

cudaError_t param_row(const std::int32_t* x, const std::int64_t* rows, int row_count, int channels, std::int32_t* y,
                      unsigned long long node_key, unsigned long long* failure, cudaStream_t stream) {
    if (channels < 1) return cudaSuccess;
    param_row_kernel<<<1, threads, 0, stream>>>(x, rows, row_count, channels, y, node_key, failure);
    return cudaGetLastError();
}

}  // namespace nvcr_sm100::fx::kernels
