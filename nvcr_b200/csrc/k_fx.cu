// nvcr.fx.v1 kernels: the profile's integer ops (docs/spec/numerics-fx-v1.md
// section 4; reference CPU arithmetic src/deterministic/fx.cpp) on batch-1
// NCHW int32 tensors. Every product fits int32 or is widened before it is
// formed, and every sum is int64, so the results are the reference's integers.
//
// All kernels are HBM-bound elementwise or gather work except the gemm, whose
// inner product this first version runs on the CUDA cores (a 32 x 32 -> 64-bit
// multiply-add per tap): each thread owns one pixel and four output groups,
// computes the rounded, saturated input digit once per input channel and
// reuses it for all 4 * group rows.
#include "fx_kernels.hpp"

#include <algorithm>

namespace nvcr_sm100::fx::kernels {
namespace {

constexpr int threads = 256;
constexpr std::int64_t digit2_max = 32639;
constexpr std::int64_t stored_max = std::int64_t{1} << 30;
constexpr std::int64_t gemm_limit = (std::int64_t{1} << 29) - 1;

unsigned grid_for(std::size_t count) {
    return static_cast<unsigned>(std::max<std::size_t>(1, std::min<std::size_t>((count + threads - 1) / threads,
                                                                                  148 * 16)));
}

// rsr(a, s) = a for s = 0, floor((a + 2^(s-1)) / 2^s) otherwise (>> on a signed
// operand is an arithmetic shift in CUDA C++).
__device__ __forceinline__ std::int64_t rsr(std::int64_t a, int s) {
    return s == 0 ? a : (a + (std::int64_t{1} << (s - 1))) >> s;
}

__device__ __forceinline__ std::int64_t delta_act(std::int64_t r, const Table& table) {
    const std::int64_t base = r > 0 ? r : 0;
    if (r < -table.h || r > table.h) return base;
    return base + table.dc[(r + table.h) >> table.shift];
}

__device__ __forceinline__ bool outside_stored(std::int64_t v) { return v > stored_max || v < -stored_max; }

__device__ __forceinline__ void record(unsigned long long* failure, unsigned long long key) { atomicMin(failure, key); }

__global__ void check_input_kernel(const std::int32_t* __restrict__ x, std::size_t count, unsigned long long base,
                                   unsigned long long* failure) {
    for (std::size_t i = static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
         i += static_cast<std::size_t>(gridDim.x) * blockDim.x) {
        if (outside_stored(x[i])) record(failure, (base + i) << 1);
    }
}

constexpr int gemm_pixels = 128;  // threads per block, one pixel each
constexpr int gemm_groups = 4;    // output groups per thread

template <int G>
__global__ void __launch_bounds__(gemm_pixels) gemm_kernel(GemmArgs a, unsigned long long node_key,
                                                           unsigned long long* failure) {
    const std::size_t p = static_cast<std::size_t>(blockIdx.x) * gemm_pixels + threadIdx.x;
    if (p >= a.pixels) return;
    constexpr int rows = gemm_groups * G;
    // Group tiles stride over gridDim.y (at most 65535), so any row count runs.
    for (int g0 = static_cast<int>(blockIdx.y) * gemm_groups; g0 < a.groups;
         g0 += static_cast<int>(gridDim.y) * gemm_groups) {
        const int owned = min(gemm_groups, a.groups - g0);  // >= 1 inside the loop
        std::int64_t acc[rows];
#pragma unroll
        for (int r = 0; r < rows; ++r) acc[r] = 0;
        const std::int16_t* w = a.weights + static_cast<std::size_t>(g0) * G * a.in_channels;
        for (int k = 0; k < a.in_channels; ++k) {
            std::int64_t digit = rsr(a.x[static_cast<std::size_t>(k) * a.pixels + p], a.input_shift);
            digit = digit > digit2_max ? digit2_max : digit < -digit2_max ? -digit2_max : digit;
            const int xi = static_cast<int>(digit);
#pragma unroll
            for (int r = 0; r < rows; ++r) {
                if (r < owned * G) {
                    const int wk = w[static_cast<std::size_t>(r) * a.in_channels + k];
                    acc[r] += static_cast<std::int64_t>(wk) * xi;
                }
            }
        }
#pragma unroll
        for (int gi = 0; gi < gemm_groups; ++gi) {
            if (gi < owned) {
                const int g = g0 + gi;
                const unsigned long long position = static_cast<unsigned long long>(p) * a.groups + g;
                std::int64_t sum = 0;
#pragma unroll
                for (int j = 0; j < G; ++j) {
                    const int o = g * G + j;
                    const std::int64_t r = rsr(acc[gi * G + j] + a.bias[o], a.shifts[o]);
                    if (r >= gemm_limit || r <= -gemm_limit) record(failure, node_key | (position << 1));
                    sum += a.table.dc != nullptr ? delta_act(r, a.table) : r;
                }
                const std::size_t at = static_cast<std::size_t>(g) * a.pixels + p;
                if (a.residual0 != nullptr) sum += a.residual0[at];
                if (a.residual1 != nullptr) sum += a.residual1[at];
                if (outside_stored(sum)) record(failure, node_key | (position << 1) | 1u);
                a.y[at] = static_cast<std::int32_t>(sum);
            }
        }
    }
}

__global__ void depthwise3x3_kernel(const std::int32_t* __restrict__ x, int channels, int height, int width,
                                    const std::int32_t* __restrict__ weights, const std::int64_t* __restrict__ bias,
                                    const std::int32_t* __restrict__ shifts, std::int32_t* __restrict__ y,
                                    unsigned long long node_key, unsigned long long* failure) {
    const std::size_t plane = static_cast<std::size_t>(height) * width;
    const std::size_t count = plane * channels;
    for (std::size_t i = static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
         i += static_cast<std::size_t>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(i / plane);
        const int row = static_cast<int>((i % plane) / width);
        const int col = static_cast<int>(i % width);
        const std::int32_t* src = x + static_cast<std::size_t>(c) * plane;
        const std::int32_t* taps = weights + static_cast<std::size_t>(c) * 9;
        std::int64_t acc = bias[c];
#pragma unroll
        for (int ti = 0; ti < 3; ++ti) {
            const int yy = row + ti - 1;
            if (yy < 0 || yy >= height) continue;
#pragma unroll
            for (int tj = 0; tj < 3; ++tj) {
                const int xx = col + tj - 1;
                if (xx < 0 || xx >= width) continue;
                acc += static_cast<std::int64_t>(taps[ti * 3 + tj]) * src[static_cast<std::size_t>(yy) * width + xx];
            }
        }
        const std::int64_t v = rsr(acc, shifts[c]);
        if (outside_stored(v)) record(failure, node_key | (static_cast<unsigned long long>(i) << 1));
        y[i] = static_cast<std::int32_t>(v);
    }
}

__global__ void mul_kernel(const std::int32_t* __restrict__ a, int channels, std::size_t plane,
                           const std::int32_t* __restrict__ b, int b_channels, std::size_t b_plane, int shift,
                           std::int32_t* __restrict__ y, unsigned long long node_key, unsigned long long* failure) {
    const std::size_t count = plane * channels;
    for (std::size_t i = static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
         i += static_cast<std::size_t>(gridDim.x) * blockDim.x) {
        const std::size_t c = b_channels == 1 ? 0 : i / plane;
        const std::size_t p = b_plane == 1 ? 0 : i % plane;
        const std::int64_t v = rsr(static_cast<std::int64_t>(a[i]) * b[c * b_plane + p], shift);
        if (outside_stored(v)) record(failure, node_key | (static_cast<unsigned long long>(i) << 1));
        y[i] = static_cast<std::int32_t>(v);
    }
}

__global__ void affine_kernel(const std::int32_t* __restrict__ x, std::size_t count, std::int64_t alpha,
                              std::int64_t beta, int shift, std::int32_t* __restrict__ y, unsigned long long node_key,
                              unsigned long long* failure) {
    for (std::size_t i = static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
         i += static_cast<std::size_t>(gridDim.x) * blockDim.x) {
        const std::int64_t v = rsr(alpha * x[i] + beta, shift);
        if (outside_stored(v)) record(failure, node_key | (static_cast<unsigned long long>(i) << 1));
        y[i] = static_cast<std::int32_t>(v);
    }
}

__global__ void add_kernel(const std::int32_t* __restrict__ a, const std::int32_t* __restrict__ b, std::size_t count,
                           std::int32_t* __restrict__ y, unsigned long long node_key, unsigned long long* failure) {
    for (std::size_t i = static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
         i += static_cast<std::size_t>(gridDim.x) * blockDim.x) {
        const std::int64_t v = static_cast<std::int64_t>(a[i]) + b[i];
        if (outside_stored(v)) record(failure, node_key | (static_cast<unsigned long long>(i) << 1));
        y[i] = static_cast<std::int32_t>(v);
    }
}

__global__ void sat_table_kernel(const std::int32_t* __restrict__ x, std::size_t count,
                                 const std::int32_t* __restrict__ table, std::int64_t n, std::int32_t top,
                                 std::int32_t* __restrict__ y) {
    for (std::size_t i = static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
         i += static_cast<std::size_t>(gridDim.x) * blockDim.x) {
        const std::int64_t v = x[i];
        y[i] = v >= n ? top : v < -n ? 0 : table[v + n];
    }
}

__global__ void delta_kernel(const std::int32_t* __restrict__ x, std::size_t count, Table table,
                             std::int32_t* __restrict__ y) {
    for (std::size_t i = static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
         i += static_cast<std::size_t>(gridDim.x) * blockDim.x) {
        y[i] = static_cast<std::int32_t>(delta_act(x[i], table));
    }
}

__global__ void clamp_kernel(const std::int32_t* __restrict__ x, std::size_t count, std::int32_t lo, std::int32_t hi,
                             std::int32_t* __restrict__ y) {
    for (std::size_t i = static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
         i += static_cast<std::size_t>(gridDim.x) * blockDim.x) {
        y[i] = min(max(x[i], lo), hi);
    }
}

// One thread per element of the wide tensor (channels / r^2 at r x the size):
// wide[c][y r + i][x r + j] <-> deep[c r^2 + i r + j][y][x].
__global__ void shuffle_kernel(const std::int32_t* __restrict__ x, int deep_channels, int height, int width, int r,
                               bool up, std::int32_t* __restrict__ y) {
    const std::size_t wide_w = static_cast<std::size_t>(width) * r;
    const std::size_t wide_plane = static_cast<std::size_t>(height) * r * wide_w;
    const std::size_t count = static_cast<std::size_t>(deep_channels) * height * width;
    for (std::size_t w = static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x; w < count;
         w += static_cast<std::size_t>(gridDim.x) * blockDim.x) {
        const std::size_t c = w / wide_plane;
        const std::size_t wy = (w % wide_plane) / wide_w;
        const std::size_t wx = w % wide_w;
        const std::size_t deep_c = c * r * r + (wy % r) * r + (wx % r);
        const std::size_t d = (deep_c * height + wy / r) * width + wx / r;
        if (up) {
            y[w] = x[d];
        } else {
            y[d] = x[w];
        }
    }
}

__global__ void im2col_kernel(const std::int32_t* __restrict__ x, int channels, int height, int width, int k,
                              int stride, int out_h, int out_w, std::int32_t* __restrict__ y) {
    const int pad = k == 3 ? 1 : 0;
    const std::size_t out_plane = static_cast<std::size_t>(out_h) * out_w;
    const std::size_t count = static_cast<std::size_t>(channels) * k * k * out_plane;
    for (std::size_t i = static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
         i += static_cast<std::size_t>(gridDim.x) * blockDim.x) {
        const std::size_t oc = i / out_plane;
        const int oy = static_cast<int>((i % out_plane) / out_w);
        const int ox = static_cast<int>(i % out_w);
        const int c = static_cast<int>(oc / (k * k));
        const int ti = static_cast<int>((oc / k) % k);
        const int tj = static_cast<int>(oc % k);
        const int iy = oy * stride - pad + ti;
        const int ix = ox * stride - pad + tj;
        const bool inside = iy >= 0 && iy < height && ix >= 0 && ix < width;
        y[i] = inside ? x[(static_cast<std::size_t>(c) * height + iy) * width + ix] : 0;
    }
}

__global__ void crop_kernel(const std::int32_t* __restrict__ x, int channels, int height, int width, int out_h,
                            int out_w, std::int32_t* __restrict__ y) {
    const std::size_t out_plane = static_cast<std::size_t>(out_h) * out_w;
    const std::size_t count = out_plane * channels;
    for (std::size_t i = static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
         i += static_cast<std::size_t>(gridDim.x) * blockDim.x) {
        const std::size_t c = i / out_plane;
        const std::size_t row = (i % out_plane) / out_w;
        const std::size_t col = i % out_w;
        y[i] = x[(c * height + row) * width + col];
    }
}

__global__ void param_row_kernel(const std::int32_t* __restrict__ x, const std::int64_t* __restrict__ rows,
                                 int row_count, int channels, std::int32_t* __restrict__ y,
                                 unsigned long long node_key, unsigned long long* failure) {
    const std::int32_t q = x[0];
    if (q < 0 || q >= row_count) {
        if (threadIdx.x == 0 && blockIdx.x == 0) record(failure, node_key);
        return;
    }
    for (int c = static_cast<int>(blockIdx.x * blockDim.x + threadIdx.x); c < channels;
         c += static_cast<int>(gridDim.x * blockDim.x)) {
        y[c] = static_cast<std::int32_t>(rows[static_cast<std::size_t>(q) * channels + c]);
    }
}

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
    const int group_tiles = (args.groups + gemm_groups - 1) / gemm_groups;
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
