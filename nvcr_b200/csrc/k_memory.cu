// Memory-bound kernels of the intconv.v1 executor: the FP16 stage boundary,
// single-operation elementwise ops, exact data movement and the FP32 conv.
// Each element is one IEEE operation with an _rn intrinsic, so results equal
// the reference's run_cpu bit for bit whatever the thread mapping. Flat ops
// move 16 bytes per thread per step (float4 / 8 x fp16) when the buffers and
// count allow, with grid-stride loops sized to a multiple of the 148 SMs.

#include "exact_math.cuh"
#include "kernels.hpp"
#include "launch.cuh"

#include <cuda_fp16.h>

#include <algorithm>

namespace nvcr_sm100::kernels {
namespace {

constexpr int threads = 256;
constexpr int sm_count = 148;

unsigned int grid_for(std::size_t work_items) {
    const std::size_t blocks = (work_items + threads - 1) / threads;
    const std::size_t cap = static_cast<std::size_t>(sm_count) * 16;
    return static_cast<unsigned int>(blocks < 1 ? 1 : (blocks > cap ? cap : blocks));
}

bool aligned16(const void* p) { return (reinterpret_cast<std::uintptr_t>(p) & 15u) == 0; }

__device__ __forceinline__ std::size_t global_index() {
    return static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
}
__device__ __forceinline__ std::size_t global_stride() {
    return static_cast<std::size_t>(gridDim.x) * blockDim.x;
}

// Exact widening: cvt.f32.f16 represents every binary16 value, subnormals included.
__global__ void half_to_float_kernel(const std::uint16_t* __restrict__ in, float* __restrict__ out,
                                     std::size_t count, int vector) {
    const auto* h = reinterpret_cast<const __half*>(in);
    if (vector) {
        const std::size_t groups = count / 8;
        for (std::size_t g = global_index(); g < groups; g += global_stride()) {
            const uint4 raw = reinterpret_cast<const uint4*>(in)[g];
            const __half2* pairs = reinterpret_cast<const __half2*>(&raw);
            float4 lo, hi;
            float2 f;
            f = __half22float2(pairs[0]); lo.x = f.x; lo.y = f.y;
            f = __half22float2(pairs[1]); lo.z = f.x; lo.w = f.y;
            f = __half22float2(pairs[2]); hi.x = f.x; hi.y = f.y;
            f = __half22float2(pairs[3]); hi.z = f.x; hi.w = f.y;
            reinterpret_cast<float4*>(out)[2 * g] = lo;
            reinterpret_cast<float4*>(out)[2 * g + 1] = hi;
        }
        for (std::size_t i = groups * 8 + global_index(); i < count; i += global_stride()) out[i] = __half2float(h[i]);
        return;
    }
    for (std::size_t i = global_index(); i < count; i += global_stride()) out[i] = __half2float(h[i]);
}

// Round to nearest-even, overflow to infinity, subnormals kept (cvt.rn.f16.f32).
__global__ void float_to_half_kernel(const float* __restrict__ in, std::uint16_t* __restrict__ out,
                                     std::size_t count, int vector) {
    auto* h = reinterpret_cast<__half*>(out);
    if (vector) {
        const std::size_t groups = count / 8;
        for (std::size_t g = global_index(); g < groups; g += global_stride()) {
            const float4 lo = reinterpret_cast<const float4*>(in)[2 * g];
            const float4 hi = reinterpret_cast<const float4*>(in)[2 * g + 1];
            uint4 raw;
            __half2* pairs = reinterpret_cast<__half2*>(&raw);
            pairs[0] = __halves2half2(__float2half_rn(lo.x), __float2half_rn(lo.y));
            pairs[1] = __halves2half2(__float2half_rn(lo.z), __float2half_rn(lo.w));
            pairs[2] = __halves2half2(__float2half_rn(hi.x), __float2half_rn(hi.y));
            pairs[3] = __halves2half2(__float2half_rn(hi.z), __float2half_rn(hi.w));
            reinterpret_cast<uint4*>(out)[g] = raw;
        }
        for (std::size_t i = groups * 8 + global_index(); i < count; i += global_stride()) h[i] = __float2half_rn(in[i]);
        return;
    }
    for (std::size_t i = global_index(); i < count; i += global_stride()) h[i] = __float2half_rn(in[i]);
}

// Generic flat map: f(element index, a) over float4 groups when aligned.
template <typename F>
__global__ void map1_kernel(const float* __restrict__ a, float* __restrict__ out, std::size_t count, int vector, F f) {
    if (vector) {
        const std::size_t groups = count / 4;
        for (std::size_t g = global_index(); g < groups; g += global_stride()) {
            float4 v = reinterpret_cast<const float4*>(a)[g];
            const std::size_t base = 4 * g;
            v.x = f(base, v.x);
            v.y = f(base + 1, v.y);
            v.z = f(base + 2, v.z);
            v.w = f(base + 3, v.w);
            reinterpret_cast<float4*>(out)[g] = v;
        }
        for (std::size_t i = groups * 4 + global_index(); i < count; i += global_stride()) out[i] = f(i, a[i]);
        return;
    }
    for (std::size_t i = global_index(); i < count; i += global_stride()) out[i] = f(i, a[i]);
}

template <typename F>
__global__ void map2_kernel(const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ out,
                            std::size_t count, int vector, F f) {
    if (vector) {
        const std::size_t groups = count / 4;
        for (std::size_t g = global_index(); g < groups; g += global_stride()) {
            float4 x = reinterpret_cast<const float4*>(a)[g];
            const float4 y = reinterpret_cast<const float4*>(b)[g];
            x.x = f(x.x, y.x);
            x.y = f(x.y, y.y);
            x.z = f(x.z, y.z);
            x.w = f(x.w, y.w);
            reinterpret_cast<float4*>(out)[g] = x;
        }
        for (std::size_t i = groups * 4 + global_index(); i < count; i += global_stride()) out[i] = f(a[i], b[i]);
        return;
    }
    for (std::size_t i = global_index(); i < count; i += global_stride()) out[i] = f(a[i], b[i]);
}

struct MulOp {
    __device__ float operator()(float x, float y) const { return __fmul_rn(x, y); }
};
struct AddOp {
    __device__ float operator()(float x, float y) const { return __fadd_rn(x, y); }
};
struct MulScalarOp {
    float s;
    __device__ float operator()(std::size_t, float x) const { return __fmul_rn(x, s); }
};
struct SigmoidOp {
    __device__ float operator()(std::size_t, float x) const { return profile_sigmoid(x); }
};
// x < lo ? lo : (x > hi ? hi : x); a NaN passes through.
struct ClampOp {
    float lo, hi;
    __device__ float operator()(std::size_t, float x) const { return x < lo ? lo : (x > hi ? hi : x); }
};
struct ScaleChannelsOp {
    const float* scale;
    std::size_t plane;
    __device__ float operator()(std::size_t i, float x) const { return __fmul_rn(x, __ldg(scale + i / plane)); }
};

__global__ void crop_kernel(const float* __restrict__ in, float* __restrict__ out, int channels, int out_h,
                            int out_w, int in_h, int in_w) {
    const std::size_t count = static_cast<std::size_t>(channels) * out_h * out_w;
    for (std::size_t i = global_index(); i < count; i += global_stride()) {
        const int x = static_cast<int>(i % out_w);
        const std::size_t row = i / out_w;
        const int y = static_cast<int>(row % out_h);
        const std::size_t c = row / out_h;
        out[i] = in[(c * in_h + y) * in_w + x];
    }
}

// CRD depth_to_space: out[c][y][x] = in[c b^2 + (y % b) b + x % b][y / b][x / b].
__global__ void depth_to_space_kernel(const float* __restrict__ in, float* __restrict__ out, int channels,
                                      int out_h, int out_w, int in_h, int in_w, int block) {
    const std::size_t count = static_cast<std::size_t>(channels) * out_h * out_w;
    for (std::size_t i = global_index(); i < count; i += global_stride()) {
        const int x = static_cast<int>(i % out_w);
        const std::size_t row = i / out_w;
        const int y = static_cast<int>(row % out_h);
        const int c = static_cast<int>(row / out_h);
        const int source = c * block * block + (y % block) * block + x % block;
        out[i] = in[(static_cast<std::size_t>(source) * in_h + y / block) * in_w + x / block];
    }
}

// PixelUnshuffle order: out[c b^2 + i b + j][y][x] = in[c][y b + i][x b + j].
__global__ void space_to_depth_kernel(const float* __restrict__ in, float* __restrict__ out, int channels,
                                      int out_h, int out_w, int in_h, int in_w, int block) {
    const std::size_t count = static_cast<std::size_t>(channels) * out_h * out_w;
    for (std::size_t i = global_index(); i < count; i += global_stride()) {
        const int x = static_cast<int>(i % out_w);
        const std::size_t row = i / out_w;
        const int y = static_cast<int>(row % out_h);
        const int c = static_cast<int>(row / out_h);
        const int source = c / (block * block);
        const int oy = (c / block) % block;
        const int ox = c % block;
        out[i] = in[(static_cast<std::size_t>(source) * in_h + y * block + oy) * in_w + x * block + ox];
    }
}

// im2col: out[(c kh + ky) kw + kx][oy][ox] = in[c][oy sy - pt + ky][ox sx - pl + kx], zero outside.
__global__ void im2col_kernel(const float* __restrict__ in, float* __restrict__ out, int channels, int out_h,
                              int out_w, int in_h, int in_w, Window w) {
    const std::size_t count = static_cast<std::size_t>(channels) * out_h * out_w;
    const int taps = w.kernel_h * w.kernel_w;
    for (std::size_t i = global_index(); i < count; i += global_stride()) {
        const int x = static_cast<int>(i % out_w);
        const std::size_t row = i / out_w;
        const int y = static_cast<int>(row % out_h);
        const int c = static_cast<int>(row / out_h);
        const int source = c / taps;
        const int ky = (c % taps) / w.kernel_w;
        const int kx = c % w.kernel_w;
        const int iy = y * w.stride_y - w.pad_top + ky;
        const int ix = x * w.stride_x - w.pad_left + kx;
        out[i] = iy >= 0 && iy < in_h && ix >= 0 && ix < in_w
            ? in[(static_cast<std::size_t>(source) * in_h + iy) * in_w + ix]
            : 0.0f;
    }
}

// FP32 conv, one thread per output: acc = bias, then for each input channel of
// the group, each kernel row and column, acc = fma(w, x, acc) with x = 0 on
// padding taps (the padding fma can still turn -0 into +0, so it is kept).
__global__ void conv_fp32_kernel(const float* __restrict__ weights, const float* __restrict__ bias,
                                 const float* __restrict__ in, float* __restrict__ out, ConvShape s) {
    const std::size_t count = static_cast<std::size_t>(s.out_channels) * s.out_h * s.out_w;
    const int group_inputs = s.depthwise ? 1 : s.in_channels;
    const int taps = s.window.kernel_h * s.window.kernel_w;
    for (std::size_t i = global_index(); i < count; i += global_stride()) {
        const int ox = static_cast<int>(i % s.out_w);
        const std::size_t row = i / s.out_w;
        const int oy = static_cast<int>(row % s.out_h);
        const int oc = static_cast<int>(row / s.out_h);
        float acc = __ldg(bias + oc);
        const int iy0 = oy * s.window.stride_y - s.window.pad_top;
        const int ix0 = ox * s.window.stride_x - s.window.pad_left;
        for (int local = 0; local < group_inputs; ++local) {
            const int ic = s.depthwise ? oc : local;
            const float* plane = in + static_cast<std::size_t>(ic) * s.in_h * s.in_w;
            const float* kernel = weights + (static_cast<std::size_t>(oc) * group_inputs + local) * taps;
            for (int ky = 0; ky < s.window.kernel_h; ++ky) {
                const int iy = iy0 + ky;
                const bool row_inside = iy >= 0 && iy < s.in_h;
                for (int kx = 0; kx < s.window.kernel_w; ++kx) {
                    const int ix = ix0 + kx;
                    const float x = row_inside && ix >= 0 && ix < s.in_w
                        ? plane[static_cast<std::size_t>(iy) * s.in_w + ix] : 0.0f;
                    acc = __fmaf_rn(__ldg(kernel + ky * s.window.kernel_w + kx), x, acc);
                }
            }
        }
        out[i] = acc;
    }
}

// Depthwise 3x3, stride 1, pad 1: a 32 x 32 output tile of one channel plane
// per block from a 34 x 34 input tile in shared memory; each thread computes a
// column of four outputs. Same fma order as conv_fp32_kernel (bias, then row,
// column; padding taps multiply zeros).
constexpr int dw_tile = 32;
__global__ void __launch_bounds__(256) depthwise3x3_kernel(const float* __restrict__ weights,
                                                           const float* __restrict__ bias,
                                                           const float* __restrict__ in, float* __restrict__ out,
                                                           int height, int width) {
    __shared__ float tile[dw_tile + 2][dw_tile + 3];
    const int c = blockIdx.z;
    const int x0 = blockIdx.x * dw_tile;
    const int y0 = blockIdx.y * dw_tile;
    const float* plane = in + static_cast<std::size_t>(c) * height * width;
    for (int i = threadIdx.x; i < (dw_tile + 2) * (dw_tile + 2); i += 256) {
        const int ty = i / (dw_tile + 2);
        const int tx = i - ty * (dw_tile + 2);
        const int y = y0 + ty - 1;
        const int x = x0 + tx - 1;
        tile[ty][tx] = (y >= 0 && y < height && x >= 0 && x < width) ? __ldg(plane + static_cast<std::size_t>(y) * width + x)
                                                                     : 0.0f;
    }
    float w[9];
#pragma unroll
    for (int k = 0; k < 9; ++k) w[k] = __ldg(weights + static_cast<std::size_t>(c) * 9 + k);
    const float b = __ldg(bias + c);
    __syncthreads();
    const int tx = threadIdx.x & 31;
    const int ty = (threadIdx.x >> 5) * 4;  // four output rows per thread
    const int x = x0 + tx;
    if (x >= width) return;
    float column[6][3];
#pragma unroll
    for (int r = 0; r < 6; ++r) {
#pragma unroll
        for (int k = 0; k < 3; ++k) column[r][k] = tile[ty + r][tx + k];
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const int y = y0 + ty + r;
        if (y >= height) break;
        float acc = b;
#pragma unroll
        for (int ky = 0; ky < 3; ++ky) {
#pragma unroll
            for (int kx = 0; kx < 3; ++kx) acc = __fmaf_rn(w[3 * ky + kx], column[r + ky][kx], acc);
        }
        out[(static_cast<std::size_t>(c) * height + y) * width + x] = acc;
    }
}

// The same depthwise 3x3 on channel-innermost tensors ([H][W][c_pad] FP32,
// padding channels zero, the layout an integer conv reads its source in). A
// block takes an 8 x 32 output tile of one 32-channel slab: it stages the
// 10 x 34 input halo of the slab in shared memory (each pixel's 32 channels
// as 128-byte runs, 36 floats apart so the reads below are conflict-free),
// then thread (x, quad) computes output rows 0..7 of column x for channels
// 4 quad .. 4 quad + 3 with the same fma order as conv_fp32_kernel (bias, then
// row, column; padding taps multiply zeros); padding channels stay zero. Each
// pixel's max |x| over the slab (bit patterns: non-negative floats order as
// their bits; +inf for a non-finite value) goes into the zeroed maxima by an
// atomic max, so the slabs combine.
constexpr int dws_rows = 8;
constexpr int dws_cols = 32;
constexpr int dws_slab = 32;
constexpr int dws_stride = dws_slab + 4;  // floats per staged pixel

__global__ void __launch_bounds__(256) depthwise3x3_staged_kernel(const float* __restrict__ weights,
                                                                  const float* __restrict__ bias, int channels,
                                                                  int c_pad, const float* __restrict__ in,
                                                                  float* __restrict__ out,
                                                                  float* __restrict__ pixel_max, int height,
                                                                  int width) {
    grid_dependency_wait();  // the input may come from the kernel before
    launch_dependents();
    __shared__ __align__(16) float tile[(dws_rows + 2) * (dws_cols + 2) * dws_stride];
    const int x0 = static_cast<int>(blockIdx.x) * dws_cols;
    const int y0 = static_cast<int>(blockIdx.y) * dws_rows;
    const int c0 = static_cast<int>(blockIdx.z) * dws_slab;
    constexpr int halo_pixels = (dws_rows + 2) * (dws_cols + 2);
    // All of a thread's halo loads are in flight before any shared-memory store.
    constexpr int halo_loads = (halo_pixels * 8 + 255) / 256;
    float4 staged[halo_loads];
#pragma unroll
    for (int u = 0; u < halo_loads; ++u) {
        const int i = static_cast<int>(threadIdx.x) + 256 * u;
        const int pixel = i >> 3;
        const int ty = pixel / (dws_cols + 2);
        const int tx = pixel - ty * (dws_cols + 2);
        const int y = y0 + ty - 1;
        const int x = x0 + tx - 1;
        staged[u] = (i < halo_pixels * 8 && y >= 0 && y < height && x >= 0 && x < width)
            ? __ldg(reinterpret_cast<const float4*>(in + (static_cast<std::size_t>(y) * width + x) * c_pad + c0) + (i & 7))
            : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
#pragma unroll
    for (int u = 0; u < halo_loads; ++u) {
        const int i = static_cast<int>(threadIdx.x) + 256 * u;
        if (i < halo_pixels * 8) *reinterpret_cast<float4*>(tile + (i >> 3) * dws_stride + 4 * (i & 7)) = staged[u];
    }
    const int quad = threadIdx.x & 7;
    const int col = threadIdx.x >> 3;  // 0..31
    float w[4][9];
    float b[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int c = c0 + 4 * quad + j;
#pragma unroll
        for (int k = 0; k < 9; ++k) w[j][k] = c < channels ? __ldg(weights + static_cast<std::size_t>(c) * 9 + k) : 0.0f;
        b[j] = c < channels ? __ldg(bias + c) : 0.0f;
    }
    __syncthreads();
    const int x = x0 + col;
    // window[r][kx]: staged input row r of columns col .. col + 2 (4 channels each).
    float4 window[3][3];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
#pragma unroll
        for (int kx = 0; kx < 3; ++kx) {
            window[r][kx] = *reinterpret_cast<const float4*>(tile + (r * (dws_cols + 2) + col + kx) * dws_stride + 4 * quad);
        }
    }
#pragma unroll
    for (int r = 0; r < dws_rows; ++r) {
#pragma unroll
        for (int kx = 0; kx < 3; ++kx) {
            window[2][kx] =
                *reinterpret_cast<const float4*>(tile + ((r + 2) * (dws_cols + 2) + col + kx) * dws_stride + 4 * quad);
        }
        const int y = y0 + r;
        float acc[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            acc[j] = b[j];
#pragma unroll
            for (int ky = 0; ky < 3; ++ky) {
#pragma unroll
                for (int kx = 0; kx < 3; ++kx) {
                    const float4& v = window[ky][kx];
                    const float in_value = j == 0 ? v.x : (j == 1 ? v.y : (j == 2 ? v.z : v.w));
                    acc[j] = __fmaf_rn(w[j][3 * ky + kx], in_value, acc[j]);
                }
            }
            if (c0 + 4 * quad + j >= channels) acc[j] = 0.0f;
        }
        std::uint32_t bits = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) bits = max(bits, __float_as_uint(acc[j]) & 0x7fffffffu);
        // The eight quads of a pixel are lanes 8 m .. 8 m + 7 of the warp.
#pragma unroll
        for (int offset = 4; offset > 0; offset >>= 1) bits = max(bits, __shfl_xor_sync(0xffffffffu, bits, offset));
        if (y < height && x < width) {
            *(reinterpret_cast<float4*>(out + (static_cast<std::size_t>(y) * width + x) * c_pad + c0) + quad) =
                make_float4(acc[0], acc[1], acc[2], acc[3]);
            if (quad == 0) {
                const std::uint32_t m = bits >= 0x7f800000u ? 0x7f800000u : bits;
                atomicMax(reinterpret_cast<unsigned int*>(pixel_max) + static_cast<std::size_t>(y) * width + x, m);
            }
        }
#pragma unroll
        for (int kx = 0; kx < 3; ++kx) {
            window[0][kx] = window[1][kx];
            window[1][kx] = window[2][kx];
        }
    }
}

}  // namespace

namespace {
// Zeroes `count` floats after the kernels before it in the stream finish (it
// may be launched early, overlapped with them, like the kernels that follow).
__global__ void __launch_bounds__(256) zero_floats_kernel(float* __restrict__ out, std::size_t count) {
    grid_dependency_wait();
    launch_dependents();
    for (std::size_t i = static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
         i += static_cast<std::size_t>(gridDim.x) * blockDim.x) {
        out[i] = 0.0f;
    }
}
}  // namespace

cudaError_t zero_floats(float* out, std::size_t count, cudaStream_t stream) {
    if (count == 0) return cudaSuccess;
    const unsigned blocks = static_cast<unsigned>(std::min<std::size_t>((count + 255) / 256, 4 * 148));
    return launch_overlapped(zero_floats_kernel, dim3(blocks), dim3(256), 0, stream, out, count);
}

cudaError_t depthwise3x3_staged(const float* weights, const float* bias, int channels, int c_pad, const float* in,
                                float* out, float* pixel_max, int height, int width, cudaStream_t stream) {
    if (height <= 0 || width <= 0) return cudaSuccess;
    if (channels < 1 || channels > c_pad || c_pad % dws_slab != 0 || (reinterpret_cast<std::uintptr_t>(in) & 15u) != 0 ||
        (reinterpret_cast<std::uintptr_t>(out) & 15u) != 0) {
        return cudaErrorInvalidValue;
    }
    const cudaError_t status = zero_floats(pixel_max, static_cast<std::size_t>(height) * width, stream);
    if (status != cudaSuccess) return status;
    const dim3 grid(static_cast<unsigned>((width + dws_cols - 1) / dws_cols),
                    static_cast<unsigned>((height + dws_rows - 1) / dws_rows), static_cast<unsigned>(c_pad / dws_slab));
    return launch_overlapped(depthwise3x3_staged_kernel, grid, dim3(256), 0, stream, weights, bias, channels, c_pad, in,
                             out, pixel_max, height, width);
}

cudaError_t half_to_float(const std::uint16_t* in, float* out, std::size_t count, cudaStream_t stream) {
    if (count == 0) return cudaSuccess;
    const int vector = aligned16(in) && aligned16(out);
    half_to_float_kernel<<<grid_for(vector ? count / 8 + 1 : count), threads, 0, stream>>>(in, out, count, vector);
    return cudaGetLastError();
}

cudaError_t float_to_half(const float* in, std::uint16_t* out, std::size_t count, cudaStream_t stream) {
    if (count == 0) return cudaSuccess;
    const int vector = aligned16(in) && aligned16(out);
    float_to_half_kernel<<<grid_for(vector ? count / 8 + 1 : count), threads, 0, stream>>>(in, out, count, vector);
    return cudaGetLastError();
}

cudaError_t binary(Binary op, const float* a, const float* b, float* out, std::size_t count, cudaStream_t stream) {
    if (count == 0) return cudaSuccess;
    const int vector = aligned16(a) && aligned16(b) && aligned16(out);
    const unsigned int grid = grid_for(vector ? count / 4 + 1 : count);
    if (op == Binary::mul) {
        map2_kernel<<<grid, threads, 0, stream>>>(a, b, out, count, vector, MulOp{});
    } else {
        map2_kernel<<<grid, threads, 0, stream>>>(a, b, out, count, vector, AddOp{});
    }
    return cudaGetLastError();
}

cudaError_t mul_scalar(const float* a, float scalar, float* out, std::size_t count, cudaStream_t stream) {
    if (count == 0) return cudaSuccess;
    const int vector = aligned16(a) && aligned16(out);
    map1_kernel<<<grid_for(vector ? count / 4 + 1 : count), threads, 0, stream>>>(a, out, count, vector,
                                                                                  MulScalarOp{scalar});
    return cudaGetLastError();
}

cudaError_t sigmoid(const float* a, float* out, std::size_t count, cudaStream_t stream) {
    if (count == 0) return cudaSuccess;
    const int vector = aligned16(a) && aligned16(out);
    map1_kernel<<<grid_for(vector ? count / 4 + 1 : count), threads, 0, stream>>>(a, out, count, vector, SigmoidOp{});
    return cudaGetLastError();
}

cudaError_t scale_channels(const float* a, const float* scale, float* out, std::size_t count, std::size_t plane,
                           cudaStream_t stream) {
    if (count == 0) return cudaSuccess;
    const int vector = aligned16(a) && aligned16(out);
    map1_kernel<<<grid_for(vector ? count / 4 + 1 : count), threads, 0, stream>>>(
        a, out, count, vector, ScaleChannelsOp{scale, plane});
    return cudaGetLastError();
}

cudaError_t clamp(const float* a, float lo, float hi, float* out, std::size_t count, cudaStream_t stream) {
    if (count == 0) return cudaSuccess;
    const int vector = aligned16(a) && aligned16(out);
    map1_kernel<<<grid_for(vector ? count / 4 + 1 : count), threads, 0, stream>>>(a, out, count, vector,
                                                                                  ClampOp{lo, hi});
    return cudaGetLastError();
}

cudaError_t chunk_add(const float* in, float* out, std::size_t half, cudaStream_t stream) {
    return binary(Binary::add, in, in + half, out, half, stream);
}

cudaError_t copy(const float* in, float* out, std::size_t count, cudaStream_t stream) {
    if (count == 0) return cudaSuccess;
    return cudaMemcpyAsync(out, in, count * sizeof(float), cudaMemcpyDeviceToDevice, stream);
}

cudaError_t crop(const float* in, float* out, int channels, int out_h, int out_w, int in_h, int in_w,
                 cudaStream_t stream) {
    const std::size_t count = static_cast<std::size_t>(channels) * out_h * out_w;
    if (count == 0) return cudaSuccess;
    crop_kernel<<<grid_for(count), threads, 0, stream>>>(in, out, channels, out_h, out_w, in_h, in_w);
    return cudaGetLastError();
}

cudaError_t depth_to_space(const float* in, float* out, int out_channels, int out_h, int out_w, int in_h, int in_w,
                           int block, cudaStream_t stream) {
    const std::size_t count = static_cast<std::size_t>(out_channels) * out_h * out_w;
    if (count == 0) return cudaSuccess;
    depth_to_space_kernel<<<grid_for(count), threads, 0, stream>>>(in, out, out_channels, out_h, out_w, in_h, in_w,
                                                                   block);
    return cudaGetLastError();
}

cudaError_t space_to_depth(const float* in, float* out, int out_channels, int out_h, int out_w, int in_h, int in_w,
                           int block, cudaStream_t stream) {
    const std::size_t count = static_cast<std::size_t>(out_channels) * out_h * out_w;
    if (count == 0) return cudaSuccess;
    space_to_depth_kernel<<<grid_for(count), threads, 0, stream>>>(in, out, out_channels, out_h, out_w, in_h, in_w,
                                                                   block);
    return cudaGetLastError();
}

cudaError_t im2col(const float* in, float* out, int out_channels, int out_h, int out_w, int in_h, int in_w,
                   Window window, cudaStream_t stream) {
    const std::size_t count = static_cast<std::size_t>(out_channels) * out_h * out_w;
    if (count == 0) return cudaSuccess;
    im2col_kernel<<<grid_for(count), threads, 0, stream>>>(in, out, out_channels, out_h, out_w, in_h, in_w, window);
    return cudaGetLastError();
}

cudaError_t conv_fp32(const float* weights, const float* bias, const float* in, float* out, ConvShape shape,
                      cudaStream_t stream) {
    const std::size_t count = static_cast<std::size_t>(shape.out_channels) * shape.out_h * shape.out_w;
    if (count == 0) return cudaSuccess;
    const Window& w = shape.window;
    if (shape.depthwise && w.kernel_h == 3 && w.kernel_w == 3 && w.stride_y == 1 && w.stride_x == 1 &&
        w.pad_top == 1 && w.pad_left == 1 && shape.out_h == shape.in_h && shape.out_w == shape.in_w &&
        shape.out_channels == shape.in_channels && shape.out_channels <= 65535) {
        const dim3 grid((shape.out_w + dw_tile - 1) / dw_tile, (shape.out_h + dw_tile - 1) / dw_tile,
                        shape.out_channels);
        depthwise3x3_kernel<<<grid, 256, 0, stream>>>(weights, bias, in, out, shape.in_h, shape.in_w);
        return cudaGetLastError();
    }
    conv_fp32_kernel<<<grid_for(count), threads, 0, stream>>>(weights, bias, in, out, shape);
    return cudaGetLastError();
}

}  // namespace nvcr_sm100::kernels
