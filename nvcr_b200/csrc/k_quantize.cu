// Activation quantiser of the integer conv (reference contract: program.hpp:33-36;
// the reference quantises an im2col'd FP32 tensor, program.cpp:416-430 and
// cuda_executor.cu:303-395).
//
// For output position p the exponent e_p comes from the largest magnitude over
// its whole receptive field (C * kh * kw values), so one input pixel quantises
// differently for different positions. The im2col tensor is never built:
//   1. pixel_max: per input pixel, max |x| over channels (+inf when any channel
//      is non-finite, which makes every position that sees the pixel NaN);
//   2. quantize: per output position, e_p = frexp(max over the window) - (bits-1),
//      then q = clamp(rint(ldexp(x, -e_p)), +-L) for every tap, written as int8
//      limbs into [positions][K] matrices (K contiguous, im2col channel order,
//      zero-padded to whole 128-byte rows) that the GEMM's TMA reads.
// Max and integer sums are order-free, so the thread mapping changes no bit.

#include "exact_math.cuh"
#include "kernels.hpp"

#include <climits>

namespace nvcr_sm100::kernels {
namespace {

constexpr int max_threads = 256;

// Block: 32 pixels x 8 channel groups.
__global__ void __launch_bounds__(max_threads) pixel_max_kernel(const float* __restrict__ in, int channels,
                                                                int pixels, float* __restrict__ out) {
    __shared__ float partial[8][32];
    const int lane = threadIdx.x & 31;
    const int group = threadIdx.x >> 5;
    const int pixel = blockIdx.x * 32 + lane;
    float maximum = 0.0f;
    bool finite = true;
    if (pixel < pixels) {
        for (int c = group; c < channels; c += 8) {
            const float x = __ldg(in + static_cast<std::size_t>(c) * pixels + pixel);
            finite = finite && is_finite_value(x);
            maximum = fmaxf(maximum, fabsf(x));
        }
    }
    partial[group][lane] = finite ? maximum : __uint_as_float(0x7f800000u);
    __syncthreads();
    if (group == 0 && pixel < pixels) {
        float m = partial[0][lane];
        for (int g = 1; g < 8; ++g) m = fmaxf(m, partial[g][lane]);
        out[pixel] = m;
    }
}

constexpr int tile_positions = 32;
constexpr int chunk_k = 64;
constexpr int row_pitch = chunk_k + 16;  // bytes per staged row

template <int Bits>
__global__ void __launch_bounds__(max_threads) quantize_kernel(QuantizeArgs a) {
    constexpr bool two_limbs = Bits == 16;
    __shared__ int exponent_of[tile_positions];
    __shared__ __align__(16) std::int8_t staged_high[tile_positions][row_pitch];
    __shared__ __align__(16) std::int8_t staged_low[two_limbs ? tile_positions : 1][row_pitch];
    __shared__ long long partial_terms[8][tile_positions];

    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int p0 = blockIdx.x * tile_positions;
    const int positions = a.out_h * a.out_w;
    const int taps = a.window.kernel_h * a.window.kernel_w;
    const int k_real = a.channels * taps;
    const int p = p0 + lane;
    const bool real_position = p < positions;
    const int oy = real_position ? p / a.out_w : 0;
    const int ox = real_position ? p - oy * a.out_w : 0;
    const int iy0 = oy * a.window.stride_y - a.window.pad_top;
    const int ix0 = ox * a.window.stride_x - a.window.pad_left;

    if (warp == 0) {
        int exponent = INT_MIN;
        if (real_position) {
            float maximum = 0.0f;
            for (int ky = 0; ky < a.window.kernel_h; ++ky) {
                const int iy = iy0 + ky;
                if (iy < 0 || iy >= a.in_h) continue;
                for (int kx = 0; kx < a.window.kernel_w; ++kx) {
                    const int ix = ix0 + kx;
                    if (ix < 0 || ix >= a.in_w) continue;
                    maximum = fmaxf(maximum, __ldg(a.pixel_max + static_cast<std::size_t>(iy) * a.in_w + ix));
                }
            }
            exponent = maximum == __uint_as_float(0x7f800000u) ? INT_MIN : activation_exponent(maximum, Bits);
            a.exponents[p] = exponent;
        }
        exponent_of[lane] = exponent;
    }
    __syncthreads();
    const int exponent = exponent_of[lane];
    const bool live = real_position && exponent != INT_MIN;
    long long high_sum = 0;
    long long low_sum = 0;
    const std::size_t plane = static_cast<std::size_t>(a.in_h) * a.in_w;

    for (int chunk = 0; chunk < a.k_padded; chunk += chunk_k) {
#pragma unroll
        for (int j = 0; j < chunk_k / 8; ++j) {
            const int local = warp * (chunk_k / 8) + j;
            const int k = chunk + local;
            int q = 0;
            const bool real_tap = live && k < k_real;
            if (real_tap) {
                const int c = k / taps;
                const int r = k - c * taps;
                const int ky = r / a.window.kernel_w;
                const int kx = r - ky * a.window.kernel_w;
                const int iy = iy0 + ky;
                const int ix = ix0 + kx;
                const float x = iy >= 0 && iy < a.in_h && ix >= 0 && ix < a.in_w
                    ? __ldg(a.in + static_cast<std::size_t>(c) * plane + static_cast<std::size_t>(iy) * a.in_w + ix)
                    : 0.0f;
                q = quantize_value<Bits>(x, exponent);
            }
            if constexpr (two_limbs) {
                const int h = q >> 8;                      // floor(q / 256), in [-128, 127]
                const int l = real_tap ? (q & 255) - 128 : 0;  // q = 256 h + l + 128
                staged_high[lane][local] = static_cast<std::int8_t>(h);
                staged_low[lane][local] = static_cast<std::int8_t>(l);
                high_sum += h;
                low_sum += l;
            } else {
                staged_high[lane][local] = static_cast<std::int8_t>(q);
                high_sum += q;
            }
        }
        __syncthreads();
        // 32 rows of 64 bytes: 128 threads store 16 bytes each.
        if (threadIdx.x < tile_positions * (chunk_k / 16)) {
            const int row = threadIdx.x / (chunk_k / 16);
            const int part = threadIdx.x % (chunk_k / 16);
            const std::size_t offset = static_cast<std::size_t>(p0 + row) * a.k_padded + chunk + part * 16;
            *reinterpret_cast<int4*>(a.high + offset) = *reinterpret_cast<const int4*>(&staged_high[row][part * 16]);
            if constexpr (two_limbs) {
                *reinterpret_cast<int4*>(a.low + offset) = *reinterpret_cast<const int4*>(&staged_low[row][part * 16]);
            }
        }
        __syncthreads();
    }
    if (a.column_terms != nullptr) {
        partial_terms[warp][lane] = a.high_factor * high_sum + a.low_factor * low_sum;
        __syncthreads();
        if (warp == 0 && real_position) {
            long long total = 0;
            for (int w = 0; w < 8; ++w) total += partial_terms[w][lane];
            a.column_terms[p] = live ? total : 0;
        }
    }
}

}  // namespace

cudaError_t quantize_activations(const QuantizeArgs& a, cudaStream_t stream) {
    const int pixels = a.in_h * a.in_w;
    if (pixels > 0) {
        pixel_max_kernel<<<(pixels + 31) / 32, max_threads, 0, stream>>>(a.in, a.channels, pixels, a.pixel_max);
        const cudaError_t launched = cudaGetLastError();
        if (launched != cudaSuccess) return launched;
    }
    const unsigned int blocks = static_cast<unsigned int>(a.positions_padded / tile_positions);
    if (a.activation_bits == 16) {
        quantize_kernel<16><<<blocks, max_threads, 0, stream>>>(a);
    } else {
        quantize_kernel<8><<<blocks, max_threads, 0, stream>>>(a);
    }
    return cudaGetLastError();
}

}  // namespace nvcr_sm100::kernels
