// Integer conv on pre-quantised activations (w8a8), sm_100a.
//
// The profile quantises the activations of each output position p with one
// exponent, e_p = frexp(max |x| over p's receptive field) - 7, so one input
// pixel may quantise differently for different positions. But frexp's exponent
// is monotone in the magnitude, so e_p is the largest of the per-pixel
// exponents e_P = frexp(max |x| over pixel P's channels) - 7 over the window's
// non-zero pixels, and when those pixels all have the same e_P, every value of
// the window quantises at its own pixel's exponent: q = clamp(rint(x * 2^-e_P),
// +-127). An all-zero pixel quantises to zero at any exponent. So:
//
//   quantise_pixels / quantise_fields  write each pixel quantised at its own
//       exponent, int8 channel-innermost [pixels][c8] (c8 = channels rounded up
//       to 32, padding zero), and the per-pixel max |x| (+inf when a channel is
//       non-finite). A pointwise conv has one pixel per window, and a conv over
//       staged receptive fields has one field per window, so for them this IS
//       the profile's quantisation.
//   direct_conv_kernel  a TMA-fed implicit GEMM: the A operand of each
//       (tap, channel block) is one 3-D TMA box of the int8 tensor (k_block
//       bytes x patch_w x patch_h pixels, shifted by the tap; the image border
//       and padding taps come back as the TMA's zero fill), already in the
//       swizzled K-major layout the MMA reads. No thread touches an activation.
//       The epilogue threads compute each position's exponent from the window's
//       pixel maxima; a window whose non-zero pixels have different exponents
//       sets the fallback word, and the quantise-on-load conv (k_conv.cu),
//       gated on that word, then recomputes the whole conv.
//
// Warp roles (15 warps, 128 registers each): warps 0-11 epilogue (three per
// TMEM lane quarter, each a third of the tile's 16-column chunks), warp 12 the
// weight TMA, warp 13 TMEM allocation and the MMA issue (one thread), warp 14
// the activation TMA. Accumulators are double-buffered in TMEM when they fit.
// Every wait is bounded (about 2 s of the global timer); after a timeout the
// CTA sets bit 0 of the status word, stops issuing, drains its MMAs and TMA
// loads, frees its TMEM and returns. No multicast load is used.

#include "exact_math.cuh"
#include "kernels.hpp"
#include "launch.cuh"
#include "tcgen05.cuh"

#include <climits>

#include <cuda_fp16.h>

namespace nvcr_sm100::kernels {
namespace {

constexpr int direct_warps = 15;
constexpr int direct_threads = direct_warps * 32;
constexpr int epilogue_warps = 12;
constexpr int epilogue_threads = epilogue_warps * 32;
constexpr int weight_warp = 12;
constexpr int mma_warp = 13;
constexpr int activation_warp = 14;
constexpr int max_direct_stages = 16;
constexpr float round_magic = 12582912.0f;  // 1.5 * 2^23

struct DirectTail {
    unsigned long long full_a[max_direct_stages];
    unsigned long long empty_a[max_direct_stages];
    unsigned long long full_b[max_direct_stages];
    unsigned long long empty_b[max_direct_stages];
    unsigned long long tmem_full[2];
    unsigned long long tmem_empty[2];
    unsigned long long drain;
    std::uint32_t tmem_base;
    int abort;
};

// Shared-memory matrix descriptor of a K-major int8 tile whose rows are
// k_block bytes long, swizzled over k_block bytes: 8-row atoms of
// 8 * k_block bytes stacked back to back (SBO), layout 2 / 4 / 6 for the
// 128 / 64 / 32-byte swizzle, descriptor version 1.
__device__ __forceinline__ std::uint64_t swizzled_descriptor(std::uint32_t address, int k_block) {
    const std::uint64_t layout = k_block == 128 ? 2u : (k_block == 64 ? 4u : 6u);
    const std::uint64_t atom = static_cast<std::uint64_t>(8 * k_block) >> 4;
    return static_cast<std::uint64_t>((address >> 4) & 0x3FFFu) | (static_cast<std::uint64_t>(1) << 16) |
        (atom << 32) | (static_cast<std::uint64_t>(1) << 46) | (layout << 61);
}

// Bytes of the per-column scales and biases after the tail.
__host__ __device__ constexpr int column_bytes(int columns) { return columns * 8; }

__host__ __device__ constexpr int tail_bytes() { return static_cast<int>((sizeof(DirectTail) + 15) / 16 * 16); }

// ---------------------------------------------------------------- prepass

// q = clamp(rint(x * 2^-e), +-127) for one value of a pixel whose exponent is
// e; `scale` = 2^-e when that is a normal float (then one fused multiply-add
// with 1.5 * 2^23 rounds x * 2^-e to the integer exactly once: |x * 2^-e| <
// 128), else the bit-level ldexp and rint.
__device__ __forceinline__ int quantise_one(float x, bool normal_scale, float scale, int exponent) {
    if (normal_scale) {
        const float y = __fmaf_rn(x, scale, round_magic);
        const int q = static_cast<int>(__float_as_uint(y) - __float_as_uint(round_magic));
        return q > 127 ? 127 : (q < -127 ? -127 : q);
    }
    return quantize_value<8>(x, exponent);
}

struct PixelScale {
    bool finite;
    bool normal;
    float scale;
    int exponent;
};

__device__ __forceinline__ PixelScale pixel_scale(float maximum) {
    PixelScale s;
    s.finite = maximum != __uint_as_float(0x7f800000u);
    s.exponent = activation_exponent(maximum, 8);
    s.normal = s.exponent >= -127 && s.exponent <= 126;
    s.scale = s.normal ? power_of_two(-s.exponent) : 0.0f;
    return s;
}

// Sixteen quantised values packed into four words, byte j of word w = value 4w + j.
__device__ __forceinline__ uint4 pack16(const int (&q)[16]) {
    std::uint32_t w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        w[k] = (static_cast<std::uint32_t>(q[4 * k]) & 0xffu) | ((static_cast<std::uint32_t>(q[4 * k + 1]) & 0xffu) << 8) |
            ((static_cast<std::uint32_t>(q[4 * k + 2]) & 0xffu) << 16) |
            ((static_cast<std::uint32_t>(q[4 * k + 3]) & 0xffu) << 24);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ std::uint32_t magnitude_bits_of(float v) { return __float_as_uint(v) & 0x7fffffffu; }
__device__ __forceinline__ float max_from_magnitude_bits(std::uint32_t m) {
    return m >= 0x7f800000u ? __uint_as_float(0x7f800000u) : __uint_as_float(m);
}

constexpr int plane_pixels = 64;  // pixels per block of the plane prepass

// NCHW planes (FP32 or FP16) -> per-pixel int8. A block takes 64 consecutive
// pixels and all channels through shared memory ([channel][pixel], coalesced
// plane reads), finds each pixel's max |x|, then writes each pixel's c8 bytes
// as 16-byte stores, consecutive threads on consecutive stores.
template <bool Half>
__global__ void __launch_bounds__(256) quantise_planes_kernel(const void* __restrict__ in, int channels, int c8,
                                                              int pixels, std::int8_t* __restrict__ out,
                                                              float* __restrict__ pixel_max,
                                                              unsigned int* __restrict__ clear_word) {
    grid_dependency_wait();
    launch_dependents();
    if (clear_word != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *clear_word = 0u;
    extern __shared__ float tile[];  // [channels][plane_pixels + 1]
    constexpr int pitch = plane_pixels + 1;
    __shared__ std::uint32_t partial[4][plane_pixels];
    __shared__ float maxima[plane_pixels];
    const long long first = static_cast<long long>(blockIdx.x) * plane_pixels;
    const int valid = static_cast<int>(pixels - first < plane_pixels ? pixels - first : plane_pixels);
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    // Loads: warp w takes channels w, w + 8, ...; lanes cover the 64 pixels twice.
    for (int c = warp; c < channels; c += 8) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int p = lane + 32 * h;
            float v = 0.0f;
            if (p < valid) {
                const std::size_t at = static_cast<std::size_t>(c) * pixels + first + p;
                v = Half ? __half2float(static_cast<const __half*>(in)[at]) : static_cast<const float*>(in)[at];
            }
            tile[c * pitch + p] = v;
        }
    }
    __syncthreads();
    // Per-pixel maxima: four threads per pixel, each a quarter of the channels.
    {
        const int p = threadIdx.x & (plane_pixels - 1);
        const int part = threadIdx.x >> 6;  // 0..3
        std::uint32_t m = 0;
        for (int c = part; c < channels; c += 4) m = max(m, magnitude_bits_of(tile[c * pitch + p]));
        partial[part][p] = m;
    }
    __syncthreads();
    if (threadIdx.x < plane_pixels) {
        const int p = threadIdx.x;
        const std::uint32_t m = max(max(partial[0][p], partial[1][p]), max(partial[2][p], partial[3][p]));
        const float maximum = max_from_magnitude_bits(m);
        maxima[p] = maximum;
        if (p < valid) pixel_max[first + p] = maximum;
    }
    __syncthreads();
    const int stores_per_pixel = c8 / 16;
    uint4* target = reinterpret_cast<uint4*>(out + first * c8);
    for (int item = threadIdx.x; item < valid * stores_per_pixel; item += 256) {
        const int p = item / stores_per_pixel;
        const int c0 = (item - p * stores_per_pixel) * 16;
        const PixelScale s = pixel_scale(maxima[p]);
        int q[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const int c = c0 + j;
            q[j] = (c < channels && s.finite) ? quantise_one(tile[c * pitch + p], s.normal, s.scale, s.exponent) : 0;
        }
        target[item] = pack16(q);
    }
}

// Staged FP32 [pixels][c_pad] with known maxima -> per-pixel int8: one thread
// per 16 channels of a pixel (four 16-byte loads, one 16-byte store).
__global__ void __launch_bounds__(256) quantise_staged_kernel(const float* __restrict__ in, int channels, int c_pad,
                                                              int c8, int pixels, const float* __restrict__ pixel_max,
                                                              std::int8_t* __restrict__ out,
                                                              unsigned int* __restrict__ clear_word) {
    grid_dependency_wait();
    launch_dependents();
    if (clear_word != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *clear_word = 0u;
    const int stores_per_pixel = c8 / 16;
    const long long item = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (item >= static_cast<long long>(pixels) * stores_per_pixel) return;
    const long long p = item / stores_per_pixel;
    const int c0 = static_cast<int>(item - p * stores_per_pixel) * 16;
    const PixelScale s = pixel_scale(__ldg(pixel_max + p));
    float v[16];
    if (c0 < c_pad) {
        const float4* source = reinterpret_cast<const float4*>(in + p * c_pad + c0);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float4 f = __ldg(source + k);
            v[4 * k] = f.x;
            v[4 * k + 1] = f.y;
            v[4 * k + 2] = f.z;
            v[4 * k + 3] = f.w;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = 0.0f;
    }
    int q[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        q[j] = (c0 + j < channels && s.finite) ? quantise_one(v[j], s.normal, s.scale, s.exponent) : 0;
    }
    reinterpret_cast<uint4*>(out)[item] = pack16(q);
}

constexpr int max_field_values = 64;

// One thread per output position: its receptive field in k = c * taps + tap
// order (padding taps and k past channels * taps zero), the field's max |x|,
// and the field quantised with its own exponent into c8 bytes.
template <bool Half>
__global__ void __launch_bounds__(256) quantise_fields_kernel(const void* __restrict__ in, int channels, int in_h,
                                                              int in_w, Window w, int out_h, int out_w, int c8,
                                                              std::int8_t* __restrict__ out,
                                                              float* __restrict__ field_max) {
    grid_dependency_wait();
    launch_dependents();
    __shared__ long long plane_at[max_field_values];  // c * in_h * in_w, or -1 past the field
    __shared__ short2 tap_at[max_field_values];       // (ky, kx)
    const int taps = w.kernel_h * w.kernel_w;
    for (int k = threadIdx.x; k < c8; k += blockDim.x) {
        const int c = k / taps;
        const int tap = k - c * taps;
        const int ky = tap / w.kernel_w;
        plane_at[k] = k < channels * taps ? static_cast<long long>(c) * in_h * in_w : -1;
        tap_at[k] = make_short2(static_cast<short>(ky), static_cast<short>(tap - ky * w.kernel_w));
    }
    __syncthreads();
    const long long position = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (position >= static_cast<long long>(out_h) * out_w) return;
    const int oy = static_cast<int>(position / out_w);
    const int ox = static_cast<int>(position - static_cast<long long>(oy) * out_w);
    const int iy0 = oy * w.stride_y - w.pad_top;
    const int ix0 = ox * w.stride_x - w.pad_left;
    float v[max_field_values];
    std::uint32_t m = 0;
#pragma unroll
    for (int k = 0; k < max_field_values; ++k) {
        v[k] = 0.0f;
        if (k < c8) {
            const long long plane = plane_at[k];
            const short2 d = tap_at[k];
            const int iy = iy0 + d.x;
            const int ix = ix0 + d.y;
            if (plane >= 0 && static_cast<unsigned>(iy) < static_cast<unsigned>(in_h) &&
                static_cast<unsigned>(ix) < static_cast<unsigned>(in_w)) {
                const long long at = plane + static_cast<long long>(iy) * in_w + ix;
                v[k] = Half ? __half2float(static_cast<const __half*>(in)[at]) : static_cast<const float*>(in)[at];
            }
            m = max(m, magnitude_bits_of(v[k]));
        }
    }
    const float maximum = max_from_magnitude_bits(m);
    field_max[position] = maximum;
    const PixelScale s = pixel_scale(maximum);
    uint4* record = reinterpret_cast<uint4*>(out + position * c8);
#pragma unroll
    for (int k0 = 0; k0 < max_field_values; k0 += 16) {
        if (k0 >= c8) break;
        int q[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) q[j] = s.finite ? quantise_one(v[k0 + j], s.normal, s.scale, s.exponent) : 0;
        record[k0 / 16] = pack16(q);
    }
}

// ---------------------------------------------------------------- the conv

// Quotient and remainder by a divisor fixed for the kernel (exact for
// 0 <= n < 2^22): a float reciprocal and one correction step.
struct TileDivider {
    int d;
    float inverse;
    __device__ explicit TileDivider(int divisor) : d(divisor), inverse(1.0f / static_cast<float>(divisor)) {}
    __device__ __forceinline__ int divide(int n, int& remainder) const {
        int q = __float2int_rz(__fmul_rn(__int2float_rn(n), inverse));
        int r = n - q * d;
        if (r < 0) {
            --q;
            r += d;
        } else if (r >= d) {
            ++q;
            r -= d;
        }
        remainder = r;
        return q;
    }
};

struct Sixteen16 {
    float v[16];
};

__device__ __noinline__ Sixteen16 direct_ldexp_add16(Sixteen16 x, Sixteen16 bias, int exponent) {
#pragma unroll
    for (int j = 0; j < 16; ++j) x.v[j] = __fadd_rn(exact_ldexp(x.v[j], exponent), bias.v[j]);
    return x;
}

// profile_wsilu of 16 values: the refined reciprocal where the denominator lies
// in [1, 2^126), the IEEE division for the rest (marked in a mask, redone).
__device__ __noinline__ Sixteen16 direct_wsilu16(Sixteen16 x, float k) {
    std::uint32_t rare = 0;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const float d = __fadd_rn(1.0f, profile_exp(-__fmul_rn(x.v[j], k)));
        const bool inside = d < sigmoid_reciprocal_limit;
        rare |= inside ? 0u : 1u << j;
        x.v[j] = inside ? __fmul_rn(sigmoid_reciprocal(d), x.v[j]) : x.v[j];
    }
    if (rare != 0) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            if ((rare >> j) & 1u) x.v[j] = profile_wsilu(x.v[j], k);
        }
    }
    return x;
}

__global__ void __launch_bounds__(direct_threads, 1)
direct_conv_kernel(const __grid_constant__ CUtensorMap a_map, const __grid_constant__ CUtensorMap b_map,
                   DirectConvArgs a, int tmem_buffers, std::uint32_t tmem_columns) {
    extern __shared__ std::uint8_t dynamic_smem[];
    const std::uint32_t raw = smem_address(dynamic_smem);
    std::uint8_t* smem = dynamic_smem + (((raw + 1023u) & ~1023u) - raw);
    const int n_tile = a.n_tile;
    const int k_block = a.k_block;
    const int a_stage_bytes = tile_positions_m * k_block;
    const int b_stage_bytes = n_tile * k_block;
    // Shared memory: [A stages][B stages][tail][column parameters]; stage sizes are
    // multiples of 1024 bytes, so every stage keeps the 1 KiB swizzle alignment.
    std::uint8_t* b_smem = smem + a.a_stages * a_stage_bytes;
    auto* tail = reinterpret_cast<DirectTail*>(b_smem + a.b_stages * b_stage_bytes);
    const int all_columns = a.n_tiles * n_tile;
    float* column_scale = reinterpret_cast<float*>(reinterpret_cast<std::uint8_t*>(tail) + tail_bytes());
    float* column_bias = column_scale + all_columns;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int total_tiles = a.p_tiles * a.n_tiles;
    const int k_blocks = a.k_blocks;
    const TileDivider by_n_tiles(a.n_tiles);
    const TileDivider by_tiles_x(a.tiles_x);

    for (int i = threadIdx.x; i < all_columns; i += direct_threads) {
        column_scale[i] = a.scales[i];
        column_bias[i] = a.bias[i];
    }
    if (warp == mma_warp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_address(&tail->tmem_base)), "r"(tmem_columns)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (warp == weight_warp && lane == 0) {
        for (int s = 0; s < a.a_stages; ++s) {
            barrier_init(smem_address(&tail->full_a[s]), 1);
            barrier_init(smem_address(&tail->empty_a[s]), 1);
        }
        for (int s = 0; s < a.b_stages; ++s) {
            barrier_init(smem_address(&tail->full_b[s]), 1);
            barrier_init(smem_address(&tail->empty_b[s]), 1);
        }
        for (int b = 0; b < 2; ++b) {
            barrier_init(smem_address(&tail->tmem_full[b]), 1);
            barrier_init(smem_address(&tail->tmem_empty[b]), epilogue_threads);
        }
        barrier_init(smem_address(&tail->drain), 1);
        tail->abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        fence_proxy_async_shared();
    }
    tmem_fence_before();
    __syncthreads();
    tmem_fence_after();
    const std::uint32_t tmem = tail->tmem_base;
    // The weight TMA and the MMA read only constant weights, shared memory and
    // TMEM; the other roles wait for the kernels before this one first.
    launch_dependents();
    volatile int* abort = &tail->abort;

    if (warp == weight_warp) {
        if (lane == 0) {
            // ---------------- weights by TMA
            const std::uint32_t bytes = static_cast<std::uint32_t>(b_stage_bytes);
            std::uint32_t g = 0;
            std::uint32_t issued = 0;
            bool ok = true;
            const int last = a.b_resident ? static_cast<int>(blockIdx.x) + 1 : total_tiles;
            for (int t = blockIdx.x; t < last && ok; t += gridDim.x) {
                int n_index;
                by_n_tiles.divide(t, n_index);
                const int n0 = n_index * n_tile;
                for (int kb = 0; kb < k_blocks; ++kb, ++g) {
                    const int s = static_cast<int>(g % a.b_stages);
                    const std::uint32_t phase = (g / a.b_stages) & 1u;
                    if (*abort || !barrier_wait(smem_address(&tail->empty_b[s]), phase ^ 1u, a.status)) {
                        *abort = 1;
                        ok = false;
                        break;
                    }
                    const std::uint32_t full = smem_address(&tail->full_b[s]);
                    barrier_expect_bytes(full, bytes);
                    tma_load_2d(smem_address(b_smem + s * b_stage_bytes), &b_map, full, kb * k_block, n0);
                    issued = g + 1;
                }
            }
            if (!ok) {
                const std::uint32_t first = issued > static_cast<std::uint32_t>(a.b_stages) ? issued - a.b_stages : 0;
                for (std::uint32_t h = first; h < issued; ++h) {
                    barrier_wait(smem_address(&tail->full_b[h % a.b_stages]), (h / a.b_stages) & 1u, a.status);
                }
            }
        }
    } else if (warp == activation_warp) {
        grid_dependency_wait();
        if (lane == 0) {
            // ---------------- activations by TMA: one box per (tap, channel block)
            const std::uint32_t bytes = static_cast<std::uint32_t>(a_stage_bytes);
            std::uint32_t g = 0;
            std::uint32_t issued = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
                int n_index, tx;
                const int p_tile = by_n_tiles.divide(t, n_index);
                const int ty = by_tiles_x.divide(p_tile, tx);
                const int y0 = ty * a.patch_h - a.window.pad_top;
                const int x0 = tx * a.patch_w - a.window.pad_left;
                int ky = 0, kx = 0, cb = 0;
                for (int kb = 0; kb < k_blocks; ++kb, ++g) {
                    const int s = static_cast<int>(g % a.a_stages);
                    const std::uint32_t phase = (g / a.a_stages) & 1u;
                    if (*abort || !barrier_wait(smem_address(&tail->empty_a[s]), phase ^ 1u, a.status)) {
                        *abort = 1;
                        ok = false;
                        break;
                    }
                    const std::uint32_t full = smem_address(&tail->full_a[s]);
                    barrier_expect_bytes(full, bytes);
                    // Innermost coordinate: the channel block's first byte, a multiple of k_block.
                    tma_load_3d(smem_address(smem + s * a_stage_bytes), &a_map, full, cb * k_block, x0 + kx, y0 + ky);
                    issued = g + 1;
                    if (++cb == a.c_blocks) {
                        cb = 0;
                        if (++kx == a.window.kernel_w) {
                            kx = 0;
                            ++ky;
                        }
                    }
                }
            }
            if (!ok) {
                const std::uint32_t first = issued > static_cast<std::uint32_t>(a.a_stages) ? issued - a.a_stages : 0;
                for (std::uint32_t h = first; h < issued; ++h) {
                    barrier_wait(smem_address(&tail->full_a[h % a.a_stages]), (h / a.a_stages) & 1u, a.status);
                }
            }
        }
    } else if (warp == mma_warp) {
        if (lane == 0) {
            // ---------------- tensor-core issue
            const std::uint32_t idesc = i8_instruction(n_tile);
            const int steps = k_block / 32;
            std::uint32_t g = 0;
            int local = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x, ++local) {
                const int buffer = local % tmem_buffers;
                const std::uint32_t use = static_cast<std::uint32_t>(local / tmem_buffers);
                if (*abort || !barrier_wait(smem_address(&tail->tmem_empty[buffer]), (use & 1u) ^ 1u, a.status)) {
                    *abort = 1;
                    break;
                }
                tmem_fence_after();
                const std::uint32_t acc = tmem + static_cast<std::uint32_t>(buffer * n_tile);
                for (int kb = 0; kb < k_blocks; ++kb, ++g) {
                    const int sa = static_cast<int>(g % a.a_stages);
                    const std::uint32_t a_phase = (g / a.a_stages) & 1u;
                    const int sb = a.b_resident ? kb : static_cast<int>(g % a.b_stages);
                    const std::uint32_t b_phase = a.b_resident ? 0u : (g / a.b_stages) & 1u;
                    if (*abort || !barrier_wait(smem_address(&tail->full_a[sa]), a_phase, a.status) ||
                        !barrier_wait(smem_address(&tail->full_b[sb]), b_phase, a.status)) {
                        *abort = 1;
                        ok = false;
                        break;
                    }
                    tmem_fence_after();
                    const std::uint32_t a_base = smem_address(smem + sa * a_stage_bytes);
                    const std::uint32_t b_base = smem_address(b_smem + sb * b_stage_bytes);
                    for (int kk = 0; kk < steps; ++kk) {
                        const std::uint32_t step = static_cast<std::uint32_t>(kk * 32);
                        const std::uint32_t accumulate = (kb == 0 && kk == 0) ? 0u : 1u;
                        mma_i8(acc, swizzled_descriptor(a_base + step, k_block),
                               swizzled_descriptor(b_base + step, k_block), idesc, accumulate);
                    }
                    mma_commit(smem_address(&tail->empty_a[sa]));
                    if (!a.b_resident) mma_commit(smem_address(&tail->empty_b[sb]));
                }
                if (!ok) break;
                mma_commit(smem_address(&tail->tmem_full[buffer]));
            }
            mma_commit(smem_address(&tail->drain));
            barrier_wait(smem_address(&tail->drain), 0u, a.status);
        }
    } else if (warp < epilogue_warps) {
        // ---------------- epilogue: thread <-> TMEM lane <-> position
        grid_dependency_wait();
        const int quarter = warp & 3;
        const int part = warp >> 2;  // third of the columns
        const int row = quarter * 32 + lane;
        const std::uint32_t lane_base = static_cast<std::uint32_t>(quarter * 32) << 16;
        const int pair_offset = a.chunk_add ? n_tile / 2 : 0;
        const int columns = a.chunk_add ? n_tile / 2 : n_tile;
        const int chunks = columns / 16;
        const int per_part = (chunks + 2) / 3;
        const int first_column = min(part * per_part, chunks) * 16;
        const int last_column = min((part + 1) * per_part, chunks) * 16;
        const int b = a.d2s_block;
        const int patch_y = row / a.patch_w;
        const int patch_x = row - patch_y * a.patch_w;
        const int out_w_full = a.out_w * (b > 0 ? b : 1);
        const int out_h_full = a.out_h * (b > 0 ? b : 1);
        const int kernel_h = a.window.kernel_h;
        const int kernel_w = a.window.kernel_w;
        int local = 0;
        for (int t = blockIdx.x; t < total_tiles; t += gridDim.x, ++local) {
            int n_index, tx;
            const int p_tile = by_n_tiles.divide(t, n_index);
            const int ty = by_tiles_x.divide(p_tile, tx);
            const int y = ty * a.patch_h + patch_y;
            const int x = tx * a.patch_w + patch_x;
            const bool real = y < a.out_h && x < a.out_w;
            const int p = real ? y * a.out_w + x : 0;
            // The window's exponent from its pixels' maxima (while the MMA runs):
            // the largest maximum sets it; a non-finite pixel makes the row NaN; a
            // non-zero pixel whose exponent differs from the largest marks the
            // window as mixed.
            int exponent = INT_MIN;
            bool mixed = false;  // the fallback conv writes this position
            if (real) {
                float largest = 0.0f;
                float smallest = __uint_as_float(0x7f800000u);  // smallest non-zero
                const int iy0 = y - a.window.pad_top;
                const int ix0 = x - a.window.pad_left;
                for (int ky = 0; ky < kernel_h; ++ky) {
                    const int iy = iy0 + ky;
                    if (iy < 0 || iy >= a.in_h) continue;
                    for (int kx = 0; kx < kernel_w; ++kx) {
                        const int ix = ix0 + kx;
                        if (ix < 0 || ix >= a.in_w) continue;
                        const float m = __ldg(a.pixel_max + static_cast<std::size_t>(iy) * a.in_w + ix);
                        largest = fmaxf(largest, m);
                        if (m > 0.0f) smallest = fminf(smallest, m);
                    }
                }
                if (largest != __uint_as_float(0x7f800000u)) {
                    exponent = activation_exponent(largest, 8);
                    mixed = a.fallback != nullptr && largest > 0.0f &&
                        frexp_exponent(smallest) != frexp_exponent(largest);
                    if (mixed && part == 0) atomicOr(a.fallback, 1u);
                }
            }
            // A mixed window's accumulators are not this position's result:
            // nothing is stored for it (nor added to a staged maximum, which
            // can only grow), and the fallback conv writes it instead.
            const bool store = real && !mixed;
            const int buffer = local % tmem_buffers;
            const std::uint32_t use = static_cast<std::uint32_t>(local / tmem_buffers);
            bool waited = *abort == 0 && barrier_wait(smem_address(&tail->tmem_full[buffer]), use & 1u, a.status);
            waited = __all_sync(0xffffffffu, waited);  // tcgen05.ld is warp-aligned
            if (!waited) {
                *abort = 1;
                break;
            }
            tmem_fence_after();
            const int physical0 = n_index * n_tile;
            const int logical0 = a.chunk_add ? n_index * (n_tile / 2) : physical0;
            const std::uint32_t acc = tmem + static_cast<std::uint32_t>(buffer * n_tile) + lane_base;
            const bool normal = exponent >= -126 && exponent <= 127;
            const bool plain = normal || exponent == INT_MIN;
            const float power = normal ? power_of_two(exponent) : 1.0f;

            // 16 output values at accumulator columns first.. of this tile.
            auto values16 = [&](int first, float (&v)[16]) {
                int hh[16];
                tmem_load16(acc + static_cast<std::uint32_t>(first), hh);
                const float4* scale4 = reinterpret_cast<const float4*>(column_scale + physical0 + first);
                const float4* bias4 = reinterpret_cast<const float4*>(column_bias + physical0 + first);
                float scales[16], biases[16];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float4 f = scale4[i];
                    const float4 h = bias4[i];
                    scales[4 * i] = f.x;
                    scales[4 * i + 1] = f.y;
                    scales[4 * i + 2] = f.z;
                    scales[4 * i + 3] = f.w;
                    biases[4 * i] = h.x;
                    biases[4 * i + 1] = h.y;
                    biases[4 * i + 2] = h.z;
                    biases[4 * i + 3] = h.w;
                }
                tmem_load_wait();
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = __fmul_rn(__int2float_rn(hh[j]), scales[j]);
                if (plain) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] = __fadd_rn(__fmul_rn(v[j], power), biases[j]);
                } else {
                    Sixteen16 xv, bv;
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        xv.v[j] = v[j];
                        bv.v[j] = biases[j];
                    }
                    xv = direct_ldexp_add16(xv, bv, exponent);
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] = xv.v[j];
                }
                if (a.wsilu) {
                    Sixteen16 xv;
#pragma unroll
                    for (int j = 0; j < 16; ++j) xv.v[j] = v[j];
                    xv = direct_wsilu16(xv, a.wsilu_scale);
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] = xv.v[j];
                }
            };

            std::uint32_t staged_max = 0;
            for (int j0 = first_column; j0 < last_column; j0 += 16) {
                float v[16];
                values16(j0, v);
                if (a.chunk_add) {
                    float w[16];
                    values16(j0 + pair_offset, w);
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] = __fadd_rn(v[j], w[j]);
                }
                const int c0 = logical0 + j0;
                const int count = a.out_channels - c0 < 16 ? a.out_channels - c0 : 16;
                if (store) {
                    if (exponent == INT_MIN) {
#pragma unroll
                        for (int j = 0; j < 16; ++j) v[j] = canonical_nan();
                    }
                    if (a.residual != nullptr) {
                        float add[16];
                        if (a.residual_c_pad > 0) {
                            if (count > 0) {
                                const float4* r = reinterpret_cast<const float4*>(
                                    a.residual + static_cast<std::size_t>(p) * a.residual_c_pad + c0);
#pragma unroll
                                for (int q = 0; q < 4; ++q) {
                                    const float4 f = __ldg(r + q);
                                    add[4 * q] = f.x;
                                    add[4 * q + 1] = f.y;
                                    add[4 * q + 2] = f.z;
                                    add[4 * q + 3] = f.w;
                                }
                            }
#pragma unroll
                            for (int j = 0; j < 16; ++j) add[j] = j < count ? add[j] : 0.0f;
                        } else {
                            const float* r = a.residual + static_cast<std::size_t>(c0) * a.positions + p;
#pragma unroll
                            for (int j = 0; j < 16; ++j) {
                                add[j] = j < count ? __ldg(r + static_cast<std::size_t>(j) * a.positions) : 0.0f;
                            }
                        }
#pragma unroll
                        for (int j = 0; j < 16; ++j) v[j] = __fadd_rn(v[j], add[j]);
                    }
                    if (a.out_max != nullptr) {
                        if (c0 < a.out_c_pad) {
                            float4* o = reinterpret_cast<float4*>(reinterpret_cast<float*>(a.out) +
                                                                  static_cast<std::size_t>(p) * a.out_c_pad + c0);
#pragma unroll
                            for (int j = 0; j < 16; ++j) {
                                v[j] = j < count ? v[j] : 0.0f;
                                staged_max = max(staged_max, __float_as_uint(v[j]) & 0x7fffffffu);
                            }
#pragma unroll
                            for (int q = 0; q < 4; ++q) o[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
                        }
                    } else if (b == 0 && count == 16) {
                        const std::size_t stride = static_cast<std::size_t>(a.positions);
                        const std::size_t at = static_cast<std::size_t>(c0) * stride + p;
                        if (a.out_half) {
                            __half* o = reinterpret_cast<__half*>(a.out) + at;
#pragma unroll
                            for (int j = 0; j < 16; ++j) o[j * stride] = __float2half_rn(v[j]);
                        } else {
                            float* o = reinterpret_cast<float*>(a.out) + at;
#pragma unroll
                            for (int j = 0; j < 16; ++j) o[j * stride] = v[j];
                        }
                    } else if (b == 2 && count == 16 && a.out_half) {
                        // depth_to_space(2): channel c0 + 4q + 2i + jj goes to plane c0 / 4 + q,
                        // row 2y + i, column 2x + jj; the jj pair is one aligned FP16 pair.
                        __half2* o = reinterpret_cast<__half2*>(a.out);
                        const std::size_t plane = static_cast<std::size_t>(out_h_full) * out_w_full;
                        const std::size_t at = (static_cast<std::size_t>(c0 / 4) * plane +
                                                static_cast<std::size_t>(2 * y) * out_w_full + 2 * x) / 2;
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
#pragma unroll
                            for (int i = 0; i < 2; ++i) {
                                const int j = 4 * q + 2 * i;
                                o[at + (q * plane + static_cast<std::size_t>(i) * out_w_full) / 2] =
                                    __floats2half2_rn(v[j], v[j + 1]);
                            }
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            if (j >= count) break;
                            const int c = c0 + j;
                            std::size_t index;
                            if (b > 0) {
                                const int oc = c / (b * b);
                                const int i = (c / b) % b;
                                const int jj = c % b;
                                index = (static_cast<std::size_t>(oc) * out_h_full + static_cast<std::size_t>(y) * b + i) *
                                        out_w_full + static_cast<std::size_t>(x) * b + jj;
                            } else {
                                index = static_cast<std::size_t>(c) * a.positions + p;
                            }
                            if (a.out_half) {
                                reinterpret_cast<__half*>(a.out)[index] = __float2half_rn(v[j]);
                            } else {
                                reinterpret_cast<float*>(a.out)[index] = v[j];
                            }
                        }
                    }
                }
                __syncwarp();  // tcgen05.ld is warp-aligned: reconverge before the next columns
            }
            if (a.out_max != nullptr && store && first_column < last_column) {
                atomicMax(reinterpret_cast<unsigned int*>(a.out_max) + p,
                          __float_as_uint(max_from_magnitude_bits(staged_max)));
            }
            tmem_fence_before();
            barrier_arrive(smem_address(&tail->tmem_empty[buffer]));
        }
    }

    tmem_fence_before();
    __syncthreads();
    if (warp == mma_warp) {
        __syncwarp();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tmem_columns)
                     : "memory");
    }
}

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled tiled_encoder() {
    static EncodeTiled function = [] {
        void* pointer = nullptr;
        cudaDriverEntryPointQueryResult found{};
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &pointer, 12000, cudaEnableDefault, &found) !=
                cudaSuccess ||
            found != cudaDriverEntryPointSuccess) {
            return static_cast<EncodeTiled>(nullptr);
        }
        return reinterpret_cast<EncodeTiled>(pointer);
    }();
    return function;
}

CUtensorMapSwizzle swizzle_for(std::uint32_t k_block) {
    return k_block == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
         : k_block == 64  ? CU_TENSOR_MAP_SWIZZLE_64B
                          : CU_TENSOR_MAP_SWIZZLE_32B;
}

bool valid_k_block(int k_block) { return k_block == 32 || k_block == 64 || k_block == 128; }

bool valid_direct(const DirectConvArgs& a) {
    const int taps = a.window.kernel_h * a.window.kernel_w;
    const bool aligned = (reinterpret_cast<std::uintptr_t>(a.scales) & 15u) == 0 &&
        (reinterpret_cast<std::uintptr_t>(a.bias) & 15u) == 0;
    return aligned && valid_k_block(a.k_block) && a.c_blocks >= 1 && a.k_blocks == taps * a.c_blocks && taps >= 1 &&
        a.window.kernel_h <= 3 && a.window.kernel_w <= 3 && a.window.stride_y == 1 && a.window.stride_x == 1 &&
        a.n_tile >= 16 && a.n_tile <= 256 && a.n_tile % 16 == 0 && (!a.chunk_add || a.n_tile % 32 == 0) &&
        a.n_tiles >= 1 && a.p_tiles >= 1 && static_cast<long long>(a.p_tiles) * a.n_tiles < (1LL << 22) &&
        a.patch_h * a.patch_w == tile_positions_m && a.patch_w >= 1 && a.patch_w <= 256 && a.patch_h <= 256 &&
        a.tiles_y * a.patch_h >= a.out_h && a.tiles_x * a.patch_w >= a.out_w && a.p_tiles == a.tiles_y * a.tiles_x &&
        a.positions == a.out_h * a.out_w && a.a_stages >= 2 && a.a_stages <= max_direct_stages && a.b_stages >= 1 &&
        a.b_stages <= max_direct_stages && (!a.b_resident || (a.n_tiles == 1 && a.b_stages == a.k_blocks)) &&
        (a.b_resident || a.b_stages >= 2) && a.d2s_block >= 0 &&
        (a.out_max == nullptr ||
         (!a.out_half && a.d2s_block == 0 && a.out_c_pad % 16 == 0 && a.out_c_pad >= a.out_channels &&
          (reinterpret_cast<std::uintptr_t>(a.out) & 15u) == 0)) &&
        (a.residual_c_pad == 0 ||
         (a.residual_c_pad % 16 == 0 && a.residual_c_pad >= a.out_channels &&
          (reinterpret_cast<std::uintptr_t>(a.residual) & 15u) == 0)) &&
        (a.chunk_add ? a.out_channels <= a.n_tiles * a.n_tile / 2 : a.out_channels <= a.n_tiles * a.n_tile) &&
        (taps == 1 || a.fallback != nullptr);
}

}  // namespace

int direct_conv_shared_bytes(int k_block, int n_tile, int n_tiles, int a_stages, int b_stages) {
    return 1024 + a_stages * tile_positions_m * k_block + b_stages * n_tile * k_block + tail_bytes() +
        column_bytes(n_tile * n_tiles);
}

cudaError_t encode_activation_map(CUtensorMap* map, const void* base, std::uint64_t c8, std::uint64_t height,
                                  std::uint64_t width, std::uint32_t k_block, std::uint32_t box_w, std::uint32_t box_h) {
    const EncodeTiled encode = tiled_encoder();
    if (encode == nullptr) return cudaErrorNotSupported;
    if ((reinterpret_cast<std::uintptr_t>(base) & 15u) != 0 || !valid_k_block(static_cast<int>(k_block)) ||
        c8 % k_block != 0 || box_w == 0 || box_w > 256 || box_h == 0 || box_h > 256) {
        return cudaErrorInvalidValue;
    }
    const cuuint64_t dims[3] = {c8, width, height};
    const cuuint64_t strides[2] = {c8, width * c8};
    const cuuint32_t box[3] = {k_block, box_w, box_h};
    const cuuint32_t element_strides[3] = {1, 1, 1};
    const CUresult result = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box,
                                   element_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle_for(k_block),
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return result == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t encode_weight_map(CUtensorMap* map, const void* base, std::uint64_t rows, std::uint64_t row_bytes,
                              std::uint32_t k_block, std::uint32_t box_rows) {
    const EncodeTiled encode = tiled_encoder();
    if (encode == nullptr) return cudaErrorNotSupported;
    if ((reinterpret_cast<std::uintptr_t>(base) & 15u) != 0 || !valid_k_block(static_cast<int>(k_block)) ||
        row_bytes % k_block != 0 || box_rows == 0 || box_rows > 256) {
        return cudaErrorInvalidValue;
    }
    const cuuint64_t dims[2] = {row_bytes, rows};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {k_block, box_rows};
    const cuuint32_t element_strides[2] = {1, 1};
    const CUresult result = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
                                   element_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle_for(k_block),
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return result == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t quantise_pixels(const void* in, PixelSource form, int channels, int c_pad_in, int c8, int pixels,
                            std::int8_t* out, float* pixel_max, unsigned int* clear_word, cudaStream_t stream) {
    if (pixels <= 0) return cudaSuccess;
    if (channels < 1 || c8 < channels || c8 % 32 != 0 || (reinterpret_cast<std::uintptr_t>(out) & 15u) != 0) {
        return cudaErrorInvalidValue;
    }
    if (form == PixelSource::staged_f32) {
        if (c_pad_in < channels || c_pad_in % 16 != 0 || (reinterpret_cast<std::uintptr_t>(in) & 15u) != 0) {
            return cudaErrorInvalidValue;
        }
        const long long items = static_cast<long long>(pixels) * (c8 / 16);
        return launch_overlapped(quantise_staged_kernel, dim3(static_cast<unsigned>((items + 255) / 256)), dim3(256),
                                 0, stream, static_cast<const float*>(in), channels, c_pad_in, c8, pixels,
                                 static_cast<const float*>(pixel_max), out, clear_word);
    }
    const int tile_bytes = channels * (plane_pixels + 1) * static_cast<int>(sizeof(float));
    if (tile_bytes > 200 * 1024) return cudaErrorInvalidValue;
    const unsigned blocks = static_cast<unsigned>((static_cast<long long>(pixels) + plane_pixels - 1) / plane_pixels);
    if (form == PixelSource::planes_f16) {
        static bool configured = false;
        if (!configured) {
            cudaFuncSetAttribute(quantise_planes_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
            configured = true;
        }
        return launch_overlapped(quantise_planes_kernel<true>, dim3(blocks), dim3(256), tile_bytes, stream, in,
                                 channels, c8, pixels, out, pixel_max, clear_word);
    }
    static bool configured = false;
    if (!configured) {
        cudaFuncSetAttribute(quantise_planes_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        configured = true;
    }
    return launch_overlapped(quantise_planes_kernel<false>, dim3(blocks), dim3(256), tile_bytes, stream, in, channels,
                             c8, pixels, out, pixel_max, clear_word);
}

cudaError_t quantise_fields(const void* in, int source_half, int channels, int in_h, int in_w, Window window,
                            int out_h, int out_w, int c8, std::int8_t* out, float* field_max, cudaStream_t stream) {
    const long long positions = static_cast<long long>(out_h) * out_w;
    if (positions <= 0) return cudaSuccess;
    if (channels < 1 || c8 % 32 != 0 || c8 > max_field_values || c8 < channels * window.kernel_h * window.kernel_w ||
        (reinterpret_cast<std::uintptr_t>(out) & 15u) != 0) {
        return cudaErrorInvalidValue;
    }
    const unsigned blocks = static_cast<unsigned>((positions + 255) / 256);
    if (source_half) {
        return launch_overlapped(quantise_fields_kernel<true>, dim3(blocks), dim3(256), 0, stream, in, channels, in_h,
                                 in_w, window, out_h, out_w, c8, out, field_max);
    }
    return launch_overlapped(quantise_fields_kernel<false>, dim3(blocks), dim3(256), 0, stream, in, channels, in_h,
                             in_w, window, out_h, out_w, c8, out, field_max);
}

cudaError_t direct_conv(const CUtensorMap& a_map, const CUtensorMap& b_map, const DirectConvArgs& args,
                        cudaStream_t stream) {
    static int sm_count = [] {
        int device = 0;
        int count = 148;
        if (cudaGetDevice(&device) == cudaSuccess) cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, device);
        return count;
    }();
    if (!valid_direct(args)) return cudaErrorInvalidValue;
    int buffers = 2;
    std::uint32_t columns = 32;
    while (static_cast<int>(columns) < 2 * args.n_tile) columns <<= 1;
    if (columns > 512) {
        buffers = 1;
        columns = 32;
        while (static_cast<int>(columns) < args.n_tile) columns <<= 1;
    }
    const int smem = direct_conv_shared_bytes(args.k_block, args.n_tile, args.n_tiles, args.a_stages, args.b_stages);
    if (smem > direct_conv_max_shared) return cudaErrorInvalidValue;
    static bool configured = false;
    if (!configured) {
        const cudaError_t set = cudaFuncSetAttribute(direct_conv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                     direct_conv_max_shared);
        if (set != cudaSuccess) return set;
        configured = true;
    }
    const int tiles = args.p_tiles * args.n_tiles;
    const int grid = tiles < sm_count ? tiles : sm_count;
    return launch_overlapped(direct_conv_kernel, dim3(grid), dim3(direct_threads), smem, stream, a_map, b_map, args,
                             buffers, columns);
}

}  // namespace nvcr_sm100::kernels
