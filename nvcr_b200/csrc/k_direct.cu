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
//       One warp computes each position's exponent from the window's pixel
//       maxima, tiles ahead of the epilogue; a window whose non-zero pixels have
//       different exponents sets the fallback word, and the quantise-on-load
//       conv (k_conv.cu), gated on that word, then recomputes the whole conv.
//
// Warp roles (16 warps, 128 registers each): warps 0-11 epilogue (three groups
// of four, one warp per TMEM lane quarter; the groups take alternate tiles when
// four or more accumulator buffers fit, else a third of every tile's 16-column
// chunks each), warp 12 the weight TMA, warp 13 TMEM allocation and the MMA
// issue (one thread), warp 14 the activation TMA, warp 15 the window exponents.
// Accumulators take as many TMEM buffers as fit (2 to 8).
// Every wait is bounded (about 2 s of the global timer); after a timeout the
// CTA sets bit 0 of the status word, stops issuing, drains its MMAs and TMA
// loads, frees its TMEM and returns. No multicast load is used.

#include "exact_math.cuh"
#include "kernels.hpp"
#include "launch.cuh"
#include "tcgen05.cuh"

#include <climits>
#include <type_traits>

#include <cuda_fp16.h>

namespace nvcr_sm100::kernels {
namespace {

constexpr int direct_warps = 16;
constexpr int direct_threads = direct_warps * 32;
constexpr int epilogue_warps = 12;
constexpr int epilogue_threads = epilogue_warps * 32;
constexpr int weight_warp = 12;
constexpr int mma_warp = 13;
constexpr int activation_warp = 14;
constexpr int window_warp = 15;
constexpr int window_slots = 6;  // tiles whose halo of pixel maxima is staged ahead
constexpr int max_direct_stages = 16;
constexpr int max_tmem_buffers = 8;
constexpr float round_magic = 12582912.0f;  // 1.5 * 2^23

// Epilogue groups: with four or more accumulator buffers the three groups of
// four warps (each covering the 128 TMEM lanes) take alternate tiles, all
// columns each, so three tiles' epilogues run at once; with fewer, the three
// take every tile, a third of its 16-column chunks each.
__host__ __device__ constexpr int epilogue_groups(int tmem_buffers) { return tmem_buffers >= 4 ? 3 : 1; }

struct DirectTail {
    unsigned long long full_a[max_direct_stages];
    unsigned long long empty_a[max_direct_stages];
    unsigned long long full_b[max_direct_stages];
    unsigned long long empty_b[max_direct_stages];
    unsigned long long tmem_full[max_tmem_buffers];
    unsigned long long tmem_empty[max_tmem_buffers];
    unsigned long long window_full[window_slots];
    unsigned long long window_empty[window_slots];
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

// Descriptor of an A block starting `dx` rows into a swizzled row-halo box
// (the box 1 KiB aligned): the start address moved by dx rows and the matrix
// base offset left 0. The tensor cores apply the swizzle by the operand's
// shared-memory address bits, as the TMA did when it wrote the box, so a start
// anywhere on a row boundary reads the rows that follow it (measured on B200:
// full-size outputs identical to the per-tap boxes' with base offset 0, wrong
// with the base offset set to the start's swizzle phase).
__device__ __forceinline__ std::uint64_t row_descriptor(std::uint32_t address, int k_block) {
    return swizzled_descriptor(address, k_block);
}

// Bytes of the per-column scales and biases after the tail.
__host__ __device__ constexpr int column_bytes(int columns) { return columns * 8; }

// After the column parameters, per epilogue warp: one block of 16 channels x
// 32 positions of FP16 results on its way from the accumulator layout (a thread
// per position) to 16-byte runs of one channel's consecutive positions.
constexpr int staging_warp_bytes = 16 * 32 * 2;
constexpr int staging_bytes = epilogue_warps * staging_warp_bytes;

__host__ __device__ constexpr int tail_bytes() { return static_cast<int>((sizeof(DirectTail) + 15) / 16 * 16); }

// The window warp stages each tile's halo of pixel maxima ((patch_h + 2) x
// (patch_w + 2) at most: 390 floats for a 1 x 128 patch, 408 with rows of
// whole 16-byte vectors) in one of window_slots slots, that many tiles ahead.
constexpr int halo_slot_floats = 416;
constexpr int halo_lane_items = (halo_slot_floats + 31) / 32;
__host__ __device__ constexpr int halo_ring_bytes(int m_tiles) { return window_slots * m_tiles * halo_slot_floats * 4; }

__device__ __forceinline__ void cp_async4(std::uint32_t dst, const void* src, int src_bytes) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
// Layout of a tile's halo of pixel maxima in its slot: rows `pitch` floats
// apart, the halo's first column at `shift`. With vector copies (image rows of
// whole 16-byte vectors, the maxima 16-byte aligned, patch_w a multiple of 4)
// every halo row starts at the 16-byte vector holding its first column
// (`shift` = that column mod 4, the same for every patch) and spans whole
// vectors; otherwise rows are halo_w floats from column 0.
struct HaloLayout {
    bool vectors;
    int shift, pitch, row_vectors;
};
__device__ __forceinline__ HaloLayout halo_layout(const DirectConvArgs& a) {
    const int halo_h = a.patch_h + a.window.kernel_h - 1;
    const int halo_w = a.patch_w + a.window.kernel_w - 1;
    HaloLayout h;
    h.shift = ((-a.window.pad_left) % 4 + 4) % 4;
    h.row_vectors = (halo_w + h.shift + 3) / 4;
    h.vectors = a.in_w % 4 == 0 && a.patch_w % 4 == 0 && (reinterpret_cast<std::uintptr_t>(a.pixel_max) & 15u) == 0 &&
        halo_h * 4 * h.row_vectors <= halo_slot_floats;
    if (!h.vectors) {
        h.shift = 0;
        h.row_vectors = 0;
    }
    h.pitch = h.vectors ? 4 * h.row_vectors : halo_w;
    return h;
}

__device__ __forceinline__ void cp_async16(std::uint32_t dst, const void* src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
// An arrival on the mbarrier once all of this thread's earlier cp.async copies
// have landed (the barrier's count includes it).
__device__ __forceinline__ void cp_async_arrive(std::uint32_t bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Exponent of a window with a non-finite value (the row is NaN), and the code
// of a window whose pixels have different exponents (the fallback writes it).
constexpr int window_nan = INT_MIN;
constexpr int window_mixed = INT_MAX;

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

// NCHW planes (FP16 or FP32) -> per-pixel int8, for planes whose length is a
// multiple of one 16-byte vector. A block takes 256 bytes of every plane (128
// FP16 or 64 FP32 pixels): each thread keeps eight 16-byte loads in flight, and
// vector v of channel c goes to shared slot v ^ ((c / 16) mod 16), so the
// threads that later read sixteen channels of one pixel, or one channel of 32
// pixels, hit different banks. Each pixel's record is then stored as
// consecutive 16-byte pieces: a block writes one contiguous run.
template <bool Half>
__global__ void __launch_bounds__(256) quantise_planes_wide_kernel(const void* __restrict__ in, int channels, int c8,
                                                                   int pixels, std::int8_t* __restrict__ out,
                                                                   float* __restrict__ pixel_max,
                                                                   unsigned int* __restrict__ clear_word) {
    constexpr int element = Half ? 2 : 4;
    constexpr int block_pixels = 256 / element;
    constexpr int per_vector = 16 / element;
    constexpr int threads_per_pixel = 256 / block_pixels;
    grid_dependency_wait();
    launch_dependents();
    if (clear_word != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *clear_word = 0u;
    extern __shared__ uint4 planes[];  // [channels][16] swizzled vectors
    __shared__ std::uint32_t partial[threads_per_pixel][block_pixels];
    __shared__ float maxima[block_pixels];
    const long long first = static_cast<long long>(blockIdx.x) * block_pixels;
    const int valid = static_cast<int>(pixels - first < block_pixels ? pixels - first : block_pixels);
    const int valid_vectors = valid / per_vector;
    const long long plane_vectors = pixels / per_vector;
    const uint4* source = reinterpret_cast<const uint4*>(in) + first / per_vector;
    const int items = channels * 16;
    for (int base = threadIdx.x; base < items; base += 256 * 8) {
        uint4 r[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int i = base + u * 256;
            const int c = i >> 4;
            const int v = i & 15;
            r[u] = make_uint4(0u, 0u, 0u, 0u);
            if (i < items && v < valid_vectors) r[u] = __ldg(source + c * plane_vectors + v);
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int i = base + u * 256;
            const int c = i >> 4;
            if (i < items) planes[c * 16 + ((i & 15) ^ (c >> 4 & 15))] = r[u];
        }
    }
    __syncthreads();
    // Element (c, p) of the swizzled tile, as magnitude bits (FP16 bits for Half).
    auto element_at = [&](int c, int p) -> std::uint32_t {
        const int slot = c * 16 + ((p / per_vector) ^ (c >> 4 & 15));
        if constexpr (Half) {
            return reinterpret_cast<const std::uint16_t*>(planes + slot)[p % per_vector];
        } else {
            return reinterpret_cast<const std::uint32_t*>(planes + slot)[p % per_vector];
        }
    };
    {
        const int p = threadIdx.x % block_pixels;
        const int part = threadIdx.x / block_pixels;
        std::uint32_t m = 0;
        for (int c = part; c < channels; c += threads_per_pixel) {
            m = max(m, element_at(c, p) & (Half ? 0x7fffu : 0x7fffffffu));
        }
        partial[part][p] = m;
    }
    __syncthreads();
    if (threadIdx.x < block_pixels) {
        const int p = threadIdx.x;
        std::uint32_t m = partial[0][p];
#pragma unroll
        for (int k = 1; k < threads_per_pixel; ++k) m = max(m, partial[k][p]);
        float maximum;
        if constexpr (Half) {
            maximum = m >= 0x7c00u ? __uint_as_float(0x7f800000u) : __half2float(__ushort_as_half(static_cast<unsigned short>(m)));
        } else {
            maximum = max_from_magnitude_bits(m);
        }
        maxima[p] = maximum;
        if (p < valid) pixel_max[first + p] = maximum;
    }
    __syncthreads();
    const int pieces = c8 / 16;
    uint4* target = reinterpret_cast<uint4*>(out + first * c8);
    for (int item = threadIdx.x; item < valid * pieces; item += 256) {
        const int p = item / pieces;
        const int c0 = (item - p * pieces) * 16;
        const PixelScale s = pixel_scale(maxima[p]);
        int q[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const int c = c0 + j;
            float x = 0.0f;
            if (c < channels) {
                const std::uint32_t bits = element_at(c, p);
                if constexpr (Half) {
                    x = __half2float(__ushort_as_half(static_cast<unsigned short>(bits)));
                } else {
                    x = __uint_as_float(bits);
                }
            }
            q[j] = (c < channels && s.finite) ? quantise_one(x, s.normal, s.scale, s.exponent) : 0;
        }
        target[item] = pack16(q);
    }
}

// FP16 NCHW planes -> per-pixel int8, for up to 256 channels (c8 <= 256) and
// planes whose length is a multiple of 8. Thread (sub-tile s, channel group
// cg, vector v) holds channels 16 cg .. 16 cg + 15 of pixels 8 v .. 8 v + 7 of
// its 128-pixel sub-tile in registers (one 16-byte load per channel; the 16
// threads of a group read 256 contiguous bytes of a plane). Per-pixel maxima
// are magnitude bits reduced two pixels to a word, then across the channel
// groups through shared memory. Quantisation, for a pixel whose 2^-e is a
// normal half and whose max * 2^-e < 127.5: fma.rn.f16x2(x, 2^-e, 1536) per
// pixel pair of one channel. x * 2^-e is exact and |x * 2^-e| < 127.5, so the
// single rounding of the sum lands in [1024, 2048), where halves are the
// integers and rounding to nearest-even is rint; the low byte of each half is
// then rint(x * 2^-e) and no clamp can act. Other pixels (non-finite ones
// write zeros) take the float path. Byte permutes turn the per-channel words
// into per-pixel records, stored as one 16-byte piece per pixel and group.
constexpr int half_planes_max_c8 = 256;

// The FP16 fast path of a pixel from its max |x| as FP16 bits (finite when
// below 0x7c00): 2^-e as FP16 bits when the pixel takes it, else 0. The pixel's
// exponent is e = frexp(max) - 7, and the path needs -15 <= e <= 14 and
// max * 2^-e < 127.5 (the FP16 fused multiply-add with 1536 then leaves q in
// the low byte). On the bits: a normal max = 1.m * 2^(E - 15) has e = E - 21, so
// the path holds for E >= 6 with m < 1016/1024 (1.m * 64 < 127.5), and 2^-e is
// the FP16 of exponent field 36 - E; an all-zero pixel (e = 0) takes it with
// 2^0; subnormal, infinite and NaN maxima do not. (Equal to the float rule for
// every FP16 pattern, checked exhaustively.)
__device__ __forceinline__ std::uint32_t half_fast_scale(std::uint32_t magnitude) {
    const std::uint32_t exponent = magnitude >> 10;
    const bool fast = exponent >= 6u && exponent < 31u && (magnitude & 0x3ffu) < 1016u;
    return magnitude == 0u ? 15u << 10 : (fast ? (36u - exponent) << 10 : 0u);
}

__device__ __forceinline__ std::uint32_t hfma2_bits(std::uint32_t x, std::uint32_t s, std::uint32_t c) {
    std::uint32_t r;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(x), "r"(s), "r"(c));
    return r;
}

__device__ __forceinline__ std::uint32_t byte_perm(std::uint32_t a, std::uint32_t b, std::uint32_t selector) {
    return __byte_perm(a, b, selector);
}

__device__ __forceinline__ std::uint32_t word_of(const uint4& v, int w) {
    return w == 0 ? v.x : (w == 1 ? v.y : (w == 2 ? v.z : v.w));
}

template <int CPT>  // channels per thread: 16 (8 also compiles: half the registers)
__global__ void __launch_bounds__(CPT == 8 ? 512 : 256, 2)
    quantise_half_planes_kernel(const __half* __restrict__ in, int channels, int c8, int pixels, int sub_tiles,
                                int octet_shift, std::int8_t* __restrict__ out, float* __restrict__ pixel_max,
                                unsigned int* __restrict__ clear_word) {
    grid_dependency_wait();
    launch_dependents();
    if (clear_word != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *clear_word = 0u;
    // A sub-tile is `octets` x 8 pixels (octets = 16, 8 or 4: fewer for small
    // inputs, so the blocks cover every SM) x c8 channels; thread (cg, v) takes
    // channels cg * CPT .. and pixels 8v ...
    extern __shared__ uint4 group_maxima[];  // [sub_tiles][groups][octets]
    const int octets = 1 << octet_shift;
    const int groups = c8 / CPT;
    const int per_tile = octets * groups;
    const int s = static_cast<int>(threadIdx.x) / per_tile;
    const int r = static_cast<int>(threadIdx.x) - s * per_tile;
    const int cg = r >> octet_shift;
    const int v = r & (octets - 1);
    const long long p0 = (static_cast<long long>(blockIdx.x) * sub_tiles + s) * (8 * octets) + v * 8;
    const bool live = p0 < pixels;
    uint4 x[CPT];
#pragma unroll
    for (int j = 0; j < CPT; ++j) {
        const int c = cg * CPT + j;
        x[j] = make_uint4(0u, 0u, 0u, 0u);
        if (live && c < channels) x[j] = __ldg(reinterpret_cast<const uint4*>(in + static_cast<std::size_t>(c) * pixels + p0));
    }
    std::uint32_t m[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int j = 0; j < CPT; ++j) {
#pragma unroll
        for (int w = 0; w < 4; ++w) m[w] = __vmaxu2(m[w], word_of(x[j], w) & 0x7fff7fffu);
    }
    group_maxima[(s * groups + cg) * octets + v] = make_uint4(m[0], m[1], m[2], m[3]);
    __syncthreads();
    if (!live) return;
    for (int g = 0; g < groups; ++g) {
        const uint4 q = group_maxima[(s * groups + g) * octets + v];
        m[0] = __vmaxu2(m[0], q.x);
        m[1] = __vmaxu2(m[1], q.y);
        m[2] = __vmaxu2(m[2], q.z);
        m[3] = __vmaxu2(m[3], q.w);
    }
    float maxima[8];
    std::uint32_t scale_bits[4] = {0u, 0u, 0u, 0u};  // 2^-e of pixels 2w, 2w + 1 as a half pair
    std::uint32_t slow = 0;                          // bit p: pixel p takes the float path
#pragma unroll
    for (int p = 0; p < 8; ++p) {
        const std::uint32_t magnitude = (m[p >> 1] >> (16 * (p & 1))) & 0xffffu;
        const bool finite = magnitude < 0x7c00u;
        const float maximum = finite ? __half2float(__ushort_as_half(static_cast<unsigned short>(magnitude)))
                                     : __uint_as_float(0x7f800000u);
        maxima[p] = maximum;
        const std::uint32_t fast_scale = half_fast_scale(magnitude);
        slow |= fast_scale != 0u ? 0u : 1u << p;
        scale_bits[p >> 1] |= fast_scale << (16 * (p & 1));
    }
    if (cg == 0) {
        float4* target = reinterpret_cast<float4*>(pixel_max + p0);
        target[0] = make_float4(maxima[0], maxima[1], maxima[2], maxima[3]);
        target[1] = make_float4(maxima[4], maxima[5], maxima[6], maxima[7]);
    }
    constexpr std::uint32_t magic = 0x66006600u;  // 1536 in both halves
    std::int8_t* row = out + p0 * c8 + cg * CPT;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        std::uint32_t even[CPT / 4], odd[CPT / 4];  // records of pixels 2w and 2w + 1, channels 4k .. 4k + 3 in word k
#pragma unroll
        for (int k = 0; k < CPT / 4; ++k) {
            const std::uint32_t r0 = hfma2_bits(word_of(x[4 * k], w), scale_bits[w], magic);
            const std::uint32_t r1 = hfma2_bits(word_of(x[4 * k + 1], w), scale_bits[w], magic);
            const std::uint32_t r2 = hfma2_bits(word_of(x[4 * k + 2], w), scale_bits[w], magic);
            const std::uint32_t r3 = hfma2_bits(word_of(x[4 * k + 3], w), scale_bits[w], magic);
            const std::uint32_t lo = byte_perm(r0, r1, 0x6240u);  // r0.b0 r1.b0 r0.b2 r1.b2
            const std::uint32_t hi = byte_perm(r2, r3, 0x6240u);
            even[k] = byte_perm(lo, hi, 0x5410u);
            odd[k] = byte_perm(lo, hi, 0x7632u);
        }
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const int p = 2 * w + e;
            std::uint32_t* words = e == 0 ? even : odd;
            if ((slow >> p) & 1u) {
                const PixelScale sc = pixel_scale(maxima[p]);
#pragma unroll
                for (int k = 0; k < CPT / 4; ++k) {
                    std::uint32_t word = 0;
#pragma unroll
                    for (int b = 0; b < 4; ++b) {
                        const std::uint32_t bits = (word_of(x[4 * k + b], w) >> (16 * e)) & 0xffffu;
                        const float value = __half2float(__ushort_as_half(static_cast<unsigned short>(bits)));
                        const int q = sc.finite ? quantise_one(value, sc.normal, sc.scale, sc.exponent) : 0;
                        word |= (static_cast<std::uint32_t>(q) & 0xffu) << (8 * b);
                    }
                    words[k] = word;
                }
            }
            if constexpr (CPT == 16) {
                *reinterpret_cast<uint4*>(row + static_cast<std::size_t>(p) * c8) =
                    make_uint4(words[0], words[1], words[2], words[3]);
            } else {
                *reinterpret_cast<uint2*>(row + static_cast<std::size_t>(p) * c8) = make_uint2(words[0], words[1]);
            }
        }
    }
}

// The same quantisation as a persistent, streamed kernel: one block of 256
// threads per SM walks its tiles (sub_tiles x 128 pixels x c8 channels), whose
// planes arrive by TMA (one [c8][128] FP16 box per sub-tile, channels past the
// last zero-filled) into a ring of streamed_stages shared-memory stages issued
// streamed_stages - 1 tiles ahead, so HBM reads of later tiles overlap the
// arithmetic and stores of the current one. Per tile the arithmetic is the
// plane kernel's above, reading the tile from shared memory.
constexpr int streamed_stages = 3;
constexpr int streamed_threads = 256;
constexpr int streamed_stage_bytes = streamed_threads * 16 * 16;  // 16 channels x 8 pixels of FP16 a thread

__global__ void __launch_bounds__(streamed_threads, 1)
    quantise_half_planes_streamed_kernel(const __grid_constant__ CUtensorMap planes, int channels, int c8, int pixels,
                                         int sub_tiles, int tiles, std::int8_t* __restrict__ out,
                                         float* __restrict__ pixel_max, unsigned int* __restrict__ clear_word) {
    extern __shared__ std::uint8_t streamed_raw[];
    // TMA destinations start 1 KiB aligned (the allocation has 1 KiB spare).
    std::uint8_t* streamed_smem =
        streamed_raw + (((smem_address(streamed_raw) + 1023u) & ~1023u) - smem_address(streamed_raw));
    constexpr int CPT = 16;
    const int groups = c8 / CPT;
    const int per_tile = 16 * groups;
    uint4* group_maxima = reinterpret_cast<uint4*>(streamed_smem + streamed_stages * streamed_stage_bytes);
    auto* full = reinterpret_cast<unsigned long long*>(group_maxima + sub_tiles * groups * 16);
    __shared__ unsigned int failed;
    if (threadIdx.x == 0) {
        for (int s = 0; s < streamed_stages; ++s) barrier_init(smem_address(&full[s]), 1);
        failed = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        fence_proxy_async_shared();
    }
    __syncthreads();
    grid_dependency_wait();
    launch_dependents();
    if (clear_word != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *clear_word = 0u;
    const int step = static_cast<int>(gridDim.x);
    const int first = static_cast<int>(blockIdx.x);
    const int my_tiles = first < tiles ? (tiles - first + step - 1) / step : 0;
    const std::uint32_t stage_base = smem_address(streamed_smem);
    const std::uint32_t sub_bytes = static_cast<std::uint32_t>(c8) * 256u;
    auto issue = [&](int local, int stage) {
        const std::uint32_t bar = smem_address(&full[stage]);
        barrier_expect_bytes(bar, sub_bytes * static_cast<std::uint32_t>(sub_tiles));
        const int tile = first + local * step;
        for (int sub = 0; sub < sub_tiles; ++sub) {
            tma_load_2d(stage_base + static_cast<std::uint32_t>(stage) * streamed_stage_bytes + sub * sub_bytes, &planes,
                        bar, (tile * sub_tiles + sub) * 128, 0);
        }
    };
    if (threadIdx.x == 0) {
        for (int k = 0; k < streamed_stages - 1 && k < my_tiles; ++k) issue(k, k);
    }
    const int s = static_cast<int>(threadIdx.x) / per_tile;
    const int r = static_cast<int>(threadIdx.x) - s * per_tile;
    const int cg = r >> 4;
    const int v = r & 15;
    const bool active = s < sub_tiles;
    int stage = 0;
    std::uint32_t phase = 0;
    for (int i = 0; i < my_tiles; ++i) {
        if (threadIdx.x == 0 && i + streamed_stages - 1 < my_tiles) {
            const int ahead = stage == 0 ? streamed_stages - 1 : stage - 1;  // (i + stages - 1) % stages
            issue(i + streamed_stages - 1, ahead);
        }
        const bool landed = barrier_wait(smem_address(&full[stage]), phase, &failed);
        if (!__syncthreads_and(landed ? 1 : 0)) return;  // a copy that never landed: nothing more is written
        const int tile = first + i * step;
        const long long p0 = (static_cast<long long>(tile) * sub_tiles + s) * 128 + v * 8;
        const bool live = active && p0 < pixels;
        const std::uint8_t* tile_smem = streamed_smem + stage * streamed_stage_bytes + s * c8 * 256;
        uint4 x[CPT];
#pragma unroll
        for (int j = 0; j < CPT; ++j) {
            x[j] = active ? *reinterpret_cast<const uint4*>(tile_smem + (cg * CPT + j) * 256 + v * 16)
                          : make_uint4(0u, 0u, 0u, 0u);
        }
        std::uint32_t m[4] = {0u, 0u, 0u, 0u};
#pragma unroll
        for (int j = 0; j < CPT; ++j) {
#pragma unroll
            for (int w = 0; w < 4; ++w) m[w] = __vmaxu2(m[w], word_of(x[j], w) & 0x7fff7fffu);
        }
        if (active) group_maxima[(s * groups + cg) * 16 + v] = make_uint4(m[0], m[1], m[2], m[3]);
        __syncthreads();
        if (live) {
            for (int g = 0; g < groups; ++g) {
                const uint4 q = group_maxima[(s * groups + g) * 16 + v];
                m[0] = __vmaxu2(m[0], q.x);
                m[1] = __vmaxu2(m[1], q.y);
                m[2] = __vmaxu2(m[2], q.z);
                m[3] = __vmaxu2(m[3], q.w);
            }
            float maxima[8];
            std::uint32_t scale_bits[4] = {0u, 0u, 0u, 0u};
            std::uint32_t slow = 0;
#pragma unroll
            for (int p = 0; p < 8; ++p) {
                const std::uint32_t magnitude = (m[p >> 1] >> (16 * (p & 1))) & 0xffffu;
                const bool finite = magnitude < 0x7c00u;
                const float maximum = finite ? __half2float(__ushort_as_half(static_cast<unsigned short>(magnitude)))
                                             : __uint_as_float(0x7f800000u);
                maxima[p] = maximum;
                const std::uint32_t fast_scale = half_fast_scale(magnitude);
                slow |= fast_scale != 0u ? 0u : 1u << p;
                scale_bits[p >> 1] |= fast_scale << (16 * (p & 1));
            }
            if (cg == 0) {
                float4* target = reinterpret_cast<float4*>(pixel_max + p0);
                target[0] = make_float4(maxima[0], maxima[1], maxima[2], maxima[3]);
                target[1] = make_float4(maxima[4], maxima[5], maxima[6], maxima[7]);
            }
            constexpr std::uint32_t magic = 0x66006600u;  // 1536 in both halves
            std::int8_t* row = out + p0 * c8 + cg * CPT;
#pragma unroll
            for (int w = 0; w < 4; ++w) {
                std::uint32_t even[CPT / 4], odd[CPT / 4];
#pragma unroll
                for (int k = 0; k < CPT / 4; ++k) {
                    const std::uint32_t r0 = hfma2_bits(word_of(x[4 * k], w), scale_bits[w], magic);
                    const std::uint32_t r1 = hfma2_bits(word_of(x[4 * k + 1], w), scale_bits[w], magic);
                    const std::uint32_t r2 = hfma2_bits(word_of(x[4 * k + 2], w), scale_bits[w], magic);
                    const std::uint32_t r3 = hfma2_bits(word_of(x[4 * k + 3], w), scale_bits[w], magic);
                    const std::uint32_t lo = byte_perm(r0, r1, 0x6240u);
                    const std::uint32_t hi = byte_perm(r2, r3, 0x6240u);
                    even[k] = byte_perm(lo, hi, 0x5410u);
                    odd[k] = byte_perm(lo, hi, 0x7632u);
                }
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int p = 2 * w + e;
                    std::uint32_t* words = e == 0 ? even : odd;
                    if ((slow >> p) & 1u) {
                        const PixelScale sc = pixel_scale(maxima[p]);
#pragma unroll
                        for (int k = 0; k < CPT / 4; ++k) {
                            std::uint32_t word = 0;
#pragma unroll
                            for (int b = 0; b < 4; ++b) {
                                const std::uint32_t bits = (word_of(x[4 * k + b], w) >> (16 * e)) & 0xffffu;
                                const float value = __half2float(__ushort_as_half(static_cast<unsigned short>(bits)));
                                const int q = sc.finite ? quantise_one(value, sc.normal, sc.scale, sc.exponent) : 0;
                                word |= (static_cast<std::uint32_t>(q) & 0xffu) << (8 * b);
                            }
                            words[k] = word;
                        }
                    }
                    *reinterpret_cast<uint4*>(row + static_cast<std::size_t>(p) * c8) =
                        make_uint4(words[0], words[1], words[2], words[3]);
                }
            }
        }
        __syncthreads();  // the stage and the group maxima are free for the next tile
        if (++stage == streamed_stages) {
            stage = 0;
            phase ^= 1u;
        }
    }
}

constexpr int field_run = 128;  // output positions per block of the row-staged field prepass

// Receptive fields of a run of 128 output positions of one output row: the
// block first copies the input rows the run's windows cover ([channels]
// [kernel_h][span] floats, zero outside the image) with coalesced loads, then
// each thread builds its position's field from shared memory through a table
// of offsets (k = c * taps + tap, -1 past channels * taps), its max |x|, and the
// field quantised with its own exponent into C8 bytes.
template <bool Half, int C8>
__global__ void __launch_bounds__(field_run) quantise_fields_rows_kernel(const void* __restrict__ in, int channels,
                                                                         int in_h, int in_w, Window w, int out_h,
                                                                         int out_w, int span,
                                                                         std::int8_t* __restrict__ out,
                                                                         float* __restrict__ field_max) {
    grid_dependency_wait();
    launch_dependents();
    extern __shared__ float rows[];  // [channels * kernel_h][span]
    __shared__ int offset_of[C8];
    const int kh = w.kernel_h;
    const int kw = w.kernel_w;
    const int taps = kh * kw;
    const int oy = blockIdx.y;
    const int ox0 = blockIdx.x * field_run;
    const int iy0 = oy * w.stride_y - w.pad_top;
    const int ix0 = ox0 * w.stride_x - w.pad_left;
    for (int k = threadIdx.x; k < C8; k += field_run) {
        const int c = k / taps;
        const int tap = k - c * taps;
        const int ky = tap / kw;
        offset_of[k] = k < channels * taps ? (c * kh + ky) * span + (tap - ky * kw) : -1;
    }
    // Columns of this thread in every staged row (span <= 4 * field_run).
    int column[4];
    bool column_inside[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        column[u] = static_cast<int>(threadIdx.x) + u * field_run;
        const int ix = ix0 + column[u];
        column_inside[u] = column[u] < span && ix >= 0 && ix < in_w;
    }
    const unsigned plane = static_cast<unsigned>(in_h) * static_cast<unsigned>(in_w);
    for (int rc = 0; rc < channels * kh; ++rc) {
        const int c = rc / kh;
        const int iy = iy0 + (rc - c * kh);
        const bool row_inside = iy >= 0 && iy < in_h;
        const unsigned row_at = static_cast<unsigned>(c) * plane + static_cast<unsigned>(row_inside ? iy : 0) * in_w +
            static_cast<unsigned>(ix0);
        float v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            v[u] = 0.0f;
            if (row_inside && column_inside[u]) {
                const unsigned at = row_at + static_cast<unsigned>(column[u]);
                v[u] = Half ? __half2float(static_cast<const __half*>(in)[at]) : static_cast<const float*>(in)[at];
            }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            if (column[u] < span) rows[rc * span + column[u]] = v[u];
        }
    }
    __syncthreads();
    const int ox = ox0 + static_cast<int>(threadIdx.x);
    if (ox >= out_w) return;
    const int col0 = static_cast<int>(threadIdx.x) * w.stride_x;
    float v[C8];
    std::uint32_t m = 0;
#pragma unroll
    for (int k = 0; k < C8; ++k) {
        const int at = offset_of[k];
        v[k] = at >= 0 ? rows[at + col0] : 0.0f;
        m = max(m, magnitude_bits_of(v[k]));
    }
    const float maximum = max_from_magnitude_bits(m);
    const long long position = static_cast<long long>(oy) * out_w + ox;
    field_max[position] = maximum;
    const PixelScale sc = pixel_scale(maximum);
    uint4* record = reinterpret_cast<uint4*>(out + position * C8);
#pragma unroll
    for (int k0 = 0; k0 < C8; k0 += 16) {
        int q[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) q[j] = sc.finite ? quantise_one(v[k0 + j], sc.normal, sc.scale, sc.exponent) : 0;
        record[k0 / 16] = pack16(q);
    }
}

// The receptive-field prepass for a fixed small window (C channels, KH x KW
// taps; C * KH * KW <= C8 <= 64): gather offsets are compile-time, FP16 rows are
// staged with 16-byte loads when the rows allow it, and the common
// quantisation is one fused multiply-add per value, q = y - 1.5 * 2^23 for
// y = fma(x, 2^-e, 1.5 * 2^23): with |x * 2^-e| < 127.5 the single rounding is
// rint and q's low byte is the low byte of y's bits, packed four at a time by
// byte permutes. A position whose max * 2^-e reaches 127.5 (the clamp may act),
// whose 2^-e is not a normal float, or whose field is non-finite takes the
// general path.
template <bool Half, int C, int KH, int KW, int C8>
__global__ void __launch_bounds__(field_run) quantise_fields_fixed_kernel(const void* __restrict__ in, int in_h,
                                                                          int in_w, Window w, int out_h, int out_w,
                                                                          int span, int vector_rows,
                                                                          std::int8_t* __restrict__ out,
                                                                          float* __restrict__ field_max) {
    grid_dependency_wait();
    launch_dependents();
    extern __shared__ float rows[];  // [C * KH][pitch], column 0 at input column ix0 - shift
    constexpr int values = C * KH * KW;
    static_assert(values <= C8 && C8 % 32 == 0 && C8 <= 64, "field width");
    const int oy = blockIdx.y;
    const int ox0 = blockIdx.x * field_run;
    const int iy0 = oy * w.stride_y - w.pad_top;
    const int ix0 = ox0 * w.stride_x - w.pad_left;
    const unsigned plane = static_cast<unsigned>(in_h) * static_cast<unsigned>(in_w);
    // Staged rows start at the aligned column at or before ix0 when 16-byte row
    // loads apply (in_w a multiple of 8: every row starts 16-byte aligned), so
    // each load becomes two 16-byte shared stores; `shift` = ix0 - that column.
    const bool vectors_apply = Half && vector_rows;
    const int a0 = vectors_apply ? (ix0 >= 0 ? (ix0 & ~7) : -((-ix0 + 7) & ~7)) : ix0;
    const int shift = ix0 - a0;
    const int pitch = (span + 7 + 7) & ~7;  // the shift (< 8) plus span, in whole 8-float vectors
    // Stride 2 with vector rows: each staged row is split by column parity, so
    // the gather's lanes (positions 2 columns apart) read consecutive floats
    // instead of every other one (two lanes per bank).
    const bool split = vectors_apply && w.stride_x == 2;
    if (vectors_apply) {
        const int vectors = (shift + span + 7) / 8;
        for (int i = threadIdx.x; i < C * KH * vectors; i += field_run) {
            const int rc = i / vectors;
            const int vcol = i - rc * vectors;
            const int c = rc / KH;
            const int iy = iy0 + (rc - c * KH);
            const int x0 = a0 + 8 * vcol;
            uint4 raw = make_uint4(0u, 0u, 0u, 0u);
            const bool row_inside = iy >= 0 && iy < in_h;
            if (row_inside && x0 >= 0 && x0 + 8 <= in_w) {
                raw = __ldg(reinterpret_cast<const uint4*>(static_cast<const __half*>(in) + static_cast<unsigned>(c) * plane +
                                                           static_cast<unsigned>(iy) * in_w + x0));
            } else if (row_inside) {
                unsigned short h[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int x = x0 + j;
                    h[j] = (x >= 0 && x < in_w)
                        ? __half_as_ushort(static_cast<const __half*>(in)[static_cast<unsigned>(c) * plane +
                                                                           static_cast<unsigned>(iy) * in_w + x])
                        : static_cast<unsigned short>(0);
                }
                raw = make_uint4(h[0] | (static_cast<unsigned>(h[1]) << 16), h[2] | (static_cast<unsigned>(h[3]) << 16),
                                 h[4] | (static_cast<unsigned>(h[5]) << 16), h[6] | (static_cast<unsigned>(h[7]) << 16));
            }
            const std::uint32_t words[4] = {raw.x, raw.y, raw.z, raw.w};
            float f[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                f[j] = __half2float(__ushort_as_half(static_cast<unsigned short>(words[j >> 1] >> (16 * (j & 1)))));
            }
            if (8 * vcol + 8 <= pitch) {
                if (split) {  // even columns in the row's first half, odd ones in its second
                    *reinterpret_cast<float4*>(rows + rc * pitch + 4 * vcol) = make_float4(f[0], f[2], f[4], f[6]);
                    *reinterpret_cast<float4*>(rows + rc * pitch + pitch / 2 + 4 * vcol) =
                        make_float4(f[1], f[3], f[5], f[7]);
                } else {
                    float4* target = reinterpret_cast<float4*>(rows + rc * pitch + 8 * vcol);
                    target[0] = make_float4(f[0], f[1], f[2], f[3]);
                    target[1] = make_float4(f[4], f[5], f[6], f[7]);
                }
            }
        }
    } else {
        for (int i = threadIdx.x; i < C * KH * span; i += field_run) {
            const int rc = i / span;
            const int col = i - rc * span;
            const int c = rc / KH;
            const int iy = iy0 + (rc - c * KH);
            const int ix = ix0 + col;
            float v = 0.0f;
            if (iy >= 0 && iy < in_h && ix >= 0 && ix < in_w) {
                const unsigned at = static_cast<unsigned>(c) * plane + static_cast<unsigned>(iy) * in_w + ix;
                v = Half ? __half2float(static_cast<const __half*>(in)[at]) : static_cast<const float*>(in)[at];
            }
            rows[rc * pitch + col] = v;
        }
    }
    __syncthreads();
    const int ox = ox0 + static_cast<int>(threadIdx.x);
    if (ox >= out_w) return;
    // Column of tap kx within a staged row: shift + stride * t + kx, or in a
    // parity-split row (column & 1) * pitch / 2 + column / 2 = offset[kx] + t.
    int column_of[KW];
#pragma unroll
    for (int kx = 0; kx < KW; ++kx) {
        const int column = shift + kx;
        column_of[kx] = split ? (column & 1) * (pitch / 2) + (column >> 1) + static_cast<int>(threadIdx.x)
                              : column + static_cast<int>(threadIdx.x) * w.stride_x;
    }
    float v[C8];
    std::uint32_t m = 0;
#pragma unroll
    for (int k = 0; k < C8; ++k) {
        if (k < values) {
            const int c = k / (KH * KW);
            const int tap = k % (KH * KW);
            v[k] = rows[(c * KH + tap / KW) * pitch + column_of[tap % KW]];
            m = max(m, magnitude_bits_of(v[k]));
        } else {
            v[k] = 0.0f;
        }
    }
    const float maximum = max_from_magnitude_bits(m);
    const long long position = static_cast<long long>(oy) * out_w + ox;
    field_max[position] = maximum;
    const PixelScale sc = pixel_scale(maximum);
    uint4* record = reinterpret_cast<uint4*>(out + position * C8);
    const bool fast = sc.finite && sc.normal && __fmul_rn(maximum, sc.scale) < 127.5f;
    if (fast) {
        std::uint32_t words[C8 / 4];
#pragma unroll
        for (int k = 0; k < C8 / 4; ++k) {
            std::uint32_t y[4];
#pragma unroll
            for (int b = 0; b < 4; ++b) y[b] = __float_as_uint(__fmaf_rn(v[4 * k + b], sc.scale, round_magic));
            words[k] = __byte_perm(__byte_perm(y[0], y[1], 0x0040u), __byte_perm(y[2], y[3], 0x0040u), 0x5410u);
        }
#pragma unroll
        for (int k = 0; k < C8 / 16; ++k) {
            record[k] = make_uint4(words[4 * k], words[4 * k + 1], words[4 * k + 2], words[4 * k + 3]);
        }
    } else {
#pragma unroll
        for (int k0 = 0; k0 < C8; k0 += 16) {
            int q[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) q[j] = sc.finite ? quantise_one(v[k0 + j], sc.normal, sc.scale, sc.exponent) : 0;
            record[k0 / 16] = pack16(q);
        }
    }
}

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

// Position in a ring of `size` slots, advanced without divisions (the roles'
// single threads are latency-bound): slot and the parity of the pass.
struct RingPosition {
    int slot;
    std::uint32_t phase;
    __device__ __forceinline__ void advance(int step, int size) {
        slot += step;
        while (slot >= size) {
            slot -= size;
            phase ^= 1u;
        }
    }
};

// One pipeline stage's MMAs as straight-line code: Group K blocks, each for
// MTiles sub-tiles of 128 positions (accumulators n_tile columns apart), of
// Steps MMAs each (K = 32 per MMA), descriptors at compile-time offsets from the
// stage's first A block (blocks ordered K block-major, sub-tile-minor) and first
// B block. The issuing thread is latency-bound, so any run-time arithmetic
// between MMAs slows the tensor pipe.
template <int Steps, int Group, int MTiles>
__device__ __forceinline__ void issue_stage(std::uint32_t acc, std::uint32_t sub_columns, std::uint64_t a_desc,
                                            std::uint64_t b_desc, std::uint32_t idesc, std::uint32_t first,
                                            int a_block16, int b_block16) {
#pragma unroll
    for (int i = 0; i < Group; ++i) {
#pragma unroll
        for (int m = 0; m < MTiles; ++m) {
#pragma unroll
            for (int kk = 0; kk < Steps; ++kk) {
                mma_i8(acc + static_cast<std::uint32_t>(m) * sub_columns,
                       a_desc + static_cast<std::uint64_t>((i * MTiles + m) * a_block16 + 2 * kk),
                       b_desc + static_cast<std::uint64_t>(i * b_block16 + 2 * kk), idesc,
                       (i == 0 && kk == 0) ? first : 1u);
            }
        }
    }
}

// The MMAs of one K block of a row-halo stage: MTiles patches x Steps K steps
// of 32 bytes, every descriptor a constant offset from the first.
template <int Steps, int MTiles>
__device__ __forceinline__ void issue_row_block(std::uint32_t acc, std::uint32_t n_tile, std::uint64_t a_desc,
                                                int a_block16, std::uint64_t b_desc, std::uint32_t idesc,
                                                std::uint32_t first) {
#pragma unroll
    for (int m = 0; m < MTiles; ++m) {
#pragma unroll
        for (int kk = 0; kk < Steps; ++kk) {
            mma_i8(acc + static_cast<std::uint32_t>(m) * n_tile,
                   a_desc + static_cast<std::uint64_t>(m * a_block16 + 2 * kk), b_desc + static_cast<std::uint64_t>(2 * kk),
                   idesc, kk == 0 ? first : 1u);
        }
    }
}

template <int Steps, int MTiles>
__device__ __forceinline__ void issue_stage_group(int group, std::uint32_t acc, std::uint32_t sub_columns,
                                                  std::uint64_t a_desc, std::uint64_t b_desc, std::uint32_t idesc,
                                                  std::uint32_t first, int a_block16, int b_block16) {
    if constexpr (MTiles == 2) {  // paired tiles use groups of 1 or 3 K blocks
        if (group == 3) {
            issue_stage<Steps, 3, 2>(acc, sub_columns, a_desc, b_desc, idesc, first, a_block16, b_block16);
        } else {
            issue_stage<Steps, 1, 2>(acc, sub_columns, a_desc, b_desc, idesc, first, a_block16, b_block16);
        }
    } else {
        switch (group) {
        case 1: issue_stage<Steps, 1, 1>(acc, sub_columns, a_desc, b_desc, idesc, first, a_block16, b_block16); break;
        case 2: issue_stage<Steps, 2, 1>(acc, sub_columns, a_desc, b_desc, idesc, first, a_block16, b_block16); break;
        case 3: issue_stage<Steps, 3, 1>(acc, sub_columns, a_desc, b_desc, idesc, first, a_block16, b_block16); break;
        default: issue_stage<Steps, 4, 1>(acc, sub_columns, a_desc, b_desc, idesc, first, a_block16, b_block16); break;
        }
    }
}

// One warp issues the TMA copies of a ring of `ring` stages, each filled by
// `per_item` copies (ring * per_item <= 32): lanes slot * per_item ..
// slot * per_item + per_item - 1 own stage `slot` and issue copy `part` of items
// slot, slot + ring, slot + 2 ring, ... of the sequence as soon as the stage is
// free (its empty barrier's previous phase completed). A copy instruction
// occupies the issuing warp for hundreds of cycles whatever the number of lanes
// that carry a copy in it, so all copies of the stages that came free go out
// in one instruction. `issue(item, stage, part)` starts copy `part` (part 0
// first arms the full barrier with the whole stage's bytes). After an abort or
// a wait that runs out (status bit 0, abort set), each stage's part-0 lane waits,
// bounded, for its last copies to land and the warp returns.
template <typename Issue>
__device__ __forceinline__ void ring_issue(int lane, int ring, int per_item, int items, std::uint32_t empty_base,
                                           std::uint32_t full_base, volatile int* abort, unsigned int* status,
                                           Issue issue) {
    const int slot = lane / per_item;
    const int part = lane - slot * per_item;
    const bool owner = slot < ring;
    const int leader = owner ? slot * per_item : lane;
    int item = slot;
    std::uint32_t phase = 0;  // parity of the stage's pass: (item / ring) & 1
    bool failed = false;
    unsigned long long since = global_timer();
    const std::uint32_t empty = empty_base + 8u * static_cast<std::uint32_t>(slot);
    for (unsigned int spin = 0;; ++spin) {
        const bool pending = owner && item < items && !failed;
        if (!__any_sync(0xffffffffu, pending)) break;
        bool ready = pending && part == 0 && barrier_test_wait(empty, phase ^ 1u);
        ready = __shfl_sync(0xffffffffu, ready, leader) && pending;  // one answer per stage
        if (__any_sync(0xffffffffu, ready)) {
            if (ready) {
                issue(item, slot, part);
                item += ring;
                phase ^= 1u;
                since = global_timer();
            }
            continue;
        }
        // No stage is free: the leader of the stage whose item comes next (stages
        // free in order) sleeps on it, then every lane tests again.
        const int next = __reduce_min_sync(0xffffffffu, pending ? item : INT_MAX);
        if (pending && part == 0 && item == next) barrier_try_wait_hint(empty, phase ^ 1u, 20000u);
        if (pending && (spin & 15u) == 15u) {
            if (*abort) {
                failed = true;
            } else if (global_timer() - since > wait_limit_ns) {
                atomicOr(status, 1u);
                *abort = 1;
                failed = true;
            }
        }
    }
    if (failed && part == 0 && item >= ring) {  // the last copy's pass has parity phase ^ 1
        barrier_sleep_wait(full_base + 8u * static_cast<std::uint32_t>(slot), phase ^ 1u, status);
    }
    __syncwarp();
}

// MTiles = 2: two patches per tile sharing each B block. Fusions = false: no
// WSiLU, chunk-add, residual or staged output (plain or depth_to_space stores);
// those instances keep registers for a TMEM load one chunk ahead in the
// epilogue. Pairs exist only without fusions.
template <int MTiles, bool Fusions>
__global__ void __launch_bounds__(direct_threads, 1)
direct_conv_kernel(const __grid_constant__ CUtensorMap a_map, const __grid_constant__ CUtensorMap b_map,
                   DirectConvArgs a, int tmem_buffers, std::uint32_t tmem_columns) {
    extern __shared__ std::uint8_t dynamic_smem[];
    const std::uint32_t raw = smem_address(dynamic_smem);
    std::uint8_t* smem = dynamic_smem + (((raw + 1023u) & ~1023u) - raw);
    const int n_tile = a.n_tile;
    const int k_block = a.k_block;
    // A stage holds `group` consecutive K blocks of one tile (their A boxes, and
    // their B boxes unless the weights are resident, one K block per stage).
    // Row halos (patches of one output row): an A stage is one input row of the
    // patch's halo (patch_w + kernel_w - 1 pixels of one channel block, row dy
    // of the window) serving the window's kernel_w K blocks (dx = 0 ..), each
    // reading the same rows shifted by dx; B stages hold one K block each.
    const int group = a.group;
    const bool row_halo = a.row_halo != 0;
    constexpr int m_tiles = MTiles;  // sub-tiles of 128 positions sharing each B stage
    static_assert(MTiles == 1 || !Fusions, "paired tiles carry no fusions");
    constexpr bool fusions = Fusions;
    const int a_block_bytes = row_halo ? a.a_row_bytes : tile_positions_m * k_block;
    const int b_block_bytes = n_tile * k_block;
    const int a_stage_bytes = (row_halo ? 1 : group) * m_tiles * a_block_bytes;
    const int b_stage_bytes = (a.b_resident || row_halo ? 1 : group) * b_block_bytes;
    // Bytes the TMA writes into an A stage (a row halo box is not a whole 1 KiB).
    const int a_stage_fill = row_halo ? m_tiles * (a.patch_w + a.window.kernel_w - 1) * k_block : a_stage_bytes;
    // Shared memory: [A stages][B stages][tail][halo ring][column parameters];
    // stage sizes are multiples of 1024 bytes, so every stage keeps the 1 KiB
    // swizzle alignment.
    std::uint8_t* b_smem = smem + a.a_stages * a_stage_bytes;
    auto* tail = reinterpret_cast<DirectTail*>(b_smem + a.b_stages * b_stage_bytes);
    const int all_columns = a.n_tiles * n_tile;
    float* halo_maxima = reinterpret_cast<float*>(reinterpret_cast<std::uint8_t*>(tail) + tail_bytes());
    float* column_scale =
        reinterpret_cast<float*>(reinterpret_cast<std::uint8_t*>(halo_maxima) + halo_ring_bytes(m_tiles));
    const int halo_slot = m_tiles * halo_slot_floats;  // floats of one tile's halos
    float* column_bias = column_scale + all_columns;
    const std::uint32_t staging = smem_address(column_scale) + static_cast<std::uint32_t>(column_bytes(all_columns));
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // A tile: m_tiles consecutive patches (p_tile = pg * m_tiles + m) of one N tile.
    const int p_groups = (a.p_tiles + m_tiles - 1) / m_tiles;
    const int total_tiles = p_groups * a.n_tiles;
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
        for (int b = 0; b < tmem_buffers; ++b) {
            barrier_init(smem_address(&tail->tmem_full[b]), 1);
            barrier_init(smem_address(&tail->tmem_empty[b]), epilogue_threads / epilogue_groups(tmem_buffers));
        }
        for (int w = 0; w < window_slots; ++w) {
            barrier_init(smem_address(&tail->window_full[w]), 32);
            barrier_init(smem_address(&tail->window_empty[w]), epilogue_threads / epilogue_groups(tmem_buffers));
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

    // Tiles of this CTA (t = blockIdx.x, blockIdx.x + gridDim.x, ...) and the
    // (tile, K block) items of its A and B sequences.
    const int my_tiles = total_tiles > static_cast<int>(blockIdx.x)
        ? (total_tiles - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) / static_cast<int>(gridDim.x)
        : 0;
    const int stages_per_tile = k_blocks / group;                   // A stages
    const int b_per_tile = row_halo ? k_blocks : stages_per_tile;  // B stages
    const int c_blocks = a.c_blocks;
    const int kernel_w = a.window.kernel_w;
    if (warp == weight_warp) {
        // ---------------- weights by TMA (resident weights: the first tile's K blocks, once)
        const int items = a.b_resident ? (my_tiles > 0 ? k_blocks : 0) : my_tiles * b_per_tile;
        const int boxes = a.b_resident || row_halo ? 1 : group;
        ring_issue(lane, a.b_stages, boxes, items, smem_address(&tail->empty_b[0]), smem_address(&tail->full_b[0]),
                   abort, a.status, [&](int item, int stage, int part) {
                       int n_index = 0;
                       int kb0 = item;
                       if (!a.b_resident) {
                           const int local_tile = item / b_per_tile;
                           const int j = item - local_tile * b_per_tile;
                           if (row_halo) {
                               // the MMA's order: row dy, channel block cb, then dx
                               const int s_row = j / kernel_w;
                               const int dx = j - s_row * kernel_w;
                               const int dy = s_row / c_blocks;
                               kb0 = (dy * kernel_w + dx) * c_blocks + (s_row - dy * c_blocks);
                           } else {
                               kb0 = j * group;
                           }
                           by_n_tiles.divide(static_cast<int>(blockIdx.x) + local_tile * static_cast<int>(gridDim.x),
                                             n_index);
                       }
                       const std::uint32_t full = smem_address(&tail->full_b[stage]);
                       if (part == 0) barrier_expect_bytes(full, static_cast<std::uint32_t>(b_stage_bytes));
                       __syncwarp(__activemask());  // the stage's bytes are armed before any copy
                       tma_load_2d(smem_address(b_smem + stage * b_stage_bytes + part * b_block_bytes), &b_map, full,
                                   (kb0 + part) * k_block, n_index * n_tile);
                   });
    } else if (warp == activation_warp) {
        // ---------------- activations by TMA: one box per (tap, channel block)
        grid_dependency_wait();
        ring_issue(lane, a.a_stages, (row_halo ? 1 : group) * m_tiles, my_tiles * stages_per_tile,
                   smem_address(&tail->empty_a[0]), smem_address(&tail->full_a[0]), abort, a.status,
                   [&](int item, int stage, int part) {
                       const int local_tile = item / stages_per_tile;
                       const int block = part / m_tiles;  // K block of the stage
                       const int m = part - block * m_tiles;
                       const int s_tile = item - local_tile * stages_per_tile;
                       int n_unused, tx;
                       const int pg = by_n_tiles.divide(
                           static_cast<int>(blockIdx.x) + local_tile * static_cast<int>(gridDim.x), n_unused);
                       // A sub-tile past the last patch loads rows below the image: zero fill.
                       const int ty = by_tiles_x.divide(pg * m_tiles + m, tx);
                       int cb, ky, kx;
                       if (row_halo) {  // stage s_tile = row ky of the window, channel block cb; all dx
                           ky = s_tile / c_blocks;
                           cb = s_tile - ky * c_blocks;
                           kx = 0;
                       } else {
                           const int kb = s_tile * group + block;
                           const int tap = kb / c_blocks;
                           cb = kb - tap * c_blocks;
                           ky = tap / kernel_w;
                           kx = tap - ky * kernel_w;
                       }
                       const std::uint32_t full = smem_address(&tail->full_a[stage]);
                       if (part == 0) barrier_expect_bytes(full, static_cast<std::uint32_t>(a_stage_fill));
                       __syncwarp(__activemask());  // the stage's bytes are armed before any copy
                       // Innermost coordinate: the channel block's first byte, a multiple of k_block.
                       tma_load_3d(smem_address(smem + stage * a_stage_bytes + part * a_block_bytes), &a_map, full,
                                   cb * k_block, tx * a.patch_w - a.window.pad_left + kx,
                                   ty * a.patch_h - a.window.pad_top + ky);
                   });
    } else if (warp == mma_warp) {
        if (lane == 0) {
            // ---------------- tensor-core issue
            const std::uint32_t idesc = i8_instruction(n_tile);
            const int steps = k_block / 32;
            const std::uint64_t a_desc0 = swizzled_descriptor(smem_address(smem), k_block);
            const std::uint64_t b_desc0 = swizzled_descriptor(smem_address(b_smem), k_block);
            const int a_block16 = a_block_bytes >> 4;
            const int b_block16 = b_block_bytes >> 4;
            // Row halos: the descriptor of the first A stage's first row; stages,
            // patches and dx rows are address offsets in its low field.
            const std::uint64_t row_desc0 = row_descriptor(smem_address(smem), k_block);
            const std::uint64_t k_block16 = static_cast<std::uint64_t>(k_block >> 4);
            const std::uint32_t tile_columns = static_cast<std::uint32_t>(m_tiles * n_tile);
            std::uint32_t g = 0;
            int local = 0;
            bool ok = true;
            int sa = 0, sb_ring = 0;                   // ring stages of the next A and B blocks
            std::uint32_t a_phase = 0, b_ring_phase = 0;
            RingPosition accumulator{0, 0u};
            for (int t = blockIdx.x; t < total_tiles && ok;
                 t += gridDim.x, ++local, accumulator.advance(1, tmem_buffers)) {
                const int buffer = accumulator.slot;
                if (*abort ||
                    !barrier_sleep_wait(smem_address(&tail->tmem_empty[buffer]), accumulator.phase ^ 1u, a.status)) {
                    *abort = 1;
                    break;
                }
                tmem_fence_after();
                const std::uint32_t acc = tmem + static_cast<std::uint32_t>(buffer) * tile_columns;
                if (row_halo) {
                    // Stages in (dy, cb) order; within one, K blocks dx = 0 ..
                    // kernel_w - 1 read the stage's rows from row dx on: the
                    // descriptor starts dx rows in, with the matching base offset.
                    int dy = 0, cb = 0;
                    for (int st = 0; st < stages_per_tile && ok; ++st, ++g) {
                        bool ready = barrier_sleep_wait(smem_address(&tail->full_a[sa]), a_phase, a.status);
                        std::uint64_t a_desc = row_desc0 + static_cast<std::uint64_t>((sa * a_stage_bytes) >> 4);
                        for (int dx = 0; dx < kernel_w && ready; ++dx, a_desc += k_block16) {
                            const int kb = (dy * kernel_w + dx) * c_blocks + cb;
                            if (!a.b_resident) {
                                ready = barrier_sleep_wait(smem_address(&tail->full_b[sb_ring]), b_ring_phase, a.status);
                            } else if (local == 0) {
                                ready = barrier_sleep_wait(smem_address(&tail->full_b[kb]), 0u, a.status);
                            }
                            if (!ready) break;
                            const std::uint64_t b_desc = b_desc0 +
                                static_cast<std::uint64_t>((a.b_resident ? kb * b_block_bytes : sb_ring * b_stage_bytes) >> 4);
                            const std::uint32_t first = (st == 0 && dx == 0) ? 0u : 1u;
                            if (steps == 4) {
                                issue_row_block<4, MTiles>(acc, static_cast<std::uint32_t>(n_tile), a_desc, a_block16,
                                                           b_desc, idesc, first);
                            } else {
                                issue_row_block<2, MTiles>(acc, static_cast<std::uint32_t>(n_tile), a_desc, a_block16,
                                                           b_desc, idesc, first);
                            }
                            if (!a.b_resident) {
                                mma_commit(smem_address(&tail->empty_b[sb_ring]));
                                if (++sb_ring == a.b_stages) {
                                    sb_ring = 0;
                                    b_ring_phase ^= 1u;
                                }
                            }
                        }
                        if (!ready) {
                            *abort = 1;
                            ok = false;
                            break;
                        }
                        mma_commit(smem_address(&tail->empty_a[sa]));
                        if (++sa == a.a_stages) {
                            sa = 0;
                            a_phase ^= 1u;
                        }
                        if (++cb == c_blocks) {
                            cb = 0;
                            ++dy;
                        }
                    }
                    if (!ok) break;
                    mma_commit(smem_address(&tail->tmem_full[buffer]));
                    continue;
                }
                for (int kb0 = 0; kb0 < k_blocks; kb0 += group, ++g) {
                    // (TMA writes are ordered before the MMA's reads by the full
                    // barriers; only TMEM reuse needs a tcgen05 fence, above.)
                    bool ready = barrier_sleep_wait(smem_address(&tail->full_a[sa]), a_phase, a.status);
                    if (ready && !a.b_resident) {
                        ready = barrier_sleep_wait(smem_address(&tail->full_b[sb_ring]), b_ring_phase, a.status);
                    }
                    for (int i = 0; ready && a.b_resident && local == 0 && i < group; ++i) {
                        ready = barrier_sleep_wait(smem_address(&tail->full_b[kb0 + i]), 0u, a.status);
                    }
                    if (!ready) {
                        *abort = 1;
                        ok = false;
                        break;
                    }
                    // Descriptors advance by address / 16 in their low bits (the
                    // address field cannot carry: shared addresses are below 2^18).
                    const std::uint64_t a_desc = a_desc0 + static_cast<std::uint64_t>((sa * a_stage_bytes) >> 4);
                    const std::uint64_t b_desc = b_desc0 +
                        static_cast<std::uint64_t>(((a.b_resident ? kb0 * b_block_bytes : sb_ring * b_stage_bytes)) >> 4);
                    const std::uint32_t first = kb0 == 0 ? 0u : 1u;
                    const std::uint32_t sub_columns = static_cast<std::uint32_t>(n_tile);
                    if (steps == 4) {
                        issue_stage_group<4, MTiles>(group, acc, sub_columns, a_desc, b_desc, idesc, first, a_block16,
                                                     b_block16);
                    } else if (steps == 2) {
                        issue_stage_group<2, MTiles>(group, acc, sub_columns, a_desc, b_desc, idesc, first, a_block16,
                                                     b_block16);
                    } else {
                        issue_stage_group<1, MTiles>(group, acc, sub_columns, a_desc, b_desc, idesc, first, a_block16,
                                                     b_block16);
                    }
                    mma_commit(smem_address(&tail->empty_a[sa]));
                    if (!a.b_resident) mma_commit(smem_address(&tail->empty_b[sb_ring]));
                    if (++sa == a.a_stages) {
                        sa = 0;
                        a_phase ^= 1u;
                    }
                    if (++sb_ring == a.b_stages) {
                        sb_ring = 0;
                        b_ring_phase ^= 1u;
                    }
                }
                if (!ok) break;
                mma_commit(smem_address(&tail->tmem_full[buffer]));
            }
            mma_commit(smem_address(&tail->drain));
            barrier_sleep_wait(smem_address(&tail->drain), 0u, a.status);
        }
    } else if (warp == window_warp) {
        // ---------------- halos of pixel maxima, up to window_slots tiles ahead
        // Each tile's halo of pixel maxima is copied by cp.async into a shared
        // slot (zero outside the image, which changes neither the largest maximum
        // of a window nor its smallest non-zero one); every lane's copies complete
        // the slot's full barrier by themselves, so this warp never waits for them.
        grid_dependency_wait();
        const int halo_h = a.patch_h + a.window.kernel_h - 1;
        const int halo_w = a.patch_w + a.window.kernel_w - 1;
        const int halo_count = halo_h * halo_w;
        // This lane's halo elements i = lane + 32 j as (row, column) in the halo.
        short2 at[halo_lane_items];
        {
            const TileDivider by_halo_w(halo_w);
#pragma unroll
            for (int j = 0; j < halo_lane_items; ++j) {
                int hx;
                const int hy = by_halo_w.divide(lane + 32 * j, hx);
                at[j] = make_short2(static_cast<short>(hy), static_cast<short>(hx));
            }
        }
        // Halos of whole 16-byte vectors where the layout allows (a copy per
        // maximum made this warp the pace of pointwise convs with two patches
        // per tile: about 3 K cycles per tile): at most 104 vectors, four per
        // lane, their (row, vector) precomputed.
        const HaloLayout layout = halo_layout(a);
        const int halo_vectors = halo_h * layout.row_vectors;
        short2 vat[4];
        {
            const TileDivider by_row_vectors(layout.vectors ? layout.row_vectors : 1);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                int vx;
                const int vy = by_row_vectors.divide(lane + 32 * j, vx);
                vat[j] = make_short2(static_cast<short>(vy), static_cast<short>(vx));
            }
        }
        RingPosition ring{0, 0u};
        for (int l = 0; l < my_tiles; ++l, ring.advance(1, window_slots)) {
            const int slot = ring.slot;
            const bool waited =
                *abort == 0 && barrier_sleep_wait(smem_address(&tail->window_empty[slot]), ring.phase ^ 1u, a.status);
            if (!__all_sync(0xffffffffu, waited)) {
                *abort = 1;
                break;
            }
            int n_unused;
            const int pg =
                by_n_tiles.divide(static_cast<int>(blockIdx.x) + l * static_cast<int>(gridDim.x), n_unused);
            for (int m = 0; m < m_tiles; ++m) {
                int tx;
                const int ty = by_tiles_x.divide(pg * m_tiles + m, tx);  // past the last patch: all outside
                const int iy0 = ty * a.patch_h - a.window.pad_top;
                const int ix0 = tx * a.patch_w - a.window.pad_left;
                float* halo = halo_maxima + slot * halo_slot + m * halo_slot_floats;
                if (layout.vectors) {
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        if (lane + 32 * j < halo_vectors) {
                            const int iy = iy0 + vat[j].x;
                            // a multiple of 4: the vector is wholly inside or outside (in_w % 4 == 0)
                            const int ix = ix0 - layout.shift + 4 * vat[j].y;
                            const bool inside = iy >= 0 && iy < a.in_h && ix >= 0 && ix < a.in_w;
                            cp_async16(smem_address(halo + vat[j].x * layout.pitch + 4 * vat[j].y),
                                       a.pixel_max + (inside ? static_cast<std::size_t>(iy) * a.in_w + ix : 0),
                                       inside ? 16 : 0);
                        }
                    }
                    continue;
                }
#pragma unroll
                for (int j = 0; j < halo_lane_items; ++j) {
                    const int i = lane + 32 * j;
                    if (i < halo_count) {
                        const int iy = iy0 + at[j].x;
                        const int ix = ix0 + at[j].y;
                        const bool inside = iy >= 0 && iy < a.in_h && ix >= 0 && ix < a.in_w;
                        cp_async4(smem_address(halo + i),
                                  a.pixel_max + (inside ? static_cast<std::size_t>(iy) * a.in_w + ix : 0),
                                  inside ? 4 : 0);
                    }
                }
            }
            cp_async_arrive(smem_address(&tail->window_full[slot]));
        }
        cp_async_wait_all();
    } else if (warp < epilogue_warps) {
        // ---------------- epilogue: thread <-> TMEM lane <-> position
        grid_dependency_wait();
        const int quarter = warp & 3;
        const int groups = epilogue_groups(tmem_buffers);
        const int group = warp >> 2;
        const int part = groups == 3 ? 0 : group;  // column third (one group: all columns)
        const int parts = 3 / groups;
        const int row = quarter * 32 + lane;
        const std::uint32_t lane_base = static_cast<std::uint32_t>(quarter * 32) << 16;
        const bool chunk_add = fusions && a.chunk_add;
        const int pair_offset = chunk_add ? n_tile / 2 : 0;
        const int columns = chunk_add ? n_tile / 2 : n_tile;
        const int chunks = columns / 16;
        const int per_part = (chunks + parts - 1) / parts;
        const int first_column = min(part * per_part, chunks) * 16;
        const int last_column = min((part + 1) * per_part, chunks) * 16;
        const int b = a.d2s_block;
        const int patch_y = row / a.patch_w;
        const int patch_x = row - patch_y * a.patch_w;
        const int out_w_full = a.out_w * (b > 0 ? b : 1);
        const int out_h_full = a.out_h * (b > 0 ? b : 1);
        const int first_local = groups == 3 ? group : 0;
        const int tile_step = groups * static_cast<int>(gridDim.x);
        const int kernel_h = a.window.kernel_h;
        const int kernel_w = a.window.kernel_w;
        const HaloLayout halo_geometry = halo_layout(a);
        RingPosition halo_ring{0, 0u};
        RingPosition accumulator{0, 0u};
        halo_ring.advance(first_local, window_slots);
        accumulator.advance(first_local, tmem_buffers);
        for (int t = static_cast<int>(blockIdx.x) + first_local * static_cast<int>(gridDim.x); t < total_tiles;
             t += tile_step, halo_ring.advance(groups, window_slots), accumulator.advance(groups, tmem_buffers)) {
            int n_index;
            const int pg = by_n_tiles.divide(t, n_index);
            // This position's window in each sub-tile, from the tile's halos of
            // pixel maxima: the largest maximum sets the exponent, a non-finite
            // pixel makes the row NaN (window_nan), and a non-zero pixel whose
            // exponent differs from the largest marks the window as mixed
            // (window_mixed: its result comes from the fallback).
            const int slot = halo_ring.slot;
            const bool ready = barrier_sleep_wait(smem_address(&tail->window_full[slot]), halo_ring.phase, a.status);
            if (!__all_sync(0xffffffffu, ready)) {
                *abort = 1;
                break;
            }
            int codes[MTiles];
#pragma unroll
            for (int m = 0; m < MTiles; ++m) codes[m] = window_nan;
            bool any_mixed = false;
#pragma unroll
#pragma unroll
            for (int m = 0; m < MTiles; ++m) {
                float largest = 0.0f;
                float smallest = __uint_as_float(0x7f800000u);  // smallest non-zero
                const float* halo = halo_maxima + slot * halo_slot + m * halo_slot_floats + halo_geometry.shift +
                    patch_y * halo_geometry.pitch + patch_x;
                if (kernel_h == 1 && kernel_w == 1) {
                    // One pixel per window: its exponent, never mixed.
                    int tx;
                    const int ty = by_tiles_x.divide(pg * m_tiles + m, tx);
                    const bool real_m = pg * m_tiles + m < a.p_tiles && ty * a.patch_h + patch_y < a.out_h &&
                        tx * a.patch_w + patch_x < a.out_w;
                    const float v = halo[0];
                    if (real_m && v != __uint_as_float(0x7f800000u)) codes[m] = activation_exponent(v, 8);
                    continue;
                }
#pragma unroll
                for (int ky = 0; ky < 3; ++ky) {
#pragma unroll
                    for (int kx = 0; kx < 3; ++kx) {
                        if (ky < kernel_h && kx < kernel_w) {
                            const float v = halo[ky * halo_geometry.pitch + kx];
                            largest = fmaxf(largest, v);
                            if (v > 0.0f) smallest = fminf(smallest, v);
                        }
                    }
                }
                int tx;
                const int ty = by_tiles_x.divide(pg * m_tiles + m, tx);
                const bool real_m = pg * m_tiles + m < a.p_tiles && ty * a.patch_h + patch_y < a.out_h &&
                    tx * a.patch_w + patch_x < a.out_w;
                if (real_m && largest != __uint_as_float(0x7f800000u)) {
                    codes[m] = activation_exponent(largest, 8);
                    if (largest > 0.0f && frexp_exponent(smallest) != frexp_exponent(largest)) {
                        codes[m] = window_mixed;
                        any_mixed = true;
                    }
                }
            }
            barrier_arrive(smem_address(&tail->window_empty[slot]));
            if (a.fallback != nullptr && part == 0 && __any_sync(0xffffffffu, any_mixed) && lane == 0) {
                atomicOr(a.fallback, 1u);
                if (a.condition != 0) cudaGraphSetConditional(a.condition, 1u);
            }
            const int buffer = accumulator.slot;
            bool waited =
                *abort == 0 && barrier_sleep_wait(smem_address(&tail->tmem_full[buffer]), accumulator.phase, a.status);
            waited = __all_sync(0xffffffffu, waited);  // tcgen05.ld is warp-aligned
            if (!waited) {
                *abort = 1;
                break;
            }
            tmem_fence_after();
            const int physical0 = n_index * n_tile;
            const int logical0 = chunk_add ? n_index * (n_tile / 2) : physical0;
            for (int m = 0; m < m_tiles; ++m) {
            int tx;
            const int ty = by_tiles_x.divide(pg * m_tiles + m, tx);
            const int y = ty * a.patch_h + patch_y;
            const int x = tx * a.patch_w + patch_x;
            const bool real = pg * m_tiles + m < a.p_tiles && y < a.out_h && x < a.out_w;
            const int p = real ? y * a.out_w + x : 0;
            const int code = (MTiles == 1 || m == 0) ? codes[0] : codes[MTiles - 1];
            // A mixed window's accumulators are not this position's result:
            // nothing is stored for it (nor added to a staged maximum, which
            // can only grow), and the fallback conv writes it instead.
            const bool store = real && code != window_mixed;
            const int exponent = code == window_mixed ? window_nan : code;
            const std::uint32_t acc = tmem + static_cast<std::uint32_t>(buffer * m_tiles * n_tile + m * n_tile) +
                lane_base;
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
                if (fusions && a.wsilu) {
                    Sixteen16 xv;
#pragma unroll
                    for (int j = 0; j < 16; ++j) xv.v[j] = v[j];
                    xv = direct_wsilu16(xv, a.wsilu_scale);
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] = xv.v[j];
                }
            };

            std::uint32_t staged_max = 0;
            // Stores (and residual adds, staged maxima) of the 16 values at columns j0..
            auto emit = [&](int j0, float (&v)[16]) {
                const int c0 = logical0 + j0;
                const int count = a.out_channels - c0 < 16 ? a.out_channels - c0 : 16;
                if (store) {
                    if (exponent == INT_MIN) {
#pragma unroll
                        for (int j = 0; j < 16; ++j) v[j] = canonical_nan();
                    }
                    if (fusions && a.residual != nullptr) {
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
                    if (fusions && a.out_max != nullptr) {
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
            };
            if constexpr (Fusions) {
                for (int j0 = first_column; j0 < last_column; j0 += 16) {
                    float v[16];
                    values16(j0, v);
                    if (chunk_add) {
                        float w[16];
                        values16(j0 + pair_offset, w);
#pragma unroll
                        for (int j = 0; j < 16; ++j) v[j] = __fadd_rn(v[j], w[j]);
                    }
                    emit(j0, v);
                    __syncwarp();  // tcgen05.ld is warp-aligned: reconverge before the next columns
                }
            } else if (a.vector_store != 0 &&
                       __all_sync(0xffffffffu, !real || (code != window_mixed && exponent >= a.fma_lo &&
                                                         exponent <= a.fma_hi && normal))) {
                // Vector stores (every real position of the warp stored, with an
                // exponent e for which y * 2^e is exact for every y = RN(x *
                // scale) of the conv, so RN(RN(y * 2^e) + bias) = fma(y, 2^e,
                // bias)). The accumulators come out in the fragment layout
                // (16x256b: a thread holds two columns of lanes g and g + 8),
                // are converted to FP16 pairs and stored transposed into the
                // warp's staging block ([16 channels][32 positions], 16-byte
                // pieces swizzled by (channel / 2) % 4: conflict-free both
                // ways), from which each lane writes 8 positions of two channels.
                const int g = lane >> 2;
                const int t4 = lane & 3;
                float powers[4];  // positions 8i + g of the warp (matrix i)
#pragma unroll
                for (int i = 0; i < 4; ++i) powers[i] = __shfl_sync(0xffffffffu, power, 8 * i + g);
                const bool piece_real = __shfl_sync(0xffffffffu, real ? 1 : 0, 8 * t4) != 0;
                const int piece_p = __shfl_sync(0xffffffffu, p, 8 * t4);
                const int store_channel = lane >> 2;
                const std::size_t plane = static_cast<std::size_t>(a.positions);
                uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__half*>(a.out) +
                                                      static_cast<std::size_t>(logical0 + first_column + store_channel) *
                                                          plane +
                                                      piece_p);
                const std::size_t dst_chunk = 2 * plane;  // 16 planes, in uint4
                const std::size_t dst_half = plane;       // 8 planes, in uint4
                // Stored channels left from the first column (multiples of 8).
                const int stored = piece_real ? a.out_channels - logical0 - first_column : 0;
                const std::uint32_t block = staging + static_cast<std::uint32_t>(warp * staging_warp_bytes);
                const int row_channel = lane & 7;
                const std::uint32_t st_address = block + static_cast<std::uint32_t>(
                    row_channel * 64 + (((lane >> 3) ^ ((row_channel >> 1) & 3)) << 4));
                const std::uint32_t ld_address = block + static_cast<std::uint32_t>(
                    store_channel * 64 + ((t4 ^ ((store_channel >> 1) & 3)) << 4));
                const std::uint32_t upper = acc + (16u << 16);  // TMEM lanes 16..31 of the warp
                const float* scale_at = column_scale + physical0 + first_column + 2 * t4;
                const float* bias_at = column_bias + physical0 + first_column + 2 * t4;
                const int chunks16 = (last_column - first_column) >> 4;
                auto load16 = [&](std::uint32_t (&r)[16], int c) {
                    tmem_load_16x256b_x2(acc + static_cast<std::uint32_t>(first_column + 16 * c), r);
                    tmem_load_16x256b_x2(upper + static_cast<std::uint32_t>(first_column + 16 * c), r + 8);
                };
                // Chunk c: channels 16c .. 16c + 15 from the first column. r[0..7]
                // hold lanes g, g + 8 and r[8..15] lanes 16 + g, 24 + g; within
                // each eight, columns 2t4, 2t4 + 1 of the first eight channels,
                // then of the second eight.
                auto columns = [&](auto small_tag) {
                    constexpr bool small = decltype(small_tag)::value;
                    std::uint32_t r[16];
                    if (chunks16 > 0) {
                        load16(r, 0);
                        tmem_load_wait_regs(r);
                    }
                    for (int c = 0; c < chunks16; ++c) {
                        const float2 s0 = *reinterpret_cast<const float2*>(scale_at + 16 * c);
                        const float2 s1 = *reinterpret_cast<const float2*>(scale_at + 16 * c + 8);
                        const float2 h0 = *reinterpret_cast<const float2*>(bias_at + 16 * c);
                        const float2 h1 = *reinterpret_cast<const float2*>(bias_at + 16 * c + 8);
                        std::uint32_t packed[2][4];
#pragma unroll
                        for (int half = 0; half < 2; ++half) {
                            const float2 s = half == 0 ? s0 : s1;
                            const float2 h = half == 0 ? h0 : h1;
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                const int at = (i >> 1) * 8 + half * 4 + (i & 1) * 2;
                                float x0, x1;
                                if (small) {  // exact: |r| < 2^22
                                    x0 = __fadd_rn(__uint_as_float(r[at] + 0x4B400000u), -round_magic);
                                    x1 = __fadd_rn(__uint_as_float(r[at + 1] + 0x4B400000u), -round_magic);
                                } else {
                                    x0 = __int2float_rn(static_cast<int>(r[at]));
                                    x1 = __int2float_rn(static_cast<int>(r[at + 1]));
                                }
                                const float v0 = __fmaf_rn(__fmul_rn(x0, s.x), powers[i], h.x);
                                const float v1 = __fmaf_rn(__fmul_rn(x1, s.y), powers[i], h.y);
                                const __half2 pair = __floats2half2_rn(v0, v1);
                                packed[half][i] = *reinterpret_cast<const std::uint32_t*>(&pair);
                            }
                        }
                        // The next chunk's TMEM loads fly during this chunk's stores
                        // (the last chunk reloads its own columns: no branch around
                        // the warp-wide loads).
                        load16(r, c + 1 < chunks16 ? c + 1 : c);
                        stmatrix_x4_trans(st_address, packed[0]);
                        stmatrix_x4_trans(st_address + 512u, packed[1]);
                        __syncwarp();
                        const uint4 first = load_shared_v4(ld_address);
                        const uint4 second = load_shared_v4(ld_address + 512u);
                        uint4* d = dst + static_cast<std::size_t>(c) * dst_chunk;
                        if (16 * c < stored) d[0] = first;
                        if (16 * c + 8 < stored) d[dst_half] = second;
                        __syncwarp();  // the block is rewritten by the next chunk
                        tmem_load_wait_regs(r);
                    }
                };
                if (a.small_accumulators != 0) {
                    columns(std::true_type{});
                } else {
                    columns(std::false_type{});
                }
            } else {
                // The next chunk's TMEM load is issued before this chunk's
                // arithmetic and stores, which hide its latency.
                int hh[16];
                if (first_column < last_column) {
                    tmem_load16(acc + static_cast<std::uint32_t>(first_column), hh);
                    tmem_load_wait();
                }
                for (int j0 = first_column; j0 < last_column; j0 += 16) {
                    const bool more = j0 + 16 < last_column;
                    int next[16];
                    if (more) tmem_load16(acc + static_cast<std::uint32_t>(j0 + 16), next);
                    const float4* scale4 = reinterpret_cast<const float4*>(column_scale + physical0 + j0);
                    const float4* bias4 = reinterpret_cast<const float4*>(column_bias + physical0 + j0);
                    float v[16];
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const float4 f = scale4[q];
                        v[4 * q] = __fmul_rn(__int2float_rn(hh[4 * q]), f.x);
                        v[4 * q + 1] = __fmul_rn(__int2float_rn(hh[4 * q + 1]), f.y);
                        v[4 * q + 2] = __fmul_rn(__int2float_rn(hh[4 * q + 2]), f.z);
                        v[4 * q + 3] = __fmul_rn(__int2float_rn(hh[4 * q + 3]), f.w);
                    }
                    if (plain) {
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const float4 h = bias4[q];
                            v[4 * q] = __fadd_rn(__fmul_rn(v[4 * q], power), h.x);
                            v[4 * q + 1] = __fadd_rn(__fmul_rn(v[4 * q + 1], power), h.y);
                            v[4 * q + 2] = __fadd_rn(__fmul_rn(v[4 * q + 2], power), h.z);
                            v[4 * q + 3] = __fadd_rn(__fmul_rn(v[4 * q + 3], power), h.w);
                        }
                    } else {
                        Sixteen16 xv, bv;
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const float4 h = bias4[q];
                            bv.v[4 * q] = h.x;
                            bv.v[4 * q + 1] = h.y;
                            bv.v[4 * q + 2] = h.z;
                            bv.v[4 * q + 3] = h.w;
                        }
#pragma unroll
                        for (int j = 0; j < 16; ++j) xv.v[j] = v[j];
                        xv = direct_ldexp_add16(xv, bv, exponent);
#pragma unroll
                        for (int j = 0; j < 16; ++j) v[j] = xv.v[j];
                    }
                    emit(j0, v);
                    if (more) {
                        tmem_load_wait();
#pragma unroll
                        for (int j = 0; j < 16; ++j) hh[j] = next[j];
                    }
                    __syncwarp();  // tcgen05.ld is warp-aligned: reconverge before the next columns
                }
            }
            if (fusions && a.out_max != nullptr && store && first_column < last_column) {
                atomicMax(reinterpret_cast<unsigned int*>(a.out_max) + p,
                          __float_as_uint(max_from_magnitude_bits(staged_max)));
            }
            }  // sub-tiles
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
        (a.patch_h + a.window.kernel_h - 1) * (a.patch_w + a.window.kernel_w - 1) <= halo_slot_floats &&
        a.tiles_y * a.patch_h >= a.out_h && a.tiles_x * a.patch_w >= a.out_w && a.p_tiles == a.tiles_y * a.tiles_x &&
        a.positions == a.out_h * a.out_w &&
        a.group >= 1 && a.group <= 4 &&
        a.k_blocks % a.group == 0 &&
        (a.m_tiles == 1 || (a.m_tiles == 2 && (a.row_halo || a.group == 1 || a.group == 3) && 2 * a.n_tile <= 512 &&
                            !a.wsilu && !a.chunk_add && a.residual == nullptr && a.out_max == nullptr)) &&
        (!a.row_halo ||
         (a.patch_h == 1 && a.group == a.window.kernel_w && a.patch_w + a.window.kernel_w - 1 <= 256 &&
          a.a_row_bytes == direct_row_bytes(a.patch_w, a.window.kernel_w, a.k_block))) &&
        a.a_stages * (a.row_halo ? 1 : a.group) * a.m_tiles <= 32 &&
        (a.b_resident || a.b_stages * (a.row_halo ? 1 : a.group) <= 32) &&
        a.a_stages >= 2 && a.a_stages <= max_direct_stages && a.b_stages >= 1 &&
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

int direct_conv_shared_bytes(int k_block, int n_tile, int n_tiles, int a_stages, int b_stages, int group,
                             bool b_resident, int m_tiles) {
    return 1024 + a_stages * group * m_tiles * tile_positions_m * k_block +
        b_stages * (b_resident ? 1 : group) * n_tile * k_block + tail_bytes() + halo_ring_bytes(m_tiles) +
        column_bytes(n_tile * n_tiles) + staging_bytes;
}

int direct_row_bytes(int patch_w, int kernel_w, int k_block) {
    return ((patch_w + kernel_w - 1) * k_block + 1023) / 1024 * 1024;
}

int direct_conv_row_shared_bytes(int k_block, int n_tile, int n_tiles, int a_stages, int b_stages, bool b_resident,
                                 int m_tiles, int row_bytes) {
    return 1024 + a_stages * m_tiles * row_bytes + b_stages * n_tile * k_block + tail_bytes() +
        halo_ring_bytes(m_tiles) + column_bytes(n_tile * n_tiles) + staging_bytes;
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
    const bool half = form == PixelSource::planes_f16;
    if (half && c8 <= half_planes_max_c8 && pixels % 8 == 0 && (reinterpret_cast<std::uintptr_t>(in) & 15u) == 0 &&
        (reinterpret_cast<std::uintptr_t>(pixel_max) & 15u) == 0) {
        // Sixteen channels per thread (16 threads per group of 16). (Eight per
        // thread, for twice the resident blocks, measured slower: the per-pixel
        // work doubles and the kernel spills.)
        const int per_tile = c8;
        const int sub_tiles = per_tile >= 256 ? 1 : 256 / per_tile;
        const long long block_pixels = 128LL * sub_tiles;
        const long long tile_count = (pixels + block_pixels - 1) / block_pixels;
        static const int sm_count = [] {
            int device = 0;
            int count = 148;
            if (cudaGetDevice(&device) == cudaSuccess) cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, device);
            return count;
        }();
        // Streamed (persistent blocks, planes by TMA: a box of 128 pixels x c8
        // channel rows per sub-tile, rows past the last channel zero-filled)
        // with several tiles per SM; with fewer, one tile per block and two
        // blocks per SM measured faster.
        const EncodeTiled encode = tiled_encoder();
        CUtensorMap planes;
        const cuuint64_t dims[2] = {static_cast<cuuint64_t>(pixels), static_cast<cuuint64_t>(channels)};
        const cuuint64_t strides[1] = {static_cast<cuuint64_t>(pixels) * 2u};
        const cuuint32_t box[2] = {128u, static_cast<cuuint32_t>(c8)};
        const cuuint32_t element_strides[2] = {1u, 1u};
        if (encode != nullptr && tile_count >= 4LL * sm_count && tile_count < (1LL << 31) &&
            encode(&planes, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(in), dims, strides, box,
                   element_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS) {
            const std::size_t bytes = 1024 + static_cast<std::size_t>(streamed_stages) * streamed_stage_bytes +
                static_cast<std::size_t>(sub_tiles) * c8 * 16 + streamed_stages * sizeof(unsigned long long);
            static bool streamed_configured = false;
            if (!streamed_configured) {
                cudaFuncSetAttribute(quantise_half_planes_streamed_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(streamed_stages * streamed_stage_bytes + 9216));
                streamed_configured = true;
            }
            const int tiles = static_cast<int>(tile_count);
            const int grid = tiles < sm_count ? tiles : sm_count;
            return launch_overlapped(quantise_half_planes_streamed_kernel, dim3(static_cast<unsigned>(grid)),
                                     dim3(streamed_threads), bytes, stream, planes, channels, c8, pixels, sub_tiles,
                                     tiles, out, pixel_max, clear_word);
        }
        // Sub-tiles of 128, 64 or 32 pixels and as many per block (up to 256
        // threads) as leave at least two blocks per SM: a small input (config
        // 2 L5: 8160 pixels of 256 channels) otherwise runs on part of the SMs.
        int octet_shift = 4;
        int sub = sub_tiles;
        for (const int shift : {4, 3, 2}) {
            const int tile_threads = (1 << shift) * (c8 / 16);
            bool found = false;
            for (int candidate = tile_threads >= 256 ? 1 : 256 / tile_threads; candidate >= 1; candidate /= 2) {
                octet_shift = shift;
                sub = candidate;
                const long long pixels_per_block = 8LL * (1 << shift) * candidate;
                if ((pixels + pixels_per_block - 1) / pixels_per_block >= 2LL * sm_count) {
                    found = true;
                    break;
                }
            }
            if (found) break;
        }
        const long long pixels_per_block = 8LL * (1 << octet_shift) * sub;
        const int tile_threads = (1 << octet_shift) * (c8 / 16);
        const unsigned blocks = static_cast<unsigned>((pixels + pixels_per_block - 1) / pixels_per_block);
        const std::size_t bytes = static_cast<std::size_t>(sub) * tile_threads * sizeof(uint4);
        return launch_overlapped(quantise_half_planes_kernel<16>, dim3(blocks),
                                 dim3(static_cast<unsigned>(tile_threads * sub)), bytes, stream,
                                 static_cast<const __half*>(in), channels, c8, pixels, sub, octet_shift, out,
                                 pixel_max, clear_word);
    }
    // Planes whose length is a whole number of 16-byte vectors and whose base is
    // 16-byte aligned take the vector-load kernel.
    const int per_vector = half ? 8 : 4;
    if (pixels % per_vector == 0 && (reinterpret_cast<std::uintptr_t>(in) & 15u) == 0 && channels * 256 <= 200 * 1024) {
        const int block_pixels = half ? 128 : 64;
        const unsigned wide_blocks = static_cast<unsigned>((static_cast<long long>(pixels) + block_pixels - 1) / block_pixels);
        const int bytes = channels * 256;
        static bool wide_configured = false;
        if (!wide_configured) {
            cudaFuncSetAttribute(quantise_planes_wide_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
            cudaFuncSetAttribute(quantise_planes_wide_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
            wide_configured = true;
        }
        if (half) {
            return launch_overlapped(quantise_planes_wide_kernel<true>, dim3(wide_blocks), dim3(256), bytes, stream, in,
                                     channels, c8, pixels, out, pixel_max, clear_word);
        }
        return launch_overlapped(quantise_planes_wide_kernel<false>, dim3(wide_blocks), dim3(256), bytes, stream, in,
                                 channels, c8, pixels, out, pixel_max, clear_word);
    }
    const int tile_bytes = channels * (plane_pixels + 1) * static_cast<int>(sizeof(float));
    if (tile_bytes > 200 * 1024) return cudaErrorInvalidValue;
    const unsigned blocks = static_cast<unsigned>((static_cast<long long>(pixels) + plane_pixels - 1) / plane_pixels);
    if (half) {
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
    // Row-staged kernel when a run's input rows fit in shared memory.
    const int span = (field_run - 1) * window.stride_x + window.kernel_w;
    if (channels == 3 && window.kernel_h == 3 && window.kernel_w == 3 && c8 == 32 && span <= 4 * field_run &&
        out_h <= 65535 && static_cast<long long>(channels) * in_h * in_w < (1LL << 31)) {
        const dim3 grid(static_cast<unsigned>((out_w + field_run - 1) / field_run), static_cast<unsigned>(out_h));
        const int pitch = (span + 7 + 7) & ~7;
        const std::size_t bytes = static_cast<std::size_t>(channels) * window.kernel_h * pitch * 4;
        const int vector_rows = source_half && in_w % 8 == 0 && (reinterpret_cast<std::uintptr_t>(in) & 15u) == 0;
        return source_half ? launch_overlapped(quantise_fields_fixed_kernel<true, 3, 3, 3, 32>, grid, dim3(field_run),
                                               bytes, stream, in, in_h, in_w, window, out_h, out_w, span, vector_rows,
                                               out, field_max)
                           : launch_overlapped(quantise_fields_fixed_kernel<false, 3, 3, 3, 32>, grid,
                                               dim3(field_run), bytes, stream, in, in_h, in_w, window, out_h, out_w,
                                               span, 0, out, field_max);
    }
    const long long row_bytes = static_cast<long long>(channels) * window.kernel_h * span * 4;
    const long long planes = static_cast<long long>(channels) * in_h * in_w;
    if (window.stride_x >= 1 && window.stride_y >= 1 && span <= 4 * field_run && row_bytes <= 48 * 1024 &&
        out_h <= 65535 && planes < (1LL << 31)) {
        const dim3 grid(static_cast<unsigned>((out_w + field_run - 1) / field_run), static_cast<unsigned>(out_h));
        const std::size_t bytes = static_cast<std::size_t>(row_bytes);
        if (c8 == 32) {
            return source_half ? launch_overlapped(quantise_fields_rows_kernel<true, 32>, grid, dim3(field_run), bytes,
                                                   stream, in, channels, in_h, in_w, window, out_h, out_w, span, out,
                                                   field_max)
                               : launch_overlapped(quantise_fields_rows_kernel<false, 32>, grid, dim3(field_run), bytes,
                                                   stream, in, channels, in_h, in_w, window, out_h, out_w, span, out,
                                                   field_max);
        }
        return source_half ? launch_overlapped(quantise_fields_rows_kernel<true, 64>, grid, dim3(field_run), bytes,
                                               stream, in, channels, in_h, in_w, window, out_h, out_w, span, out,
                                               field_max)
                           : launch_overlapped(quantise_fields_rows_kernel<false, 64>, grid, dim3(field_run), bytes,
                                               stream, in, channels, in_h, in_w, window, out_h, out_w, span, out,
                                               field_max);
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
    // As many accumulator buffers as fit in TMEM's 512 columns (n_tile <= 256: two
    // at least), up to eight; the allocation is the next power of two.
    const int tile_columns = args.m_tiles * args.n_tile;
    const int buffers = std::min(max_tmem_buffers, 512 / tile_columns);
    std::uint32_t columns = 32;
    while (static_cast<int>(columns) < buffers * tile_columns) columns <<= 1;
    const int smem = args.row_halo
        ? direct_conv_row_shared_bytes(args.k_block, args.n_tile, args.n_tiles, args.a_stages, args.b_stages,
                                       args.b_resident != 0, args.m_tiles, args.a_row_bytes)
        : direct_conv_shared_bytes(args.k_block, args.n_tile, args.n_tiles, args.a_stages, args.b_stages, args.group,
                                   args.b_resident != 0, args.m_tiles);
    if (smem > direct_conv_max_shared) return cudaErrorInvalidValue;
    static bool configured = false;
    if (!configured) {
        cudaError_t set = cudaFuncSetAttribute(direct_conv_kernel<1, true>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, direct_conv_max_shared);
        if (set == cudaSuccess) {
            set = cudaFuncSetAttribute(direct_conv_kernel<1, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       direct_conv_max_shared);
        }
        if (set == cudaSuccess) {
            set = cudaFuncSetAttribute(direct_conv_kernel<2, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       direct_conv_max_shared);
        }
        if (set != cudaSuccess) return set;
        configured = true;
    }
    const int tiles = (args.p_tiles + args.m_tiles - 1) / args.m_tiles * args.n_tiles;
    const int grid = tiles < sm_count ? tiles : sm_count;
    if (args.m_tiles == 2) {
        return launch_overlapped(direct_conv_kernel<2, false>, dim3(grid), dim3(direct_threads), smem, stream, a_map,
                                 b_map, args, buffers, columns);
    }
    const bool fusions = args.wsilu || args.chunk_add || args.residual != nullptr || args.out_max != nullptr;
    if (fusions) {
        return launch_overlapped(direct_conv_kernel<1, true>, dim3(grid), dim3(direct_threads), smem, stream, a_map,
                                 b_map, args, buffers, columns);
    }
    return launch_overlapped(direct_conv_kernel<1, false>, dim3(grid), dim3(direct_threads), smem, stream, a_map, b_map,
                             args, buffers, columns);
}

}  // namespace nvcr_sm100::kernels
