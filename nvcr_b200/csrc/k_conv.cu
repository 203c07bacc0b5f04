// Fused integer conv on sm_100a: quantise-on-load implicit GEMM.
//
// A prepass (stage_source) rewrites the conv's source channel-innermost,
// [in_h][in_w][c_pad] in its own type (FP16 stays FP16), and writes the
// per-pixel max |x| (a conv with channels * taps <= 64 instead stages each
// output position's whole receptive field as one record, stage_receptive_fields,
// and runs here as a 1x1 conv). Then one persistent CTA per SM walks tiles of 128 output
// positions (a 2-D patch of patch_h x patch_w output pixels) x n_tile output
// channels. Warp roles (15 warps, 128 registers each):
//   warps 0..E-1    epilogue: one TMEM lane (= one position) per thread, the
//                   profile's output arithmetic and the folded ops, then the
//                   store; E = 8 (two warps per TMEM lane quarter, each half of
//                   the columns) or E = 4 (one per quarter, all columns);
//   warps E..11     producers, one or two sets of four warps (a set takes the
//                   CTA's tiles s, s + sets, ...; each set has its own A-stage
//                   ring and halo ring): one thread per position quantises its
//                   receptive field from the shared-memory halo into the
//                   128-byte-swizzled A tile, 16 channels of one tap per 16-byte
//                   A chunk; the im2col tensor and the quantised activation
//                   matrix never exist in memory;
//   warp 12         TMA: int8 weight tiles (n_tile x 128 B per K block);
//   warp 13         allocates TMEM and issues the tcgen05 MMAs (one thread);
//   warp 14         TMA: the activation halo of each tile, `group` channels at a
//                   time, into the halo rings (2..8 buffers). Padding taps and
//                   the image border come back as the TMA's zero fill.
// The accumulators are double-buffered in TMEM when they fit, so the epilogue
// of one tile overlaps the main loop of the next. The per-column scale, bias
// and row term of every output column are copied to shared memory once.
//
// Halo layout: one record of `group` channels (record_bytes = 16..128) per
// pixel, pixels row-major; the TMA swizzles 16-byte pieces inside each
// 128-byte line (piece ^= line bits), so the 32 positions of a warp read
// distinct banks. A producer reads 8 FP16 (or 4 FP32) channels per 16-byte load.
//
// K is channel-group-major over the padded channels: k = g * (taps * group) +
// tap * group + c; the weights are laid out to match on the host. Integer sums
// do not depend on the K order.
//
// Activation quantisation per position p: e_p = frexp(max |x| over the
// receptive field) - (bits - 1) from the per-pixel maxima; then
// q = clamp(rint(x * 2^-e_p), +-L). Three exact ways, chosen per position:
//  * FP16 pairs (FP16 source, 8-bit, 2^-e_p a normal half, max * 2^-e_p <
//    127.5 so no clamp can act): fma.rn.f16x2(x, 2^-e_p, 1536) is exact in the
//    product and rounds once; |x * 2^-e_p| < 128 keeps it in [1024, 2048)
//    where halves are the integers, so the low byte of each half is q.
//  * FP32 (2^-e_p a normal float): fma(x, 2^-e_p, 1.5 * 2^23) likewise rounds
//    once to the integer (|x * 2^-e_p| < 2^15 < 2^22), low 16 bits = q, with
//    the clamp applied only when max * 2^-e_p can round past L.
//  * otherwise the bit-level ldexp + rint of each element.
//
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

constexpr int conv_warps = 15;
constexpr int conv_threads = conv_warps * 32;
// Warps 0-11 split between the epilogue and the producers at launch: eight
// epilogue warps (two per TMEM lane quarter) and one producer set of four, or
// four epilogue warps and two producer sets that take alternate tiles.
constexpr int role_warps = 12;
constexpr int tma_warp = 12;
constexpr int mma_warp = 13;
constexpr int halo_warp = 14;
constexpr int max_halo_buffers = 8;  // halo ring depth: as many buffers as shared memory holds, 2..8
constexpr int max_stages = 8;
constexpr float round_magic = 12582912.0f;              // 1.5 * 2^23
constexpr std::uint32_t half_magic_pair = 0x66006600u;  // (1536, 1536) as an FP16 pair

struct ConvTail {
    unsigned long long full_a[max_stages];
    unsigned long long empty_a[max_stages];
    unsigned long long full_b[max_stages];
    unsigned long long empty_b[max_stages];
    unsigned long long tmem_full[2];
    unsigned long long tmem_empty[2];
    unsigned long long info_full[2];
    unsigned long long info_empty[2];
    unsigned long long halo_full[max_halo_buffers];
    unsigned long long halo_empty[max_halo_buffers];
    unsigned long long drain;
    std::uint32_t tmem_base;
    int abort;
    int exponents[2][tile_positions_m];
    long long column_terms[2][tile_positions_m];
};

// Bytes of the per-column parameters after the tail: scales, biases and (two-
// limb activations) row terms of all n_tiles * n_tile physical columns.
__host__ __device__ constexpr int parameter_bytes(int columns, int activation_limbs) {
    return columns * 8 + (activation_limbs == 2 ? columns * 8 : 0);
}

template <int WL, int AL>
struct ConvLayout {
    static constexpr int accumulators = 1 + ((WL == 2 || AL == 2) ? 1 : 0) + ((WL == 2 && AL == 2) ? 1 : 0);
    static constexpr int a_bytes = tile_positions_m * tile_k_bytes;
    static __host__ __device__ int b_bytes(int n_tile) { return n_tile * tile_k_bytes; }
    static constexpr int a_stage_bytes = AL * a_bytes;
    static __host__ __device__ int b_stage_bytes(int n_tile) { return WL * b_bytes(n_tile); }
};

__device__ __forceinline__ uint4 load_shared_v4(std::uint32_t address) {
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(address));
    return v;
}

__device__ __forceinline__ void store_shared_v4(std::uint32_t address, const std::uint32_t (&w)[4]) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(address), "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3])
                 : "memory");
}

// Byte N of each of a, b, c, d packed into one word, a lowest.
template <int N>
__device__ __forceinline__ std::uint32_t pack_byte(std::uint32_t a, std::uint32_t b, std::uint32_t c, std::uint32_t d) {
    constexpr std::uint32_t pair = static_cast<std::uint32_t>(N) | (static_cast<std::uint32_t>(N + 4) << 4);
    return __byte_perm(__byte_perm(a, b, pair), __byte_perm(c, d, pair), 0x5410u);
}

// RN(x * s + 1536) for a pair of FP16 channels: q in the low byte of each half.
__device__ __forceinline__ std::uint32_t round_half_pair(std::uint32_t x, std::uint32_t s) {
    std::uint32_t y;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(y) : "r"(x), "r"(s), "r"(half_magic_pair));
    return y;
}

__device__ __forceinline__ float half_low(std::uint32_t pair) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(pair & 0xffffu)));
}
__device__ __forceinline__ float half_high(std::uint32_t pair) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(pair >> 16)));
}

// Sum of the four signed bytes of w.
__device__ __forceinline__ int byte_sum(std::uint32_t w) { return __dp4a(static_cast<int>(w), 0x01010101, 0); }

// ---------------------------------------------------------------- prepass

// Maxima of |x| on bit patterns: non-negative floats (and halves) order as
// their bits, and a NaN or infinity has bits at or above the infinity
// pattern, so max |x| is one integer max per value (two per packed FP16
// word) and a non-finite value anywhere gives +inf.
__device__ __forceinline__ float max_from_half_bits(std::uint32_t m) {
    return m >= 0x7c00u ? __uint_as_float(0x7f800000u) : __half2float(__ushort_as_half(static_cast<unsigned short>(m)));
}
__device__ __forceinline__ float max_from_float_bits(std::uint32_t m) {
    return m >= 0x7f800000u ? __uint_as_float(0x7f800000u) : __uint_as_float(m);
}
// |x| bits of one FP16 (in the low 16 bits) or FP32 value.
template <bool Half, typename T>
__device__ __forceinline__ std::uint32_t magnitude_bits(T v) {
    if constexpr (Half) {
        return static_cast<std::uint32_t>(v) & 0x7fffu;
    } else {
        return __float_as_uint(v) & 0x7fffffffu;
    }
}
template <bool Half>
__device__ __forceinline__ float max_from_bits(std::uint32_t m) {
    return Half ? max_from_half_bits(m) : max_from_float_bits(m);
}

// One thread per pixel: the channels of its pixel in blocks of 16 bytes (8 FP16
// or 4 FP32 channels), each element load coalesced across the warp's 32
// consecutive pixels, each block one 16-byte store into the pixel's record; the
// pixel's max |x| (+inf when any channel is non-finite) stays in a register.
template <bool Half>
__global__ void __launch_bounds__(256) stage_pixels_kernel(const void* __restrict__ in, int channels, int c_pad,
                                                           int pixels, void* __restrict__ out,
                                                           float* __restrict__ pixel_max,
                                                           const unsigned int* __restrict__ gate) {
    grid_dependency_wait();  // the source may come from the kernel before
    launch_dependents();
    if (gate != nullptr && *gate == 0u) return;  // a direct conv's fallback that is not needed
    using T = std::conditional_t<Half, unsigned short, float>;
    constexpr int per_block = 16 / static_cast<int>(sizeof(T));  // channels per 16-byte store
    constexpr int blocks_per_pass = Half ? 2 : 4;                 // 16 loads in flight
    const long long pixel = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (pixel >= pixels) return;
    const T* source = static_cast<const T*>(in) + pixel;
    uint4* record = reinterpret_cast<uint4*>(static_cast<T*>(out) + pixel * c_pad);
    std::uint32_t maximum = 0;  // max |x| bits
    for (int c0 = 0; c0 < c_pad; c0 += per_block * blocks_per_pass) {
        T v[blocks_per_pass][per_block];
#pragma unroll
        for (int b = 0; b < blocks_per_pass; ++b) {
#pragma unroll
            for (int i = 0; i < per_block; ++i) {
                const int c = c0 + b * per_block + i;
                v[b][i] = c < channels ? source[static_cast<std::size_t>(c) * pixels] : T(0);
            }
        }
#pragma unroll
        for (int b = 0; b < blocks_per_pass; ++b) {
            if (c0 + b * per_block >= c_pad) break;
            std::uint32_t w[4];
#pragma unroll
            for (int i = 0; i < per_block; ++i) maximum = max(maximum, magnitude_bits<Half>(v[b][i]));
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                if constexpr (Half) {
                    w[k] = static_cast<std::uint32_t>(v[b][2 * k]) | (static_cast<std::uint32_t>(v[b][2 * k + 1]) << 16);
                } else {
                    w[k] = __float_as_uint(v[b][k]);
                }
            }
            record[(c0 + b * per_block) / per_block] = make_uint4(w[0], w[1], w[2], w[3]);
        }
    }
    pixel_max[pixel] = max_from_bits<Half>(maximum);
}

// Wide records (more than 32 channels): pixels through shared memory in slabs.
template <bool Half>
struct StageShape {
    static constexpr int max_slab = Half ? 256 : 128;  // channels per pass through shared memory
    static constexpr int tile_elements = Half ? 9216 : 4352;
    static constexpr int max_pixels = Half ? 512 : 256;  // pixels per block
    static __host__ __device__ constexpr int pitch(int slab) { return slab + (Half ? 2 : 1); }  // odd words apart
    // Pixels per block for c_pad channels: the largest power-of-two multiple
    // of 32 whose tile fits.
    static int pixels(int c_pad) {
        const int slab = c_pad < max_slab ? c_pad : max_slab;
        int p = max_pixels;
        while (p > 32 && p * pitch(slab) > tile_elements) p /= 2;
        return p;
    }
};

// Pixels consecutive pixels per block, the channels in slabs through shared
// memory: coalesced reads of each channel plane (up to 16 loads in flight per
// thread), contiguous channel-innermost writes, and the per-pixel maximum.
template <bool Half, int Pixels>
__global__ void __launch_bounds__(256) stage_source_kernel(const void* __restrict__ in, int channels, int c_pad,
                                                           int pixels, void* __restrict__ out,
                                                           float* __restrict__ pixel_max,
                                                           const unsigned int* __restrict__ gate) {
    grid_dependency_wait();  // the source may come from the kernel before
    launch_dependents();
    if (gate != nullptr && *gate == 0u) return;  // a direct conv's fallback that is not needed
    using T = std::conditional_t<Half, unsigned short, float>;
    using S = StageShape<Half>;
    constexpr int per_word = Half ? 2 : 1;
    constexpr int groups = Pixels / 32;                     // pixel groups of 32 per thread
    constexpr int batch = groups >= 16 ? 1 : 16 / groups;  // channels per thread per pass
    __shared__ __align__(16) T tile[S::tile_elements];
    __shared__ std::uint32_t partial[8][Pixels];  // max |x| bits per warp
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int slab = c_pad < S::max_slab ? c_pad : S::max_slab;
    const int pitch = S::pitch(slab);
    const long long first = static_cast<long long>(blockIdx.x) * Pixels;
    const int valid = static_cast<int>(pixels - first < Pixels ? pixels - first : Pixels);
    const T* source = static_cast<const T*>(in);
    std::uint32_t* target = static_cast<std::uint32_t*>(out);
    std::uint32_t maximum[groups];  // max |x| bits
#pragma unroll
    for (int k = 0; k < groups; ++k) maximum[k] = 0;
    for (int base = 0; base < c_pad; base += slab) {
        const int count = c_pad - base < slab ? c_pad - base : slab;
        for (int c0 = warp; c0 < count; c0 += 8 * batch) {
            T v[batch][groups];
#pragma unroll
            for (int u = 0; u < batch; ++u) {
                const int channel = base + c0 + 8 * u;
#pragma unroll
                for (int k = 0; k < groups; ++k) {
                    const int p = k * 32 + lane;
                    v[u][k] = (p < valid && channel < channels && c0 + 8 * u < count)
                        ? source[static_cast<std::size_t>(channel) * pixels + first + p]
                        : T(0);
                }
            }
#pragma unroll
            for (int u = 0; u < batch; ++u) {
                const int c = c0 + 8 * u;
                if (c >= count) break;
#pragma unroll
                for (int k = 0; k < groups; ++k) {
                    maximum[k] = max(maximum[k], magnitude_bits<Half>(v[u][k]));
                    tile[(k * 32 + lane) * pitch + c] = v[u][k];
                }
            }
        }
        __syncthreads();
        // Pixel p's `count` channels go to words ((first + p) * c_pad + base) / per_word onwards.
        const int words = count / per_word;
        const int row_words = pitch / per_word;
        const std::uint32_t* rows = reinterpret_cast<const std::uint32_t*>(tile);
        if (words <= 32) {
            const int per_pass = 32 / words;  // pixels one warp writes per pass
            const int sub = lane / words;
            const int w = lane - sub * words;
            if (sub < per_pass) {
                for (int p = warp * per_pass + sub; p < valid; p += 8 * per_pass) {
                    const std::size_t origin = ((static_cast<std::size_t>(first) + p) * c_pad + base) / per_word;
                    target[origin + w] = rows[p * row_words + w];
                }
            }
        } else {
            for (int p = warp; p < valid; p += 8) {
                const std::size_t origin = ((static_cast<std::size_t>(first) + p) * c_pad + base) / per_word;
                for (int w = lane; w < words; w += 32) target[origin + w] = rows[p * row_words + w];
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int k = 0; k < groups; ++k) partial[warp][k * 32 + lane] = maximum[k];
    __syncthreads();
    for (int p = threadIdx.x; p < valid; p += 256) {
        std::uint32_t m = partial[0][p];
        for (int g = 1; g < 8; ++g) m = max(m, partial[g][p]);
        pixel_max[first + p] = max_from_bits<Half>(m);
    }
}

template <bool Half>
cudaError_t launch_stage(const void* in, int channels, int c_pad, int pixels, void* out, float* pixel_max,
                         const unsigned int* gate, cudaStream_t stream) {
    const int block = StageShape<Half>::pixels(c_pad);
    const unsigned blocks = static_cast<unsigned>((static_cast<long long>(pixels) + block - 1) / block);
    switch (block) {
    case 32: return launch_overlapped(stage_source_kernel<Half, 32>, dim3(blocks), dim3(256), 0, stream, in, channels,
                                      c_pad, pixels, out, pixel_max, gate);
    case 64: return launch_overlapped(stage_source_kernel<Half, 64>, dim3(blocks), dim3(256), 0, stream, in, channels,
                                       c_pad, pixels, out, pixel_max, gate);
    case 128: return launch_overlapped(stage_source_kernel<Half, 128>, dim3(blocks), dim3(256), 0, stream, in, channels,
                                       c_pad, pixels, out, pixel_max, gate);
    case 256: return launch_overlapped(stage_source_kernel<Half, 256>, dim3(blocks), dim3(256), 0, stream, in, channels,
                                       c_pad, pixels, out, pixel_max, gate);
    default:
        if constexpr (Half) {
            return launch_overlapped(stage_source_kernel<Half, 512>, dim3(blocks), dim3(256), 0, stream, in, channels,
                                     c_pad, pixels, out, pixel_max, gate);
        } else {
            return cudaErrorInvalidValue;
        }
    }
    return cudaGetLastError();
}


// One thread per output position: its receptive field in k = c * taps + tap
// order as 16-byte stores, zeros for padding taps and past channels * taps.
// A per-block table holds each k's channel plane offset and (ky, kx), so the
// per-element work is two adds, a bounds test and a load.
constexpr int max_field = 64;  // K values per staged receptive field

template <bool Half>
__global__ void __launch_bounds__(256) stage_fields_kernel(const void* __restrict__ in, int channels, int in_h,
                                                           int in_w, Window w, int out_h, int out_w, int c_pad,
                                                           void* __restrict__ out, float* __restrict__ field_max) {
    grid_dependency_wait();  // the source may come from the kernel before
    launch_dependents();
    using T = std::conditional_t<Half, unsigned short, float>;
    constexpr int per_store = 16 / static_cast<int>(sizeof(T));
    __shared__ long long plane_at[max_field];  // c * in_h * in_w, or -1 for padding
    __shared__ short2 tap_at[max_field];       // (ky, kx)
    const int taps = w.kernel_h * w.kernel_w;
    for (int k = threadIdx.x; k < c_pad; k += blockDim.x) {
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
    const T* source = static_cast<const T*>(in);
    uint4* record = reinterpret_cast<uint4*>(static_cast<T*>(out) + position * c_pad);
    std::uint32_t maximum = 0;  // max |x| bits
#pragma unroll
    for (int k0 = 0; k0 < max_field; k0 += per_store) {
        if (k0 >= c_pad) break;
        T v[per_store];
#pragma unroll
        for (int i = 0; i < per_store; ++i) {
            const long long plane = plane_at[k0 + i];
            const short2 d = tap_at[k0 + i];
            const int iy = iy0 + d.x;
            const int ix = ix0 + d.y;
            const bool inside = plane >= 0 && static_cast<unsigned>(iy) < static_cast<unsigned>(in_h) &&
                static_cast<unsigned>(ix) < static_cast<unsigned>(in_w);
            v[i] = inside ? source[plane + static_cast<long long>(iy) * in_w + ix] : T(0);
        }
#pragma unroll
        for (int i = 0; i < per_store; ++i) maximum = max(maximum, magnitude_bits<Half>(v[i]));
        std::uint32_t word[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            if constexpr (Half) {
                word[q] = static_cast<std::uint32_t>(v[2 * q]) | (static_cast<std::uint32_t>(v[2 * q + 1]) << 16);
            } else {
                word[q] = __float_as_uint(v[q]);
            }
        }
        record[k0 / per_store] = make_uint4(word[0], word[1], word[2], word[3]);
    }
    field_max[position] = max_from_bits<Half>(maximum);
}

// ---------------------------------------------------------------- fused conv

// Out-of-line helpers for the rare paths, so the hot loops stay compact in the
// instruction cache.
struct Sixteen {
    float v[16];
};
struct SixteenWords {
    std::uint32_t w[16];
};

// q of each element by the bit-level ldexp and rint (exponents whose 2^-e is
// not a normal float).
template <int Bits>
__device__ __noinline__ SixteenWords quantize_exact16(Sixteen x, int exponent) {
    SixteenWords q;
#pragma unroll
    for (int j = 0; j < 16; ++j) q.w[j] = static_cast<std::uint32_t>(quantize_value<Bits>(x.v[j], exponent));
    return q;
}

// ldexp(x, e) + bias per element, for e outside [-126, 127].
__device__ __noinline__ Sixteen ldexp_add16(Sixteen x, Sixteen bias, int exponent) {
#pragma unroll
    for (int j = 0; j < 16; ++j) x.v[j] = __fadd_rn(exact_ldexp(x.v[j], exponent), bias.v[j]);
    return x;
}

// profile_wsilu of 16 values as straight-line code: each value with the refined
// reciprocal when its denominator lies in [1, 2^126), the others (kept as the
// input, marked in a mask) redone with the IEEE division afterwards.
__device__ __noinline__ Sixteen wsilu16(Sixteen x, float k) {
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

// Quotient and remainder by a divisor fixed for the kernel: a float reciprocal
// and one correction step, exact for 0 <= n < 2^22 (tile indices are far below).
struct Divider {
    int d;
    float inverse;
    __device__ explicit Divider(int divisor) : d(divisor), inverse(1.0f / static_cast<float>(divisor)) {}
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

// How one position's activations are quantised in a tile.
enum QuantMode : int { quant_skip = 0, quant_half = 1, quant_float = 2, quant_float_clamp = 3, quant_exact = 4 };

// Quantises 16 channels of one tap of this position from the halo pieces
// d[0 .. 16 / (channels per piece) - 1] (8 FP16 or 4 FP32 channels each).
// `high` gets the 16 high-limb bytes (the whole q for 8-bit), `low` the low limbs.
template <int WL, int AL, bool SourceHalf>
__device__ __forceinline__ void quantize_chunk(const uint4* d, int mode, std::uint32_t scale_pair, float scale,
                                               int exponent, std::uint32_t (&high)[4], std::uint32_t (&low)[4],
                                               int& sum_high, int& sum_low) {
    constexpr int bits = AL == 2 ? 16 : 8;
    constexpr float limit = AL == 2 ? 32767.0f : 127.0f;
    auto piece = [&](int b) { return d[b]; };
    if (mode == quant_skip) {
        high[0] = high[1] = high[2] = high[3] = 0;
        low[0] = low[1] = low[2] = low[3] = 0;
        return;
    }
    if constexpr (SourceHalf && AL == 1) {
        if (mode == quant_half) {
            const uint4 d0 = piece(0);
            const uint4 d1 = piece(1);
            const std::uint32_t x[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
            std::uint32_t y[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) y[i] = round_half_pair(x[i], scale_pair);
#pragma unroll
            for (int w = 0; w < 4; ++w) {
                high[w] = __byte_perm(y[2 * w], y[2 * w + 1], 0x6420u);
                if constexpr (WL == 2) sum_high += byte_sum(high[w]);
            }
            return;
        }
    }
    float v[16];
    if constexpr (SourceHalf) {
        const uint4 d0 = piece(0);
        const uint4 d1 = piece(1);
        const std::uint32_t x[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            v[2 * i] = half_low(x[i]);
            v[2 * i + 1] = half_high(x[i]);
        }
    } else {
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const uint4 d = piece(b);
            v[4 * b] = __uint_as_float(d.x);
            v[4 * b + 1] = __uint_as_float(d.y);
            v[4 * b + 2] = __uint_as_float(d.z);
            v[4 * b + 3] = __uint_as_float(d.w);
        }
    }
    std::uint32_t u[16];
    if (mode == quant_exact) {
        Sixteen x;
#pragma unroll
        for (int j = 0; j < 16; ++j) x.v[j] = v[j];
        const SixteenWords q = quantize_exact16<bits>(x, exponent);
#pragma unroll
        for (int j = 0; j < 16; ++j) u[j] = q.w[j];
    } else {
        // The bits of magic + q: the low 16 bits are q in two's complement.
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            float y = __fmaf_rn(v[j], scale, round_magic);
            if (mode == quant_float_clamp) y = fminf(fmaxf(y, round_magic - limit), round_magic + limit);
            u[j] = __float_as_uint(y);
        }
    }
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        if constexpr (AL == 2) {
            // h = q >> 8 is byte 1 of q; l' = (q & 255) - 128 is byte 0 with its top bit flipped.
            high[w] = pack_byte<1>(u[4 * w], u[4 * w + 1], u[4 * w + 2], u[4 * w + 3]);
            low[w] = pack_byte<0>(u[4 * w], u[4 * w + 1], u[4 * w + 2], u[4 * w + 3]) ^ 0x80808080u;
            if constexpr (WL == 2) {
                sum_high += byte_sum(high[w]);
                sum_low += byte_sum(low[w]);
            }
        } else {
            high[w] = pack_byte<0>(u[4 * w], u[4 * w + 1], u[4 * w + 2], u[4 * w + 3]);
            if constexpr (WL == 2) sum_high += byte_sum(high[w]);
        }
    }
}

// Next use of a ring of `depth` slots starting at slot `base`: its slot and
// the mbarrier phase parity of that use, advanced one use at a time.
struct RingCursor {
    int base;
    int depth;
    int index;
    std::uint32_t phase;
    __device__ int slot() const { return base + index; }
    __device__ void advance() {
        if (++index == depth) {
            index = 0;
            phase ^= 1u;
        }
    }
};

struct ChunkLimbs {
    std::uint32_t high[4];
    std::uint32_t low[4];
    int sum_high;
    int sum_low;
};

// quantize_chunk for any mode, out of line: only warps in which some position
// leaves the common rounding call it, so the common path keeps its registers.
// FP16 sources use d0 and d1 only.
template <int WL, int AL, bool SourceHalf>
__device__ __noinline__ ChunkLimbs quantize_chunk_any(uint4 d0, uint4 d1, uint4 d2, uint4 d3, int mode,
                                                      std::uint32_t scale_pair, float scale, int exponent) {
    const uint4 d[4] = {d0, d1, d2, d3};
    ChunkLimbs r;
    r.sum_high = 0;
    r.sum_low = 0;
    quantize_chunk<WL, AL, SourceHalf>(d, mode, scale_pair, scale, exponent, r.high, r.low, r.sum_high, r.sum_low);
    return r;
}

template <int WL, int AL, bool SourceHalf>
__global__ void __launch_bounds__(conv_threads, 1)
fused_conv_kernel(const __grid_constant__ CUtensorMap b_high, const __grid_constant__ CUtensorMap b_low,
                  const __grid_constant__ CUtensorMap halo_map, FusedConvArgs a, int tmem_buffers,
                  std::uint32_t tmem_columns) {
    using L = ConvLayout<WL, AL>;
    constexpr int bits = AL == 2 ? 16 : 8;
    if (a.gate != nullptr) {
        // A direct conv's fallback: runs only when that conv found a window whose
        // pixels have different exponents.
        grid_dependency_wait();
        if (*a.gate == 0u) return;
    }
    extern __shared__ std::uint8_t dynamic_smem[];
    const std::uint32_t raw = smem_address(dynamic_smem);
    std::uint8_t* smem = dynamic_smem + (((raw + 1023u) & ~1023u) - raw);
    const int n_tile = a.n_tile;
    const int a_stages = a.a_stages;
    const int b_stages = a.b_stages;
    // Shared memory: [A stages][B stages][halo buffers][tail][column parameters],
    // the first three 1 KiB aligned.
    std::uint8_t* b_smem = smem + a_stages * L::a_stage_bytes;
    std::uint8_t* halo_smem = b_smem + b_stages * L::b_stage_bytes(n_tile);
    const int halo_buffers = a.halo_buffers;
    ConvTail* tail = reinterpret_cast<ConvTail*>(halo_smem + halo_buffers * a.halo_bytes);
    const int all_columns = a.n_tiles * n_tile;
    float* column_scale = reinterpret_cast<float*>(reinterpret_cast<std::uint8_t*>(tail) +
                                                   ((sizeof(ConvTail) + 15) / 16) * 16);
    float* column_bias = column_scale + all_columns;
    long long* column_row_terms = reinterpret_cast<long long*>(column_bias + all_columns);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int total_tiles = a.p_tiles * a.n_tiles;
    const int k_blocks = a.k_blocks;
    const int producer_sets = a.producer_sets;
    const int epilogue_warps = role_warps - 4 * producer_sets;
    const int epilogue_threads = epilogue_warps * 32;
    // Each producer set has its own A-stage ring and halo ring (the set's
    // tiles use them in order, as do the MMA and halo TMA for that set's tiles),
    // so every mbarrier wait is for the current or the previous phase.
    const int ring_stages = a_stages / producer_sets;
    const int ring_halos = halo_buffers / producer_sets;
    const Divider by_n_tiles(a.n_tiles);
    const Divider by_tiles_x(a.tiles_x);

    for (int i = threadIdx.x; i < all_columns; i += conv_threads) {
        column_scale[i] = a.scales[i];
        column_bias[i] = a.bias[i];
        if constexpr (AL == 2) column_row_terms[i] = a.row_terms[i];
    }
    if (warp == mma_warp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_address(&tail->tmem_base)), "r"(tmem_columns)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (warp == tma_warp && lane == 0) {
        for (int s = 0; s < a_stages; ++s) {
            barrier_init(smem_address(&tail->full_a[s]), tile_positions_m);
            barrier_init(smem_address(&tail->empty_a[s]), 1);
        }
        for (int s = 0; s < b_stages; ++s) {
            barrier_init(smem_address(&tail->full_b[s]), 1);
            barrier_init(smem_address(&tail->empty_b[s]), 1);
        }
        for (int b = 0; b < 2; ++b) {
            barrier_init(smem_address(&tail->tmem_full[b]), 1);
            barrier_init(smem_address(&tail->tmem_empty[b]), epilogue_threads);
            barrier_init(smem_address(&tail->info_full[b]), tile_positions_m);
            barrier_init(smem_address(&tail->info_empty[b]), epilogue_threads);
        }
        for (int h = 0; h < halo_buffers; ++h) {
            barrier_init(smem_address(&tail->halo_full[h]), 1);
            barrier_init(smem_address(&tail->halo_empty[h]), tile_positions_m);
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
    // The weight TMA and the MMA touch only constant weights, shared memory and
    // TMEM; the other roles wait for the kernels before this one first.
    launch_dependents();
    volatile int* abort = &tail->abort;

    if (warp == tma_warp) {
        if (lane == 0) {
            // ---------------- weights by TMA
            const std::uint32_t bytes = static_cast<std::uint32_t>(WL * L::b_bytes(n_tile));
            std::uint32_t g = 0;
            std::uint32_t issued = 0;
            bool ok = true;
            // Resident weights: the first tile's pass loads every K block into its own stage, once.
            const int last = a.b_resident ? static_cast<int>(blockIdx.x) + 1 : total_tiles;
            for (int t = blockIdx.x; t < last && ok; t += gridDim.x) {
                int n_index;
                by_n_tiles.divide(t, n_index);
                const int n0 = n_index * n_tile;
                for (int kb = 0; kb < k_blocks; ++kb, ++g) {
                    const int s = static_cast<int>(g % b_stages);
                    const std::uint32_t phase = (g / b_stages) & 1u;
                    if (*abort || !barrier_wait(smem_address(&tail->empty_b[s]), phase ^ 1u, a.status)) {
                        *abort = 1;
                        ok = false;
                        break;
                    }
                    const std::uint32_t full = smem_address(&tail->full_b[s]);
                    barrier_expect_bytes(full, bytes);
                    const std::uint32_t b_base = smem_address(b_smem + s * L::b_stage_bytes(n_tile));
                    tma_load_2d(b_base, &b_high, full, kb * tile_k_bytes, n0);
                    if constexpr (WL == 2) {
                        tma_load_2d(b_base + static_cast<std::uint32_t>(L::b_bytes(n_tile)), &b_low, full,
                                    kb * tile_k_bytes, n0);
                    }
                    issued = g + 1;
                }
            }
            if (!ok) {
                // Every issued load must land before the CTA may exit.
                const std::uint32_t first = issued > static_cast<std::uint32_t>(b_stages) ? issued - b_stages : 0;
                for (std::uint32_t h = first; h < issued; ++h) {
                    barrier_wait(smem_address(&tail->full_b[h % b_stages]), (h / b_stages) & 1u, a.status);
                }
            }
        }
    } else if (warp == mma_warp) {
        if (lane == 0) {
            // ---------------- tensor-core issue
            const std::uint32_t idesc = i8_instruction(n_tile);
            const int last_steps = (a.k_real - (k_blocks - 1) * tile_k_bytes + 31) / 32;
            const std::uint32_t buffer_columns = static_cast<std::uint32_t>(L::accumulators * n_tile);
            std::uint32_t g = 0;  // K blocks so far (weight ring)
            RingCursor rings0{0, ring_stages, 0, 0u};  // per producer set, kept in registers
            RingCursor rings1{ring_stages, ring_stages, 0, 0u};
            int local = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x, ++local) {
                const bool second = producer_sets == 2 && (local & 1) != 0;
                RingCursor a_ring = second ? rings1 : rings0;
                const int buffer = local % tmem_buffers;
                const std::uint32_t use = static_cast<std::uint32_t>(local / tmem_buffers);
                if (*abort || !barrier_wait(smem_address(&tail->tmem_empty[buffer]), (use & 1u) ^ 1u, a.status)) {
                    *abort = 1;
                    break;
                }
                tmem_fence_after();
                const std::uint32_t acc = tmem + static_cast<std::uint32_t>(buffer) * buffer_columns;
                const std::uint32_t mid = acc + static_cast<std::uint32_t>(n_tile);
                const std::uint32_t low = acc + static_cast<std::uint32_t>(2 * n_tile);
                for (int kb = 0; kb < k_blocks; ++kb, ++g) {
                    const int sa = a_ring.slot();
                    const std::uint32_t a_phase = a_ring.phase;
                    a_ring.advance();
                    const int sb = a.b_resident ? kb : static_cast<int>(g % b_stages);
                    const std::uint32_t b_phase = a.b_resident ? 0u : (g / b_stages) & 1u;
                    if (*abort || !barrier_wait(smem_address(&tail->full_a[sa]), a_phase, a.status) ||
                        !barrier_wait(smem_address(&tail->full_b[sb]), b_phase, a.status)) {
                        *abort = 1;
                        ok = false;
                        break;
                    }
                    tmem_fence_after();
                    const std::uint32_t a_hi = smem_address(smem + sa * L::a_stage_bytes);
                    const std::uint32_t a_lo = a_hi + L::a_bytes;
                    const std::uint32_t b_hi = smem_address(b_smem + sb * L::b_stage_bytes(n_tile));
                    const std::uint32_t b_lo = b_hi + static_cast<std::uint32_t>(L::b_bytes(n_tile));
                    // The last K block issues only the 32-byte steps that hold K.
                    const int steps = kb == k_blocks - 1 ? last_steps : tile_k_bytes / 32;
#pragma unroll
                    for (int kk = 0; kk < tile_k_bytes / 32; ++kk) {
                        if (kk >= steps) break;
                        const std::uint32_t step = static_cast<std::uint32_t>(kk * 32);
                        const std::uint32_t first = (kb == 0 && kk == 0) ? 0u : 1u;
                        mma_i8(acc, sw128_descriptor(a_hi + step), sw128_descriptor(b_hi + step), idesc, first);
                        if constexpr (AL == 2) {
                            mma_i8(mid, sw128_descriptor(a_lo + step), sw128_descriptor(b_hi + step), idesc, first);
                        }
                        if constexpr (WL == 2) {
                            mma_i8(mid, sw128_descriptor(a_hi + step), sw128_descriptor(b_lo + step), idesc,
                                   AL == 2 ? 1u : first);
                        }
                        if constexpr (WL == 2 && AL == 2) {
                            mma_i8(low, sw128_descriptor(a_lo + step), sw128_descriptor(b_lo + step), idesc, first);
                        }
                    }
                    mma_commit(smem_address(&tail->empty_a[sa]));
                    if (!a.b_resident) mma_commit(smem_address(&tail->empty_b[sb]));
                }
                if (second) {
                    rings1 = a_ring;
                } else {
                    rings0 = a_ring;
                }
                if (!ok) break;
                mma_commit(smem_address(&tail->tmem_full[buffer]));
            }
            // Arrives once every MMA issued above has completed.
            mma_commit(smem_address(&tail->drain));
            barrier_wait(smem_address(&tail->drain), 0u, a.status);
        }
    } else if (warp == halo_warp) {
        grid_dependency_wait();
        if (lane == 0) {
            // ---------------- activation halo by TMA, one channel group per load
            // The two rings' cursors stay in registers: a tile works on a copy of
            // its ring's cursor, written back after the tile.
            RingCursor ring0{0, ring_halos, 0, 0u};
            RingCursor ring1{ring_halos, ring_halos, 0, 0u};
            std::uint32_t issued0 = 0;
            std::uint32_t issued1 = 0;
            bool ok = true;
            const std::uint32_t box_bytes =
                static_cast<std::uint32_t>(a.record_bytes) * static_cast<std::uint32_t>(a.halo_box_w * a.halo_rows);
            int local = 0;
            for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x, ++local) {
                const bool second = producer_sets == 2 && (local & 1) != 0;
                RingCursor cursor = second ? ring1 : ring0;
                std::uint32_t count = second ? issued1 : issued0;
                int n_index, tx;
                const int p_tile = by_n_tiles.divide(t, n_index);
                const int ty = by_tiles_x.divide(p_tile, tx);
                const int y0 = ty * a.patch_h * a.window.stride_y - a.window.pad_top;
                const int x0 = tx * a.patch_w * a.window.stride_x - a.window.pad_left;
                for (int g = 0; g < a.groups; ++g) {
                    const int h = cursor.slot();
                    if (*abort || !barrier_wait(smem_address(&tail->halo_empty[h]), cursor.phase ^ 1u, a.status)) {
                        *abort = 1;
                        ok = false;
                        break;
                    }
                    const std::uint32_t full = smem_address(&tail->halo_full[h]);
                    barrier_expect_bytes(full, box_bytes);
                    // Innermost coordinate: the group's first channel, a multiple of 16 bytes.
                    tma_load_3d(smem_address(halo_smem + h * a.halo_bytes), &halo_map, full, g * a.group, x0, y0);
                    cursor.advance();
                    ++count;
                }
                if (second) {
                    ring1 = cursor;
                    issued1 = count;
                } else {
                    ring0 = cursor;
                    issued0 = count;
                }
            }
            if (!ok) {
                // Every issued load must land before the CTA may exit: the last
                // (up to depth) uses of each ring.
                const std::uint32_t depth = static_cast<std::uint32_t>(ring_halos);
                for (int r = 0; r < producer_sets; ++r) {
                    const std::uint32_t n = r == 0 ? issued0 : issued1;
                    const std::uint32_t first = n > depth ? n - depth : 0;
                    for (std::uint32_t u = first; u < n; ++u) {
                        const int h = r * ring_halos + static_cast<int>(u % depth);
                        barrier_wait(smem_address(&tail->halo_full[h]), (u / depth) & 1u, a.status);
                    }
                }
            }
        }
    } else if (warp >= epilogue_warps) {
        grid_dependency_wait();
        // ---------------- activation producers: thread <-> position; set s of
        // the producer_sets takes the CTA's tiles s, s + sets, ...
        const int producer_thread = threadIdx.x - epilogue_threads;
        const int set = producer_thread >> 7;
        const int row = producer_thread & (tile_positions_m - 1);
        const int py = row / a.patch_w;
        const int px = row - py * a.patch_w;
        const int kernel_w = a.window.kernel_w;
        const int taps = a.window.kernel_h * kernel_w;
        const int record_bytes = a.record_bytes;
        // Byte offset r * record_bytes >> 7 picks the 128-byte line; its low bits
        // (as many as there are 16-byte pieces in a record) swizzle the pieces.
        const std::uint32_t swizzle_mask = static_cast<std::uint32_t>(record_bytes / 16 - 1);
        const int chunks_per_tap = a.group / 16;
        constexpr int pieces_per_chunk = SourceHalf ? 2 : 4;
        const int base_record = py * a.window.stride_y * a.halo_box_w + px * a.window.stride_x;
        const std::uint32_t slot_key = static_cast<std::uint32_t>(row & 7);
        RingCursor stages{set * ring_stages, ring_stages, 0, 0u};  // this set's A-stage ring
        RingCursor halos{set * ring_halos, ring_halos, 0, 0u};     // this set's halo ring
        int local = set;  // the CTA's tile index
        const int tile_step = producer_sets * static_cast<int>(gridDim.x);
        bool ok = true;
        // Pixel maxima of this position's window in the tile t: windows of up to
        // 3x3 taps load into registers one tile ahead (their latency hides
        // behind the tile before); larger windows load when needed.
        constexpr int window_taps = 9;
        const bool small_window = a.window.kernel_h <= 3 && kernel_w <= 3;
        // The loads are unconditional (pixel 0 stands in outside the window) and
        // the returned mask marks the taps inside it: the mask is applied one
        // tile later, so no select waits for the loads before then.
        // Tile coordinates (N tile, patch column, patch row) of the tiles this set
        // walks, advanced by the constant tile step instead of divided out per tile.
        struct TileAt {
            int n_index, tx, ty;
        };
        const int first_tile = static_cast<int>(blockIdx.x) + set * static_cast<int>(gridDim.x);
        int step_n;
        const int step_p = by_n_tiles.divide(tile_step, step_n);
        int step_x;
        const int step_y = by_tiles_x.divide(step_p, step_x);
        auto tile_at = [&](int t) {
            TileAt c;
            const int p_tile = by_n_tiles.divide(t, c.n_index);
            c.ty = by_tiles_x.divide(p_tile, c.tx);
            return c;
        };
        auto advance = [&](TileAt& c) {
            int carry = 0;
            c.n_index += step_n;
            if (c.n_index >= a.n_tiles) {
                c.n_index -= a.n_tiles;
                carry = 1;
            }
            c.tx += step_x + carry;  // < 2 tiles_x: one wrap at most
            c.ty += step_y;
            if (c.tx >= a.tiles_x) {
                c.tx -= a.tiles_x;
                c.ty += 1;
            }
        };
        const bool pointwise = a.window.kernel_h == 1 && kernel_w == 1;
        auto window_loads = [&](const TileAt& c, float (&m)[window_taps]) -> std::uint32_t {
            const int oy = c.ty * a.patch_h + py;
            const int ox = c.tx * a.patch_w + px;
            const int iy0 = oy * a.window.stride_y - a.window.pad_top;
            const int ix0 = ox * a.window.stride_x - a.window.pad_left;
            const bool real = oy < a.out_h && ox < a.out_w;
            if (pointwise) {
                // One pixel: one load.
                const bool inside = real && iy0 >= 0 && iy0 < a.in_h && ix0 >= 0 && ix0 < a.in_w;
                m[0] = __ldg(a.pixel_max + (inside ? static_cast<std::size_t>(iy0) * a.in_w + ix0 : 0));
                return inside ? 1u : 0u;
            }
            std::uint32_t inside_mask = 0;
#pragma unroll
            for (int ky = 0; ky < 3; ++ky) {
#pragma unroll
                for (int kx = 0; kx < 3; ++kx) {
                    const int iy = iy0 + ky;
                    const int ix = ix0 + kx;
                    const bool inside = real && ky < a.window.kernel_h && kx < kernel_w && iy >= 0 && iy < a.in_h &&
                        ix >= 0 && ix < a.in_w;
                    m[3 * ky + kx] = __ldg(a.pixel_max + (inside ? static_cast<std::size_t>(iy) * a.in_w + ix : 0));
                    inside_mask |= inside ? 1u << (3 * ky + kx) : 0u;
                }
            }
            return inside_mask;
        };
        float next_window[window_taps];
        std::uint32_t next_mask = 0;
        TileAt next_at = tile_at(first_tile < total_tiles ? first_tile : 0);
        if (small_window && first_tile < total_tiles) next_mask = window_loads(next_at, next_window);
        for (int t = first_tile; t < total_tiles && ok; t += tile_step, local += producer_sets) {
            const TileAt at = next_at;
            advance(next_at);
            const int ty = at.ty;
            const int tx = at.tx;
            const int oy = ty * a.patch_h + py;
            const int ox = tx * a.patch_w + px;
            const bool real = oy < a.out_h && ox < a.out_w;
            const int iy0 = oy * a.window.stride_y - a.window.pad_top;
            const int ix0 = ox * a.window.stride_x - a.window.pad_left;
            float maximum = 0.0f;
            if (small_window) {
#pragma unroll
                for (int i = 0; i < window_taps; ++i) {
                    if ((next_mask >> i) & 1u) maximum = fmaxf(maximum, next_window[i]);
                }
                if (t + tile_step < total_tiles) next_mask = window_loads(next_at, next_window);
            } else if (real) {
                for (int ky = 0; ky < a.window.kernel_h; ++ky) {
                    const int iy = iy0 + ky;
                    if (iy < 0 || iy >= a.in_h) continue;
                    for (int kx = 0; kx < kernel_w; ++kx) {
                        const int ix = ix0 + kx;
                        if (ix < 0 || ix >= a.in_w) continue;
                        maximum = fmaxf(maximum, __ldg(a.pixel_max + static_cast<std::size_t>(iy) * a.in_w + ix));
                    }
                }
            }
            int exponent = INT_MIN;
            int mode = quant_skip;
            float scale = 0.0f;
            std::uint32_t scale_pair = 0;
            if (real) {
                if (maximum != __uint_as_float(0x7f800000u)) {
                    exponent = activation_exponent(maximum, bits);
                    if (exponent >= -127 && exponent <= 126) {
                        scale = power_of_two(-exponent);
                        const float scaled = __fmul_rn(maximum, scale);  // exact: a power-of-two scaling
                        constexpr float bound = AL == 2 ? 32767.5f : 127.5f;
                        mode = scaled < bound ? quant_float : quant_float_clamp;
                        if (SourceHalf && AL == 1 && mode == quant_float && exponent >= -15 && exponent <= 14) {
                            const std::uint32_t h = static_cast<std::uint32_t>(15 - exponent) << 10;
                            scale_pair = h | (h << 16);
                            mode = quant_half;
                        }
                    } else {
                        mode = quant_exact;
                    }
                }
            }
            int sum_high = 0;
            int sum_low = 0;
            int chunk = 0;            // 16-byte chunk of the open A stage, 0..7
            std::uint32_t a_key = 0;  // this position's row in the open A stage, xor its swizzle key
            auto open_stage = [&]() -> bool {
                if (*abort || !barrier_wait(smem_address(&tail->empty_a[stages.slot()]), stages.phase ^ 1u, a.status)) {
                    return false;
                }
                // Rows are 128-byte aligned: row + ((chunk ^ key) << 4) == (row ^ (key << 4)) ^ (chunk << 4).
                a_key = smem_address(smem + stages.slot() * L::a_stage_bytes + row * tile_k_bytes) ^ (slot_key << 4);
                return true;
            };
            auto close_stage = [&]() {
                fence_proxy_async_shared();
                barrier_arrive(smem_address(&tail->full_a[stages.slot()]));
                stages.advance();
            };
            // A warp whose positions all take the common rounding (or produce
            // nothing) quantises inline with that mode fixed at compile time;
            // other warps call the out-of-line any-mode quantiser.
            constexpr int fast_mode = (SourceHalf && AL == 1) ? quant_half : quant_float;
            const bool fast = __all_sync(__activemask(), mode == fast_mode || mode == quant_skip);
            auto walk = [&](auto fast_tag) {
                constexpr bool Fast = decltype(fast_tag)::value;
                // One 16-channel chunk from its pieces (FP16: p0, p1; FP32: p0..p3) into the A row at `at`.
                auto emit = [&](std::uint32_t at, const uint4& p0, const uint4& p1, const uint4& p2, const uint4& p3) {
                    std::uint32_t high[4], low[4];
                    if constexpr (Fast) {
                        const uint4 d[4] = {p0, p1, p2, p3};
                        quantize_chunk<WL, AL, SourceHalf>(d, fast_mode, scale_pair, scale, exponent, high, low,
                                                           sum_high, sum_low);
                    } else {
                        const ChunkLimbs limbs =
                            quantize_chunk_any<WL, AL, SourceHalf>(p0, p1, p2, p3, mode, scale_pair, scale, exponent);
#pragma unroll
                        for (int w = 0; w < 4; ++w) {
                            high[w] = limbs.high[w];
                            low[w] = limbs.low[w];
                        }
                        sum_high += limbs.sum_high;
                        sum_low += limbs.sum_low;
                    }
                    store_shared_v4(at, high);
                    if constexpr (AL == 2) store_shared_v4(at + L::a_bytes, low);
                };
                for (int g = 0; g < a.groups && ok; ++g) {
                    if (*abort || !barrier_wait(smem_address(&tail->halo_full[halos.slot()]), halos.phase, a.status)) {
                        ok = false;
                        break;
                    }
                    const std::uint32_t halo = smem_address(halo_smem + halos.slot() * a.halo_bytes);
                    int ky = 0;
                    int kx = 0;
                    for (int tap = 0; tap < taps; ++tap) {
                        const int r = base_record + ky * a.halo_box_w + kx;
                        const std::uint32_t offset = static_cast<std::uint32_t>(r * record_bytes);
                        const std::uint32_t record = (halo + offset) ^ (((offset >> 7) & swizzle_mask) << 4);
                        auto piece = [&](std::uint32_t b) { return load_shared_v4(record ^ (b << 4)); };
                        // A tap's chunks never straddle a K block: chunks per tap (1, 2 or 4) divide 8.
                        if (chunk == 0 && !open_stage()) {
                            ok = false;
                            break;
                        }
                        // chunk is a multiple of the chunks per tap, so chunk + q == chunk ^ q.
                        const std::uint32_t at = a_key ^ (static_cast<std::uint32_t>(chunk) << 4);
                        // The tap's whole record is loaded before its chunks.
                        if (chunks_per_tap * pieces_per_chunk == 8) {
                            const uint4 p0 = piece(0), p1 = piece(1), p2 = piece(2), p3 = piece(3);
                            const uint4 p4 = piece(4), p5 = piece(5), p6 = piece(6), p7 = piece(7);
                            if constexpr (SourceHalf) {
                                emit(at, p0, p1, p0, p1);
                                emit(at ^ 16u, p2, p3, p2, p3);
                                emit(at ^ 32u, p4, p5, p4, p5);
                                emit(at ^ 48u, p6, p7, p6, p7);
                            } else {
                                emit(at, p0, p1, p2, p3);
                                emit(at ^ 16u, p4, p5, p6, p7);
                            }
                        } else if (chunks_per_tap * pieces_per_chunk == 4) {
                            const uint4 p0 = piece(0), p1 = piece(1), p2 = piece(2), p3 = piece(3);
                            if constexpr (SourceHalf) {
                                emit(at, p0, p1, p0, p1);
                                emit(at ^ 16u, p2, p3, p2, p3);
                            } else {
                                emit(at, p0, p1, p2, p3);
                            }
                        } else {
                            const uint4 p0 = piece(0), p1 = piece(1);
                            emit(at, p0, p1, p0, p1);  // FP16 only: 16 channels in two pieces
                        }
                        chunk += chunks_per_tap;
                        if (chunk == tile_k_bytes / 16) {
                            close_stage();
                            chunk = 0;
                        }
                        if (++kx == kernel_w) {
                            kx = 0;
                            ++ky;
                        }
                    }
                    barrier_arrive(smem_address(&tail->halo_empty[halos.slot()]));
                    halos.advance();
                }
            };
            if (fast) {
                walk(std::true_type{});
            } else {
                walk(std::false_type{});
            }
            if (ok && chunk > 0) {
                // K ends inside this stage: zero limbs up to the end of the last
                // 32-byte MMA step (the MMA reads no further; the weights are zero there too).
                const std::uint32_t zero[4] = {0, 0, 0, 0};
                const int used = (chunk + 1) & ~1;
                for (; chunk < used; ++chunk) {
                    const std::uint32_t at = a_key ^ (static_cast<std::uint32_t>(chunk) << 4);
                    store_shared_v4(at, zero);
                    if constexpr (AL == 2) store_shared_v4(at + L::a_bytes, zero);
                }
                close_stage();
                chunk = 0;
            }
            if (!ok) {
                *abort = 1;
                break;
            }
            const int info = local & 1;
            if (!barrier_wait(smem_address(&tail->info_empty[info]), ((local >> 1) & 1) ^ 1u, a.status)) {
                *abort = 1;
                break;
            }
            tail->exponents[info][row] = real ? exponent : INT_MIN;
            tail->column_terms[info][row] =
                mode != quant_skip ? a.column_high_factor * sum_high + a.column_low_factor * sum_low : 0;
            barrier_arrive(smem_address(&tail->info_full[info]));
        }
    } else {
        // ---------------- epilogue: thread <-> TMEM lane <-> position
        grid_dependency_wait();
        // Warp w reads TMEM lane quarter w % 4 (positions 32(w % 4) .. +31); with
        // eight epilogue warps, w and w + 4 take the first and second half of the
        // tile's 16-column chunks, with four each warp takes them all.
        const int row = threadIdx.x & (tile_positions_m - 1);
        const int half = epilogue_warps == 8 ? warp >> 2 : -1;
        const std::uint32_t lane_base = static_cast<std::uint32_t>((warp & 3) * 32) << 16;
        const std::uint32_t buffer_columns = static_cast<std::uint32_t>(L::accumulators * n_tile);
        constexpr long long high_factor = (WL == 2 ? 256LL : 1LL) * (AL == 2 ? 256LL : 1LL);
        constexpr long long mid_factor = (WL == 2 && AL == 2) ? 256LL : 1LL;
        const int pair_offset = a.chunk_add ? n_tile / 2 : 0;
        const int columns = a.chunk_add ? n_tile / 2 : n_tile;
        const int half_columns = (columns / 2 + 15) / 16 * 16;
        const int first_column = half == 1 ? half_columns : 0;
        const int last_column = half == 0 ? half_columns : columns;
        const int b = a.d2s_block;
        const int patch_y = row / a.patch_w;
        const int patch_x = row - patch_y * a.patch_w;
        const int out_w_full = a.out_w * (b > 0 ? b : 1);
        const int out_h_full = a.out_h * (b > 0 ? b : 1);
        int local = 0;
        for (int t = blockIdx.x; t < total_tiles; t += gridDim.x, ++local) {
            const int buffer = local % tmem_buffers;
            const std::uint32_t use = static_cast<std::uint32_t>(local / tmem_buffers);
            const int info = local & 1;
            bool waited = *abort == 0 && barrier_wait(smem_address(&tail->tmem_full[buffer]), use & 1u, a.status) &&
                barrier_wait(smem_address(&tail->info_full[info]), (local >> 1) & 1u, a.status);
            // tcgen05.ld below is warp-aligned: the whole warp takes one decision.
            waited = __all_sync(0xffffffffu, waited);
            if (!waited) {
                *abort = 1;
                break;
            }
            tmem_fence_after();
            const int exponent = tail->exponents[info][row];
            const long long column = tail->column_terms[info][row];
            barrier_arrive(smem_address(&tail->info_empty[info]));
            int n_index, tx;
            const int p_tile = by_n_tiles.divide(t, n_index);
            const int ty = by_tiles_x.divide(p_tile, tx);
            const int y = ty * a.patch_h + patch_y;
            const int x = tx * a.patch_w + patch_x;
            const bool real = y < a.out_h && x < a.out_w;
            const int p = real ? y * a.out_w + x : 0;
            const int physical0 = n_index * n_tile;
            const int logical0 = a.chunk_add ? n_index * (n_tile / 2) : physical0;
            const std::uint32_t acc = tmem + static_cast<std::uint32_t>(buffer) * buffer_columns + lane_base;
            // out = ((float(acc) * scale) * 2^e) + bias. ldexp by e is one multiply
            // by 2^e when e is in [-126, 127]; rows without an exponent become NaN.
            const bool normal = exponent >= -126 && exponent <= 127;
            const bool plain = normal || exponent == INT_MIN;
            const float power = normal ? power_of_two(exponent) : 1.0f;

            // The exact integer sum of accumulator column j of a chunk, times the column scale.
            auto scaled_at = [&](int physical, int hh, int md, int lo, float scale) -> float {
                if constexpr (WL == 1 && AL == 1) {
                    return __fmul_rn(__int2float_rn(hh), scale);
                } else {
                    long long sum = high_factor * hh + column + mid_factor * md;
                    if constexpr (AL == 2) sum += column_row_terms[physical];
                    if constexpr (WL == 2 && AL == 2) sum += lo;
                    return __fmul_rn(__ll2float_rn(sum), scale);
                }
            };
            // 16 output values of the chunk at accumulator columns first.. (one
            // decision per chunk for the rare wide-exponent path and for WSiLU).
            auto values16 = [&](int first, float (&v)[16]) {
                int hh[16], md[16], lo[16];
                tmem_load16(acc + static_cast<std::uint32_t>(first), hh);
                if constexpr (L::accumulators > 1) tmem_load16(acc + static_cast<std::uint32_t>(n_tile + first), md);
                if constexpr (L::accumulators > 2) tmem_load16(acc + static_cast<std::uint32_t>(2 * n_tile + first), lo);
                const float4* scale4 = reinterpret_cast<const float4*>(column_scale + physical0 + first);
                const float4* bias4 = reinterpret_cast<const float4*>(column_bias + physical0 + first);
                float scales[16], biases[16];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float4 f = scale4[i];
                    const float4 g = bias4[i];
                    scales[4 * i] = f.x;
                    scales[4 * i + 1] = f.y;
                    scales[4 * i + 2] = f.z;
                    scales[4 * i + 3] = f.w;
                    biases[4 * i] = g.x;
                    biases[4 * i + 1] = g.y;
                    biases[4 * i + 2] = g.z;
                    biases[4 * i + 3] = g.w;
                }
                tmem_load_wait();
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    v[j] = scaled_at(physical0 + first + j, hh[j], L::accumulators > 1 ? md[j] : 0,
                                     L::accumulators > 2 ? lo[j] : 0, scales[j]);
                }
                if (plain) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] = __fadd_rn(__fmul_rn(v[j], power), biases[j]);
                } else {
                    Sixteen x, bias;
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        x.v[j] = v[j];
                        bias.v[j] = biases[j];
                    }
                    x = ldexp_add16(x, bias, exponent);
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] = x.v[j];
                }
                if (a.wsilu) {
                    Sixteen x;
#pragma unroll
                    for (int j = 0; j < 16; ++j) x.v[j] = v[j];
                    x = wsilu16(x, a.wsilu_scale);
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] = x.v[j];
                }
            };

            std::uint32_t staged_max = 0;  // max |x| bits of this position's staged outputs
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
                if (real) {
                    if (exponent == INT_MIN) {
#pragma unroll
                        for (int j = 0; j < 16; ++j) v[j] = canonical_nan();
                    }
                    if (a.residual != nullptr) {
                        float add[16];
                        if (a.residual_c_pad > 0) {
                            // Channel-innermost residual: the position's 16 channels are contiguous.
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
                        // Staged store: the position's 16 channels as four 16-byte stores,
                        // zeros past out_channels (up to out_c_pad), and their max |x| bits.
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
                        // Sixteen channel planes of this position.
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
            if (a.out_max != nullptr && real) {
                // Non-negative floats order as their bits; NaN bits become +inf.
                atomicMax(reinterpret_cast<unsigned int*>(a.out_max) + p,
                          __float_as_uint(max_from_float_bits(staged_max)));
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

EncodeTiled encoder() {
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

int shared_bytes(int weight_limbs, int activation_limbs, int n_tile, int n_tiles, int a_stages, int b_stages,
                 int halo_region) {
    return 1024 + a_stages * activation_limbs * tile_positions_m * tile_k_bytes +
        b_stages * weight_limbs * n_tile * tile_k_bytes + halo_region +
        static_cast<int>((sizeof(ConvTail) + 15) / 16 * 16) + parameter_bytes(n_tile * n_tiles, activation_limbs);
}

// Host-side checks of everything the kernel's indexing relies on.
bool valid_geometry(const FusedConvArgs& a, int accumulators) {
    const int element = a.source_half ? 2 : 4;
    const int taps = a.window.kernel_h * a.window.kernel_w;
    const bool record_ok = a.record_bytes == 16 || a.record_bytes == 32 || a.record_bytes == 64 ||
        a.record_bytes == 128;
    const bool aligned = (reinterpret_cast<std::uintptr_t>(a.scales) & 15u) == 0 &&
        (reinterpret_cast<std::uintptr_t>(a.bias) & 15u) == 0;
    return aligned && static_cast<long long>(a.p_tiles) * a.n_tiles < (1LL << 22) && a.n_tile >= 16 && a.n_tile <= 256 && a.n_tile % 16 == 0 &&
        (!a.chunk_add || a.n_tile % 32 == 0) && accumulators * a.n_tile <= 512 && a.k_blocks >= 1 &&
        a.p_tiles >= 1 && a.n_tiles >= 1 && taps >= 1 && a.patch_h * a.patch_w == tile_positions_m &&
        a.patch_w >= 1 && record_ok && a.group % 16 == 0 && a.group * element == a.record_bytes &&
        a.c_pad % a.group == 0 && a.groups * a.group == a.c_pad && a.c_pad >= a.channels &&
        a.k_real == taps * a.c_pad && a.k_blocks == (a.k_real + tile_k_bytes - 1) / tile_k_bytes &&
        a.halo_rows == (a.patch_h - 1) * a.window.stride_y + a.window.kernel_h &&
        a.halo_box_w >= (a.patch_w - 1) * a.window.stride_x + a.window.kernel_w && a.halo_box_w <= 256 &&
        a.halo_rows <= 256 && a.halo_bytes % 1024 == 0 && a.halo_buffers >= 2 &&
        (a.producer_sets == 1 || a.producer_sets == 2) && a.a_stages % a.producer_sets == 0 &&
        (a.out_max == nullptr ||
         (!a.out_half && a.d2s_block == 0 && a.out_c_pad % 16 == 0 && a.out_c_pad >= a.out_channels &&
          (reinterpret_cast<std::uintptr_t>(a.out) & 15u) == 0)) &&
        (a.residual_c_pad == 0 ||
         (a.residual_c_pad % 16 == 0 && a.residual_c_pad >= a.out_channels &&
          (reinterpret_cast<std::uintptr_t>(a.residual) & 15u) == 0)) &&
        a.halo_buffers <= max_halo_buffers &&
        a.halo_bytes >= a.halo_rows * a.halo_box_w * a.record_bytes && a.a_stages >= 1 &&
        a.a_stages <= max_stages && a.b_stages >= 1 && a.b_stages <= max_stages &&
        (!a.b_resident || (a.n_tiles == 1 && a.b_stages == a.k_blocks)) && a.tiles_y * a.patch_h >= a.out_h &&
        a.tiles_x * a.patch_w >= a.out_w && a.p_tiles == a.tiles_y * a.tiles_x &&
        a.positions == a.out_h * a.out_w && a.d2s_block >= 0 &&
        (a.chunk_add ? a.out_channels <= a.n_tiles * a.n_tile / 2 : a.out_channels <= a.n_tiles * a.n_tile);
}

template <int WL, int AL, bool SourceHalf>
cudaError_t launch_fused(const CUtensorMap& b_high, const CUtensorMap& b_low, const CUtensorMap& halo,
                         const FusedConvArgs& args, int sm_count, cudaStream_t stream) {
    using L = ConvLayout<WL, AL>;
    constexpr int max_dynamic = 232448;
    const int n_tile = args.n_tile;
    if (!valid_geometry(args, L::accumulators)) return cudaErrorInvalidValue;
    int buffers = 2;
    std::uint32_t columns = 32;
    while (static_cast<int>(columns) < 2 * L::accumulators * n_tile) columns <<= 1;
    if (columns > 512) {
        buffers = 1;
        columns = 32;
        while (static_cast<int>(columns) < L::accumulators * n_tile) columns <<= 1;
        if (columns > 512) return cudaErrorInvalidValue;
    }
    const int smem = shared_bytes(WL, AL, n_tile, args.n_tiles, args.a_stages, args.b_stages,
                                  args.halo_buffers * args.halo_bytes);
    if (smem > max_dynamic) return cudaErrorInvalidValue;
    static bool configured = false;
    if (!configured) {
        const cudaError_t set = cudaFuncSetAttribute(fused_conv_kernel<WL, AL, SourceHalf>,
                                                     cudaFuncAttributeMaxDynamicSharedMemorySize, max_dynamic);
        if (set != cudaSuccess) return set;
        configured = true;
    }
    const int tiles = args.p_tiles * args.n_tiles;
    const int grid = tiles < sm_count ? tiles : sm_count;
    return launch_overlapped(fused_conv_kernel<WL, AL, SourceHalf>, dim3(grid), dim3(conv_threads), smem, stream,
                             b_high, b_low, halo, args, buffers, columns);
}

template <int WL, int AL>
cudaError_t dispatch_source(const CUtensorMap& b_high, const CUtensorMap& b_low, const CUtensorMap& halo,
                            const FusedConvArgs& args, int sm_count, cudaStream_t stream) {
    return args.source_half ? launch_fused<WL, AL, true>(b_high, b_low, halo, args, sm_count, stream)
                            : launch_fused<WL, AL, false>(b_high, b_low, halo, args, sm_count, stream);
}

}  // namespace

cudaError_t encode_int8_map(CUtensorMap* map, const void* base, std::uint64_t rows, std::uint64_t row_bytes,
                            std::uint32_t box_rows) {
    const EncodeTiled encode = encoder();
    if (encode == nullptr) return cudaErrorNotSupported;
    if ((reinterpret_cast<std::uintptr_t>(base) & 15u) != 0 || row_bytes % tile_k_bytes != 0 || box_rows == 0 ||
        box_rows > 256) {
        return cudaErrorInvalidValue;
    }
    const cuuint64_t dims[2] = {row_bytes, rows};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(tile_k_bytes), box_rows};
    const cuuint32_t element_strides[2] = {1, 1};
    const CUresult result = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
                                   element_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return result == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

int fused_conv_shared_bytes(int weight_limbs, int activation_limbs, int n_tile, int n_tiles, int a_stages,
                            int b_stages, int halo_region) {
    return shared_bytes(weight_limbs, activation_limbs, n_tile, n_tiles, a_stages, b_stages, halo_region);
}

cudaError_t encode_halo_map(CUtensorMap* map, const void* base, int half, std::uint64_t c_pad, std::uint64_t height,
                            std::uint64_t width, std::uint32_t group, std::uint32_t box_w, std::uint32_t box_h) {
    const EncodeTiled encode = encoder();
    if (encode == nullptr) return cudaErrorNotSupported;
    const std::uint64_t element = half ? 2 : 4;
    const std::uint64_t record = group * element;
    if ((reinterpret_cast<std::uintptr_t>(base) & 15u) != 0 || (c_pad * element) % 16 != 0 || group == 0 ||
        c_pad % group != 0 || (record != 16 && record != 32 && record != 64 && record != 128) || box_w == 0 ||
        box_w > 256 || box_h == 0 || box_h > 256) {
        return cudaErrorInvalidValue;
    }
    const CUtensorMapSwizzle swizzle = record == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
        : record == 64                               ? CU_TENSOR_MAP_SWIZZLE_64B
        : record == 32                               ? CU_TENSOR_MAP_SWIZZLE_32B
                                                     : CU_TENSOR_MAP_SWIZZLE_NONE;
    const cuuint64_t dims[3] = {c_pad, width, height};
    const cuuint64_t strides[2] = {c_pad * element, width * c_pad * element};
    const cuuint32_t box[3] = {group, box_w, box_h};
    const cuuint32_t element_strides[3] = {1, 1, 1};
    const CUresult result = encode(map, half ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3,
                                   const_cast<void*>(base), dims, strides, box, element_strides,
                                   CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return result == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t stage_source(const void* in, int source_half, int channels, int c_pad, int pixels, void* out,
                         float* pixel_max, cudaStream_t stream, const unsigned int* gate) {
    if (pixels <= 0) return cudaSuccess;
    if (channels < 1 || c_pad < channels || c_pad % 16 != 0 || (reinterpret_cast<std::uintptr_t>(out) & 15u) != 0) {
        return cudaErrorInvalidValue;
    }
    if (c_pad > 32) {
        return source_half ? launch_stage<true>(in, channels, c_pad, pixels, out, pixel_max, gate, stream)
                           : launch_stage<false>(in, channels, c_pad, pixels, out, pixel_max, gate, stream);
    }
    const unsigned blocks = static_cast<unsigned>((static_cast<long long>(pixels) + 255) / 256);
    if (source_half) {
        return launch_overlapped(stage_pixels_kernel<true>, dim3(blocks), dim3(256), 0, stream, in, channels, c_pad,
                                 pixels, out, pixel_max, gate);
    } else {
        return launch_overlapped(stage_pixels_kernel<false>, dim3(blocks), dim3(256), 0, stream, in, channels, c_pad,
                                 pixels, out, pixel_max, gate);
    }
    return cudaGetLastError();
}

namespace {
__global__ void wait_timeout_kernel(unsigned long long limit_ns, unsigned int* status) {
    __shared__ unsigned long long never;
    if (threadIdx.x == 0) {
        barrier_init(smem_address(&never), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        barrier_wait_for(smem_address(&never), 0u, status, limit_ns);  // phase 0 never completes
    }
}
}  // namespace

namespace {
// Counts the floats d with bit patterns first .. first + count - 1 for which the
// sigmoid's reciprocal differs in any bit from the IEEE division 1 / d.
__global__ void reciprocal_check_kernel(std::uint32_t first, std::uint32_t count, unsigned long long* mismatches) {
    unsigned int local = 0;
    for (std::uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < count; i += gridDim.x * blockDim.x) {
        const float d = __uint_as_float(first + i);
        local += __float_as_uint(sigmoid_reciprocal(d)) != __float_as_uint(__fdiv_rn(1.0f, d)) ? 1u : 0u;
    }
    local = __reduce_add_sync(0xffffffffu, local);
    if ((threadIdx.x & 31) == 0 && local != 0) atomicAdd(mismatches, static_cast<unsigned long long>(local));
}
}  // namespace

cudaError_t check_reciprocal(std::uint32_t first, std::uint32_t count, unsigned long long* mismatches,
                             cudaStream_t stream) {
    // Only the range the sigmoid uses it on: 1 <= d < 2^126.
    if (first < 0x3f800000u || count > 0x7e800000u - first) return cudaErrorInvalidValue;
    reciprocal_check_kernel<<<1184, 256, 0, stream>>>(first, count, mismatches);
    return cudaGetLastError();
}

cudaError_t wait_timeout(unsigned long long limit_ns, unsigned int* status, cudaStream_t stream) {
    if (limit_ns > 4000000000ull) return cudaErrorInvalidValue;
    wait_timeout_kernel<<<1, 32, 0, stream>>>(limit_ns, status);
    return cudaGetLastError();
}

cudaError_t stage_receptive_fields(const void* in, int source_half, int channels, int in_h, int in_w,
                                   Window window, int out_h, int out_w, int c_pad, void* out, float* field_max,
                                   cudaStream_t stream) {
    const long long positions = static_cast<long long>(out_h) * out_w;
    if (positions <= 0) return cudaSuccess;
    if (channels < 1 || c_pad % 16 != 0 || c_pad > max_field || c_pad < channels * window.kernel_h * window.kernel_w ||
        (reinterpret_cast<std::uintptr_t>(out) & 15u) != 0) {
        return cudaErrorInvalidValue;
    }
    const unsigned blocks = static_cast<unsigned>((positions + 255) / 256);
    if (source_half) {
        return launch_overlapped(stage_fields_kernel<true>, dim3(blocks), dim3(256), 0, stream, in, channels, in_h,
                                 in_w, window, out_h, out_w, c_pad, out, field_max);
    } else {
        return launch_overlapped(stage_fields_kernel<false>, dim3(blocks), dim3(256), 0, stream, in, channels, in_h,
                                 in_w, window, out_h, out_w, c_pad, out, field_max);
    }
    return cudaGetLastError();
}

cudaError_t fused_conv(const CUtensorMap& b_high, const CUtensorMap& b_low, const CUtensorMap& halo, int weight_limbs,
                       int activation_limbs, const FusedConvArgs& args, cudaStream_t stream) {
    static int sm_count = [] {
        int device = 0;
        int count = 148;
        if (cudaGetDevice(&device) == cudaSuccess) {
            cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, device);
        }
        return count;
    }();
    if (weight_limbs == 1 && activation_limbs == 1) return dispatch_source<1, 1>(b_high, b_low, halo, args, sm_count, stream);
    if (weight_limbs == 2 && activation_limbs == 1) return dispatch_source<2, 1>(b_high, b_low, halo, args, sm_count, stream);
    if (weight_limbs == 1 && activation_limbs == 2) return dispatch_source<1, 2>(b_high, b_low, halo, args, sm_count, stream);
    if (weight_limbs == 2 && activation_limbs == 2) return dispatch_source<2, 2>(b_high, b_low, halo, args, sm_count, stream);
    return cudaErrorInvalidValue;
}

}  // namespace nvcr_sm100::kernels
