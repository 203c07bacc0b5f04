// Fused integer conv on sm_100a: quantise-on-load implicit GEMM.
//
// One persistent CTA per SM walks tiles of 128 output positions (a 2-D patch
// of patch_h x patch_w output pixels) x n_tile output channels. Warp roles:
//   warps 0-3  epilogue: one TMEM lane (= one position) per thread, the
//              profile's output arithmetic and the folded ops, then the store;
//   warp 4     TMA: int8 weight tiles (n_tile x 128 B per K block);
//   warp 5     allocates TMEM and issues the tcgen05 MMAs (one thread);
//   warps 6-9  producers: one thread per position quantises its receptive
//              field from the shared-memory halo into the 128-byte-swizzled A
//              tile; the im2col tensor and the quantised activation matrix
//              never exist in memory;
//   warp 10    TMA: the activation halo of the tile, one channel group at a
//              time, into a double-buffered shared-memory ring. Padding taps
//              and the image border come back as the TMA's zero fill.
// The accumulators are double-buffered in TMEM when they fit, so the epilogue
// of one tile overlaps the main loop of the next.
//
// K is channel-group-major: k = g * (taps * G) + tap * G_g + c, for groups of
// G channels (the last group holds G_g <= G); the weights are laid out to
// match on the host. Integer sums do not depend on the K order.
//
// Activation quantisation per position p: e_p = frexp(max |x| over the
// receptive field) - (bits - 1) from the per-pixel maxima; then
// q = clamp(rint(x * 2^-e_p), +-L). With 2^-e_p a normal float the rounding is
// one fma: fma(x, 2^-e_p, 1.5 * 2^23) is exact in the product and rounds once
// to the nearest integer at the 2^23 scale, ties to even, so its low bits hold
// rint(x * 2^-e_p) for |x * 2^-e_p| < 2^22 (always < 2^15 here). Positions whose
// 2^-e_p is not a normal float take the exact bit-level path.
//
// Every wait is bounded (about 2 s of the global timer); after a timeout the
// CTA sets bit 0 of the status word, stops issuing, drains its MMAs and TMA
// loads, frees its TMEM and returns. No multicast load is used.

#include "exact_math.cuh"
#include "kernels.hpp"
#include "tcgen05.cuh"

#include <climits>

#include <cuda_fp16.h>

namespace nvcr_sm100::kernels {
namespace {

constexpr int conv_warps = 11;
constexpr int conv_threads = conv_warps * 32;
constexpr int tma_warp = 4;
constexpr int mma_warp = 5;
constexpr int first_producer_warp = 6;
constexpr int halo_warp = 10;
constexpr int halo_buffers = 2;
constexpr int max_stages = 8;
constexpr float round_magic = 12582912.0f;           // 1.5 * 2^23
constexpr int round_magic_bits = 0x4B400000;

struct ConvTail {
    unsigned long long full_a[max_stages];
    unsigned long long empty_a[max_stages];
    unsigned long long full_b[max_stages];
    unsigned long long empty_b[max_stages];
    unsigned long long tmem_full[2];
    unsigned long long tmem_empty[2];
    unsigned long long info_full[2];
    unsigned long long info_empty[2];
    unsigned long long halo_full[halo_buffers];
    unsigned long long halo_empty[halo_buffers];
    unsigned long long drain;
    std::uint32_t tmem_base;
    int abort;
    int exponents[2][tile_positions_m];
    long long column_terms[2][tile_positions_m];
};

template <int WL, int AL>
struct ConvLayout {
    static constexpr int accumulators = 1 + ((WL == 2 || AL == 2) ? 1 : 0) + ((WL == 2 && AL == 2) ? 1 : 0);
    static constexpr int a_bytes = tile_positions_m * tile_k_bytes;
    static __host__ __device__ int b_bytes(int n_tile) { return n_tile * tile_k_bytes; }
    static constexpr int a_stage_bytes = AL * a_bytes;
    static __host__ __device__ int b_stage_bytes(int n_tile) { return WL * b_bytes(n_tile); }
};

template <bool Half>
__device__ __forceinline__ float load_halo(std::uint32_t address) {
    if constexpr (Half) {
        unsigned short bits;
        asm volatile("ld.shared.u16 %0, [%1];" : "=h"(bits) : "r"(address));
        return __half2float(__ushort_as_half(bits));
    } else {
        float value;
        asm volatile("ld.shared.f32 %0, [%1];" : "=f"(value) : "r"(address));
        return value;
    }
}

// Bytes 0 of a, b, c, d packed into one word, a lowest.
__device__ __forceinline__ std::uint32_t pack_low_bytes(std::uint32_t a, std::uint32_t b, std::uint32_t c,
                                                        std::uint32_t d) {
    return __byte_perm(__byte_perm(a, b, 0x0040u), __byte_perm(c, d, 0x0040u), 0x5410u);
}
__device__ __forceinline__ std::uint32_t pack_low_bytes(int a, int b, int c, int d) {
    return pack_low_bytes(static_cast<std::uint32_t>(a), static_cast<std::uint32_t>(b), static_cast<std::uint32_t>(c),
                          static_cast<std::uint32_t>(d));
}

// Sixteen bytes assembled one at a time in two 64-bit registers.
struct ByteRow {
    unsigned long long lo{0}, hi{0};
    __device__ __forceinline__ void put(int j, int value) {
        const unsigned long long b = static_cast<unsigned long long>(static_cast<std::uint32_t>(value) & 255u);
        if (j < 8) {
            lo |= b << (8 * j);
        } else {
            hi |= b << (8 * (j - 8));
        }
    }
    __device__ __forceinline__ void words(std::uint32_t (&w)[4]) const {
        w[0] = static_cast<std::uint32_t>(lo);
        w[1] = static_cast<std::uint32_t>(lo >> 32);
        w[2] = static_cast<std::uint32_t>(hi);
        w[3] = static_cast<std::uint32_t>(hi >> 32);
    }
};

__device__ __forceinline__ void store_shared_v4(std::uint32_t address, const std::uint32_t (&w)[4]) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(address), "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3])
                 : "memory");
}

template <bool Half>
__device__ __forceinline__ float load_source(const void* base, std::size_t index) {
    if constexpr (Half) {
        return __half2float(__ldg(static_cast<const __half*>(base) + index));
    } else {
        return __ldg(static_cast<const float*>(base) + index);
    }
}

// Per-pixel max |x| over channels; +inf when any channel is non-finite.
template <bool Half>
__global__ void __launch_bounds__(256) pixel_max_kernel(const void* __restrict__ in, int channels, int pixels,
                                                        float* __restrict__ out) {
    __shared__ float partial[8][32];
    const int lane = threadIdx.x & 31;
    const int group = threadIdx.x >> 5;
    const int pixel = blockIdx.x * 32 + lane;
    float maximum = 0.0f;
    bool finite = true;
    if (pixel < pixels) {
        for (int c = group; c < channels; c += 8) {
            const float x = load_source<Half>(in, static_cast<std::size_t>(c) * pixels + pixel);
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

template <int WL, int AL, bool SourceHalf>
__global__ void __launch_bounds__(conv_threads, 1)
fused_conv_kernel(const __grid_constant__ CUtensorMap b_high, const __grid_constant__ CUtensorMap b_low,
                  const __grid_constant__ CUtensorMap halo_map, FusedConvArgs a, int tmem_buffers,
                  std::uint32_t tmem_columns) {
    using L = ConvLayout<WL, AL>;
    constexpr int bits = AL == 2 ? 16 : 8;
    extern __shared__ std::uint8_t dynamic_smem[];
    const std::uint32_t raw = smem_address(dynamic_smem);
    std::uint8_t* smem = dynamic_smem + (((raw + 1023u) & ~1023u) - raw);
    const int n_tile = a.n_tile;
    const int a_stages = a.a_stages;
    const int b_stages = a.b_stages;
    // Shared memory: [A stages][B stages][halo buffers][tail], each part 1 KiB aligned.
    std::uint8_t* b_smem = smem + a_stages * L::a_stage_bytes;
    std::uint8_t* halo_smem = b_smem + b_stages * L::b_stage_bytes(n_tile);
    ConvTail* tail = reinterpret_cast<ConvTail*>(halo_smem + halo_buffers * a.halo_bytes);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int total_tiles = a.p_tiles * a.n_tiles;
    const int k_blocks = a.k_blocks;

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
            barrier_init(smem_address(&tail->tmem_empty[b]), tile_positions_m);
            barrier_init(smem_address(&tail->info_full[b]), tile_positions_m);
            barrier_init(smem_address(&tail->info_empty[b]), tile_positions_m);
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
    volatile int* abort = &tail->abort;

    if (warp == tma_warp) {
        if (lane == 0) {
            // ---------------- weights by TMA
            const std::uint32_t bytes = static_cast<std::uint32_t>(WL * L::b_bytes(n_tile));
            std::uint32_t g = 0;
            std::uint32_t issued = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
                const int n0 = (t % a.n_tiles) * n_tile;
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
            const std::uint32_t buffer_columns = static_cast<std::uint32_t>(L::accumulators * n_tile);
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
                const std::uint32_t acc = tmem + static_cast<std::uint32_t>(buffer) * buffer_columns;
                const std::uint32_t mid = acc + static_cast<std::uint32_t>(n_tile);
                const std::uint32_t low = acc + static_cast<std::uint32_t>(2 * n_tile);
                for (int kb = 0; kb < k_blocks; ++kb, ++g) {
                    const int sa = static_cast<int>(g % a_stages);
                    const int sb = static_cast<int>(g % b_stages);
                    if (*abort || !barrier_wait(smem_address(&tail->full_a[sa]), (g / a_stages) & 1u, a.status) ||
                        !barrier_wait(smem_address(&tail->full_b[sb]), (g / b_stages) & 1u, a.status)) {
                        *abort = 1;
                        ok = false;
                        break;
                    }
                    tmem_fence_after();
                    const std::uint32_t a_hi = smem_address(smem + sa * L::a_stage_bytes);
                    const std::uint32_t a_lo = a_hi + L::a_bytes;
                    const std::uint32_t b_hi = smem_address(b_smem + sb * L::b_stage_bytes(n_tile));
                    const std::uint32_t b_lo = b_hi + static_cast<std::uint32_t>(L::b_bytes(n_tile));
#pragma unroll
                    for (int kk = 0; kk < tile_k_bytes / 32; ++kk) {
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
                    mma_commit(smem_address(&tail->empty_b[sb]));
                }
                if (!ok) break;
                mma_commit(smem_address(&tail->tmem_full[buffer]));
            }
            // Arrives once every MMA issued above has completed.
            mma_commit(smem_address(&tail->drain));
            barrier_wait(smem_address(&tail->drain), 0u, a.status);
        }
    } else if (warp == halo_warp) {
        if (lane == 0) {
            // ---------------- activation halo by TMA, one channel group per load
            std::uint32_t job = 0;
            std::uint32_t issued = 0;
            bool ok = true;
            const int align = a.source_half ? 8 : 4;  // 16 bytes of elements
            for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
                const int p_tile = t / a.n_tiles;
                const int ty = p_tile / a.tiles_x;
                const int tx = p_tile - ty * a.tiles_x;
                const int y0 = ty * a.patch_h * a.window.stride_y - a.window.pad_top;
                const int x0 = tx * a.patch_w * a.window.stride_x - a.window.pad_left;
                const int x_start = x0 >= 0 ? (x0 / align) * align : -(((-x0) + align - 1) / align) * align;
                for (int g = 0; g < a.groups; ++g, ++job) {
                    const int h = static_cast<int>(job % halo_buffers);
                    const std::uint32_t phase = (job / halo_buffers) & 1u;
                    if (*abort || !barrier_wait(smem_address(&tail->halo_empty[h]), phase ^ 1u, a.status)) {
                        *abort = 1;
                        ok = false;
                        break;
                    }
                    const std::uint32_t full = smem_address(&tail->halo_full[h]);
                    // The TMA delivers exactly the box: group x halo_rows x halo_box_w elements.
                    barrier_expect_bytes(full, static_cast<std::uint32_t>(a.group * a.halo_rows * a.halo_box_w *
                                                                          (SourceHalf ? 2 : 4)));
                    tma_load_3d(smem_address(halo_smem + h * a.halo_bytes), &halo_map, full, x_start, y0, g * a.group);
                    issued = job + 1;
                }
            }
            if (!ok) {
                const std::uint32_t first = issued > halo_buffers ? issued - halo_buffers : 0;
                for (std::uint32_t j = first; j < issued; ++j) {
                    barrier_wait(smem_address(&tail->halo_full[j % halo_buffers]), (j / halo_buffers) & 1u, a.status);
                }
            }
        }
    } else if (warp >= first_producer_warp) {
        // ---------------- activation producers: thread <-> position
        const int row = threadIdx.x - first_producer_warp * 32;
        const int py = row / a.patch_w;
        const int px = row - py * a.patch_w;
        const int kernel_w = a.window.kernel_w;
        const int taps = a.window.kernel_h * kernel_w;
        const int align = a.source_half ? 8 : 4;
        const int channel_stride = a.halo_rows * a.halo_box_w;  // elements per channel plane of the halo
        constexpr float limit = AL == 2 ? 32767.0f : 127.0f;
        std::uint32_t g_stage = 0;  // K blocks issued so far (stage ring)
        std::uint32_t job = 0;      // halo groups consumed so far (halo ring)
        int local = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x, ++local) {
            const int p_tile = t / a.n_tiles;
            const int ty = p_tile / a.tiles_x;
            const int tx = p_tile - ty * a.tiles_x;
            const int oy = ty * a.patch_h + py;
            const int ox = tx * a.patch_w + px;
            const bool real = oy < a.out_h && ox < a.out_w;
            const int iy0 = oy * a.window.stride_y - a.window.pad_top;
            const int ix0 = ox * a.window.stride_x - a.window.pad_left;
            int exponent = INT_MIN;
            if (real) {
                float maximum = 0.0f;
                for (int ky = 0; ky < a.window.kernel_h; ++ky) {
                    const int iy = iy0 + ky;
                    if (iy < 0 || iy >= a.in_h) continue;
                    for (int kx = 0; kx < kernel_w; ++kx) {
                        const int ix = ix0 + kx;
                        if (ix < 0 || ix >= a.in_w) continue;
                        maximum = fmaxf(maximum, __ldg(a.pixel_max + static_cast<std::size_t>(iy) * a.in_w + ix));
                    }
                }
                exponent = maximum == __uint_as_float(0x7f800000u) ? INT_MIN : activation_exponent(maximum, bits);
            }
            const bool live = exponent != INT_MIN;
            const bool fast = live && exponent >= -127 && exponent <= 126;  // 2^-e is a normal float
            const float scale = fast ? power_of_two(-exponent) : 0.0f;
            // Halo coordinates of this position's (0, 0) tap.
            const int x0 = tx * a.patch_w * a.window.stride_x - a.window.pad_left;
            const int x_start = x0 >= 0 ? (x0 / align) * align : -(((-x0) + align - 1) / align) * align;
            const int base_y = py * a.window.stride_y;
            const int base_x = px * a.window.stride_x + (x0 - x_start);
            int sum_high = 0;
            int sum_low = 0;
            // Walk state: group, channels in it, tap, channel, element offset in the halo.
            int group = 0;
            int group_channels = a.group < a.channels ? a.group : a.channels;
            int tap = 0;
            int c = 0;
            int index = base_y * a.halo_box_w + base_x;
            std::uint32_t halo = 0;  // shared address of the current halo buffer
            auto acquire_halo = [&]() -> bool {
                const int h = static_cast<int>(job % halo_buffers);
                if (!barrier_wait(smem_address(&tail->halo_full[h]), (job / halo_buffers) & 1u, a.status)) return false;
                halo = smem_address(halo_smem + h * a.halo_bytes);
                return true;
            };
            // After the last channel of a tap: the next tap, or the next channel group.
            auto next_tap = [&]() -> bool {
                c = 0;
                if (++tap == taps) {
                    tap = 0;
                    barrier_arrive(smem_address(&tail->halo_empty[job % halo_buffers]));
                    ++job;
                    if (++group < a.groups) {
                        const int left = a.channels - group * a.group;
                        group_channels = left < a.group ? left : a.group;
                        if (!acquire_halo()) return false;
                    }
                }
                const int ky = tap / kernel_w;
                const int kx = tap - ky * kernel_w;
                index = (base_y + ky) * a.halo_box_w + base_x + kx;
                return true;
            };
            auto load = [&](int element) -> float {
                return load_halo<SourceHalf>(halo + static_cast<std::uint32_t>(element) * (SourceHalf ? 2u : 4u));
            };
            if (*abort || !acquire_halo()) {
                *abort = 1;
                break;
            }
            for (int kb = 0; kb < k_blocks; ++kb, ++g_stage) {
                const int s = static_cast<int>(g_stage % a_stages);
                const std::uint32_t phase = (g_stage / a_stages) & 1u;
                if (*abort || !barrier_wait(smem_address(&tail->empty_a[s]), phase ^ 1u, a.status)) {
                    *abort = 1;
                    ok = false;
                    break;
                }
                const std::uint32_t a_hi = smem_address(smem + s * L::a_stage_bytes + row * tile_k_bytes);
                const std::uint32_t a_lo = a_hi + L::a_bytes;
                int k = kb * tile_k_bytes;
#pragma unroll 1
                for (int chunk = 0; chunk < tile_k_bytes / 16; ++chunk) {
                    std::uint32_t high_words[4] = {0, 0, 0, 0};
                    std::uint32_t low_words[4] = {0, 0, 0, 0};
                    if (c + 16 <= group_channels && k + 16 <= a.k_real) {
                        // Sixteen channels of one tap: independent loads, then the rounding.
                        if (fast) {
                            std::uint32_t rounded[16];
#pragma unroll
                            for (int j = 0; j < 16; ++j) rounded[j] = __float_as_uint(load(index + j * channel_stride));
#pragma unroll
                            for (int j = 0; j < 16; ++j) {
                                float y = __fmaf_rn(__uint_as_float(rounded[j]), scale, round_magic);
                                y = fminf(fmaxf(y, round_magic - limit), round_magic + limit);
                                rounded[j] = __float_as_uint(y);
                            }
#pragma unroll
                            for (int w = 0; w < 4; ++w) {
                                const std::uint32_t* b = rounded + 4 * w;
                                if constexpr (AL == 2) {
                                    // q = bits - bits(magic); h = q >> 8; l' = (q & 255) - 128.
                                    int h[4];
#pragma unroll
                                    for (int j = 0; j < 4; ++j) {
                                        const int q = static_cast<int>(b[j]) - round_magic_bits;
                                        h[j] = q >> 8;
                                        if constexpr (WL == 2) {
                                            sum_high += h[j];
                                            sum_low += (q & 255) - 128;
                                        }
                                    }
                                    high_words[w] = pack_low_bytes(h[0], h[1], h[2], h[3]);
                                    low_words[w] = pack_low_bytes(b[0], b[1], b[2], b[3]) ^ 0x80808080u;
                                } else {
                                    // The low byte of bits(magic + q) is q in two's complement.
                                    high_words[w] = pack_low_bytes(b[0], b[1], b[2], b[3]);
                                    if constexpr (WL == 2) {
#pragma unroll
                                        for (int j = 0; j < 4; ++j) sum_high += static_cast<int>(b[j]) - round_magic_bits;
                                    }
                                }
                            }
                        } else if (live) {
                            ByteRow hb, lb;
#pragma unroll 1
                            for (int j = 0; j < 16; ++j) {
                                const int q = quantize_value<bits>(load(index + j * channel_stride), exponent);
                                const int h = AL == 2 ? (q >> 8) : q;
                                const int l = AL == 2 ? (q & 255) - 128 : 0;
                                hb.put(j, h);
                                lb.put(j, l);
                                if constexpr (WL == 2) {
                                    sum_high += h;
                                    sum_low += l;
                                }
                            }
                            hb.words(high_words);
                            lb.words(low_words);
                        } else if constexpr (AL == 2) {
                            // q = 0 for every real tap of a non-finite position: l' = -128.
                            low_words[0] = low_words[1] = low_words[2] = low_words[3] = 0x80808080u;
                        }
                        index += 16 * channel_stride;
                        c += 16;
                        k += 16;
                        if (c == group_channels && !next_tap()) {
                            *abort = 1;
                            ok = false;
                        }
                    } else {
                        // General walk, one k at a time (tap or group changes inside the chunk).
                        ByteRow hb, lb;
#pragma unroll 1
                        for (int j = 0; j < 16; ++j, ++k) {
                            if (k >= a.k_real) continue;
                            int q = 0;
                            if (live) {
                                const float x = load(index);
                                if (fast) {
                                    float y = __fmaf_rn(x, scale, round_magic);
                                    y = fminf(fmaxf(y, round_magic - limit), round_magic + limit);
                                    q = __float_as_int(y) - round_magic_bits;
                                } else {
                                    q = quantize_value<bits>(x, exponent);
                                }
                            }
                            const int h = AL == 2 ? (q >> 8) : q;
                            const int l = AL == 2 ? (q & 255) - 128 : 0;
                            hb.put(j, h);
                            lb.put(j, l);
                            if constexpr (WL == 2) {
                                sum_high += h;
                                sum_low += l;
                            }
                            index += channel_stride;
                            if (++c == group_channels && !next_tap()) {
                                *abort = 1;
                                ok = false;
                            }
                        }
                        hb.words(high_words);
                        lb.words(low_words);
                    }
                    const std::uint32_t slot = static_cast<std::uint32_t>((chunk ^ (row & 7)) * 16);
                    store_shared_v4(a_hi + slot, high_words);
                    if constexpr (AL == 2) store_shared_v4(a_lo + slot, low_words);
                }
                fence_proxy_async_shared();
                barrier_arrive(smem_address(&tail->full_a[s]));
                if (!ok) break;
            }
            if (!ok) break;
            const int info = local & 1;
            if (!barrier_wait(smem_address(&tail->info_empty[info]), ((local >> 1) & 1) ^ 1u, a.status)) {
                *abort = 1;
                break;
            }
            tail->exponents[info][row] = real ? exponent : INT_MIN;
            tail->column_terms[info][row] =
                live ? a.column_high_factor * sum_high + a.column_low_factor * sum_low : 0;
            barrier_arrive(smem_address(&tail->info_full[info]));
        }
    } else {
        // ---------------- epilogue: thread <-> TMEM lane <-> position
        const int row = threadIdx.x;  // warps 0-3
        const std::uint32_t lane_base = static_cast<std::uint32_t>(warp * 32) << 16;
        const std::uint32_t buffer_columns = static_cast<std::uint32_t>(L::accumulators * n_tile);
        constexpr long long high_factor = (WL == 2 ? 256LL : 1LL) * (AL == 2 ? 256LL : 1LL);
        constexpr long long mid_factor = (WL == 2 && AL == 2) ? 256LL : 1LL;
        const int pair_offset = a.chunk_add ? n_tile / 2 : 0;
        const int columns = a.chunk_add ? n_tile / 2 : n_tile;
        const int b = a.d2s_block;
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
            const int p_tile = t / a.n_tiles;
            const int n_index = t % a.n_tiles;
            const int ty = p_tile / a.tiles_x;
            const int y = ty * a.patch_h + row / a.patch_w;
            const int x = (p_tile - ty * a.tiles_x) * a.patch_w + row % a.patch_w;
            const bool real = y < a.out_h && x < a.out_w;
            const int p = real ? y * a.out_w + x : 0;
            const int physical0 = n_index * n_tile;
            const int logical0 = a.chunk_add ? n_index * (n_tile / 2) : physical0;
            const std::uint32_t acc = tmem + static_cast<std::uint32_t>(buffer) * buffer_columns + lane_base;

            // Per-channel parameters of one 16-column chunk, one coalesced load per
            // warp: lane l < 16 holds column j0 + l, lane 16 + l its chunk-add
            // partner j0 + pair_offset + l. Shuffled to every lane when used, and
            // fetched one chunk ahead.
            auto fetch = [&](int j0, float& scale, float& bias, long long& terms) {
                const int column = j0 + (lane < 16 ? lane : pair_offset + lane - 16);
                const int physical = physical0 + (column < n_tile ? column : 0);
                scale = __ldg(a.scales + physical);
                bias = __ldg(a.bias + physical);
                terms = AL == 2 ? __ldg(a.row_terms + physical) : 0;
            };
            float next_scale, next_bias;
            long long next_terms;
            fetch(0, next_scale, next_bias, next_terms);

            auto value_at = [&](int source_lane, int hh, int md, int lo, float scales, float biases,
                                long long terms) -> float {
                const float scale = __shfl_sync(0xffffffffu, scales, source_lane);
                const float bias = __shfl_sync(0xffffffffu, biases, source_lane);
                const long long row_term = AL == 2 ? __shfl_sync(0xffffffffu, terms, source_lane) : 0;
                float v;
                if constexpr (WL == 1 && AL == 1) {
                    v = integer_output32(hh, scale, exponent, bias);
                } else {
                    long long sum = high_factor * hh + column + mid_factor * md + row_term;
                    if constexpr (WL == 2 && AL == 2) sum += lo;
                    v = integer_output(sum, scale, exponent, bias);
                }
                if (a.wsilu) v = profile_wsilu(v, a.wsilu_scale);
                return v;
            };

            for (int j0 = 0; j0 < columns; j0 += 16) {
                const float scales = next_scale;
                const float biases = next_bias;
                const long long terms = next_terms;
                if (j0 + 16 < columns) fetch(j0 + 16, next_scale, next_bias, next_terms);
                int hh[16], md[16], lo[16], hh2[16], md2[16], lo2[16];
                tmem_load16(acc + static_cast<std::uint32_t>(j0), hh);
                if constexpr (L::accumulators > 1) tmem_load16(acc + static_cast<std::uint32_t>(n_tile + j0), md);
                if constexpr (L::accumulators > 2) tmem_load16(acc + static_cast<std::uint32_t>(2 * n_tile + j0), lo);
                if (a.chunk_add) {
                    const std::uint32_t second = static_cast<std::uint32_t>(j0 + pair_offset);
                    tmem_load16(acc + second, hh2);
                    if constexpr (L::accumulators > 1) tmem_load16(acc + static_cast<std::uint32_t>(n_tile) + second, md2);
                    if constexpr (L::accumulators > 2) {
                        tmem_load16(acc + static_cast<std::uint32_t>(2 * n_tile) + second, lo2);
                    }
                }
                tmem_load_wait();
                // Shuffles need the whole warp, so values are computed for every lane.
                float v[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    v[j] = value_at(j, hh[j], L::accumulators > 1 ? md[j] : 0, L::accumulators > 2 ? lo[j] : 0,
                                    scales, biases, terms);
                }
                if (a.chunk_add) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const float w = value_at(16 + j, hh2[j], L::accumulators > 1 ? md2[j] : 0,
                                                 L::accumulators > 2 ? lo2[j] : 0, scales, biases, terms);
                        v[j] = __fadd_rn(v[j], w);
                    }
                }
                const int c0 = logical0 + j0;
                const int count = a.out_channels - c0 < 16 ? a.out_channels - c0 : 16;
                if (real) {
                    if (exponent == INT_MIN) {
#pragma unroll
                        for (int j = 0; j < 16; ++j) v[j] = canonical_nan();
                    }
                    if (a.residual != nullptr) {
                        float r[16];
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            r[j] = j < count ? __ldg(a.residual + static_cast<std::size_t>(c0 + j) * a.positions + p) : 0.0f;
                        }
#pragma unroll
                        for (int j = 0; j < 16; ++j) v[j] = __fadd_rn(v[j], r[j]);
                    }
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        if (j >= count) break;
                        const int c = c0 + j;
                        std::size_t index;
                        if (b > 0) {
                            const int bb = b * b;
                            const int oc = c / bb;
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
                __syncwarp();  // tcgen05.ld is warp-aligned: reconverge before the next columns
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

template <int WL, int AL, bool SourceHalf>
cudaError_t launch_fused(const CUtensorMap& b_high, const CUtensorMap& b_low, const CUtensorMap& halo,
                         const FusedConvArgs& args, int sm_count, cudaStream_t stream) {
    using L = ConvLayout<WL, AL>;
    constexpr int max_dynamic = 232448;
    const int n_tile = args.n_tile;
    if (n_tile < 16 || n_tile > 256 || n_tile % 16 != 0 || (args.chunk_add && n_tile % 32 != 0) ||
        args.k_blocks < 1 || args.p_tiles < 1 || args.n_tiles < 1) {
        return cudaErrorInvalidValue;
    }
    int buffers = 2;
    std::uint32_t columns = 32;
    while (static_cast<int>(columns) < 2 * L::accumulators * n_tile) columns <<= 1;
    if (columns > 512) {
        buffers = 1;
        columns = 32;
        while (static_cast<int>(columns) < L::accumulators * n_tile) columns <<= 1;
        if (columns > 512) return cudaErrorInvalidValue;
    }
    if (args.a_stages < 1 || args.a_stages > max_stages || args.b_stages < 1 || args.b_stages > max_stages ||
        args.halo_bytes % 1024 != 0 || args.halo_bytes <= 0) {
        return cudaErrorInvalidValue;
    }
    const int smem = 1024 + args.a_stages * L::a_stage_bytes + args.b_stages * L::b_stage_bytes(n_tile) +
        halo_buffers * args.halo_bytes + static_cast<int>(sizeof(ConvTail));
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
    fused_conv_kernel<WL, AL, SourceHalf><<<grid, conv_threads, smem, stream>>>(b_high, b_low, halo, args, buffers,
                                                                                columns);
    return cudaGetLastError();
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

int fused_conv_shared_bytes(int weight_limbs, int activation_limbs, int n_tile, int a_stages, int b_stages,
                            int halo_bytes) {
    return 1024 + a_stages * activation_limbs * tile_positions_m * tile_k_bytes +
        b_stages * weight_limbs * n_tile * tile_k_bytes + halo_buffers * halo_bytes + static_cast<int>(sizeof(ConvTail));
}

cudaError_t encode_halo_map(CUtensorMap* map, const void* base, int half, std::uint64_t channels,
                            std::uint64_t height, std::uint64_t width, std::uint32_t box_w, std::uint32_t box_h,
                            std::uint32_t box_c) {
    const EncodeTiled encode = encoder();
    if (encode == nullptr) return cudaErrorNotSupported;
    const std::uint64_t element = half ? 2 : 4;
    if ((reinterpret_cast<std::uintptr_t>(base) & 15u) != 0 || (width * element) % 16 != 0 || box_w == 0 ||
        box_w > 256 || box_h == 0 || box_h > 256 || box_c == 0 || box_c > 256 || (box_w * element) % 16 != 0) {
        return cudaErrorInvalidValue;
    }
    const cuuint64_t dims[3] = {width, height, channels};
    const cuuint64_t strides[2] = {width * element, width * height * element};
    const cuuint32_t box[3] = {box_w, box_h, box_c};
    const cuuint32_t element_strides[3] = {1, 1, 1};
    const CUresult result = encode(map, half ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3,
                                   const_cast<void*>(base), dims, strides, box, element_strides,
                                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return result == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t pixel_max(const void* in, int source_half, int channels, int pixels, float* out, cudaStream_t stream) {
    if (pixels <= 0) return cudaSuccess;
    if (source_half) {
        pixel_max_kernel<true><<<(pixels + 31) / 32, 256, 0, stream>>>(in, channels, pixels, out);
    } else {
        pixel_max_kernel<false><<<(pixels + 31) / 32, 256, 0, stream>>>(in, channels, pixels, out);
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
