// Integer pointwise conv on sm_100a tensor cores (tcgen05, kind::i8).
//
// Orientation: the GEMM's M dimension is output positions (128 per CTA, one
// TMEM lane each) and N is output channels (n_tile per CTA, TMEM columns), so
// a thread of the epilogue owns one position: its activation exponent e_p is a
// register and the per-channel scale and bias come from shared memory. K is
// C * kh * kw in im2col order.
//
// 16-bit operands are split into signed int8 limbs q = 256 h + l' + 128
// (h = q >> 8, l' = (q & 255) - 128). With aw, ax = 256 for a two-limb operand
// and cw, cx = 128 its limb offset:
//   sum W X = aw ax sum(Wh Xh) + aw sum(Wh Xl') + ax sum(Wl' Xh) + sum(Wl' Xl')
//           + cx (aw sum Wh + sum Wl') + cw (ax sum Xh + sum Xl') + K cw cx
// The tensor cores produce the limb products (exact int32); the row term (per
// output channel, computed on the host) and the column term (per position,
// from the quantiser) are added in int64 in the epilogue. Integer sums are
// exact in any order, so tiling and tensor-core order cannot change a bit.
//
// Per CTA: warp 0 allocates TMEM and its lane 0 streams A (activation limbs,
// 128 x 128 B) and B (weight limbs, n_tile x 128 B) tiles by TMA into a ring of
// shared-memory stages (128-byte swizzle); warp 1 lane 0 issues the MMAs and
// returns each stage with tcgen05.commit; then all four warps read their 32
// TMEM lanes and run the profile's epilogue:
//   v = ((float(acc) * scale) * 2^e) + bias, [v = v * sigmoid(k v)],
//   [v = v + v_pair (chunk-add)], [v = v + residual], store FP32 or FP16.
// Every wait is bounded (about 2 s of the global timer); on a timeout the CTA
// sets bit 0 of the status word, stops issuing, drains what it issued, frees
// its TMEM and returns. No TMA multicast is used anywhere.

#include "exact_math.cuh"
#include "kernels.hpp"

#include <climits>

#include <cuda_fp16.h>

namespace nvcr_sm100::kernels {
namespace {

constexpr int block_m = 128;
constexpr int block_k = 128;  // bytes of K per stage (one 128-byte swizzle row)
constexpr int gemm_threads = 128;
constexpr unsigned long long wait_limit_ns = 2000000000ull;

__device__ __forceinline__ std::uint32_t smem_address(const void* p) {
    return static_cast<std::uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_timer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void barrier_init(std::uint32_t bar, std::uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void barrier_expect_bytes(std::uint32_t bar, std::uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool barrier_try_wait(std::uint32_t bar, std::uint32_t parity) {
    std::uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}

// Waits for the phase of `parity` to complete; false (and status bit 0) after
// about two seconds.
__device__ bool barrier_wait(std::uint32_t bar, std::uint32_t parity, unsigned int* status) {
    if (barrier_try_wait(bar, parity)) return true;
    const unsigned long long start = global_timer();
    for (unsigned int spin = 0;; ++spin) {
        if (barrier_try_wait(bar, parity)) return true;
        if ((spin & 63u) == 63u) {
            if (global_timer() - start > wait_limit_ns) {
                atomicOr(status, 1u);
                return false;
            }
            __nanosleep(128);
        }
    }
}

__device__ __forceinline__ void tma_load_2d(std::uint32_t dst, const CUtensorMap* map, std::uint32_t bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
        ::"r"(dst), "l"(reinterpret_cast<std::uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
        : "memory");
}

// Shared-memory matrix descriptor for a K-major tile with 128-byte swizzle:
// 8-row x 128-byte atoms stacked 1024 bytes apart (SBO), LBO unused (1),
// descriptor version 1 (bits 46-47), layout 2 = SWIZZLE_128B (bits 61-63).
__device__ __forceinline__ std::uint64_t sw128_descriptor(std::uint32_t address) {
    return static_cast<std::uint64_t>((address >> 4) & 0x3FFFu) | (static_cast<std::uint64_t>(1) << 16) |
        (static_cast<std::uint64_t>(1024 >> 4) << 32) | (static_cast<std::uint64_t>(1) << 46) |
        (static_cast<std::uint64_t>(2) << 61);
}

// Instruction descriptor, kind::i8: D s32 (bits 4-5 = 2), A and B signed 8-bit
// (bits 7-9 and 10-12 = 1), both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
__device__ __forceinline__ std::uint32_t i8_instruction(int n) {
    return (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<std::uint32_t>(n >> 3) << 17) |
        (static_cast<std::uint32_t>(block_m >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(std::uint32_t d_tmem, std::uint64_t a, std::uint64_t b, std::uint32_t idesc,
                                       std::uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mma_commit(std::uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

__device__ __forceinline__ void tmem_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 16 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_load16(std::uint32_t address, int (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(address));
}

__device__ __forceinline__ void tmem_load_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

template <int WL, int AL>
struct Layout {
    static constexpr int accumulators = 1 + ((WL == 2 || AL == 2) ? 1 : 0) + ((WL == 2 && AL == 2) ? 1 : 0);
    static constexpr int a_bytes = block_m * block_k;  // one limb
    static __host__ __device__ int b_bytes(int n_tile) { return n_tile * block_k; }
    static __host__ __device__ int stage_bytes(int n_tile) { return AL * a_bytes + WL * b_bytes(n_tile); }
};

struct SharedTail {
    unsigned long long full[8];
    unsigned long long empty[8];
    unsigned long long accumulated;
    std::uint32_t tmem_base;
    int abort;
};

template <int WL, int AL>
__global__ void __launch_bounds__(gemm_threads, 1)
integer_gemm_kernel(const __grid_constant__ CUtensorMap a_high, const __grid_constant__ CUtensorMap a_low,
                    const __grid_constant__ CUtensorMap b_high, const __grid_constant__ CUtensorMap b_low,
                    GemmShape shape, GemmEpilogue ep, int stages, std::uint32_t tmem_columns) {
    using L = Layout<WL, AL>;
    extern __shared__ std::uint8_t dynamic_smem[];
    // Swizzled tiles need 1024-byte alignment; the launch reserves the slack.
    const std::uint32_t raw = smem_address(dynamic_smem);
    std::uint8_t* smem = dynamic_smem + (((raw + 1023u) & ~1023u) - raw);
    const int n_tile = shape.n_tile;
    const int stage_bytes = L::stage_bytes(n_tile);
    SharedTail* tail = reinterpret_cast<SharedTail*>(smem + stages * stage_bytes);
    float* channel_scale = reinterpret_cast<float*>(tail + 1);
    float* channel_bias = channel_scale + n_tile;
    long long* channel_terms = reinterpret_cast<long long*>(channel_bias + n_tile + (n_tile & 1));

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * n_tile;    // physical weight row
    const int p0 = blockIdx.y * block_m;   // first position
    const int k_blocks = shape.k_padded / block_k;

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_address(&tail->tmem_base)), "r"(tmem_columns)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (warp == 1 && lane == 0) {
        for (int s = 0; s < stages; ++s) {
            barrier_init(smem_address(&tail->full[s]), 1);
            barrier_init(smem_address(&tail->empty[s]), 1);
        }
        barrier_init(smem_address(&tail->accumulated), 1);
        tail->abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    for (int j = threadIdx.x; j < n_tile; j += gemm_threads) {
        channel_scale[j] = ep.scales[n0 + j];
        channel_bias[j] = ep.bias[n0 + j];
        channel_terms[j] = ep.row_terms != nullptr ? ep.row_terms[n0 + j] : 0;
    }
    tmem_fence_before();
    __syncthreads();
    tmem_fence_after();
    const std::uint32_t tmem = tail->tmem_base;

    const std::uint32_t a_high_base = smem_address(smem);
    auto stage_base = [&](int s) { return a_high_base + static_cast<std::uint32_t>(s * stage_bytes); };

    if (warp == 0 && lane == 0) {
        // TMA producer.
        const std::uint32_t bytes = static_cast<std::uint32_t>(stage_bytes);
        int issued = 0;
        for (int kb = 0; kb < k_blocks; ++kb) {
            const int s = kb % stages;
            const std::uint32_t phase = static_cast<std::uint32_t>((kb / stages) & 1);
            if (!barrier_wait(smem_address(&tail->empty[s]), phase ^ 1u, ep.status)) {
                tail->abort = 1;
                break;
            }
            const std::uint32_t full = smem_address(&tail->full[s]);
            barrier_expect_bytes(full, bytes);
            const std::uint32_t base = stage_base(s);
            const int x = kb * block_k;
            tma_load_2d(base, &a_high, full, x, p0);
            if constexpr (AL == 2) tma_load_2d(base + L::a_bytes, &a_low, full, x, p0);
            const std::uint32_t b_base = base + AL * L::a_bytes;
            tma_load_2d(b_base, &b_high, full, x, n0);
            if constexpr (WL == 2) tma_load_2d(b_base + L::b_bytes(n_tile), &b_low, full, x, n0);
            issued = kb + 1;
        }
        if (*reinterpret_cast<volatile int*>(&tail->abort) != 0) {
            // Drain: every issued load must land before the CTA may exit.
            const int first = issued > stages ? issued - stages : 0;
            for (int kb = first; kb < issued; ++kb) {
                barrier_wait(smem_address(&tail->full[kb % stages]),
                             static_cast<std::uint32_t>((kb / stages) & 1), ep.status);
            }
        }
    } else if (warp == 1 && lane == 0) {
        // MMA issuer.
        const std::uint32_t idesc = i8_instruction(n_tile);
        const std::uint32_t mid = tmem + static_cast<std::uint32_t>(n_tile);
        const std::uint32_t low = tmem + static_cast<std::uint32_t>(2 * n_tile);
        for (int kb = 0; kb < k_blocks; ++kb) {
            const int s = kb % stages;
            const std::uint32_t phase = static_cast<std::uint32_t>((kb / stages) & 1);
            if (!barrier_wait(smem_address(&tail->full[s]), phase, ep.status)) {
                tail->abort = 1;
                break;
            }
            tmem_fence_after();
            const std::uint32_t base = stage_base(s);
            const std::uint32_t a_hi = base;
            const std::uint32_t a_lo = base + L::a_bytes;
            const std::uint32_t b_hi = base + AL * L::a_bytes;
            const std::uint32_t b_lo = b_hi + static_cast<std::uint32_t>(L::b_bytes(n_tile));
#pragma unroll
            for (int kk = 0; kk < block_k / 32; ++kk) {
                const std::uint32_t step = static_cast<std::uint32_t>(kk * 32);
                const std::uint32_t first = (kb == 0 && kk == 0) ? 0u : 1u;
                mma_i8(tmem, sw128_descriptor(a_hi + step), sw128_descriptor(b_hi + step), idesc, first);
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
            mma_commit(smem_address(&tail->empty[s]));
        }
        // Arrives once every MMA issued above has completed.
        mma_commit(smem_address(&tail->accumulated));
    }
    __syncwarp();

    // Epilogue: thread <-> TMEM lane <-> position.
    const bool accumulated = barrier_wait(smem_address(&tail->accumulated), 0u, ep.status);
    tmem_fence_after();
    const int quarter = warp & 3;
    const int p = p0 + quarter * 32 + lane;
    const bool real = p < ep.positions;
    const int exponent = real ? ep.exponents[p] : INT_MIN;
    const long long column = (real && ep.column_terms != nullptr) ? ep.column_terms[p] : 0;
    const std::uint32_t lane_base = tmem + (static_cast<std::uint32_t>(quarter * 32) << 16);
    const bool store = accumulated && *reinterpret_cast<volatile int*>(&tail->abort) == 0 && real;
    constexpr long long high_factor = (WL == 2 ? 256LL : 1LL) * (AL == 2 ? 256LL : 1LL);
    constexpr long long mid_factor = (WL == 2 && AL == 2) ? 256LL : 1LL;
    const int pair_offset = ep.chunk_add ? n_tile / 2 : 0;
    const int columns = ep.chunk_add ? n_tile / 2 : n_tile;
    const int logical0 = ep.chunk_add ? blockIdx.x * (n_tile / 2) : n0;

    auto value_at = [&](int j, int hh, int md, int lo) -> float {
        float v;
        if constexpr (WL == 1 && AL == 1) {
            v = integer_output32(hh, channel_scale[j], exponent, channel_bias[j]);
        } else {
            long long acc = high_factor * hh + channel_terms[j] + column;
            acc += mid_factor * md;
            if constexpr (WL == 2 && AL == 2) acc += lo;
            v = integer_output(acc, channel_scale[j], exponent, channel_bias[j]);
        }
        if (ep.wsilu) v = profile_wsilu(v, ep.wsilu_scale);
        return v;
    };

    for (int j0 = 0; j0 < columns; j0 += 16) {
        int hh[16], md[16], lo[16], hh2[16], md2[16], lo2[16];
        tmem_load16(lane_base + static_cast<std::uint32_t>(j0), hh);
        if constexpr (L::accumulators > 1) tmem_load16(lane_base + static_cast<std::uint32_t>(n_tile + j0), md);
        if constexpr (L::accumulators > 2) tmem_load16(lane_base + static_cast<std::uint32_t>(2 * n_tile + j0), lo);
        if (ep.chunk_add) {
            const std::uint32_t second = static_cast<std::uint32_t>(j0 + pair_offset);
            tmem_load16(lane_base + second, hh2);
            if constexpr (L::accumulators > 1) tmem_load16(lane_base + static_cast<std::uint32_t>(n_tile) + second, md2);
            if constexpr (L::accumulators > 2) tmem_load16(lane_base + static_cast<std::uint32_t>(2 * n_tile) + second, lo2);
        }
        tmem_load_wait();
        if (store) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const int c = logical0 + j0 + j;
            if (c >= ep.out_channels) break;
            float v;
            if (exponent == INT_MIN) {
                v = canonical_nan();
            } else {
                v = value_at(j0 + j, hh[j], L::accumulators > 1 ? md[j] : 0, L::accumulators > 2 ? lo[j] : 0);
                if (ep.chunk_add) {
                    const float w = value_at(j0 + pair_offset + j, hh2[j], L::accumulators > 1 ? md2[j] : 0,
                                             L::accumulators > 2 ? lo2[j] : 0);
                    v = __fadd_rn(v, w);
                }
            }
            const std::size_t index = static_cast<std::size_t>(c) * ep.positions + p;
            if (ep.residual != nullptr) v = __fadd_rn(v, ep.residual[index]);
            if (ep.out_half) {
                reinterpret_cast<__half*>(ep.out)[index] = __float2half_rn(v);
            } else {
                reinterpret_cast<float*>(ep.out)[index] = v;
            }
        }
        }
        __syncwarp();  // tcgen05.ld is warp-aligned: reconverge before the next columns
    }

    tmem_fence_before();
    __syncthreads();
    if (warp == 0) {
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

template <int WL, int AL>
cudaError_t launch_gemm(const GemmMaps& maps, const GemmShape& shape, const GemmEpilogue& ep, cudaStream_t stream) {
    using L = Layout<WL, AL>;
    constexpr int max_dynamic = 232448;  // 227 KiB per CTA on sm_100
    const int n_tile = shape.n_tile;
    if (n_tile < 16 || n_tile > 256 || n_tile % 16 != 0 || shape.k_padded % block_k != 0 ||
        shape.positions_padded % block_m != 0 || shape.n_tiles < 1 || (ep.chunk_add && n_tile % 32 != 0)) {
        return cudaErrorInvalidValue;
    }
    const int needed_columns = L::accumulators * n_tile;
    std::uint32_t columns = 32;
    while (static_cast<int>(columns) < needed_columns) columns <<= 1;
    if (columns > 512) return cudaErrorInvalidValue;
    const int stage_bytes = L::stage_bytes(n_tile);
    const int fixed = 1024 + static_cast<int>(sizeof(SharedTail)) + n_tile * 16 + 16;
    int stages = (max_dynamic - fixed) / stage_bytes;
    if (stages > 6) stages = 6;
    if (stages < 2) return cudaErrorInvalidValue;
    int smem = fixed + stages * stage_bytes;
    // Two resident CTAs must not need more than the SM's 512 TMEM columns.
    if (columns > 256 && smem < 120 * 1024) smem = 120 * 1024;
    static int configured = 0;
    if (smem > configured) {
        const cudaError_t set = cudaFuncSetAttribute(integer_gemm_kernel<WL, AL>,
                                                     cudaFuncAttributeMaxDynamicSharedMemorySize, max_dynamic);
        if (set != cudaSuccess) return set;
        configured = max_dynamic;
    }
    const dim3 grid(static_cast<unsigned int>(shape.n_tiles), static_cast<unsigned int>(shape.positions_padded / block_m));
    if (grid.y > 65535u) return cudaErrorInvalidValue;
    integer_gemm_kernel<WL, AL><<<grid, gemm_threads, smem, stream>>>(maps.a_high, maps.a_low, maps.b_high,
                                                                      maps.b_low, shape, ep, stages, columns);
    return cudaGetLastError();
}

}  // namespace

cudaError_t encode_int8_map(CUtensorMap* map, const void* base, std::uint64_t rows, std::uint64_t row_bytes,
                            std::uint32_t box_rows) {
    const EncodeTiled encode = encoder();
    if (encode == nullptr) return cudaErrorNotSupported;
    if ((reinterpret_cast<std::uintptr_t>(base) & 15u) != 0 || row_bytes % block_k != 0 || box_rows == 0 ||
        box_rows > 256) {
        return cudaErrorInvalidValue;
    }
    const cuuint64_t dims[2] = {row_bytes, rows};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(block_k), box_rows};
    const cuuint32_t element_strides[2] = {1, 1};
    const CUresult result = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
                                   element_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return result == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t integer_gemm(const GemmMaps& maps, const GemmShape& shape, const GemmEpilogue& ep, cudaStream_t stream) {
    if (shape.weight_limbs == 1 && shape.activation_limbs == 1) return launch_gemm<1, 1>(maps, shape, ep, stream);
    if (shape.weight_limbs == 2 && shape.activation_limbs == 1) return launch_gemm<2, 1>(maps, shape, ep, stream);
    if (shape.weight_limbs == 1 && shape.activation_limbs == 2) return launch_gemm<1, 2>(maps, shape, ep, stream);
    if (shape.weight_limbs == 2 && shape.activation_limbs == 2) return launch_gemm<2, 2>(maps, shape, ep, stream);
    return cudaErrorInvalidValue;
}

}  // namespace nvcr_sm100::kernels
