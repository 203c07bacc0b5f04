#pragma once

// Launchers of the nvcr.fx.v1 kernels (k_fx.cu). Tensors are batch-1 NCHW
// int32 in device memory; every sum is taken in int64, which the profile's
// load-time bounds make exact. Each launcher enqueues on `stream` and returns
// the launch status.
//
// Stage failures are not returned: a kernel that meets one records it in the
// run's failure word with atomicMin of
//     node_key | (loop position << 1) | rule
// where node_key = (node index + 1) << 47 (0 for the input checks), the loop
// position is the output's index in the reference's loop order
// (src/deterministic/fx.cpp) and rule is 1 for a stored-bound failure after a
// gemm's pre-activation failure at the same position. The smallest key is the
// failure the reference meets first. Values written after a failure are
// unspecified, but every index a kernel forms stays in bounds whatever the
// values are (table lookups and param_row check their range first).

#include <cstddef>
#include <cstdint>

#include <cuda_runtime.h>

namespace nvcr_sm100::fx::kernels {

inline constexpr int node_shift = 47;
inline constexpr unsigned long long no_failure = ~0ull;

struct Table {
    const std::int16_t* dc{nullptr};  // null: no table activation
    std::int64_t h{0};
    int shift{0};
};

struct GemmArgs {
    const std::int32_t* x{nullptr};  // [in_channels][pixels]
    std::size_t pixels{0};
    int in_channels{0};
    int group{1};   // 1, 2 or 4 adjacent rows summed
    int groups{0};  // out_channels / group
    int input_shift{0};
    const std::int16_t* weights{nullptr};  // [out][in]
    const std::int64_t* bias{nullptr};
    const std::int32_t* shifts{nullptr};
    Table table;
    const std::int32_t* residual0{nullptr};  // [groups][pixels] or null
    const std::int32_t* residual1{nullptr};
    std::int32_t* y{nullptr};  // [groups][pixels]
};

cudaError_t check_input(const std::int32_t* x, std::size_t count, unsigned long long position_base,
                        unsigned long long* failure, cudaStream_t stream);
cudaError_t gemm(const GemmArgs& args, unsigned long long node_key, unsigned long long* failure, cudaStream_t stream);
cudaError_t depthwise3x3(const std::int32_t* x, int channels, int height, int width, const std::int32_t* weights,
                         const std::int64_t* bias, const std::int32_t* shifts, std::int32_t* y,
                         unsigned long long node_key, unsigned long long* failure, cudaStream_t stream);
cudaError_t mul(const std::int32_t* a, int channels, std::size_t plane, const std::int32_t* b, int b_channels,
                std::size_t b_plane, int shift, std::int32_t* y, unsigned long long node_key,
                unsigned long long* failure, cudaStream_t stream);
cudaError_t affine(const std::int32_t* x, std::size_t count, std::int64_t alpha, std::int64_t beta, int shift,
                   std::int32_t* y, unsigned long long node_key, unsigned long long* failure, cudaStream_t stream);
cudaError_t add(const std::int32_t* a, const std::int32_t* b, std::size_t count, std::int32_t* y,
                unsigned long long node_key, unsigned long long* failure, cudaStream_t stream);
cudaError_t sat_table(const std::int32_t* x, std::size_t count, const std::int32_t* table, std::int64_t n,
                      std::int32_t top, std::int32_t* y, cudaStream_t stream);
cudaError_t delta(const std::int32_t* x, std::size_t count, Table table, std::int32_t* y, cudaStream_t stream);
cudaError_t clamp(const std::int32_t* x, std::size_t count, std::int32_t lo, std::int32_t hi, std::int32_t* y,
                  cudaStream_t stream);
// pixel_shuffle (up) / pixel_unshuffle, PyTorch's channel order; extents are the input's.
cudaError_t shuffle(const std::int32_t* x, int channels, int height, int width, int factor, bool up, std::int32_t* y,
                    cudaStream_t stream);
// Channels (c, i, j) of the k x k taps, zero outside; 3x3 pads 1, 2x2 pads 0.
cudaError_t im2col(const std::int32_t* x, int channels, int height, int width, int kernel, int stride, int out_h,
                   int out_w, std::int32_t* y, cudaStream_t stream);
cudaError_t crop(const std::int32_t* x, int channels, int height, int width, int out_h, int out_w, std::int32_t* y,
                 cudaStream_t stream);
// y[c] = rows[q * channels + c] for the one value q of x; q outside [0, row_count) is a failure.
cudaError_t param_row(const std::int32_t* x, const std::int64_t* rows, int row_count, int channels, std::int32_t* y,
                      unsigned long long node_key, unsigned long long* failure, cudaStream_t stream);

}  // namespace nvcr_sm100::fx::kernels
