#pragma once

// Host-side launchers of the sm_100a kernels. Every launcher enqueues on the
// given stream and returns the launch status; tensors are batch-1 NCHW FP32 in
// device memory unless stated otherwise.

#include <cstddef>
#include <cstdint>

#include <cuda.h>
#include <cuda_runtime.h>

namespace nvcr_sm100::kernels {

// ---- stage boundary (FP16 <-> FP32) ----
cudaError_t half_to_float(const std::uint16_t* in, float* out, std::size_t count, cudaStream_t stream);
cudaError_t float_to_half(const float* in, std::uint16_t* out, std::size_t count, cudaStream_t stream);

// ---- elementwise FP32, one IEEE operation per element ----
enum class Binary { mul, add };
cudaError_t binary(Binary op, const float* a, const float* b, float* out, std::size_t count, cudaStream_t stream);
cudaError_t mul_scalar(const float* a, float scalar, float* out, std::size_t count, cudaStream_t stream);
cudaError_t sigmoid(const float* a, float* out, std::size_t count, cudaStream_t stream);
cudaError_t scale_channels(const float* a, const float* scale, float* out, std::size_t count,
                           std::size_t plane, cudaStream_t stream);
cudaError_t clamp(const float* a, float lo, float hi, float* out, std::size_t count, cudaStream_t stream);
// out[i] = in[i] + in[i + half] (slice(0, C) + slice(C, 2C) of one tensor)
cudaError_t chunk_add(const float* in, float* out, std::size_t half, cudaStream_t stream);

// ---- exact data movement ----
cudaError_t copy(const float* in, float* out, std::size_t count, cudaStream_t stream);
cudaError_t crop(const float* in, float* out, int channels, int out_h, int out_w, int in_h, int in_w,
                 cudaStream_t stream);
cudaError_t depth_to_space(const float* in, float* out, int out_channels, int out_h, int out_w, int in_h,
                           int in_w, int block, cudaStream_t stream);
cudaError_t space_to_depth(const float* in, float* out, int out_channels, int out_h, int out_w, int in_h,
                           int in_w, int block, cudaStream_t stream);
struct Window {
    int kernel_h, kernel_w, stride_y, stride_x, pad_top, pad_left;
};
cudaError_t im2col(const float* in, float* out, int out_channels, int out_h, int out_w, int in_h, int in_w,
                   Window window, cudaStream_t stream);

// ---- FP32 conv in the profile's fma order (bias, then channel, row, column) ----
struct ConvShape {
    int in_channels, out_channels, depthwise;
    int in_h, in_w, out_h, out_w;
    Window window;
};
cudaError_t conv_fp32(const float* weights, const float* bias, const float* in, float* out, ConvShape shape,
                      cudaStream_t stream);

// ---- integer conv: activation quantiser ----
// Positions are the output pixels of the (implicit) im2col window over `in`
// ([channels][in_h][in_w]); K = channels * kernel_h * kernel_w in im2col order.
struct QuantizeArgs {
    const float* in;
    int channels, in_h, in_w, out_h, out_w;
    Window window;
    int k_padded;            // row length of the limb matrices (multiple of 128)
    int positions_padded;    // rows of the limb matrices (multiple of 128)
    float* pixel_max;        // [in_h * in_w] scratch: max |x| over channels, +inf if non-finite
    std::int8_t* high;       // [positions_padded][k_padded] first limb (the value for 8 bits)
    std::int8_t* low;        // second limb l - 128 (16-bit activations), else unused
    int* exponents;          // [positions] activation exponent, INT_MIN if non-finite
    long long* column_terms; // [positions] exact correction for 2-limb weights, else unused
    int activation_bits;     // 8 or 16
    long long high_factor;   // correction: sum over k of (high_factor * h + low_factor * l')
    long long low_factor;
};
cudaError_t quantize_activations(const QuantizeArgs& args, cudaStream_t stream);

// ---- integer conv: tcgen05 GEMM with the profile's epilogue ----
struct GemmEpilogue {
    const float* scales;           // [n_padded] per physical weight row
    const float* bias;             // [n_padded]
    const long long* row_terms;    // [n_padded] exact correction for 2-limb activations
    const int* exponents;          // [positions]
    const long long* column_terms; // [positions] or null
    int wsilu;                     // apply v * sigmoid(k v)
    float wsilu_scale;
    int chunk_add;                 // physical tile columns j and j + n_tile/2 are one pair
    const float* residual;         // [out_channels][positions] added last, or null
    void* out;                     // [out_channels][positions] FP32, or FP16 when out_half
    int out_half;
    int out_channels;              // logical output channels (after chunk-add)
    int positions;
    unsigned int* status;          // device word; bit 0: a bounded wait gave up
};
struct GemmShape {
    int weight_limbs, activation_limbs;
    int n_tile;                  // output columns per CTA (multiple of 16, <= 256)
    int n_tiles;                 // CTAs along N
    int k_padded;                // multiple of 128
    int positions_padded;        // multiple of 128
};
struct GemmMaps {
    CUtensorMap a_high, a_low, b_high, b_low;  // unused limbs may be copies of the high maps
};
cudaError_t integer_gemm(const GemmMaps& maps, const GemmShape& shape, const GemmEpilogue& epilogue,
                         cudaStream_t stream);

// Encodes a 2D tensor map over an int8 [rows][row_bytes] matrix with 128x`box_rows`
// boxes and 128-byte swizzle, the layout the GEMM's shared-memory descriptors expect.
cudaError_t encode_int8_map(CUtensorMap* map, const void* base, std::uint64_t rows, std::uint64_t row_bytes,
                            std::uint32_t box_rows);

}  // namespace nvcr_sm100::kernels
