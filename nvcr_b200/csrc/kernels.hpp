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
// Zeroes `count` floats once the kernels before it in the stream are done
// (launched overlapped, so the chain of early-starting kernels is not broken).
cudaError_t zero_floats(float* out, std::size_t count, cudaStream_t stream);
// Depthwise 3x3 s1 p1 on channel-innermost FP32 tensors [H][W][c_pad] (c_pad
// 128 or 256, padding channels zero), with each pixel's max |x| (+inf when a
// value is non-finite): the layout and maxima an integer conv reads.
cudaError_t depthwise3x3_staged(const float* weights, const float* bias, int channels, int c_pad, const float* in,
                                float* out, float* pixel_max, int height, int width, cudaStream_t stream);

// ---- integer conv: fused quantise-on-load implicit GEMM (persistent, tcgen05) ----
// The conv reads its source from a channel-innermost copy [in_h][in_w][c_pad]
// (FP16 or FP32, channels c_pad > channels zero) made by stage_source(), which
// also writes the per-pixel maxima. K is channel-group-major over the padded
// channels: k = g * (taps * group) + tap * group + c, K = taps * c_pad; the
// weight matrices must use the same order.
struct FusedConvArgs {
    int source_half;               // staged copy is FP16 (else FP32)
    const float* pixel_max;        // [in_h][in_w] from stage_source()
    int channels, c_pad, in_h, in_w, out_h, out_w;
    Window window;
    int k_real, k_blocks;          // K = taps * c_pad, blocks of 128 bytes
    int positions, p_tiles;        // out_h * out_w; p_tiles = tiles_y * tiles_x
    int patch_h, patch_w;          // a tile is a patch_h x patch_w block of output pixels (product 128)
    int tiles_y, tiles_x;
    int group, groups;             // channels per halo load (divides c_pad), halo loads per tile
    int record_bytes;              // group * element bytes: 16, 32, 64 or 128 (the halo swizzle span)
    int halo_rows, halo_box_w;     // halo box: halo_rows x halo_box_w pixels of `group` channels
    int halo_bytes;                // bytes per halo buffer (multiple of 1024)
    int halo_buffers;              // halo ring depth, 2..8
    int producer_sets;             // 1: eight epilogue + four producer warps; 2: four + eight (alternate tiles)
    int a_stages, b_stages;        // shared-memory ring depths for activations and weights
    int b_resident;                // weights stay in shared memory: one N tile, b_stages == k_blocks
    int n_tile, n_tiles;
    long long column_high_factor, column_low_factor;  // column term (two-limb weights), else 0
    const float* scales;           // [n_tiles * n_tile] per physical weight row (16-byte aligned)
    const float* bias;             // (16-byte aligned)
    const long long* row_terms;    // two-limb activations, else null
    int wsilu;
    float wsilu_scale;
    int chunk_add;
    const float* residual;         // [out_channels][positions] FP32, or null
    int residual_c_pad;            // 0: residual as above; else [positions][residual_c_pad] FP32
    void* out;                     // FP32, or FP16 when out_half
    int out_half;
    // Staged output: out is [positions][out_c_pad] FP32 (the layout an integer
    // conv reads its source in, padding channels zero) and out_max gets each
    // position's max |x| (+inf when a value is non-finite) by atomic max into a
    // zeroed buffer. Null for the NCHW store.
    float* out_max;
    int out_c_pad;
    int out_channels;              // logical channels stored (after chunk-add)
    int d2s_block;                 // 0: NCHW store; b: store through depth_to_space(b)
    unsigned int* status;
    // When not null, the kernel runs only if *gate is non-zero (read once the
    // kernels before it are done): the fallback of a direct conv.
    const unsigned int* gate;
};
// Channel-innermost copy of a [channels][pixels] FP16 or FP32 tensor with
// c_pad >= channels channels per pixel (c_pad a multiple of 16, the extra
// channels zero), and per pixel max |x| over the channels (+inf when any
// channel is non-finite).
cudaError_t stage_source(const void* in, int source_half, int channels, int c_pad, int pixels, void* out,
                         float* pixel_max, cudaStream_t stream, const unsigned int* gate = nullptr);
// For convs with few input channels: per output position its whole receptive
// field, [out_h][out_w][c_pad] with k = c * taps + tap (padding taps and k past
// channels * taps zero), in the source's type, and the max |x| over the field
// (+inf when a value is non-finite). The conv then runs as a 1x1 conv on it.
cudaError_t stage_receptive_fields(const void* in, int source_half, int channels, int in_h, int in_w,
                                   Window window, int out_h, int out_w, int c_pad, void* out, float* field_max,
                                   cudaStream_t stream);
cudaError_t fused_conv(const CUtensorMap& b_high, const CUtensorMap& b_low, const CUtensorMap& halo, int weight_limbs,
                       int activation_limbs, const FusedConvArgs& args, cudaStream_t stream);
// Dynamic shared memory the fused conv needs for these ring depths and halo
// buffers, with the per-column parameters of all n_tiles * n_tile columns.
int fused_conv_shared_bytes(int weight_limbs, int activation_limbs, int n_tile, int n_tiles, int a_stages,
                            int b_stages, int halo_region);
constexpr int fused_conv_max_shared = 232448;
// Encodes the 3-D halo map over a staged [height][width][c_pad] tensor with a
// box of box_h x box_w pixels x `group` channels, zero fill outside the tensor,
// and the shared-memory swizzle whose span is group * element bytes (none for 16).
cudaError_t encode_halo_map(CUtensorMap* map, const void* base, int half, std::uint64_t c_pad, std::uint64_t height,
                            std::uint64_t width, std::uint32_t group, std::uint32_t box_w, std::uint32_t box_h);

// Encodes a 2D tensor map over an int8 [rows][row_bytes] matrix with 128x`box_rows`
// boxes and 128-byte swizzle, the layout the MMA's shared-memory descriptors expect.
cudaError_t encode_int8_map(CUtensorMap* map, const void* base, std::uint64_t rows, std::uint64_t row_bytes,
                            std::uint32_t box_rows);

// ---- integer conv on pre-quantised activations (w8a8; persistent, tcgen05) ----
// When every window of a conv takes its activation exponent from pixels that
// share one exponent, the profile's per-position quantisation of the window
// equals each pixel quantised with its own exponent. A prepass writes that
// per-pixel int8 copy, channel-innermost [pixels][c8] (c8 = channels rounded up
// to 32, padding zero), with each pixel's max |x|; the conv then loads its A
// operand by TMA straight from it, one (tap, channel block) box of 128 output
// positions at a time, and checks every window: a window whose non-zero pixels
// have different exponents sets *fallback, and the quantise-on-load path is
// then run for the whole conv (it gates on the same word and otherwise returns
// at once). A 1x1 conv, or a conv over staged receptive fields, has one pixel
// per window and never falls back.
struct DirectConvArgs {
    const float* pixel_max;        // [in_h][in_w] per-pixel max |x| (+inf when non-finite)
    int in_h, in_w, out_h, out_w;
    Window window;                 // stride 1 (any window up to 3x3), or 1x1
    int k_block;                   // K bytes per stage: 32, 64 or 128 (the A and B swizzle span)
    int c_blocks;                  // K blocks per tap: c8 / k_block
    int k_blocks;                  // taps * c_blocks
    int group;                     // K blocks per pipeline stage (1-4, dividing k_blocks; resident weights stay
                                   // one block per stage)
    int m_tiles;                   // patches of 128 positions per tile sharing each B block (1 or 2): two
                                   // accumulators of n_tile columns; plain or depth_to_space stores only
    int positions, p_tiles;        // out_h * out_w; tiles_y * tiles_x
    int patch_h, patch_w, tiles_y, tiles_x;
    int a_stages, b_stages;
    int b_resident;                // one N tile whose K blocks all stay in shared memory
    int n_tile, n_tiles;
    const float* scales;           // [n_tiles * n_tile] per physical weight row (16-byte aligned)
    const float* bias;             // (16-byte aligned)
    int wsilu;
    float wsilu_scale;
    int chunk_add;
    const float* residual;         // as FusedConvArgs
    int residual_c_pad;
    void* out;
    int out_half;
    float* out_max;
    int out_c_pad;
    int out_channels;
    int d2s_block;
    // 1 when the plain FP16 output may be written as 16-byte runs of 8 positions
    // of one channel: no fusions, no depth_to_space, patch_w, out_w and
    // out_channels multiples of 8, `out` 16-byte aligned, finite scales and biases.
    int vector_store;
    // 1 when every accumulator is below 2^22 in magnitude (127 * the largest
    // row sum of |weights|), so it converts to float exactly by integer addition.
    int small_accumulators;
    // Window exponents for which the vector stores fuse the power-of-two scale
    // and the bias add into one multiply-add (exact there); others take the
    // per-channel stores.
    int fma_lo, fma_hi;
    // 1: patches of one output row (patch_h 1), each A stage one halo row of
    // patch_w + kernel_w - 1 pixels of one channel block (a_row_bytes apart per
    // patch, direct_row_bytes) serving the window row's kernel_w K blocks; group
    // = kernel_w and B stages hold one K block each.
    int row_halo;
    int a_row_bytes;
    unsigned int* fallback;        // multi-tap windows: set to 1 when a window mixes exponents; else null
    unsigned int* status;
    // When not zero, a conditional-node handle of the graph this launch belongs
    // to: set to 1 (cudaGraphSetConditional) when a window mixes exponents.
    unsigned long long condition;
};
// Source forms of quantise_pixels: NCHW FP32 or FP16 planes, or a staged FP32
// tensor [pixels][c_pad] whose per-pixel maxima are already known.
enum class PixelSource { planes_f32, planes_f16, staged_f32 };
// Per-pixel int8 quantisation into [pixels][c8] (c8 a multiple of 32, >= channels)
// with each pixel's max |x| written to pixel_max (read from it for staged_f32);
// clears *clear_word (when not null) for the conv that follows.
cudaError_t quantise_pixels(const void* in, PixelSource form, int channels, int c_pad_in, int c8, int pixels,
                            std::int8_t* out, float* pixel_max, unsigned int* clear_word, cudaStream_t stream);
// The receptive field of each output position (k = c * taps + tap, padding
// taps zero) quantised with the field's own exponent into [out_h][out_w][c8],
// and the field's max |x|.
cudaError_t quantise_fields(const void* in, int source_half, int channels, int in_h, int in_w, Window window,
                            int out_h, int out_w, int c8, std::int8_t* out, float* field_max, cudaStream_t stream);
// Tensor maps: the int8 activations [height][width][c8] with a box of k_block
// bytes x box_w x box_h pixels, and the int8 weights [rows][row_bytes] with a
// box of k_block bytes x box_rows rows; both with the swizzle of span k_block.
cudaError_t encode_activation_map(CUtensorMap* map, const void* base, std::uint64_t c8, std::uint64_t height,
                                  std::uint64_t width, std::uint32_t k_block, std::uint32_t box_w, std::uint32_t box_h);
cudaError_t encode_weight_map(CUtensorMap* map, const void* base, std::uint64_t rows, std::uint64_t row_bytes,
                              std::uint32_t k_block, std::uint32_t box_rows);
cudaError_t direct_conv(const CUtensorMap& a_map, const CUtensorMap& b_map, const DirectConvArgs& args,
                        cudaStream_t stream);
int direct_conv_shared_bytes(int k_block, int n_tile, int n_tiles, int a_stages, int b_stages, int group,
                             bool b_resident, int m_tiles);
// Row halos: the bytes of one patch's A box ((patch_w + kernel_w - 1) pixels x
// k_block bytes, rounded up to 1 KiB) and the shared memory of that layout.
int direct_row_bytes(int patch_w, int kernel_w, int k_block);
int direct_conv_row_shared_bytes(int k_block, int n_tile, int n_tiles, int a_stages, int b_stages, bool b_resident,
                                 int m_tiles, int row_bytes);
constexpr int direct_conv_max_shared = 232448;

// Diagnostics: one thread waits on an mbarrier that nothing arrives on, with the
// kernels' bounded-wait loop and a limit of `limit_ns`, then sets bit 0 of
// `status` and returns (the path every kernel takes when a wait runs out).
cudaError_t wait_timeout(unsigned long long limit_ns, unsigned int* status, cudaStream_t stream);

// Diagnostics: adds to *mismatches (device memory) the count of floats d with
// bit patterns first .. first + count - 1 (within [1, 2^126)) whose sigmoid
// reciprocal differs from the IEEE division 1 / d.
cudaError_t check_reciprocal(std::uint32_t first, std::uint32_t count, unsigned long long* mismatches,
                             cudaStream_t stream);

}  // namespace nvcr_sm100::kernels
