/*
 * nvcr_sm100: C ABI of the Blackwell (sm_100a) executor for the
 * nvcr.intconv.v1 exact-convolution profile.
 *
 * This is the shim a new execution provider calls (one process, one GPU, one
 * executor per stream). It replaces the reference's CUDA executor behind the
 * provider boundary:
 *   reference src/deterministic/cuda_executor.hpp:26-53   (CudaExecutor)
 *   reference src/deterministic/normative_stage.hpp:28-65 (normative helpers)
 *   reference src/provider/tensorrt/session.cpp:1464-1467,1526-1594 (exact stages)
 * Every output is bit-identical to the reference's CPU executor run_cpu
 * (src/deterministic/program.cpp:702-820); NaN payloads are unspecified.
 * The nvcr_sm100_fx_* functions at the end load and run programs of the other
 * profile, nvcr.fx.v1 (reference src/deterministic/fx_program.hpp:70-79).
 *
 * Plain C types only. Every function returns NVCR_SM100_OK (0) or
 * 1 + the reference's nvcr::ErrorCode value (include/nvcr/common/error.hpp:11-34),
 * and leaves a message for nvcr_sm100_last_error() on the calling thread. No
 * exception crosses the ABI.
 */
#ifndef NVCR_SM100_H
#define NVCR_SM100_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NVCR_SM100_ABI_VERSION 1

/* Status codes: 0, or 1 + nvcr::ErrorCode. */
#define NVCR_SM100_OK 0
#define NVCR_SM100_INVALID_ARGUMENT 1
#define NVCR_SM100_INVALID_STATE 2
#define NVCR_SM100_IO_ERROR 3
#define NVCR_SM100_MALFORMED_BITSTREAM 4
#define NVCR_SM100_RESOURCE_EXHAUSTED 5
#define NVCR_SM100_BACKEND_ERROR 7
#define NVCR_SM100_NOT_IMPLEMENTED 8
#define NVCR_SM100_INTERNAL_ERROR 9
#define NVCR_SM100_MISSING_ARTIFACT 12
#define NVCR_SM100_INCOMPATIBLE_TARGET 16
#define NVCR_SM100_INCOMPATIBLE_PRECISION 17
#define NVCR_SM100_DIGEST_MISMATCH 19

typedef struct nvcr_sm100_executor nvcr_sm100_executor;
typedef struct nvcr_sm100_program nvcr_sm100_program;

/* A named batch-1 NCHW tensor. `data` is device FP16 for run_half, device
 * FP32 for run_float and host FP32 for run_host (reference HalfDeviceTensor,
 * cuda_executor.hpp:19-24, and Tensor, program.hpp:116-127). */
typedef struct nvcr_sm100_tensor {
    const char* name;
    int32_t channels;
    int32_t height;
    int32_t width;
    void* data;
} nvcr_sm100_tensor;

/* One timed step of a profiled run (see nvcr_sm100_set_profiling). */
typedef struct nvcr_sm100_step_time {
    char label[96];
    char kernel[32];
    double milliseconds;
    double algorithmic_ops;   /* 2 * C_in * kh * kw * C_out * P for integer convs */
    double algorithmic_bytes; /* each input read once and the output written once */
} nvcr_sm100_step_time;

int nvcr_sm100_abi_version(void);

/* Message of the last failed call on this thread; returns its full length. */
size_t nvcr_sm100_last_error(char* buffer, size_t size);

/* 1 when `profile` is nvcr.intconv.v1 and the current device is sm_100, else 0
 * (reference IProviderSession::supports_numerics_profile,
 * include/nvcr/provider/experimental/session.hpp:147-150, as the TensorRT
 * provider answers it at src/provider/tensorrt/session.cpp:1464-1467). */
int nvcr_sm100_supports_profile(const char* profile);

/* Reference is_normative (normative_stage.hpp:28-31): *normative = 0 for an
 * empty profile (a native stage), 1 for nvcr.intconv.v1; any other profile is
 * NVCR_SM100_INCOMPATIBLE_PRECISION. */
int nvcr_sm100_is_normative(const char* profile, int* normative);

/* A loaded program without a device (reference Program, program.hpp:105-115,
 * from load_program, program.cpp:537-626): for output sizing and validation
 * on hosts that have not created an executor yet. No GPU is needed. */
int nvcr_sm100_program_load(const char* program_json_path, nvcr_sm100_program** program);
int nvcr_sm100_program_load_memory(const char* program_json, size_t json_size, const float* weights,
                                   size_t weight_count, nvcr_sm100_program** program);
void nvcr_sm100_program_destroy(nvcr_sm100_program* program);
int nvcr_sm100_program_tensor_count(const nvcr_sm100_program* program, int is_output, size_t* count);
int nvcr_sm100_program_tensor_info(const nvcr_sm100_program* program, int is_output, size_t index,
                                   const char** name, int32_t* channels);
/* Reference infer_output_extents (normative_stage.cpp:42-65) on a program handle. */
int nvcr_sm100_program_infer_output_extents(const nvcr_sm100_program* program, const nvcr_sm100_tensor* inputs,
                                            size_t input_count, nvcr_sm100_tensor* outputs, size_t output_count);
/* An executor over a copy of a loaded program (CudaExecutor::create). */
int nvcr_sm100_executor_create_from_program(const nvcr_sm100_program* program, void* stream,
                                            nvcr_sm100_executor** executor);

/* Reference load_program + CudaExecutor::create (program.cpp:537-626,
 * cuda_executor.cu:1279-1313): loads <path> (.detprog.json) and the .detw it
 * names, checks the weight digest, uploads and quantises the weights on the
 * current device. `stream` is a cudaStream_t, or NULL for an executor-owned
 * non-blocking stream; with a stream, all work is ordered on it. */
int nvcr_sm100_executor_create(const char* program_json_path, void* stream, nvcr_sm100_executor** executor);

/* The same from JSON text with the weights given as FP32 values (the in-memory
 * Program form of the reference's tests, tests/deterministic_executor_tests.cpp:96-179);
 * `weight_count` must equal the JSON's weights.count. */
int nvcr_sm100_executor_create_from_memory(const char* program_json, size_t json_size, const float* weights,
                                           size_t weight_count, void* stream, nvcr_sm100_executor** executor);

/* Reference load_normative_program (normative_stage.cpp:71-91): the program is
 * <directory>/<component>.detprog.json and its SHA-256 must equal
 * `expected_sha256_hex` (64 lowercase hex digits); a missing file is
 * NVCR_SM100_MISSING_ARTIFACT, a different digest NVCR_SM100_DIGEST_MISMATCH. */
int nvcr_sm100_load_normative(const char* directory, const char* component, const char* expected_sha256_hex,
                              void* stream, nvcr_sm100_executor** executor);

void nvcr_sm100_executor_destroy(nvcr_sm100_executor* executor);

/* Program metadata: names and channel counts of inputs (is_output = 0) and
 * outputs (is_output = 1). `name` stays valid for the executor's lifetime. */
int nvcr_sm100_tensor_count(const nvcr_sm100_executor* executor, int is_output, size_t* count);
int nvcr_sm100_tensor_info(const nvcr_sm100_executor* executor, int is_output, size_t index, const char** name,
                           int32_t* channels);

/* Reference infer_output_extents (normative_stage.cpp:42-65): inputs in
 * program order (names ignored); fills name/channels/height/width of
 * `outputs[0..output_count)` in program order. */
int nvcr_sm100_infer_output_extents(const nvcr_sm100_executor* executor, const nvcr_sm100_tensor* inputs,
                                    size_t input_count, nvcr_sm100_tensor* outputs, size_t output_count);

/* Reference CudaExecutor::run_half (cuda_executor.cu:1315-1373): named device
 * FP16 tensors; inputs widen exactly, outputs round to nearest even. Returns
 * once the work is enqueued; outputs are complete in stream order. */
int nvcr_sm100_run_half(nvcr_sm100_executor* executor, const nvcr_sm100_tensor* inputs, size_t input_count,
                        const nvcr_sm100_tensor* outputs, size_t output_count);

/* As run_half with device FP32 tensors on both sides (no boundary rounding). */
int nvcr_sm100_run_float(nvcr_sm100_executor* executor, const nvcr_sm100_tensor* inputs, size_t input_count,
                         const nvcr_sm100_tensor* outputs, size_t output_count);

/* Reference CudaExecutor::run (cuda_executor.cu:1375-1397): host FP32 tensors,
 * synchronous; the output buffers are caller-allocated. */
int nvcr_sm100_run_host(nvcr_sm100_executor* executor, const nvcr_sm100_tensor* inputs, size_t input_count,
                        const nvcr_sm100_tensor* outputs, size_t output_count);

/* Waits for the executor's stream; NVCR_SM100_BACKEND_ERROR if a CUDA error
 * occurred or a device-side bounded wait gave up. */
int nvcr_sm100_synchronize(nvcr_sm100_executor* executor);

/* Failure-detection self-test (no counterpart in the reference): enqueues on the
 * executor's stream one device wait on a barrier that nothing completes, bounded
 * by limit_ms (1..4000), which gives up the way a kernel's wait does. The next
 * nvcr_sm100_synchronize returns NVCR_SM100_BACKEND_ERROR ("a device-side wait
 * gave up") and clears the status; the executor and its CUDA context stay usable. */
int nvcr_sm100_test_wait_timeout(nvcr_sm100_executor* executor, unsigned int limit_ms);

/* Arithmetic self-test (no counterpart in the reference): the sigmoid in the
 * fused WSiLU epilogues takes 1 / d for d = 1 + exp(-x) in [1, 2^126) as a
 * refined hardware reciprocal instead of an IEEE division. This counts, in
 * *mismatches, the floats d with bit patterns first_bits .. first_bits + count - 1
 * (within [1, 2^126): 0x3f800000 .. 0x7e7fffff) for which the two differ in any
 * bit. Uses the current device; allocates and frees eight bytes of device memory. */
int nvcr_sm100_test_reciprocal(unsigned int first_bits, unsigned int count, unsigned long long* mismatches);

/* The stream all work is ordered on (a cudaStream_t). */
void* nvcr_sm100_stream(const nvcr_sm100_executor* executor);

/* Kernels launched by the last run, and the workspace bytes held. */
int nvcr_sm100_last_launch_count(const nvcr_sm100_executor* executor);
size_t nvcr_sm100_workspace_bytes(const nvcr_sm100_executor* executor);

/* Per-step CUDA-event timing of subsequent runs (off by default). */
int nvcr_sm100_set_profiling(nvcr_sm100_executor* executor, int enabled);
/* Synchronises and copies up to `capacity` kernel-segment times recorded by
 * the profiled runs since the previous call (which are then forgotten);
 * *count receives the number of segments. */
int nvcr_sm100_profile(nvcr_sm100_executor* executor, nvcr_sm100_step_time* steps, size_t capacity, size_t* count);

/* The numerics-identity payload (reference include/nvcr/bitstream/
 * numerics_identity.hpp, NumericsIdentityIO::make + serialize,
 * src/bitstream/numerics_identity.cpp): names the numerics profile and the
 * exact programs of the codec's normative stages. stage_ids[i] with the 32-byte
 * program SHA-256 stage_digests[32 i .. 32 i + 31], in the codec's stage order;
 * ids are 1..128 bytes of printable ASCII without space, 1..64 unique stages.
 * Writes u8 profile length, the profile id and the 32-byte program-set digest
 * (SHA-256 of, per stage, u8 id length, id bytes, program digest) to payload;
 * *payload_size gets its length (at most 161 bytes). Errors:
 * NVCR_SM100_INVALID_ARGUMENT for bad ids, a duplicate stage, a stage count
 * outside 1..64 or a payload buffer that is too small. */
int nvcr_sm100_numerics_identity(const char* profile, const char* const* stage_ids, const unsigned char* stage_digests,
                                 size_t stage_count, unsigned char* payload, size_t capacity, size_t* payload_size);

/* Reads a numerics-identity payload (reference NumericsIdentityIO::deserialize):
 * profile gets the NUL-terminated profile id (profile_capacity >= 129 always
 * suffices), program_set_digest its 32 bytes. NVCR_SM100_MALFORMED_BITSTREAM
 * for a truncated payload, trailing bytes or an invalid profile id. */
int nvcr_sm100_numerics_identity_parse(const unsigned char* payload, size_t size, char* profile,
                                       size_t profile_capacity, unsigned char* program_set_digest);

/* run_half without device allocation. No counterpart in the reference: it
 * exists for hosts that cannot call cudaMalloc while they run (an enqueue
 * inside a framework that owns all device memory, a real-time decode thread
 * that must not block on the allocator). Every scratch tensor of the run lives
 * in one file-scope static device array of NVCR_SM100_STATIC_WORKSPACE_BYTES,
 * which each GPU that loads the library keeps until exit. The first call on a
 * device looks the array's address up (cudaGetSymbolAddress): make it before
 * any stream capture. The executor's device (current at create) must be
 * current: otherwise NVCR_SM100_INVALID_STATE, with nothing enqueued. All
 * calls share the array: calls whose work overlaps on
 * the GPU race and must be ordered by the caller. A run needing more than the
 * array holds fails with NVCR_SM100_INVALID_ARGUMENT before enqueuing work.
 * Inputs, outputs and their meaning are those of nvcr_sm100_run_half. */
#define NVCR_SM100_STATIC_WORKSPACE_BYTES (64u * 1024u * 1024u)
int nvcr_sm100_run_half_static(nvcr_sm100_executor* executor, const nvcr_sm100_tensor* inputs, size_t input_count,
                               const nvcr_sm100_tensor* outputs, size_t output_count);

/* nvcr.fx.v1 stage programs (format nvcr.fx-program.v1): the reference's
 * fx::load_program and fx::program_digest (src/deterministic/fx_program.hpp:
 * 70-75, fx_program.cpp:394-466). */
typedef struct nvcr_sm100_fx_program nvcr_sm100_fx_program;

/* Loads <directory>/<stage>.fxprog.json and the data file it names, with the
 * profile's load-time refusals (weight, bias, shift and table bounds, every
 * tensor and data reference in range). Errors as the reference's loader:
 * NVCR_SM100_MISSING_ARTIFACT (no program file), NVCR_SM100_IO_ERROR (no data
 * file), NVCR_SM100_DIGEST_MISMATCH (the data file's SHA-256 differs from the
 * one the JSON pins), NVCR_SM100_INVALID_ARGUMENT (any other refusal). */
int nvcr_sm100_fx_program_load(const char* directory, const char* stage, nvcr_sm100_fx_program** program);
void nvcr_sm100_fx_program_destroy(nvcr_sm100_fx_program* program);
/* Lowercase hex SHA-256 of <directory>/<stage>.fxprog.json, NUL-terminated
 * (65 bytes): the program's identity. */
int nvcr_sm100_fx_program_digest(const char* directory, const char* stage, char* digest_hex);
/* Counts of a loaded program, and its digest (65 bytes). No counterpart in the
 * reference (its Program fields are read directly). */
int nvcr_sm100_fx_program_summary(const nvcr_sm100_fx_program* program, size_t* tensor_count, size_t* node_count,
                                  size_t* input_count, size_t* output_count, char* digest_hex);
/* Node `index` of a loaded program: its op name (as in the program file), the
 * number of inputs and the output tensor id. No counterpart in the reference. */
int nvcr_sm100_fx_program_node(const nvcr_sm100_fx_program* program, size_t index, const char** op,
                               size_t* input_count, uint32_t* output);

/* Name and channel count of a loaded program's input (is_output = 0) or output
 * (is_output = 1) `index`, in program.inputs / program.outputs order: the order
 * nvcr_sm100_fx_run takes tensors in. `name` lives as long as the program
 * handle. The reference reads these as Program fields (fx_program.hpp:62-66). */
int nvcr_sm100_fx_program_tensor(const nvcr_sm100_fx_program* program, int is_output, size_t index,
                                 const char** name, int32_t* channels);

/* An executor of one loaded fx program on the current device and `stream`
 * (a cudaStream_t; NULL for the default stream). It replaces the reference's
 * fx::run (src/deterministic/fx_program.cpp:468-525): the same int32 outputs,
 * and on any input the same outcome. The executor keeps a copy of the program
 * (the handle may be destroyed afterwards) and uploads its parameters at the
 * first run; creation and extent inference touch no device. */
typedef struct nvcr_sm100_fx_executor nvcr_sm100_fx_executor;
int nvcr_sm100_fx_executor_create(const nvcr_sm100_fx_program* program, void* stream,
                                  nvcr_sm100_fx_executor** executor);
void nvcr_sm100_fx_executor_destroy(nvcr_sm100_fx_executor* executor);
/* (channels, height, width) of each output for these input extents (3 int32
 * per tensor, program.inputs / program.outputs order). No counterpart in the
 * reference (its run sizes outputs as it goes). */
int nvcr_sm100_fx_infer_output_extents(nvcr_sm100_fx_executor* executor, const int32_t* input_extents,
                                       size_t input_count, int32_t* output_extents, size_t output_count);
/* Runs the program on batch-1 NCHW int32 tensors: host memory when
 * device_memory is 0 (copies inside the call), device memory otherwise. Returns
 * after the run (the stream is synchronised). NVCR_SM100_MALFORMED_BITSTREAM
 * for a stage failure (a gemm pre-activation with |r| >= 2^29 - 1, a stored
 * value outside [-2^30, 2^30], an input outside that bound, a qp outside a
 * param_row table): the failure the reference meets first, outputs
 * unspecified. NVCR_SM100_INVALID_ARGUMENT for inputs whose count or shapes the
 * program cannot take. */
int nvcr_sm100_fx_run(nvcr_sm100_fx_executor* executor, const int32_t* const* inputs, const int32_t* input_extents,
                      size_t input_count, int32_t* const* outputs, size_t output_count, int device_memory);
/* Kernels launched by the last run. No counterpart in the reference. */
int nvcr_sm100_fx_last_launch_count(const nvcr_sm100_fx_executor* executor);

/* DCVC-RT inter-stage glue on the device, exact numerics: the steps between a
 * decoder's spatial stages, on the caller's stream (a cudaStream_t; NULL for
 * the default stream), so no host round trip is needed between steps. FP16
 * tensors are bit patterns, batch-first NCHW, in device memory. Each returns
 * once its kernel is enqueued; NVCR_SM100_INVALID_ARGUMENT for what the
 * reference's host ops refuse. */

/* Reference build_decode_indexes(..., exact = true) (src/dcvcrt/host_ops.cpp:
 * 542-556; GPU form src/dcvcrt/backend/tensorrt/cuda_ops.cu:463-476, 807-820):
 * the entropy table of each scale, #{ i : clamp(scale, 0.11, 16) >= T[i] } over
 * the 127 exact thresholds, or 0 where a positive force-zero threshold is not
 * exceeded. */
int nvcr_sm100_dcvc_build_decode_indexes(const uint16_t* scales, uint8_t* indexes, size_t count,
                                         float force_zero_threshold, void* stream);
/* Reference build_encode_indexes(..., exact = true) (host_ops.cpp:523-540):
 * (symbol << 8) | table, 0 where forced to zero; symbols are integers in
 * [-128, 127]. */
int nvcr_sm100_dcvc_build_encode_indexes(const uint16_t* symbols, const uint16_t* scales, int16_t* indexes,
                                         size_t count, float force_zero_threshold, void* stream);
/* Reference make_four_way_mask / make_two_way_mask (host_ops.cpp:307-349):
 * ways 4 (stage 0..3) or 2 (stage 0..1); channels a multiple of ways. */
int nvcr_sm100_dcvc_make_mask(uint16_t* mask, int32_t batch, int32_t channels, int32_t height, int32_t width,
                              int ways, int stage, void* stream);
/* Reference restore_four_way / restore_two_way (host_ops.cpp:412-428, 456-472):
 * output[d] = (symbol + mean[d]) * mask[d] for the `ways` destinations of each
 * symbol; symbols hold volume / ways values, the rest the full output shape. */
int nvcr_sm100_dcvc_restore(const uint16_t* symbols, const uint16_t* means, const uint16_t* mask, uint16_t* output,
                            int32_t batch, int32_t channels, int32_t height, int32_t width, int ways, void* stream);

/* Reference process_with_mask (host_ops.cpp:351-377): per element, the masked
 * scale, mean and residual (values - mean) * mask, the symbol round(residual)
 * (half away from zero; 0 where a positive force-zero threshold is not
 * exceeded) clamped to [-128, 127], and symbol + mean. `residual` may be NULL;
 * every tensor holds `count` values. */
int nvcr_sm100_dcvc_process_with_mask(const uint16_t* values, const uint16_t* scales, const uint16_t* means,
                                      const uint16_t* mask, uint16_t* residual, uint16_t* symbols,
                                      uint16_t* reconstructed, uint16_t* masked_scales, size_t count,
                                      float force_zero_threshold, void* stream);
/* Reference reduce_channel_quarters / _halves (mask NULL) and
 * reduce_masked_quarters / _halves (host_ops.cpp:379-454): the ways (4 or 2)
 * channel slices of the input shape summed into one, each multiplied by the
 * mask first when it is given. */
int nvcr_sm100_dcvc_reduce(const uint16_t* input, const uint16_t* mask, uint16_t* output, int32_t batch,
                           int32_t channels, int32_t height, int32_t width, int ways, void* stream);

/* The elementwise steps between stages (reference host_ops.cpp:101-118,
 * 474-521), in place where the reference works in place; each value rounds to
 * FP16 after every step, and min / max follow IEEE 754-2008 minNum / maxNum.
 * round_to_int8: values = clamp(round(values), -128, 127), also as int8.
 * int8_to_half: output = values. clamp_min: values = max(values, minimum).
 * clamp_reciprocal_with_quant: quant_step = max(quant_step, 0.5), values *=
 * the FP16 reciprocal of it. add_in_place: first += second.
 * multiply_broadcast (reference multiply_broadcast_in_place): values[c][p] *=
 * factors[p] for each of `channels` planes of spatial_count values.
 * add_and_multiply: first = FP16(first + second) * quant_step. */
int nvcr_sm100_dcvc_round_to_int8(uint16_t* values, int8_t* quantized, size_t count, void* stream);
int nvcr_sm100_dcvc_int8_to_half(const int8_t* values, uint16_t* output, size_t count, void* stream);
int nvcr_sm100_dcvc_clamp_min(uint16_t* values, size_t count, float minimum, void* stream);
int nvcr_sm100_dcvc_clamp_reciprocal_with_quant(uint16_t* quant_step, uint16_t* values, size_t count, void* stream);
int nvcr_sm100_dcvc_add_in_place(uint16_t* first, const uint16_t* second, size_t count, void* stream);
int nvcr_sm100_dcvc_multiply_broadcast(uint16_t* values, const uint16_t* factors, size_t spatial_count,
                                       int32_t channels, void* stream);
int nvcr_sm100_dcvc_add_and_multiply(uint16_t* first, const uint16_t* second, const uint16_t* quant_step, size_t count,
                                     void* stream);
/* Reference replicate_pad and crop_spatial (host_ops.cpp:120-167): edge
 * replication up to padded_height x padded_width, or the crop from the origin. */
int nvcr_sm100_dcvc_replicate_pad(const uint16_t* input, uint16_t* output, int32_t batch, int32_t channels,
                                  int32_t height, int32_t width, int32_t padded_height, int32_t padded_width,
                                  void* stream);
int nvcr_sm100_dcvc_crop_spatial(const uint16_t* input, uint16_t* output, int32_t batch, int32_t channels,
                                 int32_t height, int32_t width, int32_t out_height, int32_t out_width, void* stream);

/* Picture conversions at the codec's edges (reference host_ops.cpp:198-305):
 * RGB24 (interleaved, width x height) or YUV 4:2:0 8-bit (planar Y, U, V; even
 * width and height) to a 3-plane FP16 YCbCr picture of padded_height x
 * padded_width with the last row and column replicated (BT.709 weights), and a
 * 1 x 3 x height x width YCbCr picture back to the visible (even) 4:2:0 planes. */
int nvcr_sm100_dcvc_rgb24_to_ycbcr_padded(const uint8_t* input, int32_t width, int32_t height, uint16_t* output,
                                          int32_t padded_height, int32_t padded_width, void* stream);
int nvcr_sm100_dcvc_yuv420p8_to_ycbcr_padded(const uint8_t* input, int32_t width, int32_t height, uint16_t* output,
                                             int32_t padded_height, int32_t padded_width, void* stream);
int nvcr_sm100_dcvc_ycbcr_padded_to_yuv420p8(const uint16_t* input, int32_t batch, int32_t channels, int32_t height,
                                             int32_t width, int32_t visible_width, int32_t visible_height,
                                             uint8_t* output, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* NVCR_SM100_H */
