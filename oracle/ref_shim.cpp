// C entry points over the reference's own CPU executor, for tests and the CPU
// baseline only. TEST INFRASTRUCTURE: compiled by oracle/Makefile together with
// the reference sources it names (src/deterministic/program.cpp,
// normative_stage.cpp, src/common/{json,sha256,error}.cpp,
// src/bitstream/numerics_identity.cpp, src/deterministic/fx.cpp,
// src/deterministic/fx_program.cpp, src/dcvcrt/host_ops.cpp) into
// oracle/_ref/libnvcr_ref.so. Nothing in the product links or loads it.
//
// Programs reach the reference through its own loader (load_program,
// src/deterministic/program.cpp:537-626) from the .detprog.json/.detw files the
// tests write, so the reference also checks the files' format and digests.
#include "deterministic/det_math.hpp"
#include "deterministic/fx_program.hpp"
#include "dcvcrt/host_ops.hpp"
#include "dcvcrt/scale_index.hpp"
#include "deterministic/normative_stage.hpp"
#include "deterministic/program.hpp"
#include "nvcr/bitstream/numerics_identity.hpp"

#include <algorithm>
#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

namespace det = nvcr::deterministic;

namespace {

void write_error(char* buffer, std::size_t size, std::string_view message) {
    if (buffer == nullptr || size == 0) return;
    std::snprintf(buffer, size, "%.*s", static_cast<int>(message.size()), message.data());
}

}  // namespace

extern "C" {

// 0 when the reference accepts the program file; otherwise the reference's
// ErrorCode value plus one, with its message.
int ref_load_check(const char* program_json, char* error, std::size_t error_size) {
    auto program = det::load_program(program_json);
    if (program) return 0;
    write_error(error, error_size, program.error().message());
    return static_cast<int>(program.error().code()) + 1;
}

// Runs run_cpu on FP32 NCHW inputs (program.inputs order). When weights is not
// null it replaces the program's FP16-widened weights with the given FP32
// values (the in-memory Program form the reference's tests use). Outputs are
// malloc'd; extents receive (c, h, w) per output. Returns 0 or ErrorCode + 1.
int ref_run(const char* program_json, const float* weights, std::int64_t weight_count,
            int input_count, const std::int32_t* input_extents, const float* const* inputs,
            int output_capacity, std::int32_t* output_extents, float** outputs, char* error,
            std::size_t error_size) {
    auto loaded = det::load_program(program_json);
    if (!loaded) {
        write_error(error, error_size, loaded.error().message());
        return static_cast<int>(loaded.error().code()) + 1;
    }
    auto& program = loaded.value();
    if (weights != nullptr) {
        if (static_cast<std::size_t>(weight_count) != program.weights.size()) {
            write_error(error, error_size, "weight override has the wrong count");
            return 1;
        }
        program.weights.assign(weights, weights + weight_count);
    }
    std::vector<det::Tensor> tensors;
    for (int index = 0; index < input_count; ++index) {
        det::Tensor tensor{input_extents[3 * index], input_extents[3 * index + 1],
                           input_extents[3 * index + 2], {}};
        tensor.values.assign(inputs[index], inputs[index] + tensor.size());
        tensors.push_back(std::move(tensor));
    }
    auto results = det::run_cpu(program, tensors);
    if (!results) {
        write_error(error, error_size, results.error().message());
        return static_cast<int>(results.error().code()) + 1;
    }
    if (static_cast<int>(results.value().size()) > output_capacity) {
        write_error(error, error_size, "too many outputs");
        return 1;
    }
    for (std::size_t slot = 0; slot < results.value().size(); ++slot) {
        const auto& result = results.value()[slot];
        output_extents[3 * slot] = result.channels;
        output_extents[3 * slot + 1] = result.height;
        output_extents[3 * slot + 2] = result.width;
        outputs[slot] = static_cast<float*>(std::malloc(result.values.size() * sizeof(float) + 4));
        std::memcpy(outputs[slot], result.values.data(), result.values.size() * sizeof(float));
    }
    return 0;
}

// Times `repeats` calls of run_cpu on the given inputs (weights as loaded) and
// returns the mean seconds per call, or a negative value on failure.
double ref_time_run(const char* program_json, int input_count, const std::int32_t* input_extents,
                    const float* const* inputs, int repeats) {
    auto loaded = det::load_program(program_json);
    if (!loaded) return -1.0;
    std::vector<det::Tensor> tensors;
    for (int index = 0; index < input_count; ++index) {
        det::Tensor tensor{input_extents[3 * index], input_extents[3 * index + 1],
                           input_extents[3 * index + 2], {}};
        tensor.values.assign(inputs[index], inputs[index] + tensor.size());
        tensors.push_back(std::move(tensor));
    }
    const auto start = std::chrono::steady_clock::now();
    for (int repeat = 0; repeat < repeats; ++repeat) {
        auto results = det::run_cpu(loaded.value(), tensors);
        if (!results) return -2.0;
    }
    const std::chrono::duration<double> elapsed = std::chrono::steady_clock::now() - start;
    return elapsed.count() / repeats;
}

// Output extents of a program for the given input extents (infer_output_extents,
// normative_stage.cpp:42-65). Returns 0 or ErrorCode + 1.
int ref_infer_extents(const char* program_json, int input_count, const std::int32_t* input_extents,
                      int output_capacity, std::int32_t* output_extents, char* error,
                      std::size_t error_size) {
    auto loaded = det::load_program(program_json);
    if (!loaded) {
        write_error(error, error_size, loaded.error().message());
        return static_cast<int>(loaded.error().code()) + 1;
    }
    std::vector<det::Extent> extents;
    for (int index = 0; index < input_count; ++index) {
        extents.push_back(det::Extent{input_extents[3 * index], input_extents[3 * index + 1],
                                      input_extents[3 * index + 2]});
    }
    auto inferred = det::infer_output_extents(loaded.value(), extents);
    if (!inferred) {
        write_error(error, error_size, inferred.error().message());
        return static_cast<int>(inferred.error().code()) + 1;
    }
    if (static_cast<int>(inferred.value().size()) > output_capacity) return 1;
    for (std::size_t slot = 0; slot < inferred.value().size(); ++slot) {
        output_extents[3 * slot] = inferred.value()[slot].channels;
        output_extents[3 * slot + 1] = inferred.value()[slot].height;
        output_extents[3 * slot + 2] = inferred.value()[slot].width;
    }
    return 0;
}

// quantize_weights (program.cpp:509-535) on one [out][in] matrix.
void ref_quantize_weights(const float* weights, std::int32_t out_channels, std::int32_t in_channels,
                          std::int32_t weight_bits, std::int16_t* values, float* scales) {
    det::Program program;
    program.weights.assign(weights, weights + static_cast<std::size_t>(out_channels) * in_channels);
    det::Node node;
    node.in_channels = in_channels;
    node.out_channels = out_channels;
    node.weight_bits = weight_bits;
    const auto quantized = det::quantize_weights(program, node);
    std::memcpy(values, quantized.values.data(), quantized.values.size() * sizeof(std::int16_t));
    std::memcpy(scales, quantized.scales.data(), quantized.scales.size() * sizeof(float));
}

float ref_det_exp(float x) { return det::det_exp(x); }
float ref_det_sigmoid(float x) { return det::det_sigmoid(x); }
float ref_det_ldexp(float x, int e) { return det::det_ldexp(x, e); }
int ref_det_int_exponent(float maximum, int bits) { return det::det_int_exponent(maximum, bits); }
int ref_det_int_quantize(float x, int e, int bits) { return det::det_int_quantize(x, e, bits); }
float ref_det_int_output(long long acc, float scale, int e, float bias) {
    return det::det_int_output(acc, scale, e, bias);
}
float ref_half_to_float(std::uint16_t h) { return det::det_half_bits_to_float(h); }
std::uint16_t ref_float_to_half(float x) { return det::det_float_to_half_bits(x); }

// NumericsIdentityIO::make + serialize (src/bitstream/numerics_identity.cpp):
// 0 and the payload, or the reference's ErrorCode value plus one.
int ref_numerics_identity(const char* profile, const char* const* stage_ids, const unsigned char* digests,
                          std::size_t count, unsigned char* payload, std::size_t capacity, std::size_t* size) {
    std::vector<nvcr::NormativeStageIdentity> stages(count);
    for (std::size_t i = 0; i < count; ++i) {
        stages[i].stage_id = stage_ids[i];
        std::memcpy(stages[i].program_digest.data(), digests + 32 * i, 32);
    }
    auto identity = nvcr::NumericsIdentityIO::make(profile, stages);
    if (!identity) return static_cast<int>(identity.error().code()) + 1;
    auto bytes = nvcr::NumericsIdentityIO::serialize(identity.value());
    if (!bytes) return static_cast<int>(bytes.error().code()) + 1;
    if (bytes.value().size() > capacity) return -1;
    std::memcpy(payload, bytes.value().data(), bytes.value().size());
    *size = bytes.value().size();
    return 0;
}

// NumericsIdentityIO::deserialize: 0 with the profile and digest, or ErrorCode + 1.
int ref_numerics_identity_parse(const unsigned char* payload, std::size_t size, char* profile,
                                std::size_t profile_capacity, unsigned char* digest) {
    auto identity = nvcr::NumericsIdentityIO::deserialize(
        std::span(reinterpret_cast<const std::byte*>(payload), size));
    if (!identity) return static_cast<int>(identity.error().code()) + 1;
    if (identity.value().profile.size() + 1 > profile_capacity) return -1;
    std::memcpy(profile, identity.value().profile.c_str(), identity.value().profile.size() + 1);
    std::memcpy(digest, identity.value().program_set_digest.data(), 32);
    return 0;
}

// nvcr.fx.v1 scalar rules (src/deterministic/fx.cpp:29-37).
std::int64_t ref_fx_rsr(std::int64_t a, int s) { return det::fx::rsr(a, s); }

std::int64_t ref_fx_delta_act(std::int64_t r, std::int64_t h, int shift, const std::int16_t* dc, std::size_t count) {
    const det::fx::DeltaTable table{h, shift, std::vector<std::int16_t>(dc, dc + count)};
    return det::fx::delta_act(r, table);
}

// fx::load_program (src/deterministic/fx_program.cpp:398-466): 0, or ErrorCode + 1
// with the reference's message.
int ref_fx_load_check(const char* directory, const char* stage, char* error, std::size_t error_size) {
    auto program = det::fx::load_program(directory, stage);
    if (program) return 0;
    write_error(error, error_size, program.error().message());
    return static_cast<int>(program.error().code()) + 1;
}

// fx::program_digest: 0 and 64 lowercase hex digits plus a terminator, or ErrorCode + 1.
int ref_fx_program_digest(const char* directory, const char* stage, char* digest) {
    auto hex = det::fx::program_digest(directory, stage);
    if (!hex) return static_cast<int>(hex.error().code()) + 1;
    std::snprintf(digest, 65, "%s", hex.value().c_str());
    return 0;
}

// fx::load_program then fx::run (fx_program.cpp:468-525) on int32 NCHW inputs
// (program.inputs order; extents are (c, h, w) per input). Outputs are malloc'd;
// output_extents receive (c, h, w) per output. 0, or ErrorCode + 1 with the
// reference's message (a stage failure is malformed_bitstream).
int ref_fx_run(const char* directory, const char* stage, int input_count, const std::int32_t* input_extents,
               const std::int32_t* const* inputs, int output_capacity, std::int32_t* output_extents,
               std::int32_t** outputs, char* error, std::size_t error_size) {
    auto program = det::fx::load_program(directory, stage);
    if (!program) {
        write_error(error, error_size, program.error().message());
        return static_cast<int>(program.error().code()) + 1;
    }
    std::vector<det::fx::Tensor> tensors;
    for (int index = 0; index < input_count; ++index) {
        det::fx::Tensor tensor{input_extents[3 * index], input_extents[3 * index + 1], input_extents[3 * index + 2], {}};
        tensor.values.assign(inputs[index], inputs[index] + static_cast<std::size_t>(tensor.channels) * tensor.plane());
        tensors.push_back(std::move(tensor));
    }
    auto result = det::fx::run(program.value(), tensors);
    if (!result) {
        write_error(error, error_size, result.error().message());
        return static_cast<int>(result.error().code()) + 1;
    }
    const auto& produced = result.value();
    if (static_cast<int>(produced.size()) > output_capacity) {
        write_error(error, error_size, "too many outputs");
        return -1;
    }
    for (std::size_t index = 0; index < produced.size(); ++index) {
        const auto& y = produced[index];
        output_extents[3 * index] = y.channels;
        output_extents[3 * index + 1] = y.height;
        output_extents[3 * index + 2] = y.width;
        outputs[index] = static_cast<std::int32_t*>(std::malloc(std::max<std::size_t>(1, y.values.size()) * 4));
        std::memcpy(outputs[index], y.values.data(), y.values.size() * 4);
    }
    return 0;
}

// DCVC-RT inter-stage glue on the host (src/dcvcrt/host_ops.cpp), exact
// numerics. Each returns the reference's bool as 1 or 0.
namespace glue = nvcr::dcvcrt::host_ops;

void ref_glue_to_half(const float* in, std::uint16_t* out, std::size_t count) {
    for (std::size_t i = 0; i < count; ++i) out[i] = glue::to_half(in[i]);
}
void ref_glue_to_float(const std::uint16_t* in, float* out, std::size_t count) {
    for (std::size_t i = 0; i < count; ++i) out[i] = glue::to_float(in[i]);
}
// exact_scale_index (src/dcvcrt/scale_index.hpp:153-169) on float scales.
void ref_glue_exact_scale_indexes(const float* in, std::uint8_t* out, std::size_t count) {
    for (std::size_t i = 0; i < count; ++i) out[i] = nvcr::dcvcrt::exact_scale_index(in[i]);
}

int ref_glue_decode_indexes(const std::uint16_t* scales, std::uint8_t* out, std::size_t count, float force_zero) {
    return glue::build_decode_indexes(std::span(scales, count), std::span(out, count), force_zero, true) ? 1 : 0;
}

int ref_glue_encode_indexes(const std::uint16_t* symbols, const std::uint16_t* scales, std::int16_t* out,
                            std::size_t count, float force_zero) {
    return glue::build_encode_indexes(std::span(symbols, count), std::span(scales, count), std::span(out, count),
                                      force_zero, true) ? 1 : 0;
}

int ref_glue_mask(std::uint16_t* mask, std::size_t capacity, int batch, int channels, int height, int width, int ways,
                  int stage) {
    const glue::Shape4D shape{batch, channels, height, width};
    return (ways == 4 ? glue::make_four_way_mask(std::span(mask, capacity), shape, stage)
                      : glue::make_two_way_mask(std::span(mask, capacity), shape, stage)) ? 1 : 0;
}

int ref_glue_restore(const std::uint16_t* symbols, const std::uint16_t* means, const std::uint16_t* mask,
                     std::uint16_t* out, std::size_t capacity, int batch, int channels, int height, int width,
                     int ways) {
    const glue::Shape4D shape{batch, channels, height, width};
    const std::size_t part = capacity / static_cast<std::size_t>(ways);
    return (ways == 4 ? glue::restore_four_way(std::span(symbols, part), std::span(means, capacity),
                                               std::span(mask, capacity), std::span(out, capacity), shape)
                      : glue::restore_two_way(std::span(symbols, part), std::span(means, capacity),
                                              std::span(mask, capacity), std::span(out, capacity), shape)) ? 1 : 0;
}

int ref_glue_process(const std::uint16_t* values, const std::uint16_t* scales, const std::uint16_t* means,
                     const std::uint16_t* mask, std::uint16_t* residual, std::uint16_t* symbols,
                     std::uint16_t* reconstructed, std::uint16_t* masked_scales, std::size_t count, float force_zero) {
    return glue::process_with_mask(std::span(values, count), std::span(scales, count), std::span(means, count),
                                   std::span(mask, count),
                                   residual != nullptr ? std::span(residual, count) : std::span<std::uint16_t>(),
                                   std::span(symbols, count), std::span(reconstructed, count),
                                   std::span(masked_scales, count), force_zero) ? 1 : 0;
}

// reduce_channel_quarters / _halves (mask null) and reduce_masked_quarters / _halves.
int ref_glue_reduce(const std::uint16_t* input, const std::uint16_t* mask, std::uint16_t* output, std::size_t capacity,
                    int batch, int channels, int height, int width, int ways) {
    const glue::Shape4D shape{batch, channels, height, width};
    const auto in = std::span(input, capacity);
    const auto out = std::span(output, capacity / static_cast<std::size_t>(ways));
    if (mask == nullptr) {
        return (ways == 4 ? glue::reduce_channel_quarters(in, out, shape) : glue::reduce_channel_halves(in, out, shape))
            ? 1 : 0;
    }
    const auto m = std::span(mask, capacity);
    return (ways == 4 ? glue::reduce_masked_quarters(in, m, out, shape) : glue::reduce_masked_halves(in, m, out, shape))
        ? 1 : 0;
}

// The elementwise steps (host_ops.cpp:101-118, 474-521), op numbered as
// nvcr_sm100::glue::PointwiseOp; a, b, c, q as there.
int ref_glue_pointwise(int op, std::uint16_t* a, std::uint16_t* b, const std::uint16_t* c, std::int8_t* q,
                       std::size_t count, float scalar, std::size_t spatial_count) {
    const auto A = std::span(a, count);
    switch (op) {
    case 0: return glue::round_to_int8(A, std::span(q, count)) ? 1 : 0;
    case 1: return glue::int8_to_half(std::span<const std::int8_t>(q, count), A) ? 1 : 0;
    case 2: return glue::clamp_min(A, scalar) ? 1 : 0;
    case 3: return glue::clamp_reciprocal_with_quant(A, std::span(b, count)) ? 1 : 0;
    case 4: return glue::add_in_place(A, std::span<const std::uint16_t>(b, count)) ? 1 : 0;
    case 5: {
        const std::size_t channels = spatial_count == 0 ? 0 : count / spatial_count;
        return glue::multiply_broadcast_in_place(A, std::span<const std::uint16_t>(b, spatial_count), spatial_count,
                                                 static_cast<std::int32_t>(channels)) ? 1 : 0;
    }
    case 6: return glue::add_and_multiply(A, std::span<const std::uint16_t>(b, count), std::span(c, count)) ? 1 : 0;
    default: return -1;
    }
}

int ref_glue_pad_or_crop(const std::uint16_t* input, std::uint16_t* output, std::size_t out_capacity, int batch,
                         int channels, int height, int width, int out_height, int out_width, int pad) {
    const glue::Shape4D shape{batch, channels, height, width};
    const std::size_t in_count = static_cast<std::size_t>(batch > 0 ? batch : 0) * (channels > 0 ? channels : 0) *
        (height > 0 ? height : 0) * (width > 0 ? width : 0);
    return (pad ? glue::replicate_pad(std::span(input, in_count), std::span(output, out_capacity), shape, out_height,
                                      out_width)
                : glue::crop_spatial(std::span(input, in_count), std::span(output, out_capacity), shape, out_height,
                                     out_width)) ? 1 : 0;
}

int ref_glue_to_ycbcr(const std::uint8_t* input, std::size_t input_size, int width, int height, std::uint16_t* output,
                      std::size_t output_size, int padded_height, int padded_width, int yuv) {
    return (yuv ? glue::yuv420p8_to_ycbcr_padded(std::span(input, input_size), width, height,
                                                 std::span(output, output_size), padded_height, padded_width)
                : glue::rgb24_to_ycbcr_padded(std::span(input, input_size), width, height,
                                              std::span(output, output_size), padded_height, padded_width)) ? 1 : 0;
}

int ref_glue_to_yuv(const std::uint16_t* input, int batch, int channels, int height, int width, int visible_width,
                    int visible_height, std::uint8_t* output, std::size_t output_size) {
    const glue::Shape4D shape{batch, channels, height, width};
    const std::size_t in_count = static_cast<std::size_t>(batch > 0 ? batch : 0) * (channels > 0 ? channels : 0) *
        (height > 0 ? height : 0) * (width > 0 ? width : 0);
    return glue::ycbcr_padded_to_yuv420p8(std::span(input, in_count), shape, visible_width, visible_height,
                                          std::span(output, output_size)) ? 1 : 0;
}

void ref_free(void* pointer) { std::free(pointer); }

}  // extern "C"
