// The extern "C" entry points of include/nvcr_sm100.h over the executor.
// Failures become 1 + the reference's ErrorCode value and a thread-local message.

#include "../../include/nvcr_sm100.h"

#include "capi_internal.hpp"
#include "fx_executor.hpp"
#include "glue_kernels.hpp"
#include "fx_program.hpp"
#include "numerics_identity.hpp"
#include "sha256.hpp"

#include <cstdio>
#include <cstring>
#include <fstream>
#include <new>
#include <sstream>
#include <string>
#include <sys/stat.h>

struct nvcr_sm100_program {
    nvcr_sm100::Program program;
};

struct nvcr_sm100_fx_program {
    nvcr_sm100::fx::FxProgram program;
};

struct nvcr_sm100_fx_executor {
    std::unique_ptr<nvcr_sm100::fx::FxExecutor> executor;
};

namespace {

using nvcr_sm100::Code;
using nvcr_sm100::Error;

thread_local std::string last_error;

int report(const Error& error) {
    last_error = error.message;
    return static_cast<int>(error.code) + 1;
}

int report(Code code, const std::string& message) { return report(Error{code, message}); }

int succeed() {
    last_error.clear();
    return NVCR_SM100_OK;
}

}  // namespace

int nvcr_sm100::report_error(const Error& error) { return report(error); }
int nvcr_sm100::report_ok() { return succeed(); }

namespace {

template <typename F>
int guarded(F&& body) {
    try {
        return body();
    } catch (const std::bad_alloc&) {
        return report(Code::resource_exhausted, "host allocation failed");
    } catch (const std::exception& exception) {
        return report(Code::internal_error, exception.what());
    } catch (...) {
        return report(Code::internal_error, "unknown exception");
    }
}

std::vector<nvcr_sm100::TensorView> views(const nvcr_sm100_tensor* tensors, size_t count) {
    std::vector<nvcr_sm100::TensorView> out;
    for (size_t i = 0; i < count; ++i) {
        out.push_back(nvcr_sm100::TensorView{tensors[i].name != nullptr ? tensors[i].name : "",
                                             {tensors[i].channels, tensors[i].height, tensors[i].width},
                                             tensors[i].data});
    }
    return out;
}

int finish_create(nvcr_sm100::Result<nvcr_sm100::Program> program, void* stream, nvcr_sm100_executor** executor) {
    if (!program) return report(program.error());
    auto created = nvcr_sm100::Executor::create(std::move(program.value()), static_cast<cudaStream_t>(stream));
    if (!created) return report(created.error());
    *executor = new nvcr_sm100_executor{std::move(created.value())};
    return succeed();
}

template <typename Run>
int run_with(nvcr_sm100_executor* executor, const nvcr_sm100_tensor* inputs, size_t input_count,
             const nvcr_sm100_tensor* outputs, size_t output_count, Run run) {
    if (executor == nullptr || (inputs == nullptr && input_count > 0) || (outputs == nullptr && output_count > 0)) {
        return report(Code::invalid_argument, "null executor or tensor array");
    }
    auto status = run(*executor->executor, views(inputs, input_count), views(outputs, output_count));
    if (!status) return report(status.error());
    return succeed();
}

int infer_extents(const nvcr_sm100::Program& program, const nvcr_sm100_tensor* inputs, size_t input_count,
                  nvcr_sm100_tensor* outputs, size_t output_count) {
    if (inputs == nullptr && input_count > 0) return report(Code::invalid_argument, "null argument");
    std::vector<nvcr_sm100::Extent> extents;
    for (size_t i = 0; i < input_count; ++i) extents.push_back({inputs[i].channels, inputs[i].height, inputs[i].width});
    auto inferred = nvcr_sm100::infer_output_extents(program, extents);
    if (!inferred) return report(inferred.error());
    if (output_count < inferred.value().size() || outputs == nullptr) {
        return report(Code::invalid_argument, "output array is too small");
    }
    for (size_t slot = 0; slot < inferred.value().size(); ++slot) {
        outputs[slot].name = program.tensor_names[program.outputs[slot]].c_str();
        outputs[slot].channels = inferred.value()[slot].channels;
        outputs[slot].height = inferred.value()[slot].height;
        outputs[slot].width = inferred.value()[slot].width;
    }
    return succeed();
}

int tensor_info(const nvcr_sm100::Program& program, int is_output, size_t index, const char** name,
                int32_t* channels) {
    const auto& ids = is_output ? program.outputs : program.inputs;
    if (index >= ids.size()) return report(Code::invalid_argument, "tensor index out of range");
    if (name != nullptr) *name = program.tensor_names[ids[index]].c_str();
    if (channels != nullptr) *channels = program.tensor_channels[ids[index]];
    return succeed();
}

}  // namespace

extern "C" {

int nvcr_sm100_abi_version(void) { return NVCR_SM100_ABI_VERSION; }

size_t nvcr_sm100_last_error(char* buffer, size_t size) {
    if (buffer != nullptr && size > 0) std::snprintf(buffer, size, "%s", last_error.c_str());
    return last_error.size();
}

int nvcr_sm100_supports_profile(const char* profile) {
    if (profile == nullptr || std::string_view(profile) != nvcr_sm100::intconv_profile) return 0;
    int device = 0;
    int major = 0;
    int minor = 0;
    if (cudaGetDevice(&device) != cudaSuccess) return 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess) return 0;
    if (cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device) != cudaSuccess) return 0;
    return major == 10 && minor == 0 ? 1 : 0;
}

int nvcr_sm100_is_normative(const char* profile, int* normative) {
    if (normative == nullptr) return report(Code::invalid_argument, "null output");
    const std::string_view text = profile != nullptr ? profile : "";
    if (text.empty()) {
        *normative = 0;
        return succeed();
    }
    if (text == nvcr_sm100::intconv_profile) {
        *normative = 1;
        return succeed();
    }
    return report(Code::incompatible_precision, "unknown numerics profile '" + std::string(text) + "'");
}

int nvcr_sm100_executor_create(const char* path, void* stream, nvcr_sm100_executor** executor) {
    return guarded([&] {
        if (path == nullptr || executor == nullptr) return report(Code::invalid_argument, "null argument");
        return finish_create(nvcr_sm100::load_program_file(path), stream, executor);
    });
}

int nvcr_sm100_executor_create_from_memory(const char* json, size_t json_size, const float* weights,
                                           size_t weight_count, void* stream, nvcr_sm100_executor** executor) {
    return guarded([&] {
        if (json == nullptr || executor == nullptr || (weights == nullptr && weight_count > 0)) {
            return report(Code::invalid_argument, "null argument");
        }
        static const float no_weights = 0.0f;
        return finish_create(nvcr_sm100::load_program_text(std::string_view(json, json_size), ".",
                                                           weights != nullptr ? weights : &no_weights, weight_count),
                             stream, executor);
    });
}

int nvcr_sm100_load_normative(const char* directory, const char* component, const char* expected, void* stream,
                              nvcr_sm100_executor** executor) {
    return guarded([&] {
        if (directory == nullptr || component == nullptr || executor == nullptr) {
            return report(Code::invalid_argument, "null argument");
        }
        const std::string name(component);
        if (expected == nullptr || std::strlen(expected) == 0) {
            return report(Code::invalid_argument, "normative stage " + name + " has no program digest");
        }
        const std::string path = std::string(directory) + "/" + name + ".detprog.json";
        struct stat info{};
        if (stat(path.c_str(), &info) != 0 || !S_ISREG(info.st_mode)) {
            return report(Code::missing_artifact, "normative program is missing: " + path);
        }
        std::ifstream stream_in(path, std::ios::binary);
        std::ostringstream contents;
        contents << stream_in.rdbuf();
        const std::string text = contents.str();
        if (nvcr_sm100::sha256_hex(text.data(), text.size()) != std::string(expected)) {
            return report(Code::digest_mismatch, "normative program digest mismatch: " + path);
        }
        return finish_create(nvcr_sm100::load_program_file(path), stream, executor);
    });
}

void nvcr_sm100_executor_destroy(nvcr_sm100_executor* executor) { delete executor; }

int nvcr_sm100_tensor_count(const nvcr_sm100_executor* executor, int is_output, size_t* count) {
    if (executor == nullptr || count == nullptr) return report(Code::invalid_argument, "null argument");
    const auto& program = executor->executor->program();
    *count = is_output ? program.outputs.size() : program.inputs.size();
    return succeed();
}

int nvcr_sm100_tensor_info(const nvcr_sm100_executor* executor, int is_output, size_t index, const char** name,
                           int32_t* channels) {
    if (executor == nullptr) return report(Code::invalid_argument, "null executor");
    const auto& program = executor->executor->program();
    const auto& ids = is_output ? program.outputs : program.inputs;
    if (index >= ids.size()) return report(Code::invalid_argument, "tensor index out of range");
    if (name != nullptr) *name = program.tensor_names[ids[index]].c_str();
    if (channels != nullptr) *channels = program.tensor_channels[ids[index]];
    return succeed();
}

int nvcr_sm100_program_load(const char* path, nvcr_sm100_program** program) {
    return guarded([&] {
        if (path == nullptr || program == nullptr) return report(Code::invalid_argument, "null argument");
        auto loaded = nvcr_sm100::load_program_file(path);
        if (!loaded) return report(loaded.error());
        *program = new nvcr_sm100_program{std::move(loaded.value())};
        return succeed();
    });
}

int nvcr_sm100_program_load_memory(const char* json, size_t json_size, const float* weights, size_t weight_count,
                                   nvcr_sm100_program** program) {
    return guarded([&] {
        if (json == nullptr || program == nullptr || (weights == nullptr && weight_count > 0)) {
            return report(Code::invalid_argument, "null argument");
        }
        static const float no_weights = 0.0f;
        auto loaded = nvcr_sm100::load_program_text(std::string_view(json, json_size), ".",
                                                    weights != nullptr ? weights : &no_weights, weight_count);
        if (!loaded) return report(loaded.error());
        *program = new nvcr_sm100_program{std::move(loaded.value())};
        return succeed();
    });
}

void nvcr_sm100_program_destroy(nvcr_sm100_program* program) { delete program; }

int nvcr_sm100_program_tensor_count(const nvcr_sm100_program* program, int is_output, size_t* count) {
    if (program == nullptr || count == nullptr) return report(Code::invalid_argument, "null argument");
    *count = is_output ? program->program.outputs.size() : program->program.inputs.size();
    return succeed();
}

int nvcr_sm100_program_tensor_info(const nvcr_sm100_program* program, int is_output, size_t index,
                                   const char** name, int32_t* channels) {
    if (program == nullptr) return report(Code::invalid_argument, "null program");
    return tensor_info(program->program, is_output, index, name, channels);
}

int nvcr_sm100_program_infer_output_extents(const nvcr_sm100_program* program, const nvcr_sm100_tensor* inputs,
                                            size_t input_count, nvcr_sm100_tensor* outputs, size_t output_count) {
    return guarded([&] {
        if (program == nullptr) return report(Code::invalid_argument, "null program");
        return infer_extents(program->program, inputs, input_count, outputs, output_count);
    });
}

int nvcr_sm100_executor_create_from_program(const nvcr_sm100_program* program, void* stream,
                                            nvcr_sm100_executor** executor) {
    return guarded([&] {
        if (program == nullptr || executor == nullptr) return report(Code::invalid_argument, "null argument");
        return finish_create(nvcr_sm100::Result<nvcr_sm100::Program>(program->program), stream, executor);
    });
}

int nvcr_sm100_infer_output_extents(const nvcr_sm100_executor* executor, const nvcr_sm100_tensor* inputs,
                                    size_t input_count, nvcr_sm100_tensor* outputs, size_t output_count) {
    return guarded([&] {
        if (executor == nullptr) return report(Code::invalid_argument, "null executor");
        return infer_extents(executor->executor->program(), inputs, input_count, outputs, output_count);
    });
}

int nvcr_sm100_run_half(nvcr_sm100_executor* executor, const nvcr_sm100_tensor* inputs, size_t input_count,
                        const nvcr_sm100_tensor* outputs, size_t output_count) {
    return guarded([&] {
        return run_with(executor, inputs, input_count, outputs, output_count,
                        [](nvcr_sm100::Executor& e, const auto& in, const auto& out) { return e.run_half(in, out); });
    });
}

int nvcr_sm100_run_float(nvcr_sm100_executor* executor, const nvcr_sm100_tensor* inputs, size_t input_count,
                         const nvcr_sm100_tensor* outputs, size_t output_count) {
    return guarded([&] {
        return run_with(executor, inputs, input_count, outputs, output_count,
                        [](nvcr_sm100::Executor& e, const auto& in, const auto& out) { return e.run_float(in, out); });
    });
}

int nvcr_sm100_run_host(nvcr_sm100_executor* executor, const nvcr_sm100_tensor* inputs, size_t input_count,
                        const nvcr_sm100_tensor* outputs, size_t output_count) {
    return guarded([&] {
        return run_with(executor, inputs, input_count, outputs, output_count,
                        [](nvcr_sm100::Executor& e, const auto& in, const auto& out) { return e.run_host(in, out); });
    });
}

int nvcr_sm100_synchronize(nvcr_sm100_executor* executor) {
    return guarded([&] {
        if (executor == nullptr) return report(Code::invalid_argument, "null executor");
        auto status = executor->executor->synchronize();
        if (!status) return report(status.error());
        return succeed();
    });
}

int nvcr_sm100_test_wait_timeout(nvcr_sm100_executor* executor, unsigned int limit_ms) {
    return guarded([&] {
        if (executor == nullptr) return report(Code::invalid_argument, "null executor");
        auto status = executor->executor->test_wait_timeout(limit_ms);
        if (!status) return report(status.error());
        return succeed();
    });
}

int nvcr_sm100_test_reciprocal(unsigned int first_bits, unsigned int count, unsigned long long* mismatches) {
    return guarded([&] {
        if (mismatches == nullptr) return report(Code::invalid_argument, "null mismatch count");
        if (first_bits < 0x3f800000u || count > 0x7e800000u - first_bits) {
            return report(Code::invalid_argument, "the range must lie within [1, 2^126)");
        }
        unsigned long long* device = nullptr;
        cudaError_t status = cudaMalloc(reinterpret_cast<void**>(&device), sizeof(unsigned long long));
        if (status != cudaSuccess) return report(Code::backend_error, std::string("cudaMalloc: ") + cudaGetErrorString(status));
        status = cudaMemset(device, 0, sizeof(unsigned long long));
        if (status == cudaSuccess) status = nvcr_sm100::kernels::check_reciprocal(first_bits, count, device, nullptr);
        if (status == cudaSuccess) {
            status = cudaMemcpy(mismatches, device, sizeof(unsigned long long), cudaMemcpyDeviceToHost);
        }
        cudaFree(device);
        if (status != cudaSuccess) return report(Code::backend_error, std::string("reciprocal check: ") + cudaGetErrorString(status));
        return succeed();
    });
}

int nvcr_sm100_numerics_identity(const char* profile, const char* const* stage_ids, const unsigned char* stage_digests,
                                 size_t stage_count, unsigned char* payload, size_t capacity, size_t* payload_size) {
    return guarded([&] {
        if (profile == nullptr || payload == nullptr || payload_size == nullptr ||
            (stage_count > 0 && (stage_ids == nullptr || stage_digests == nullptr))) {
            return report(Code::invalid_argument, "null argument");
        }
        std::vector<nvcr_sm100::StageDigest> stages(stage_count);
        for (std::size_t i = 0; i < stage_count; ++i) {
            if (stage_ids[i] == nullptr) return report(Code::invalid_argument, "null stage id");
            stages[i].stage_id = stage_ids[i];
            std::memcpy(stages[i].program_digest.data(), stage_digests + 32 * i, 32);
        }
        auto identity = nvcr_sm100::make_numerics_identity(profile, stages);
        if (!identity) return report(identity.error());
        auto bytes = nvcr_sm100::serialize_numerics_identity(identity.value());
        if (!bytes) return report(bytes.error());
        if (bytes.value().size() > capacity) return report(Code::invalid_argument, "payload buffer is too small");
        std::memcpy(payload, bytes.value().data(), bytes.value().size());
        *payload_size = bytes.value().size();
        return succeed();
    });
}

int nvcr_sm100_numerics_identity_parse(const unsigned char* payload, size_t size, char* profile,
                                       size_t profile_capacity, unsigned char* program_set_digest) {
    return guarded([&] {
        if (profile == nullptr || program_set_digest == nullptr) return report(Code::invalid_argument, "null argument");
        auto identity = nvcr_sm100::parse_numerics_identity(payload, size);
        if (!identity) return report(identity.error());
        if (identity.value().profile.size() + 1 > profile_capacity) {
            return report(Code::invalid_argument, "profile buffer is too small");
        }
        std::memcpy(profile, identity.value().profile.c_str(), identity.value().profile.size() + 1);
        std::memcpy(program_set_digest, identity.value().program_set_digest.data(), 32);
        return succeed();
    });
}

void* nvcr_sm100_stream(const nvcr_sm100_executor* executor) {
    return executor == nullptr ? nullptr : static_cast<void*>(executor->executor->stream());
}

int nvcr_sm100_last_launch_count(const nvcr_sm100_executor* executor) {
    return executor == nullptr ? 0 : executor->executor->launches_last_run();
}

size_t nvcr_sm100_workspace_bytes(const nvcr_sm100_executor* executor) {
    return executor == nullptr ? 0 : executor->executor->workspace_bytes();
}

int nvcr_sm100_set_profiling(nvcr_sm100_executor* executor, int enabled) {
    if (executor == nullptr) return report(Code::invalid_argument, "null executor");
    executor->executor->set_profiling(enabled != 0);
    return succeed();
}

int nvcr_sm100_profile(nvcr_sm100_executor* executor, nvcr_sm100_step_time* steps, size_t capacity, size_t* count) {
    return guarded([&] {
        if (executor == nullptr || count == nullptr) return report(Code::invalid_argument, "null argument");
        auto timings = executor->executor->profile();
        if (!timings) return report(timings.error());
        *count = timings.value().size();
        for (size_t i = 0; i < timings.value().size() && i < capacity && steps != nullptr; ++i) {
            const auto& t = timings.value()[i];
            std::snprintf(steps[i].label, sizeof(steps[i].label), "%s", t.label.c_str());
            std::snprintf(steps[i].kernel, sizeof(steps[i].kernel), "%s", t.kernel.c_str());
            steps[i].milliseconds = t.milliseconds;
            steps[i].algorithmic_ops = t.algorithmic_ops;
            steps[i].algorithmic_bytes = t.algorithmic_bytes;
        }
        return succeed();
    });
}

int nvcr_sm100_fx_program_load(const char* directory, const char* stage, nvcr_sm100_fx_program** program) {
    return guarded([&] {
        if (directory == nullptr || stage == nullptr || program == nullptr) {
            return report(Code::invalid_argument, "null argument");
        }
        *program = nullptr;
        auto loaded = nvcr_sm100::fx::load_fx_program(directory, stage);
        if (!loaded) return report(loaded.error());
        *program = new nvcr_sm100_fx_program{std::move(loaded.value())};
        return succeed();
    });
}

void nvcr_sm100_fx_program_destroy(nvcr_sm100_fx_program* program) { delete program; }

int nvcr_sm100_fx_program_digest(const char* directory, const char* stage, char* digest_hex) {
    return guarded([&] {
        if (directory == nullptr || stage == nullptr || digest_hex == nullptr) {
            return report(Code::invalid_argument, "null argument");
        }
        auto digest = nvcr_sm100::fx::fx_program_digest(directory, stage);
        if (!digest) return report(digest.error());
        std::memcpy(digest_hex, digest.value().c_str(), digest.value().size() + 1);
        return succeed();
    });
}

int nvcr_sm100_fx_program_summary(const nvcr_sm100_fx_program* program, size_t* tensor_count, size_t* node_count,
                                  size_t* input_count, size_t* output_count, char* digest_hex) {
    if (program == nullptr || tensor_count == nullptr || node_count == nullptr || input_count == nullptr ||
        output_count == nullptr || digest_hex == nullptr) {
        return report(Code::invalid_argument, "null argument");
    }
    const auto& p = program->program;
    *tensor_count = p.tensor_names.size();
    *node_count = p.nodes.size();
    *input_count = p.inputs.size();
    *output_count = p.outputs.size();
    std::memcpy(digest_hex, p.digest_hex.c_str(), p.digest_hex.size() + 1);
    return succeed();
}

int nvcr_sm100_fx_program_node(const nvcr_sm100_fx_program* program, size_t index, const char** op,
                               size_t* input_count, uint32_t* output) {
    if (program == nullptr || op == nullptr || input_count == nullptr || output == nullptr) {
        return report(Code::invalid_argument, "null argument");
    }
    if (index >= program->program.nodes.size()) return report(Code::invalid_argument, "node index out of range");
    const auto& node = program->program.nodes[index];
    *op = nvcr_sm100::fx::op_name(node.op);
    *input_count = node.inputs.size();
    *output = node.output;
    return succeed();
}

int nvcr_sm100_fx_program_tensor(const nvcr_sm100_fx_program* program, int is_output, size_t index,
                                 const char** name, int32_t* channels) {
    if (program == nullptr || name == nullptr || channels == nullptr) {
        return report(Code::invalid_argument, "null argument");
    }
    const auto& p = program->program;
    const auto& ids = is_output ? p.outputs : p.inputs;
    if (index >= ids.size()) return report(Code::invalid_argument, "tensor index out of range");
    *name = p.tensor_names[ids[index]].c_str();
    *channels = p.tensor_channels[ids[index]];
    return succeed();
}

int nvcr_sm100_fx_executor_create(const nvcr_sm100_fx_program* program, void* stream,
                                   nvcr_sm100_fx_executor** executor) {
    return guarded([&] {
        if (program == nullptr || executor == nullptr) return report(Code::invalid_argument, "null argument");
        *executor = nullptr;
        auto created = nvcr_sm100::fx::FxExecutor::create(program->program, static_cast<cudaStream_t>(stream));
        if (!created) return report(created.error());
        *executor = new nvcr_sm100_fx_executor{std::move(created.value())};
        return succeed();
    });
}

void nvcr_sm100_fx_executor_destroy(nvcr_sm100_fx_executor* executor) { delete executor; }

namespace {

std::vector<nvcr_sm100::fx::FxExtent> fx_extents(const int32_t* extents, size_t count) {
    std::vector<nvcr_sm100::fx::FxExtent> out(count);
    for (size_t i = 0; i < count; ++i) out[i] = {extents[3 * i], extents[3 * i + 1], extents[3 * i + 2]};
    return out;
}

}  // namespace

int nvcr_sm100_fx_infer_output_extents(nvcr_sm100_fx_executor* executor, const int32_t* input_extents,
                                       size_t input_count, int32_t* output_extents, size_t output_count) {
    return guarded([&] {
        if (executor == nullptr || (input_count > 0 && input_extents == nullptr) ||
            (output_count > 0 && output_extents == nullptr)) {
            return report(Code::invalid_argument, "null argument");
        }
        auto inferred = executor->executor->infer_output_extents(fx_extents(input_extents, input_count));
        if (!inferred) return report(inferred.error());
        if (inferred.value().size() != output_count) return report(Code::invalid_argument, "wrong number of outputs");
        for (size_t i = 0; i < output_count; ++i) {
            output_extents[3 * i] = inferred.value()[i].channels;
            output_extents[3 * i + 1] = inferred.value()[i].height;
            output_extents[3 * i + 2] = inferred.value()[i].width;
        }
        return succeed();
    });
}

int nvcr_sm100_fx_run(nvcr_sm100_fx_executor* executor, const int32_t* const* inputs, const int32_t* input_extents,
                      size_t input_count, int32_t* const* outputs, size_t output_count, int device_memory) {
    return guarded([&] {
        if (executor == nullptr || (input_count > 0 && (inputs == nullptr || input_extents == nullptr)) ||
            (output_count > 0 && outputs == nullptr)) {
            return report(Code::invalid_argument, "null argument");
        }
        std::vector<const std::int32_t*> in(inputs, inputs + input_count);
        std::vector<std::int32_t*> out(outputs, outputs + output_count);
        auto ran = executor->executor->run(in, fx_extents(input_extents, input_count), out, device_memory != 0);
        if (!ran) return report(ran.error());
        return succeed();
    });
}

int nvcr_sm100_fx_last_launch_count(const nvcr_sm100_fx_executor* executor) {
    return executor == nullptr ? -1 : executor->executor->last_launch_count();
}

namespace {

int glue_status(cudaError_t status, const char* refusal) {
    if (status == cudaErrorInvalidValue) return report(Code::invalid_argument, refusal);
    if (status != cudaSuccess) return report(Code::backend_error, cudaGetErrorString(status));
    return succeed();
}

}  // namespace

int nvcr_sm100_dcvc_build_decode_indexes(const uint16_t* scales, uint8_t* indexes, size_t count,
                                         float force_zero_threshold, void* stream) {
    return glue_status(nvcr_sm100::glue::build_decode_indexes(scales, indexes, count, force_zero_threshold,
                                                               static_cast<cudaStream_t>(stream)),
                       "empty or null tensor");
}

int nvcr_sm100_dcvc_build_encode_indexes(const uint16_t* symbols, const uint16_t* scales, int16_t* indexes,
                                         size_t count, float force_zero_threshold, void* stream) {
    return glue_status(nvcr_sm100::glue::build_encode_indexes(symbols, scales, indexes, count, force_zero_threshold,
                                                               static_cast<cudaStream_t>(stream)),
                       "empty or null tensor");
}

int nvcr_sm100_dcvc_make_mask(uint16_t* mask, int32_t batch, int32_t channels, int32_t height, int32_t width,
                              int ways, int stage, void* stream) {
    return glue_status(nvcr_sm100::glue::make_mask(mask, batch, channels, height, width, ways, stage,
                                                   static_cast<cudaStream_t>(stream)),
                       "mask shape, ways or stage invalid");
}

int nvcr_sm100_dcvc_restore(const uint16_t* symbols, const uint16_t* means, const uint16_t* mask, uint16_t* output,
                            int32_t batch, int32_t channels, int32_t height, int32_t width, int ways, void* stream) {
    return glue_status(nvcr_sm100::glue::restore(symbols, means, mask, output, batch, channels, height, width, ways,
                                                 static_cast<cudaStream_t>(stream)),
                       "restore shape or ways invalid");
}

int nvcr_sm100_dcvc_process_with_mask(const uint16_t* values, const uint16_t* scales, const uint16_t* means,
                                      const uint16_t* mask, uint16_t* residual, uint16_t* symbols,
                                      uint16_t* reconstructed, uint16_t* masked_scales, size_t count,
                                      float force_zero_threshold, void* stream) {
    return glue_status(nvcr_sm100::glue::process_with_mask(values, scales, means, mask, residual, symbols, reconstructed,
                                                            masked_scales, count, force_zero_threshold,
                                                            static_cast<cudaStream_t>(stream)),
                       "empty or null tensor");
}

int nvcr_sm100_dcvc_reduce(const uint16_t* input, const uint16_t* mask, uint16_t* output, int32_t batch,
                           int32_t channels, int32_t height, int32_t width, int ways, void* stream) {
    return glue_status(nvcr_sm100::glue::reduce(input, mask, output, batch, channels, height, width, ways,
                                                static_cast<cudaStream_t>(stream)),
                       "reduce shape or ways invalid");
}

namespace {

int glue_pointwise(nvcr_sm100::glue::PointwiseOp op, uint16_t* a, uint16_t* b, const uint16_t* c, int8_t* q,
                   size_t count, float scalar, size_t spatial_count, void* stream) {
    return glue_status(nvcr_sm100::glue::pointwise(op, a, b, c, q, count, scalar, spatial_count,
                                                   static_cast<cudaStream_t>(stream)),
                       "empty or null tensor");
}

}  // namespace

int nvcr_sm100_dcvc_round_to_int8(uint16_t* values, int8_t* quantized, size_t count, void* stream) {
    return glue_pointwise(nvcr_sm100::glue::PointwiseOp::round_to_int8, values, nullptr, nullptr, quantized, count, 0.0f,
                          0, stream);
}

int nvcr_sm100_dcvc_int8_to_half(const int8_t* values, uint16_t* output, size_t count, void* stream) {
    return glue_pointwise(nvcr_sm100::glue::PointwiseOp::int8_to_half, output, nullptr, nullptr,
                          const_cast<int8_t*>(values), count, 0.0f, 0, stream);
}

int nvcr_sm100_dcvc_clamp_min(uint16_t* values, size_t count, float minimum, void* stream) {
    return glue_pointwise(nvcr_sm100::glue::PointwiseOp::clamp_min, values, nullptr, nullptr, nullptr, count, minimum, 0,
                          stream);
}

int nvcr_sm100_dcvc_clamp_reciprocal_with_quant(uint16_t* quant_step, uint16_t* values, size_t count, void* stream) {
    return glue_pointwise(nvcr_sm100::glue::PointwiseOp::clamp_reciprocal_with_quant, quant_step, values, nullptr,
                          nullptr, count, 0.0f, 0, stream);
}

int nvcr_sm100_dcvc_add_in_place(uint16_t* first, const uint16_t* second, size_t count, void* stream) {
    return glue_pointwise(nvcr_sm100::glue::PointwiseOp::add_in_place, first, const_cast<uint16_t*>(second), nullptr,
                          nullptr, count, 0.0f, 0, stream);
}

int nvcr_sm100_dcvc_multiply_broadcast(uint16_t* values, const uint16_t* factors, size_t spatial_count,
                                       int32_t channels, void* stream) {
    if (channels <= 0) return report(Code::invalid_argument, "channels must be positive");
    return glue_pointwise(nvcr_sm100::glue::PointwiseOp::multiply_broadcast, values, const_cast<uint16_t*>(factors),
                          nullptr, nullptr, spatial_count * static_cast<size_t>(channels), 0.0f, spatial_count, stream);
}

int nvcr_sm100_dcvc_add_and_multiply(uint16_t* first, const uint16_t* second, const uint16_t* quant_step, size_t count,
                                     void* stream) {
    return glue_pointwise(nvcr_sm100::glue::PointwiseOp::add_and_multiply, first, const_cast<uint16_t*>(second),
                          quant_step, nullptr, count, 0.0f, 0, stream);
}

int nvcr_sm100_dcvc_replicate_pad(const uint16_t* input, uint16_t* output, int32_t batch, int32_t channels,
                                  int32_t height, int32_t width, int32_t padded_height, int32_t padded_width,
                                  void* stream) {
    return glue_status(nvcr_sm100::glue::replicate_pad(input, output, batch, channels, height, width, padded_height,
                                                       padded_width, static_cast<cudaStream_t>(stream)),
                       "pad shape invalid");
}

int nvcr_sm100_dcvc_crop_spatial(const uint16_t* input, uint16_t* output, int32_t batch, int32_t channels,
                                 int32_t height, int32_t width, int32_t out_height, int32_t out_width, void* stream) {
    return glue_status(nvcr_sm100::glue::crop_spatial(input, output, batch, channels, height, width, out_height,
                                                      out_width, static_cast<cudaStream_t>(stream)),
                       "crop shape invalid");
}

int nvcr_sm100_dcvc_rgb24_to_ycbcr_padded(const uint8_t* input, int32_t width, int32_t height, uint16_t* output,
                                          int32_t padded_height, int32_t padded_width, void* stream) {
    return glue_status(nvcr_sm100::glue::to_ycbcr_padded(input, width, height, output, padded_height, padded_width,
                                                         false, static_cast<cudaStream_t>(stream)),
                       "picture size invalid");
}

int nvcr_sm100_dcvc_yuv420p8_to_ycbcr_padded(const uint8_t* input, int32_t width, int32_t height, uint16_t* output,
                                             int32_t padded_height, int32_t padded_width, void* stream) {
    return glue_status(nvcr_sm100::glue::to_ycbcr_padded(input, width, height, output, padded_height, padded_width,
                                                         true, static_cast<cudaStream_t>(stream)),
                       "picture size invalid");
}

int nvcr_sm100_dcvc_ycbcr_padded_to_yuv420p8(const uint16_t* input, int32_t batch, int32_t channels, int32_t height,
                                             int32_t width, int32_t visible_width, int32_t visible_height,
                                             uint8_t* output, void* stream) {
    return glue_status(nvcr_sm100::glue::ycbcr_padded_to_yuv420p8(input, batch, channels, height, width, visible_width,
                                                                  visible_height, output,
                                                                  static_cast<cudaStream_t>(stream)),
                       "picture size invalid");
}

}  // extern "C"
