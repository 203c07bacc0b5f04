// C entry points over the sm_100a provider session (nvcr_b200/provider), for
// the tests in tests/test_provider.py. TEST INFRASTRUCTURE: built by
// nvcr_b200/provider/build.py together with the provider and the reference's
// registry and error sources it needs, into
// nvcr_b200/provider/_build/libnvcr_sm100_provider.so.
//
// Each call builds its own session (or uses the registry's factory), so a test
// sees exactly the provider boundary the reference's runtime would use.
#include "sm100_session.hpp"

#include "nvcr/runtime/registry.hpp"

#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

namespace api = nvcr::provider::experimental;

namespace {

void write_message(char* buffer, std::size_t size, std::string_view message) {
    if (buffer == nullptr || size == 0) return;
    std::snprintf(buffer, size, "%.*s", static_cast<int>(message.size()), message.data());
}

int report(const nvcr::Error& error, char* message, std::size_t size) {
    write_message(message, size, error.message());
    return static_cast<int>(error.code()) + 1;
}

api::ExecutableStageDescriptor descriptor(const char* directory, const char* component, const unsigned char* digest,
                                          const char* profile) {
    api::ExecutableStageDescriptor d;
    d.stage_id = component;
    d.artifact.component_id = component;
    d.artifact.path = directory;
    d.artifact.provider_id = "sm100";
    if (digest != nullptr) {
        for (int i = 0; i < 32; ++i) d.artifact.expected_digest.push_back(static_cast<std::byte>(digest[i]));
    }
    d.numerics_profile = profile != nullptr ? profile : "";
    return d;
}

}  // namespace

extern "C" {

// supports_numerics_profile of a fresh session.
int ph_supports(const char* profile) {
    auto session = nvcr::provider::sm100::create_session();
    return session && session.value()->supports_numerics_profile(profile) ? 1 : 0;
}

// load_stage on a fresh session: 0, or the refusal's ErrorCode + 1.
int ph_load(const char* directory, const char* component, const unsigned char* digest, const char* profile,
            char* message, std::size_t size) {
    auto session = nvcr::provider::sm100::create_session();
    if (!session) return report(session.error(), message, size);
    auto stage = session.value()->load_stage(descriptor(directory, component, digest, profile));
    if (!stage) return report(stage.error(), message, size);
    return 0;
}

// Registers the provider and checks the registry finds it and its session
// factory builds a session that claims nvcr.intconv.v1 exactly when the
// library does. 0 on success.
int ph_registry(char* message, std::size_t size) {
    nvcr::provider::sm100::register_provider();
    auto entry = nvcr::runtime::Registry::instance().find_provider("sm100");
    if (!entry) {
        write_message(message, size, "not registered");
        return 1;
    }
    if (!entry->session_factory) {
        write_message(message, size, "no session factory");
        return 2;
    }
    nvcr::RuntimeConfiguration configuration{};
    auto session = entry->session_factory(configuration);
    if (!session) return report(session.error(), message, size);
    write_message(message, size, entry->descriptor.display_name);
    return session.value()->supports_numerics_profile("nvcr.fx.v1") ? 3 : 0;
}

// One stage through load_stage and submit: FP16 inputs and outputs as host
// arrays, the session's buffers in `domain` (0 host, 1 pinned host, 2 device;
// device buffers are filled and read with cudaMemcpy here). Shapes are
// (c, h, w) per tensor. 0, or ErrorCode + 1.
int ph_run(const char* directory, const char* component, const unsigned char* digest, int input_count,
           const char* const* input_names, const std::int32_t* input_shapes, const std::uint16_t* const* inputs,
           int output_count, const char* const* output_names, const std::int32_t* output_shapes,
           std::uint16_t* const* outputs, int domain, int repeats, char* message, std::size_t size);

}  // extern "C"

int ph_run(const char* directory, const char* component, const unsigned char* digest, int input_count,
           const char* const* input_names, const std::int32_t* input_shapes, const std::uint16_t* const* inputs,
           int output_count, const char* const* output_names, const std::int32_t* output_shapes,
           std::uint16_t* const* outputs, int domain, int repeats, char* message, std::size_t size) {
    auto created = nvcr::provider::sm100::create_session();
    if (!created) return report(created.error(), message, size);
    auto session = created.value();
    auto stage = session->load_stage(descriptor(directory, component, digest, "nvcr.intconv.v1"));
    if (!stage) return report(stage.error(), message, size);
    const auto memory = domain == 2 ? api::MemoryDomain::provider_device
        : domain == 1                ? api::MemoryDomain::pinned_host
                                     : api::MemoryDomain::host;
    struct Slot {
        api::BufferHandle buffer;
        std::size_t bytes;
    };
    std::vector<Slot> slots;
    std::vector<api::TensorView> views;
    auto add = [&](const char* name, const std::int32_t* shape, bool output) -> int {
        const std::size_t bytes = 2u * static_cast<std::size_t>(shape[0]) * shape[1] * shape[2];
        auto buffer = session->allocate(bytes, memory);
        if (!buffer) return report(buffer.error(), message, size);
        slots.push_back({buffer.value(), bytes});
        api::TensorView view;
        view.name = name;
        view.data_type = api::TensorDataType::float16;
        view.shape = {1, shape[0], shape[1], shape[2]};
        view.access = output ? api::TensorAccess::write : api::TensorAccess::read;
        view.storage = {buffer.value(), 0, bytes};
        views.push_back(std::move(view));
        return 0;
    };
    for (int i = 0; i < input_count; ++i) {
        if (int s = add(input_names[i], input_shapes + 3 * i, false)) return s;
        auto& slot = slots.back();
        if (memory == api::MemoryDomain::provider_device) {
            void* device = nvcr::provider::sm100::device_address(*slot.buffer);
            const cudaError_t status = cudaMemcpy(device, inputs[i], slot.bytes, cudaMemcpyHostToDevice);
            if (status != cudaSuccess) {
                write_message(message, size, cudaGetErrorString(status));
                return static_cast<int>(nvcr::ErrorCode::backend_error) + 1;
            }
            continue;
        }
        std::memcpy(slot.buffer->host_bytes().data(), inputs[i], slot.bytes);
    }
    for (int i = 0; i < output_count; ++i) {
        if (int s = add(output_names[i], output_shapes + 3 * i, true)) return s;
    }
    for (int r = 0; r < repeats; ++r) {
        auto done = session->submit(stage.value(), views, {});
        if (!done) return report(done.error(), message, size);
        auto waited = done.value()->wait();
        if (!waited) return report(waited.error(), message, size);
    }
    for (int i = 0; i < output_count; ++i) {
        const auto& slot = slots[static_cast<std::size_t>(input_count + i)];
        if (memory == api::MemoryDomain::provider_device) {
            const cudaError_t status = cudaMemcpy(outputs[i], nvcr::provider::sm100::device_address(*slot.buffer),
                                                  slot.bytes, cudaMemcpyDeviceToHost);
            if (status != cudaSuccess) {
                write_message(message, size, cudaGetErrorString(status));
                return static_cast<int>(nvcr::ErrorCode::backend_error) + 1;
            }
        } else {
            std::memcpy(outputs[i], slot.buffer->host_bytes().data(), slot.bytes);
        }
    }
    auto reset = session->reset();
    if (!reset) return report(reset.error(), message, size);
    return 0;
}
