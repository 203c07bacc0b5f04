// The sm_100a execution provider (see sm100_session.hpp): an IProviderSession
// over libnvcr_sm100's C ABI for nvcr.intconv.v1 stages.
#include "sm100_session.hpp"

#include "nvcr/runtime/registry.hpp"
#include "nvcr_sm100.h"

#include <cuda_runtime.h>

#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <mutex>
#include <string>
#include <vector>

namespace nvcr::provider::sm100 {
namespace {

namespace api = nvcr::provider::experimental;
constexpr const char* subsystem = "provider.sm100";
constexpr const char* intconv = "nvcr.intconv.v1";

Error from_status(int status) {  // status = 1 + nvcr::ErrorCode
    char message[512] = {};
    nvcr_sm100_last_error(message, sizeof(message));
    return Error(static_cast<ErrorCode>(status - 1), message, subsystem);
}

Error failure(ErrorCode code, std::string message) { return Error(code, std::move(message), subsystem); }

Error cuda_failure(const char* what, cudaError_t status) {
    return failure(ErrorCode::backend_error, std::string(what) + ": " + cudaGetErrorString(status));
}

std::string hex(const std::vector<std::byte>& bytes) {
    static const char digits[] = "0123456789abcdef";
    std::string out;
    for (const std::byte b : bytes) {
        out.push_back(digits[static_cast<unsigned>(b) >> 4]);
        out.push_back(digits[static_cast<unsigned>(b) & 15u]);
    }
    return out;
}

// Storage of one allocate() call: device memory, pinned host memory or plain
// host memory, freed with the last handle.
class Buffer final : public api::IProviderBuffer {
public:
    Buffer(void* data, std::size_t size, api::MemoryDomain domain, std::string owner)
        : data_(data), size_(size), domain_(domain), owner_(std::move(owner)) {}
    ~Buffer() override {
        switch (domain_) {
        case api::MemoryDomain::provider_device: cudaFree(data_); break;
        case api::MemoryDomain::pinned_host: cudaFreeHost(data_); break;
        case api::MemoryDomain::host: std::free(data_); break;
        }
    }
    std::size_t size_bytes() const noexcept override { return size_; }
    api::MemoryDomain domain() const noexcept override { return domain_; }
    std::string_view owner_id() const noexcept override { return owner_; }
    std::span<std::byte> host_bytes() noexcept override {
        if (domain_ == api::MemoryDomain::provider_device) return {};
        return {static_cast<std::byte*>(data_), size_};
    }
    void* data() const { return data_; }

private:
    void* data_;
    std::size_t size_;
    api::MemoryDomain domain_;
    std::string owner_;
};

// A loaded nvcr.intconv.v1 stage: its descriptor and the executor (which holds
// the digest-checked program and its quantised weights on the device).
class Stage final : public api::IExecutableStage {
public:
    Stage(api::ExecutableStageDescriptor descriptor, std::string owner, nvcr_sm100_executor* executor)
        : descriptor_(std::move(descriptor)), owner_(std::move(owner)), executor_(executor) {}
    ~Stage() override { nvcr_sm100_executor_destroy(executor_); }
    const api::ExecutableStageDescriptor& descriptor() const noexcept override { return descriptor_; }
    std::string_view owner_id() const noexcept override { return owner_; }
    nvcr_sm100_executor* executor() const { return executor_; }

private:
    api::ExecutableStageDescriptor descriptor_;
    std::string owner_;
    nvcr_sm100_executor* executor_;
};

// An event recorded on the session's stream after a submission; for host
// buffers the copies back are in front of it.
class Completion final : public api::ICompletion {
public:
    Completion(std::string owner, cudaEvent_t event, nvcr_sm100_executor* executor)
        : owner_(std::move(owner)), event_(event), executor_(executor) {}
    ~Completion() override {
        if (event_ != nullptr) cudaEventDestroy(event_);
    }
    std::string_view owner_id() const noexcept override { return owner_; }
    bool ready() const noexcept override { return event_ == nullptr || cudaEventQuery(event_) == cudaSuccess; }
    Result<void> wait() override {
        if (event_ != nullptr) {
            const cudaError_t status = cudaEventSynchronize(event_);
            if (status != cudaSuccess) return cuda_failure("cudaEventSynchronize", status);
        }
        // A device-side wait of the executor's kernels that gave up is reported here.
        if (executor_ != nullptr) {
            if (const int status = nvcr_sm100_synchronize(executor_); status != NVCR_SM100_OK) {
                return from_status(status);
            }
        }
        return {};
    }
    cudaEvent_t event() const { return event_; }

private:
    std::string owner_;
    cudaEvent_t event_;
    nvcr_sm100_executor* executor_;
};

std::atomic<unsigned long long> session_counter{0};

class Session final : public api::IProviderSession {
public:
    Session() : owner_("sm100-session-" + std::to_string(++session_counter)) {}
    ~Session() override {
        if (stream_ != nullptr) {
            cudaStreamSynchronize(stream_);
            cudaStreamDestroy(stream_);
        }
    }

    std::string_view owner_id() const noexcept override { return owner_; }

    bool supports_numerics_profile(std::string_view profile) const noexcept override {
        return nvcr_sm100_supports_profile(std::string(profile).c_str()) == 1;
    }

    Result<api::BufferHandle> allocate(std::size_t size_bytes, api::MemoryDomain domain) override {
        void* data = nullptr;
        cudaError_t status = cudaSuccess;
        switch (domain) {
        case api::MemoryDomain::provider_device: status = cudaMalloc(&data, size_bytes == 0 ? 1 : size_bytes); break;
        case api::MemoryDomain::pinned_host: status = cudaMallocHost(&data, size_bytes == 0 ? 1 : size_bytes); break;
        case api::MemoryDomain::host:
            data = std::malloc(size_bytes == 0 ? 1 : size_bytes);
            if (data == nullptr) return failure(ErrorCode::resource_exhausted, "host buffer allocation failed");
            break;
        }
        if (status != cudaSuccess) {
            return failure(ErrorCode::resource_exhausted, std::string("buffer allocation: ") + cudaGetErrorString(status));
        }
        return api::BufferHandle(std::make_shared<Buffer>(data, size_bytes, domain, owner_));
    }

    Result<api::ExecutableStage> load_stage(api::ExecutableStageDescriptor descriptor) override {
        int normative = 0;
        if (const int status = nvcr_sm100_is_normative(descriptor.numerics_profile.c_str(), &normative)) {
            return from_status(status);  // a profile this provider does not know: incompatible_precision
        }
        if (!normative) {
            return failure(ErrorCode::incompatible_precision,
                           descriptor.stage_id + " is a native stage; this provider runs only " + intconv + " stages");
        }
        if (!supports_numerics_profile(descriptor.numerics_profile)) {
            return failure(ErrorCode::incompatible_precision,
                           descriptor.stage_id + " requires " + descriptor.numerics_profile +
                               ", which needs an sm_100 device here");
        }
        if (auto ready = ensure_stream(); !ready) return ready.error();
        nvcr_sm100_executor* executor = nullptr;
        const std::string digest = hex(descriptor.artifact.expected_digest);
        if (const int status = nvcr_sm100_load_normative(descriptor.artifact.path.c_str(),
                                                         descriptor.artifact.component_id.c_str(), digest.c_str(),
                                                         stream_, &executor)) {
            return from_status(status);
        }
        return api::ExecutableStage(std::make_shared<const Stage>(std::move(descriptor), owner_, executor));
    }

    Result<api::Completion> submit(const api::ExecutableStage& stage, std::span<const api::TensorView> tensors,
                                   std::span<const api::ExecutionDependency> dependencies) override {
        auto exact = std::dynamic_pointer_cast<const Stage>(stage);
        if (!exact || exact->owner_id() != owner_) {
            return failure(ErrorCode::invalid_argument, "the stage belongs to another provider session");
        }
        for (const auto& dependency : dependencies) {
            auto done = std::dynamic_pointer_cast<Completion>(dependency.completion);
            if (!done || done->owner_id() != owner_) {
                return failure(ErrorCode::invalid_argument, "a dependency belongs to another provider session");
            }
            // Same stream: its work is already ordered before this submission.
        }
        // Views and, for host buffers, device staging copies.
        struct Bound {
            std::string name;
            nvcr_sm100_tensor view;
            Buffer* buffer;
            std::size_t offset;
            std::size_t bytes;
            bool output;
            bool staged;
        };
        std::vector<Bound> bound;
        bound.reserve(tensors.size());
        std::size_t staging_bytes = 0;
        for (const auto& tensor : tensors) {
            auto* buffer = dynamic_cast<Buffer*>(tensor.storage.buffer.get());
            if (tensor.data_type != api::TensorDataType::float16 || buffer == nullptr || buffer->owner_id() != owner_) {
                return failure(ErrorCode::invalid_argument,
                               "normative tensor " + std::string(tensor.name) + " must be an FP16 buffer of this session");
            }
            if (tensor.shape.size() != 4 || tensor.shape[0] != 1 || tensor.shape[1] <= 0 || tensor.shape[2] <= 0 ||
                tensor.shape[3] <= 0 || tensor.shape[1] > INT32_MAX || tensor.shape[2] > INT32_MAX ||
                tensor.shape[3] > INT32_MAX) {
                return failure(ErrorCode::invalid_argument,
                               "normative tensor " + std::string(tensor.name) + " must be a batch-1 NCHW tensor");
            }
            const std::size_t bytes = 2u * static_cast<std::size_t>(tensor.shape[1]) *
                static_cast<std::size_t>(tensor.shape[2]) * static_cast<std::size_t>(tensor.shape[3]);
            const std::size_t offset = tensor.storage.offset_bytes;
            if (offset > buffer->size_bytes() || tensor.storage.size_bytes > buffer->size_bytes() - offset ||
                tensor.storage.size_bytes != bytes || offset % 16 != 0) {
                return failure(ErrorCode::invalid_argument,
                               "normative tensor " + std::string(tensor.name) + " is out of bounds or misaligned");
            }
            const bool staged = buffer->domain() != api::MemoryDomain::provider_device;
            if (staged) staging_bytes += (bytes + 255) / 256 * 256;
            bound.push_back({std::string(tensor.name),
                             {nullptr, static_cast<std::int32_t>(tensor.shape[1]),
                              static_cast<std::int32_t>(tensor.shape[2]), static_cast<std::int32_t>(tensor.shape[3]),
                              static_cast<std::byte*>(buffer->data()) + offset},
                             buffer, offset, bytes, tensor.access != api::TensorAccess::read, staged});
        }
        if (auto ready = ensure_stream(); !ready) return ready.error();
        if (auto grown = ensure_staging(staging_bytes); !grown) return grown.error();
        std::size_t cursor = 0;
        std::vector<nvcr_sm100_tensor> inputs, outputs;
        for (auto& b : bound) {
            b.view.name = b.name.c_str();
            if (b.staged) {
                void* device = static_cast<std::byte*>(staging_) + cursor;
                cursor += (b.bytes + 255) / 256 * 256;
                if (!b.output) {
                    const cudaError_t status =
                        cudaMemcpyAsync(device, b.view.data, b.bytes, cudaMemcpyHostToDevice, stream_);
                    if (status != cudaSuccess) return cuda_failure("cudaMemcpyAsync", status);
                }
                b.view.data = device;
            }
            (b.output ? outputs : inputs).push_back(b.view);
        }
        if (const int status =
                nvcr_sm100_run_half(exact->executor(), inputs.data(), inputs.size(), outputs.data(), outputs.size())) {
            return from_status(status);
        }
        for (const auto& b : bound) {
            if (!b.staged || !b.output) continue;
            void* host = static_cast<std::byte*>(b.buffer->data()) + b.offset;
            const cudaError_t status = cudaMemcpyAsync(host, b.view.data, b.bytes, cudaMemcpyDeviceToHost, stream_);
            if (status != cudaSuccess) return cuda_failure("cudaMemcpyAsync", status);
        }
        cudaEvent_t event = nullptr;
        cudaError_t status = cudaEventCreateWithFlags(&event, cudaEventDisableTiming);
        if (status == cudaSuccess) status = cudaEventRecord(event, stream_);
        if (status != cudaSuccess) {
            if (event != nullptr) cudaEventDestroy(event);
            return cuda_failure("cudaEventRecord", status);
        }
        auto completion = std::make_shared<Completion>(owner_, event, exact->executor());
        // Host staging buffers are reused by the next submission, so a submission
        // with host buffers completes before it returns, as the CPU provider does.
        if (staging_bytes > 0) {
            auto waited = completion->wait();
            if (!waited) return waited.error();
        }
        return api::Completion(completion);
    }

    Result<void> reset() override {
        if (stream_ != nullptr) {
            const cudaError_t status = cudaStreamSynchronize(stream_);
            if (status != cudaSuccess) return cuda_failure("cudaStreamSynchronize", status);
        }
        return {};
    }

private:
    Result<void> ensure_stream() {
        if (stream_ != nullptr) return {};
        const cudaError_t status = cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking);
        if (status != cudaSuccess) return cuda_failure("cudaStreamCreate", status);
        return {};
    }
    Result<void> ensure_staging(std::size_t bytes) {
        if (bytes <= staging_bytes_) return {};
        if (staging_ != nullptr) {
            cudaStreamSynchronize(stream_);
            cudaFree(staging_);
            staging_ = nullptr;
            staging_bytes_ = 0;
        }
        const cudaError_t status = cudaMalloc(&staging_, bytes);
        if (status != cudaSuccess) return failure(ErrorCode::resource_exhausted, "device staging allocation failed");
        staging_bytes_ = bytes;
        return {};
    }

    std::string owner_;
    cudaStream_t stream_{nullptr};
    void* staging_{nullptr};
    std::size_t staging_bytes_{0};
};

}  // namespace

Result<std::shared_ptr<experimental::IProviderSession>> create_session() {
    return std::shared_ptr<experimental::IProviderSession>(std::make_shared<Session>());
}

void* device_address(const experimental::IProviderBuffer& buffer) noexcept {
    const auto* own = dynamic_cast<const Buffer*>(&buffer);
    return own != nullptr && own->domain() == api::MemoryDomain::provider_device ? own->data() : nullptr;
}

void register_provider() {
    runtime::ProviderEntry entry;
    entry.descriptor.kind = ProviderKind::cuda_fused;
    entry.descriptor.id = "sm100";
    entry.descriptor.version = "1";
    entry.descriptor.display_name = "NVIDIA sm_100a exact-numerics executor (nvcr.intconv.v1)";
    entry.capabilities.supports_fp16 = true;
    entry.capabilities.supports_int8 = true;
    entry.capabilities.supports_dynamic_shapes = true;
    entry.capabilities.supports_cuda_graphs = true;
    entry.capabilities.target_device = "NVIDIA B200 (sm_100)";
    entry.session_factory = [](const RuntimeConfiguration&) { return create_session(); };
    runtime::Registry::instance().register_provider(std::move(entry));
}

}  // namespace nvcr::provider::sm100
