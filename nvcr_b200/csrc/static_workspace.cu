// nvcr_sm100_run_half_static: run_half for callers that must not allocate
// device memory while they run. A host that enqueues work from a context where
// cudaMalloc is forbidden or unsafe cannot use run_half's first call (which may
// grow the executor's workspace): for example a provider whose enqueue happens
// inside a framework that owns every device allocation, a real-time decode
// thread that must not block on the driver's allocator, or code running while
// another component holds the device at its memory limit. Such a caller
// creates its executor at set-up time, then runs through this entry point,
// which places every scratch tensor of the run (the FP32 intermediates, the
// quantised activation matrices, per-position exponents and correction terms)
// in the fixed device array below instead.
//
// The array is a file-scope static __device__ object of
// NVCR_SM100_STATIC_WORKSPACE_BYTES (64 MiB). Every GPU that loads this code
// holds it until the process exits. Its address is looked up once per device
// with cudaGetSymbolAddress, with that device current, by the first call made
// on the device: make that first call before any stream capture begins. The
// executor's own device (the one current when it was created) must be current
// for every call; with another device current the call is refused with
// NVCR_SM100_INVALID_STATE and nothing is enqueued. All
// calls on a device share the one array and it keeps the previous call's
// contents; every byte a run reads is written earlier in the same run, so
// nothing needs clearing, but two calls whose work overlaps on the GPU (other
// streams, other executors, or other threads) race on it and must be ordered
// by the caller. A run whose plan needs more than the array holds is refused
// with NVCR_SM100_INVALID_ARGUMENT before any work is enqueued.

#include "../../include/nvcr_sm100.h"

#include "capi_internal.hpp"

#include <mutex>
#include <string>

namespace {

static __device__ __align__(256) unsigned char static_workspace[NVCR_SM100_STATIC_WORKSPACE_BYTES];

constexpr int max_devices = 64;
std::mutex setup_lock;
void* workspace_address[max_devices] = {};

int static_report(nvcr_sm100::Code code, const std::string& message) {
    return nvcr_sm100::report_error(nvcr_sm100::Error{code, message});
}

// The device address of static_workspace on the executor's device, looked up
// once. That device must be the current one: cudaGetSymbolAddress answers for
// the current device, and the executor's stream, weights and tensor maps live
// on its own device, so a call made with another device current is refused
// before anything is enqueued.
int workspace_for_device(int executor_device, void** address) {
    int device = 0;
    cudaError_t status = cudaGetDevice(&device);
    if (status != cudaSuccess) return static_report(nvcr_sm100::Code::backend_error, cudaGetErrorString(status));
    if (device != executor_device) {
        return static_report(nvcr_sm100::Code::invalid_state,
                             "the current device (" + std::to_string(device) + ") is not the executor's device (" +
                                 std::to_string(executor_device) + "); make it current before the call");
    }
    if (device < 0 || device >= max_devices) {
        return static_report(nvcr_sm100::Code::invalid_state, "device index outside the static workspace table");
    }
    std::lock_guard<std::mutex> guard(setup_lock);
    if (workspace_address[device] == nullptr) {
        void* pointer = nullptr;
        status = cudaGetSymbolAddress(&pointer, static_workspace);
        if (status != cudaSuccess || pointer == nullptr) {
            return static_report(nvcr_sm100::Code::backend_error,
                                 std::string("cudaGetSymbolAddress(static workspace): ") + cudaGetErrorString(status));
        }
        workspace_address[device] = pointer;
    }
    *address = workspace_address[device];
    return NVCR_SM100_OK;
}

}  // namespace

extern "C" int nvcr_sm100_run_half_static(nvcr_sm100_executor* executor, const nvcr_sm100_tensor* inputs,
                                          size_t input_count, const nvcr_sm100_tensor* outputs, size_t output_count) {
    try {
        if (executor == nullptr || (inputs == nullptr && input_count > 0) || (outputs == nullptr && output_count > 0)) {
            return static_report(nvcr_sm100::Code::invalid_argument, "null executor or tensor array");
        }
        void* workspace = nullptr;
        const int found = workspace_for_device(executor->executor->device(), &workspace);
        if (found != NVCR_SM100_OK) return found;
        std::vector<nvcr_sm100::TensorView> in, out;
        for (size_t i = 0; i < input_count; ++i) {
            in.push_back({inputs[i].name != nullptr ? inputs[i].name : "",
                          {inputs[i].channels, inputs[i].height, inputs[i].width}, inputs[i].data});
        }
        for (size_t i = 0; i < output_count; ++i) {
            out.push_back({outputs[i].name != nullptr ? outputs[i].name : "",
                           {outputs[i].channels, outputs[i].height, outputs[i].width}, outputs[i].data});
        }
        auto status = executor->executor->run_half_in_workspace(in, out, workspace, NVCR_SM100_STATIC_WORKSPACE_BYTES);
        if (!status) return static_report(status.error().code, status.error().message);
        return nvcr_sm100::report_ok();
    } catch (const std::exception& exception) {
        return static_report(nvcr_sm100::Code::internal_error, exception.what());
    }
}
