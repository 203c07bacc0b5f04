// C entry points over the reference's own CUDA executor (CudaExecutor,
// src/deterministic/cuda_executor.{hpp,cu}), the GPU comparator the new sm_100a
// path is measured against. TEST AND BENCHMARK INFRASTRUCTURE: compiled by
// oracle/Makefile, with the reference's kernel flags (CMakeLists.txt:243-256:
// -ftz=false -prec-div=true -prec-sqrt=true -fmad=false) for sm_100a, together
// with the reference sources it needs, into oracle/_ref/libnvcr_ref_cuda.so.
// Nothing in the product links or loads it.
//
// Programs reach it through the reference's own loader (load_program), from the
// .detprog.json/.detw files the caller writes; runs go through its public
// run_half on FP16 device tensors, the path its TensorRT provider takes
// (src/provider/tensorrt/session.cpp:1549-1594).
#include "deterministic/cuda_executor.hpp"
#include "deterministic/program.hpp"

#include <cuda_runtime.h>

#include <cstdio>
#include <memory>
#include <string>
#include <string_view>
#include <vector>

namespace det = nvcr::deterministic;

namespace {

struct Handle {
    std::unique_ptr<det::Program> program;  // must outlive the executor
    std::unique_ptr<det::CudaExecutor> executor;
};

void write_error(char* buffer, std::size_t size, std::string_view message) {
    if (buffer == nullptr || size == 0) return;
    std::snprintf(buffer, size, "%.*s", static_cast<int>(message.size()), message.data());
}

std::vector<det::HalfDeviceTensor> views(int count, const char* const* names, const std::int32_t* extents,
                                         void* const* data) {
    std::vector<det::HalfDeviceTensor> out;
    for (int i = 0; i < count; ++i) {
        out.push_back({names[i], det::Extent{extents[3 * i], extents[3 * i + 1], extents[3 * i + 2]}, data[i]});
    }
    return out;
}

}  // namespace

extern "C" {

// Loads the program and creates the reference's executor on the current
// device, ordered on `stream` (a cudaStream_t, or null for its own stream).
// Returns 0, or the reference's ErrorCode + 1 with its message.
int refgpu_create(const char* program_json, void* stream, void** handle, char* error, std::size_t error_size) {
    auto loaded = det::load_program(program_json);
    if (!loaded) {
        write_error(error, error_size, loaded.error().message());
        return static_cast<int>(loaded.error().code()) + 1;
    }
    auto h = std::make_unique<Handle>();
    h->program = std::make_unique<det::Program>(std::move(loaded.value()));
    auto created = det::CudaExecutor::create(*h->program, static_cast<CUstream_st*>(stream));
    if (!created) {
        write_error(error, error_size, created.error().message());
        return static_cast<int>(created.error().code()) + 1;
    }
    h->executor = std::make_unique<det::CudaExecutor>(std::move(created.value()));
    *handle = h.release();
    return 0;
}

// CudaExecutor::run_half on named NCHW FP16 device tensors (extents c, h, w).
int refgpu_run_half(void* handle, int input_count, const char* const* input_names,
                    const std::int32_t* input_extents, void* const* inputs, int output_count,
                    const char* const* output_names, const std::int32_t* output_extents, void* const* outputs,
                    char* error, std::size_t error_size) {
    auto* h = static_cast<Handle*>(handle);
    const auto in = views(input_count, input_names, input_extents, inputs);
    const auto out = views(output_count, output_names, output_extents, outputs);
    auto status = h->executor->run_half(in, out);
    if (!status) {
        write_error(error, error_size, status.error().message());
        return static_cast<int>(status.error().code()) + 1;
    }
    return 0;
}

void refgpu_destroy(void* handle) { delete static_cast<Handle*>(handle); }

}  // extern "C"
