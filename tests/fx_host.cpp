// Host build of the nvcr.fx.v1 device path, for CPU tests only. TEST
// INFRASTRUCTURE: built by tests/fx_host.py into tests/_build/libfx_host.so;
// the product never links or loads it, and it is no substitute for running the
// kernels on a GPU.
//
// It compiles the product's own fx executor (csrc/fx_executor.cpp: planning,
// value buffers, failure-word decoding), fx program loader and the per-element
// functions the kernels run (csrc/fx_elements.cuh) for the host, and replaces
// what needs a GPU:
//   * the kernel launchers of csrc/fx_kernels.hpp become loops that visit
//     every index the kernel's threads visit and call the same element
//     function (the gemm: every pixel of every four-group tile);
//   * the CUDA runtime calls the executor makes become host stand-ins: device
//     memory is host memory, copies are memcpy, streams complete at once, and
//     the failure word's atomicMin is a plain minimum.
// What it checks: the integers and failures the element functions and the
// executor produce, against the CPU oracle. What it cannot check: launch
// geometry, concurrency, and anything about the GPU itself.
#include "fx_elements.cuh"
#include "fx_executor.hpp"
#include "fx_program.hpp"

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

namespace nvcr_sm100::fx::kernels {
namespace {

namespace el = nvcr_sm100::fx::elements;

struct HostRecord {
    unsigned long long* failure;
    void operator()(unsigned long long key) const {
        if (key < *failure) *failure = key;
    }
};

}  // namespace

cudaError_t check_input(const std::int32_t* x, std::size_t count, unsigned long long position_base,
                        unsigned long long* failure, cudaStream_t) {
    const HostRecord record{failure};
    for (std::size_t i = 0; i < count; ++i) el::check_input(x, i, position_base, record);
    return cudaSuccess;
}

cudaError_t gemm(const GemmArgs& args, unsigned long long node_key, unsigned long long* failure, cudaStream_t) {
    if (args.pixels == 0 || args.groups == 0) return cudaSuccess;
    if (args.in_channels < 1 || (args.group != 1 && args.group != 2 && args.group != 4)) return cudaErrorInvalidValue;
    const HostRecord record{failure};
    for (int g0 = 0; g0 < args.groups; g0 += el::gemm_groups) {
        for (std::size_t p = 0; p < args.pixels; ++p) {
            switch (args.group) {
            case 1: el::gemm_tile<1>(args, p, g0, node_key, record); break;
            case 2: el::gemm_tile<2>(args, p, g0, node_key, record); break;
            default: el::gemm_tile<4>(args, p, g0, node_key, record); break;
            }
        }
    }
    return cudaSuccess;
}

cudaError_t depthwise3x3(const std::int32_t* x, int channels, int height, int width, const std::int32_t* weights,
                         const std::int64_t* bias, const std::int32_t* shifts, std::int32_t* y,
                         unsigned long long node_key, unsigned long long* failure, cudaStream_t) {
    const HostRecord record{failure};
    const std::size_t count = static_cast<std::size_t>(channels) * height * width;
    for (std::size_t i = 0; i < count; ++i) el::depthwise3x3(x, height, width, weights, bias, shifts, y, i, node_key, record);
    return cudaSuccess;
}

cudaError_t mul(const std::int32_t* a, int channels, std::size_t plane, const std::int32_t* b, int b_channels,
                std::size_t b_plane, int shift, std::int32_t* y, unsigned long long node_key,
                unsigned long long* failure, cudaStream_t) {
    const HostRecord record{failure};
    for (std::size_t i = 0; i < plane * channels; ++i) el::mul(a, plane, b, b_channels, b_plane, shift, y, i, node_key, record);
    return cudaSuccess;
}

cudaError_t affine(const std::int32_t* x, std::size_t count, std::int64_t alpha, std::int64_t beta, int shift,
                   std::int32_t* y, unsigned long long node_key, unsigned long long* failure, cudaStream_t) {
    const HostRecord record{failure};
    for (std::size_t i = 0; i < count; ++i) el::affine(x, alpha, beta, shift, y, i, node_key, record);
    return cudaSuccess;
}

cudaError_t add(const std::int32_t* a, const std::int32_t* b, std::size_t count, std::int32_t* y,
                unsigned long long node_key, unsigned long long* failure, cudaStream_t) {
    const HostRecord record{failure};
    for (std::size_t i = 0; i < count; ++i) el::add(a, b, y, i, node_key, record);
    return cudaSuccess;
}

cudaError_t sat_table(const std::int32_t* x, std::size_t count, const std::int32_t* table, std::int64_t n,
                      std::int32_t top, std::int32_t* y, cudaStream_t) {
    for (std::size_t i = 0; i < count; ++i) el::sat_table(x, table, n, top, y, i);
    return cudaSuccess;
}

cudaError_t delta(const std::int32_t* x, std::size_t count, Table table, std::int32_t* y, cudaStream_t) {
    if (count == 0) return cudaSuccess;
    if (table.dc == nullptr) return cudaErrorInvalidValue;
    for (std::size_t i = 0; i < count; ++i) el::delta(x, table, y, i);
    return cudaSuccess;
}

cudaError_t clamp(const std::int32_t* x, std::size_t count, std::int32_t lo, std::int32_t hi, std::int32_t* y,
                  cudaStream_t) {
    for (std::size_t i = 0; i < count; ++i) el::clamp(x, lo, hi, y, i);
    return cudaSuccess;
}

cudaError_t shuffle(const std::int32_t* x, int channels, int height, int width, int factor, bool up, std::int32_t* y,
                    cudaStream_t) {
    // The extents the device launcher derives: the deep tensor's.
    const int r = factor;
    const int deep_channels = up ? channels : channels * r * r;
    const int deep_h = up ? height : height / r;
    const int deep_w = up ? width : width / r;
    const std::size_t count = static_cast<std::size_t>(deep_channels) * deep_h * deep_w;
    for (std::size_t w = 0; w < count; ++w) el::shuffle(x, deep_h, deep_w, r, up, y, w);
    return cudaSuccess;
}

cudaError_t im2col(const std::int32_t* x, int channels, int height, int width, int kernel, int stride, int out_h,
                   int out_w, std::int32_t* y, cudaStream_t) {
    const std::size_t count = static_cast<std::size_t>(channels) * kernel * kernel * out_h * out_w;
    for (std::size_t i = 0; i < count; ++i) el::im2col(x, height, width, kernel, stride, out_h, out_w, y, i);
    return cudaSuccess;
}

cudaError_t crop(const std::int32_t* x, int channels, int height, int width, int out_h, int out_w, std::int32_t* y,
                 cudaStream_t) {
    if (out_h > height || out_w > width) return cudaErrorInvalidValue;
    const std::size_t count = static_cast<std::size_t>(channels) * out_h * out_w;
    for (std::size_t i = 0; i < count; ++i) el::crop(x, height, width, out_h, out_w, y, i);
    return cudaSuccess;
}

cudaError_t param_row(const std::int32_t* x, const std::int64_t* rows, int row_count, int channels, std::int32_t* y,
                      unsigned long long node_key, unsigned long long* failure, cudaStream_t) {
    const HostRecord record{failure};
    for (int c = 0; c < channels; ++c) el::param_row(x, rows, row_count, channels, y, c, node_key, record);
    return cudaSuccess;
}

}  // namespace nvcr_sm100::fx::kernels

// Host stand-ins for the CUDA runtime calls of the fx executor.
extern "C" {

cudaError_t cudaMalloc(void** pointer, size_t size) {
    *pointer = std::malloc(size == 0 ? 1 : size);
    return *pointer != nullptr ? cudaSuccess : cudaErrorMemoryAllocation;
}
cudaError_t cudaMallocHost(void** pointer, size_t size) { return cudaMalloc(pointer, size); }
cudaError_t cudaFree(void* pointer) {
    std::free(pointer);
    return cudaSuccess;
}
cudaError_t cudaFreeHost(void* pointer) { return cudaFree(pointer); }
cudaError_t cudaMemcpy(void* to, const void* from, size_t size, cudaMemcpyKind) {
    std::memmove(to, from, size);
    return cudaSuccess;
}
cudaError_t cudaMemcpyAsync(void* to, const void* from, size_t size, cudaMemcpyKind, cudaStream_t) {
    std::memmove(to, from, size);
    return cudaSuccess;
}
cudaError_t cudaMemsetAsync(void* to, int value, size_t size, cudaStream_t) {
    std::memset(to, value, size);
    return cudaSuccess;
}
cudaError_t cudaStreamSynchronize(cudaStream_t) { return cudaSuccess; }
const char* cudaGetErrorString(cudaError_t) { return "host build"; }

// Loads <directory>/<stage> and runs it on int32 NCHW tensors through the
// executor, as nvcr_b200.fx.FxExecutor.run does, taking the executor's
// host-memory branch (device_memory 0) or its device-memory branch (1; here both
// are host memory), or the device branch and then the host branch twice on the
// same executor (2): outputs are malloc'd with their extents in out_extents.
// Returns 0 or ErrorCode + 1, with the message.
int fxh_run(const char* directory, const char* stage, int input_count, const std::int32_t* extents,
            const std::int32_t* const* inputs, int output_capacity, std::int32_t* out_extents, std::int32_t** outputs,
            char* message, size_t message_size, int device_memory) {
    using namespace nvcr_sm100;
    const auto report = [&](const Error& error) {
        std::snprintf(message, message_size, "%s", error.message.c_str());
        return static_cast<int>(error.code) + 1;
    };
    auto program = fx::load_fx_program(directory, stage);
    if (!program) return report(program.error());
    auto created = fx::FxExecutor::create(std::move(program.value()), nullptr);
    if (!created) return report(created.error());
    auto& executor = *created.value();
    std::vector<fx::FxExtent> shapes;
    std::vector<const std::int32_t*> in;
    for (int i = 0; i < input_count; ++i) {
        shapes.push_back({extents[3 * i], extents[3 * i + 1], extents[3 * i + 2]});
        in.push_back(inputs[i]);
    }
    auto inferred = executor.infer_output_extents(shapes);
    if (!inferred) {
        // Run anyway, so a stage failure met before the refusal is what is reported.
        auto ran = executor.run(in, shapes, {}, device_memory != 0);
        return report(ran ? inferred.error() : ran.error());
    }
    if (static_cast<int>(inferred.value().size()) > output_capacity) return -1;
    std::vector<std::int32_t*> out;
    for (std::size_t i = 0; i < inferred.value().size(); ++i) {
        const auto& e = inferred.value()[i];
        out_extents[3 * i] = e.channels;
        out_extents[3 * i + 1] = e.height;
        out_extents[3 * i + 2] = e.width;
        outputs[i] = static_cast<std::int32_t*>(std::malloc((e.count() == 0 ? 1 : e.count()) * sizeof(std::int32_t)));
        out.push_back(outputs[i]);
    }
    auto ran = executor.run(in, shapes, out, device_memory != 0);
    if (!ran) return report(ran.error());
    if (device_memory == 2) {
        // Again on the same executor through the host-memory branch, twice (the
        // cached plan, its input buffers made at the first of these runs): the
        // outputs must not change.
        for (int again = 0; again < 2; ++again) {
            std::vector<std::vector<std::int32_t>> copies;
            std::vector<std::int32_t*> second;
            for (std::size_t i = 0; i < inferred.value().size(); ++i) {
                copies.emplace_back(std::max<std::size_t>(1, inferred.value()[i].count()), 0);
                second.push_back(copies.back().data());
            }
            auto rerun = executor.run(in, shapes, second, false);
            if (!rerun) return report(rerun.error());
            for (std::size_t i = 0; i < second.size(); ++i) {
                if (std::memcmp(second[i], out[i], inferred.value()[i].count() * sizeof(std::int32_t)) != 0) {
                    std::snprintf(message, message_size, "repeated run differs");
                    return -2;
                }
            }
        }
    }
    return 0;
}

void fxh_free(void* pointer) { std::free(pointer); }

}  // extern "C"
