#pragma once

// The sm_100a executor of intconv.v1 programs: the counterpart of the
// reference's CudaExecutor (src/deterministic/cuda_executor.hpp:26-53).
//
//  * create(): uploads FP32 weights, quantises every integer pointwise conv's
//    weights once into int8 limb matrices with their exact row terms, and plans
//    fusions (im2col into the quantiser; WSiLU, chunk-add and residual add into
//    the GEMM epilogue; slice/slice/add into one kernel).
//  * run_half(): named batch-1 NCHW FP16 device tensors in and out; enqueues
//    on the executor's stream and returns. The memory plan for a set of input
//    extents is computed once (liveness-based offsets into one arena, TMA maps
//    encoded against it) and reused: no allocation on the steady-state path.
//  * run_host(): FP32 host tensors, synchronous (the conformance path).
// One executor per stream; not thread-safe (as the reference's).

#include "kernels.hpp"
#include "program.hpp"
#include "status.hpp"

#include <cuda_runtime.h>

#include <functional>
#include <map>
#include <tuple>
#include <memory>
#include <optional>
#include <string>
#include <vector>

namespace nvcr_sm100 {

struct TensorView {
    std::string name;
    Extent extent;
    void* data{nullptr};
};

struct StepTiming {
    std::string label;  // "<op>:<output tensor>"
    std::string kernel; // dominant kernel of the step
    double milliseconds{0.0};
    double algorithmic_ops{0.0};    // 2 * C_in * kh * kw * C_out * P for integer convs
    double algorithmic_bytes{0.0};  // bytes read once + written once at the step's I/O types
};

class Executor {
public:
    static Result<std::unique_ptr<Executor>> create(Program program, cudaStream_t stream);
    ~Executor();
    Executor(const Executor&) = delete;
    Executor& operator=(const Executor&) = delete;

    const Program& program() const { return program_; }
    cudaStream_t stream() const { return stream_; }
    // The device that was current at create: the stream, weights and tensor
    // maps belong to it.
    int device() const { return device_; }

    Status run_half(const std::vector<TensorView>& inputs, const std::vector<TensorView>& outputs);
    Status run_float(const std::vector<TensorView>& inputs, const std::vector<TensorView>& outputs);
    Status run_host(const std::vector<TensorView>& inputs, const std::vector<TensorView>& outputs);
    // run_half with every scratch tensor placed in the caller-provided device
    // workspace instead of the executor's own arena: nothing is allocated.
    // Fails with invalid_argument when the plan needs more than `bytes`.
    Status run_half_in_workspace(const std::vector<TensorView>& inputs, const std::vector<TensorView>& outputs,
                                 void* workspace, std::size_t bytes);
    // Waits for the stream and reports a device-side wait that gave up.
    Status synchronize();
    // Diagnostics: enqueues a device wait that runs out after `limit_ms` and
    // sets this executor's status word, as a kernel whose wait gives up does.
    Status test_wait_timeout(unsigned int limit_ms);

    int launches_last_run() const { return launches_; }
    std::size_t workspace_bytes() const { return arena_bytes_; }
    void set_profiling(bool enabled) { profiling_ = enabled; }
    // Per-kernel device times of every profiled run since the last call
    // (synchronises, then forgets them).
    Result<std::vector<StepTiming>> profile();

    struct IntegerConv;
    struct Step;
    struct Plan;

private:
    Executor() = default;
    Status prepare();
    Status prepare_integer_conv(std::size_t step_index);
    Status prepare_direct(IntegerConv& conv, const Step& step, const Node& node, const IntegerWeights& quantized);
    void plan_fusions();
    enum class Boundary { half, float32, host };
    Result<Plan*> plan_for(const std::vector<Extent>& input_extents, Boundary boundary);
    Status ensure_arena(std::size_t bytes);
    Status execute(const std::vector<TensorView>& inputs, const std::vector<TensorView>& outputs, Boundary boundary,
                   void* workspace = nullptr, std::size_t workspace_bytes = 0);

    Status launch_step(const Step& step, Plan& plan, std::size_t index);
    struct GraphKey {
        const Plan* plan;
        const void* base;
        int boundary;
        std::vector<const void*> tensors;
        bool operator<(const GraphKey& other) const {
            return std::tie(plan, base, boundary, tensors) <
                std::tie(other.plan, other.base, other.boundary, other.tensors);
        }
    };
    struct CachedGraph {
        cudaGraphExec_t exec{nullptr};
        int launches{0};
    };
    Status run_graph(const GraphKey& key, const std::function<Status()>& enqueue);
    void clear_graphs();
    std::map<GraphKey, CachedGraph> graphs_;
    Status mark(const std::string& label, const std::string& kernel, double ops, double bytes);

    Program program_;
    int device_{0};
    int sm_count_{148};  // streaming multiprocessors of device_
    cudaStream_t stream_{nullptr};
    bool owns_stream_{false};
    float* weights_{nullptr};
    unsigned int* status_{nullptr};
    std::vector<Step> steps_;
    std::vector<IntegerConv> convs_;
    // Per program input: every reader is an integer conv reading it as its
    // source, so on device runs the conv prepass reads the caller's buffer.
    std::vector<bool> input_conv_only_;
    // Per program output: the integer conv step that produces it when no step
    // reads it (the epilogue stores into the caller's buffer), else -1.
    std::vector<std::ptrdiff_t> output_step_;
    // Per tensor: kept channel-innermost ([H][W][c_pad] FP32, then the per-pixel
    // maxima) because an integer conv produces it and only integer convs read
    // it, as their source or residual; their staging prepass is skipped.
    std::vector<bool> staged_tensor_;
    std::size_t tensor_bytes(const Extent& extent, std::size_t id) const;
    std::size_t staged_max_offset(const Extent& extent, std::size_t id) const;
    // The run in progress: caller buffers for direct inputs (by tensor id) and
    // direct outputs (by step), with their element type.
    struct Direct {
        void* data{nullptr};
        bool half{false};
    };
    std::vector<Direct> run_inputs_;
    std::vector<Direct> run_outputs_;
    std::map<std::vector<std::int32_t>, std::unique_ptr<Plan>> plans_;
    void* arena_{nullptr};
    std::uint8_t* run_base_{nullptr};  // arena_ or a caller's workspace, for the run in progress
    std::size_t arena_bytes_{0};
    std::uint64_t arena_generation_{0};
    int launches_{0};
    bool profiling_{false};
    // Set while run_graph captures a run: a direct conv's fallback then goes into
    // a conditional graph node (captured on fallback_stream_) that runs only when
    // the conv found a window whose pixels have different exponents.
    bool capturing_{false};
    cudaStream_t fallback_stream_{nullptr};
    std::vector<cudaEvent_t> events_;
    std::size_t marks_{0};
    bool run_started_{false};
    std::vector<std::size_t> segment_starts_;
    std::vector<StepTiming> timings_;
};

}  // namespace nvcr_sm100
