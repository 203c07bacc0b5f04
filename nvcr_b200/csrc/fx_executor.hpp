#pragma once

// Runs nvcr.fx.v1 programs on one GPU: the device counterpart of the
// reference's fx::run (src/deterministic/fx_program.cpp:468-525). Same
// integers, and the same outcome on every input: success, a stage failure
// (malformed_bitstream, the failure the reference meets first) or a refusal
// (invalid_argument, for tensors whose shapes the program cannot take).
//
// Every value a node writes gets its own int32 NCHW device buffer, sized once
// per set of input extents (a plan, cached), so a program that writes a tensor
// id twice, or reads and writes the same id in one node, behaves as the
// reference's value semantics say. Parameters are uploaded once, at the first
// run; creating an executor and inferring extents touch no device.

#include "fx_kernels.hpp"
#include "fx_program.hpp"

#include <cuda_runtime.h>

#include <array>
#include <map>
#include <memory>
#include <vector>

namespace nvcr_sm100::fx {

struct FxExtent {
    std::int32_t channels{0};
    std::int32_t height{0};
    std::int32_t width{0};
    [[nodiscard]] std::size_t count() const {
        return static_cast<std::size_t>(channels) * static_cast<std::size_t>(height) * static_cast<std::size_t>(width);
    }
    bool operator<(const FxExtent& other) const {
        return std::array{channels, height, width} < std::array{other.channels, other.height, other.width};
    }
};

class FxExecutor {
public:
    static Result<std::unique_ptr<FxExecutor>> create(FxProgram program, cudaStream_t stream);
    ~FxExecutor();
    FxExecutor(const FxExecutor&) = delete;
    FxExecutor& operator=(const FxExecutor&) = delete;

    [[nodiscard]] const FxProgram& program() const { return program_; }
    [[nodiscard]] cudaStream_t stream() const { return stream_; }

    // Output extents for these input extents (program.inputs order), or the
    // refusal the reference's run would give for shapes alone.
    Result<std::vector<FxExtent>> infer_output_extents(const std::vector<FxExtent>& inputs);

    // Runs on int32 NCHW tensors in device memory (device = true) or host
    // memory; outputs are written in program.outputs order. Returns after the
    // run's failure word has been read (the stream is synchronised).
    Status run(const std::vector<const std::int32_t*>& inputs, const std::vector<FxExtent>& extents,
               const std::vector<std::int32_t*>& outputs, bool device);

    [[nodiscard]] int last_launch_count() const { return launches_; }

private:
    struct DeviceNode {
        std::int16_t* gemm_weights{nullptr};
        std::int64_t* bias{nullptr};
        std::int32_t* shifts{nullptr};
        std::int32_t* depthwise_weights{nullptr};
        std::int64_t* rows{nullptr};
        std::int32_t* table{nullptr};
    };
    // What the reference's run does with these extents: the value buffer each
    // node reads and writes, and where (if anywhere) it stops on a shape.
    struct Plan {
        std::vector<FxExtent> value_extents;  // inputs first, then one per node
        std::vector<std::vector<std::size_t>> node_inputs;  // value ids
        std::vector<std::size_t> output_values;
        std::size_t input_stop{0};   // inputs [0, input_stop) have valid shapes
        std::size_t nodes_run{0};    // nodes [0, nodes_run) are launched
        bool stopped{false};
        Error stop;                  // the error the reference reports if no earlier stage failure
        std::vector<std::int32_t*> values;  // device buffers; inputs' only after a host-memory run
    };

    FxExecutor(FxProgram program, cudaStream_t stream) : program_(std::move(program)), stream_(stream) {}
    Status upload();  // parameters and the failure word, once
    Plan make_plan(const std::vector<FxExtent>& inputs) const;
    Result<Plan*> plan_for(const std::vector<FxExtent>& inputs);
    Status launch(const Plan& plan, std::size_t node_index, const std::vector<std::int32_t*>& values);
    Error failure_error(unsigned long long key) const;

    FxProgram program_;
    cudaStream_t stream_{nullptr};
    std::vector<DeviceNode> device_nodes_;
    std::vector<std::int16_t*> device_tables_;
    std::vector<void*> allocations_;
    unsigned long long* failure_{nullptr};       // device word
    unsigned long long* failure_host_{nullptr};  // pinned copy
    std::map<std::vector<FxExtent>, std::unique_ptr<Plan>> plans_;
    int launches_{0};
};

}  // namespace nvcr_sm100::fx
