#include "fx_executor.hpp"

#include <cstring>
#include <optional>

namespace nvcr_sm100::fx {
namespace {

Error invalid(const std::string& message) { return fail(Code::invalid_argument, "fx program: " + message); }
Error stage_failure(const std::string& message) { return fail(Code::malformed_bitstream, "nvcr.fx.v1: " + message); }
Error cuda_error(cudaError_t status, const char* what) {
    return fail(Code::backend_error, std::string(what) + ": " + cudaGetErrorString(status));
}

// Largest value a run may hold: loop positions in the failure word need 46 bits.
constexpr std::size_t max_value_count = std::size_t{1} << 38;

template <typename T>
Result<T*> upload_array(const std::vector<T>& values, std::vector<void*>& allocations) {
    if (values.empty()) return static_cast<T*>(nullptr);
    void* device = nullptr;
    cudaError_t status = cudaMalloc(&device, values.size() * sizeof(T));
    if (status != cudaSuccess) return cuda_error(status, "cudaMalloc");
    allocations.push_back(device);
    status = cudaMemcpy(device, values.data(), values.size() * sizeof(T), cudaMemcpyHostToDevice);
    if (status != cudaSuccess) return cuda_error(status, "cudaMemcpy");
    return static_cast<T*>(device);
}

}  // namespace

Result<std::unique_ptr<FxExecutor>> FxExecutor::create(FxProgram program, cudaStream_t stream) {
    return std::unique_ptr<FxExecutor>(new FxExecutor(std::move(program), stream));
}

FxExecutor::~FxExecutor() {
    if (failure_ != nullptr) cudaStreamSynchronize(stream_);
    for (auto& [extents, plan] : plans_) {
        for (std::size_t i = 0; i < plan->values.size(); ++i) cudaFree(plan->values[i]);
    }
    for (void* pointer : allocations_) cudaFree(pointer);
    if (failure_ != nullptr) cudaFree(failure_);
    if (failure_host_ != nullptr) cudaFreeHost(failure_host_);
}

Status FxExecutor::upload() {
    if (failure_ != nullptr) return Ok{};
    cudaError_t status = cudaMalloc(reinterpret_cast<void**>(&failure_), sizeof(unsigned long long));
    if (status != cudaSuccess) return cuda_error(status, "cudaMalloc");
    status = cudaMallocHost(reinterpret_cast<void**>(&failure_host_), sizeof(unsigned long long));
    if (status != cudaSuccess) return cuda_error(status, "cudaMallocHost");
    for (const auto& table : program_.delta_tables) {
        auto dc = upload_array(table.dc, allocations_);
        if (!dc) return dc.error();
        device_tables_.push_back(dc.value());
    }
    for (const auto& node : program_.nodes) {
        DeviceNode device;
        auto gemm_weights = upload_array(node.gemm_weights, allocations_);
        if (!gemm_weights) return gemm_weights.error();
        auto bias = upload_array(node.bias, allocations_);
        if (!bias) return bias.error();
        auto shifts = upload_array(node.shifts, allocations_);
        if (!shifts) return shifts.error();
        auto depthwise_weights = upload_array(node.depthwise_weights, allocations_);
        if (!depthwise_weights) return depthwise_weights.error();
        auto rows = upload_array(node.rows, allocations_);
        if (!rows) return rows.error();
        auto table = upload_array(node.table, allocations_);
        if (!table) return table.error();
        device = {gemm_weights.value(), bias.value(), shifts.value(), depthwise_weights.value(), rows.value(),
                  table.value()};
        device_nodes_.push_back(device);
    }
    return Ok{};
}

// The checks of fx::run (fx_program.cpp:468-525), in its order, on extents
// alone. A stop records the error the reference returns there; the nodes
// before it (and, for a wrong output channel count, the node itself, whose op
// the reference runs before that check) are still launched, because a stage
// failure in them is what the reference reports first.
FxExecutor::Plan FxExecutor::make_plan(const std::vector<FxExtent>& inputs) const {
    Plan plan;
    const auto stop = [&plan](Error error, std::size_t nodes_run) {
        plan.stopped = true;
        plan.stop = std::move(error);
        plan.nodes_run = nodes_run;
    };
    const std::string& name = program_.name;
    if (inputs.size() != program_.inputs.size()) {
        stop(invalid(name + ": wrong number of inputs"), 0);
        return plan;
    }
    std::vector<std::optional<std::size_t>> current(program_.tensor_names.size());
    for (std::size_t slot = 0; slot < inputs.size(); ++slot) {
        const auto id = program_.inputs[slot];
        const FxExtent& x = inputs[slot];
        if (x.channels != program_.tensor_channels[id] || x.height < 0 || x.width < 0) {
            plan.input_stop = slot;
            stop(invalid(name + ": input " + program_.tensor_names[id] + " has the wrong shape"), 0);
            return plan;
        }
        plan.value_extents.push_back(x);
        current[id] = slot;
    }
    plan.input_stop = inputs.size();
    for (std::size_t n = 0; n < program_.nodes.size(); ++n) {
        const FxNode& node = program_.nodes[n];
        std::vector<std::size_t> ins;
        for (const auto id : node.inputs) {
            if (!current[id]) {
                stop(invalid(name + ": tensor read before it is written"), n);
                return plan;
            }
            ins.push_back(*current[id]);
        }
        const FxExtent x = plan.value_extents[ins[0]];
        const bool sized = node.op == FxOp::gemm || node.op == FxOp::add || node.op == FxOp::concat;
        for (const auto value : ins) {
            const FxExtent& t = plan.value_extents[value];
            if (sized && (t.height != x.height || t.width != x.width)) {
                stop(invalid(name + ": node inputs differ in size"), n);
                return plan;
            }
        }
        FxExtent out = x;
        switch (node.op) {
        case FxOp::gemm:
            if (x.channels != node.in_channels) {
                stop(invalid(name + ": gemm input channels"), n);
                return plan;
            }
            for (std::size_t r = 1; r < ins.size(); ++r) {
                if (plan.value_extents[ins[r]].channels != node.out_channels / node.group) {
                    stop(invalid(name + ": residual channels"), n);
                    return plan;
                }
            }
            out.channels = node.out_channels / node.group;
            break;
        case FxOp::mul: {
            const FxExtent& b = plan.value_extents[ins[1]];
            if (!(b.height == 1 && b.width == 1) && (b.height != x.height || b.width != x.width)) {
                stop(invalid(name + ": mul factor size"), n);
                return plan;
            }
            if (b.channels != 1 && b.channels != x.channels) {
                stop(invalid(name + ": mul factor channels"), n);
                return plan;
            }
            break;
        }
        case FxOp::param_row:
            if (x.count() != 1) {
                stop(stage_failure(name + ": qp outside the parameter table"), n);
                return plan;
            }
            out = {program_.tensor_channels[node.output], 1, 1};
            break;
        case FxOp::crop_like: {
            const FxExtent& ref = plan.value_extents[ins[1]];
            if (ref.height > x.height || ref.width > x.width) {
                stop(invalid(name + ": crop larger than input"), n);
                return plan;
            }
            out = {x.channels, ref.height, ref.width};
            break;
        }
        case FxOp::add:
            if (plan.value_extents[ins[1]].channels != x.channels) {
                stop(invalid(name + ": add channels"), n);
                return plan;
            }
            break;
        case FxOp::concat:
            out.channels = x.channels + plan.value_extents[ins[1]].channels;
            break;
        case FxOp::slice:
            out.channels = node.end - node.begin;
            break;
        case FxOp::pixel_shuffle:
        case FxOp::pixel_unshuffle: {
            const int r = node.factor;
            const bool up = node.op == FxOp::pixel_shuffle;
            if (up ? x.channels % (r * r) != 0 : (x.height % r != 0 || x.width % r != 0)) {
                stop(invalid(name + ": pixel shuffle size"), n);
                return plan;
            }
            out = up ? FxExtent{x.channels / (r * r), x.height * r, x.width * r}
                     : FxExtent{x.channels * r * r, x.height / r, x.width / r};
            break;
        }
        case FxOp::im2col: {
            const int pad = node.kernel == 3 ? 1 : 0;
            // C++ division truncates toward zero, as the reference's does.
            out = {x.channels * node.kernel * node.kernel, (x.height + 2 * pad - node.kernel) / node.stride + 1,
                   (x.width + 2 * pad - node.kernel) / node.stride + 1};
            break;
        }
        case FxOp::depthwise3x3:
        case FxOp::affine:
        case FxOp::sat_table:
        case FxOp::delta:
        case FxOp::clamp:
            break;
        }
        if (out.count() > max_value_count) {
            stop(fail(Code::resource_exhausted, name + ": a value exceeds 2^38 elements"), n);
            return plan;
        }
        plan.node_inputs.push_back(ins);
        plan.value_extents.push_back(out);
        if (out.channels != program_.tensor_channels[node.output]) {
            stop(invalid(name + ": node output has the wrong channel count"), n + 1);
            return plan;
        }
        current[node.output] = plan.value_extents.size() - 1;
    }
    plan.nodes_run = program_.nodes.size();
    for (const auto id : program_.outputs) {
        if (!current[id]) {
            stop(invalid(name + ": output not produced"), program_.nodes.size());
            return plan;
        }
        plan.output_values.push_back(*current[id]);
    }
    return plan;
}

Result<FxExecutor::Plan*> FxExecutor::plan_for(const std::vector<FxExtent>& inputs) {
    auto found = plans_.find(inputs);
    if (found != plans_.end()) return found->second.get();
    auto plan = std::make_unique<Plan>(make_plan(inputs));
    // Node values get buffers now; the inputs' values are the caller's buffers
    // on device-memory runs, and get buffers at the first host-memory run.
    plan->values.assign(plan->value_extents.size(), nullptr);
    for (std::size_t v = plan->input_stop; v < plan->value_extents.size(); ++v) {
        void* device = nullptr;
        const cudaError_t status =
            cudaMalloc(&device, std::max<std::size_t>(1, plan->value_extents[v].count()) * sizeof(std::int32_t));
        if (status != cudaSuccess) {
            for (std::size_t i = plan->input_stop; i < v; ++i) cudaFree(plan->values[i]);
            return cuda_error(status, "cudaMalloc");
        }
        plan->values[v] = static_cast<std::int32_t*>(device);
    }
    return plans_.emplace(inputs, std::move(plan)).first->second.get();
}

Result<std::vector<FxExtent>> FxExecutor::infer_output_extents(const std::vector<FxExtent>& inputs) {
    const Plan plan = make_plan(inputs);
    if (plan.stopped) return plan.stop;
    std::vector<FxExtent> outputs;
    for (const auto value : plan.output_values) outputs.push_back(plan.value_extents[value]);
    return outputs;
}

Status FxExecutor::launch(const Plan& plan, std::size_t n, const std::vector<std::int32_t*>& values) {
    const FxNode& node = program_.nodes[n];
    const DeviceNode& device = device_nodes_[n];
    const auto& ins = plan.node_inputs[n];
    const std::size_t out_value = program_.inputs.size() + n;
    const FxExtent& x = plan.value_extents[ins[0]];
    const FxExtent& out = plan.value_extents[out_value];
    const std::int32_t* in0 = values[ins[0]];
    std::int32_t* y = values[out_value];
    const unsigned long long key = static_cast<unsigned long long>(n + 1) << kernels::node_shift;
    const std::size_t count = x.count();
    const std::size_t plane = static_cast<std::size_t>(x.height) * static_cast<std::size_t>(x.width);
    cudaError_t status = cudaSuccess;
    int launched = 1;
    switch (node.op) {
    case FxOp::gemm: {
        kernels::GemmArgs args;
        args.x = in0;
        args.pixels = plane;
        args.in_channels = node.in_channels;
        args.group = node.group;
        args.groups = node.out_channels / node.group;
        args.input_shift = node.input_shift;
        args.weights = device.gemm_weights;
        args.bias = device.bias;
        args.shifts = device.shifts;
        if (node.delta_table >= 0) {
            const auto& table = program_.delta_tables[static_cast<std::size_t>(node.delta_table)];
            args.table = {device_tables_[static_cast<std::size_t>(node.delta_table)], table.h, table.shift};
        }
        args.residual0 = ins.size() > 1 ? values[ins[1]] : nullptr;
        args.residual1 = ins.size() > 2 ? values[ins[2]] : nullptr;
        args.y = y;
        status = kernels::gemm(args, key, failure_, stream_);
        break;
    }
    case FxOp::depthwise3x3:
        status = kernels::depthwise3x3(in0, x.channels, x.height, x.width, device.depthwise_weights, device.bias,
                                       device.shifts, y, key, failure_, stream_);
        break;
    case FxOp::mul: {
        const FxExtent& b = plan.value_extents[ins[1]];
        status = kernels::mul(in0, x.channels, plane, values[ins[1]], b.channels,
                              static_cast<std::size_t>(b.height) * static_cast<std::size_t>(b.width), node.shift, y,
                              key, failure_, stream_);
        break;
    }
    case FxOp::affine:
        status = kernels::affine(in0, count, node.alpha, node.beta, node.shift, y, key, failure_, stream_);
        break;
    case FxOp::add:
        status = kernels::add(in0, values[ins[1]], count, y, key, failure_, stream_);
        break;
    case FxOp::sat_table:
        status = kernels::sat_table(in0, count, device.table, static_cast<std::int64_t>(node.table.size() / 2),
                                    static_cast<std::int32_t>(node.hi), y, stream_);
        break;
    case FxOp::delta: {
        const auto& table = program_.delta_tables[static_cast<std::size_t>(node.delta_table)];
        status = kernels::delta(in0, count, {device_tables_[static_cast<std::size_t>(node.delta_table)], table.h,
                                             table.shift}, y, stream_);
        break;
    }
    case FxOp::clamp:
        status = kernels::clamp(in0, count, static_cast<std::int32_t>(node.lo), static_cast<std::int32_t>(node.hi), y,
                                stream_);
        break;
    case FxOp::concat: {
        const std::size_t second = plan.value_extents[ins[1]].count();
        launched = 0;
        if (count > 0) status = cudaMemcpyAsync(y, in0, count * 4, cudaMemcpyDeviceToDevice, stream_);
        if (status == cudaSuccess && second > 0) {
            status = cudaMemcpyAsync(y + count, values[ins[1]], second * 4, cudaMemcpyDeviceToDevice, stream_);
        }
        break;
    }
    case FxOp::slice:
        launched = 0;
        if (out.count() > 0) {
            status = cudaMemcpyAsync(y, in0 + static_cast<std::size_t>(node.begin) * plane, out.count() * 4,
                                     cudaMemcpyDeviceToDevice, stream_);
        }
        break;
    case FxOp::pixel_shuffle:
    case FxOp::pixel_unshuffle:
        status = kernels::shuffle(in0, x.channels, x.height, x.width, node.factor, node.op == FxOp::pixel_shuffle, y,
                                  stream_);
        break;
    case FxOp::im2col:
        status = kernels::im2col(in0, x.channels, x.height, x.width, node.kernel, node.stride, out.height, out.width, y,
                                 stream_);
        break;
    case FxOp::crop_like:
        status = kernels::crop(in0, x.channels, x.height, x.width, out.height, out.width, y, stream_);
        break;
    case FxOp::param_row:
        status = kernels::param_row(in0, device.rows, static_cast<int>(node.rows.size() / out.channels), out.channels,
                                    y, key, failure_, stream_);
        break;
    }
    if (status != cudaSuccess) return cuda_error(status, op_name(node.op));
    launches_ += launched;
    return Ok{};
}

Error FxExecutor::failure_error(unsigned long long key) const {
    const auto node = key >> kernels::node_shift;
    const bool second_rule = (key & 1u) != 0;
    if (node == 0) return stage_failure(program_.name + ": input value out of range");
    switch (program_.nodes[node - 1].op) {
    case FxOp::gemm:
        return stage_failure(second_rule ? "gemm output out of range" : "gemm pre-activation out of range");
    case FxOp::depthwise3x3: return stage_failure("depthwise output out of range");
    case FxOp::mul: return stage_failure("mul output out of range");
    case FxOp::affine: return stage_failure("affine output out of range");
    case FxOp::add: return stage_failure("add output out of range");
    case FxOp::param_row: return stage_failure(program_.name + ": qp outside the parameter table");
    default: return stage_failure("unexpected failure record");
    }
}

Status FxExecutor::run(const std::vector<const std::int32_t*>& inputs, const std::vector<FxExtent>& extents,
                       const std::vector<std::int32_t*>& outputs, bool device) {
    if (inputs.size() != extents.size()) return invalid("one extent per input");
    auto uploaded = upload();
    if (!uploaded) return uploaded.error();
    auto planned = plan_for(extents);
    if (!planned) return planned.error();
    Plan& plan = *planned.value();
    if (!plan.stopped && outputs.size() != plan.output_values.size()) return invalid("wrong number of outputs");
    if (!device) {
        for (std::size_t slot = 0; slot < plan.input_stop; ++slot) {
            if (plan.values[slot] != nullptr) continue;
            void* buffer = nullptr;
            const cudaError_t status =
                cudaMalloc(&buffer, std::max<std::size_t>(1, extents[slot].count()) * sizeof(std::int32_t));
            if (status != cudaSuccess) return cuda_error(status, "cudaMalloc");
            plan.values[slot] = static_cast<std::int32_t*>(buffer);
        }
    }
    launches_ = 0;
    std::vector<std::int32_t*> values = plan.values;
    cudaError_t status = cudaMemsetAsync(failure_, 0xFF, sizeof(unsigned long long), stream_);
    unsigned long long base = 0;
    for (std::size_t slot = 0; slot < plan.input_stop && status == cudaSuccess; ++slot) {
        const std::size_t count = extents[slot].count();
        if (count > 0 && inputs[slot] == nullptr) return invalid("null input");
        if (device) {
            values[slot] = const_cast<std::int32_t*>(inputs[slot]);
        } else if (count > 0) {
            status = cudaMemcpyAsync(values[slot], inputs[slot], count * 4, cudaMemcpyHostToDevice, stream_);
            if (status != cudaSuccess) break;
        }
        status = kernels::check_input(values[slot], count, base, failure_, stream_);
        launches_ += count > 0 ? 1 : 0;
        base += count;
    }
    if (status != cudaSuccess) return cuda_error(status, "input");
    for (std::size_t n = 0; n < plan.nodes_run; ++n) {
        auto launched = launch(plan, n, values);
        if (!launched) return launched.error();
    }
    if (!plan.stopped) {
        for (std::size_t i = 0; i < outputs.size() && status == cudaSuccess; ++i) {
            const std::size_t count = plan.value_extents[plan.output_values[i]].count();
            if (count == 0) continue;
            if (outputs[i] == nullptr) return invalid("null output");
            status = cudaMemcpyAsync(outputs[i], values[plan.output_values[i]], count * 4,
                                     device ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, stream_);
        }
    }
    if (status == cudaSuccess) {
        status = cudaMemcpyAsync(failure_host_, failure_, sizeof(unsigned long long), cudaMemcpyDeviceToHost, stream_);
    }
    if (status == cudaSuccess) status = cudaStreamSynchronize(stream_);
    if (status != cudaSuccess) return cuda_error(status, "fx run");
    if (*failure_host_ != kernels::no_failure) return failure_error(*failure_host_);
    if (plan.stopped) return plan.stop;
    return Ok{};
}

}  // namespace nvcr_sm100::fx
