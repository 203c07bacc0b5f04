#include "program.hpp"

#include "json.hpp"
#include "sha256.hpp"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <fstream>
#include <iterator>
#include <map>
#include <sstream>

namespace nvcr_sm100 {
namespace {

Error invalid(const std::string& message) { return fail(Code::invalid_argument, message); }

Result<std::int64_t> get_int(const json::Value& object, std::string_view key) {
    const auto* v = object.get(key);
    if (v == nullptr || v->kind != json::Value::Kind::number || !v->integer) {
        return invalid("program field '" + std::string(key) + "' must be an integer");
    }
    return *v->integer;
}

Result<std::string> get_text(const json::Value& object, std::string_view key) {
    const auto* v = object.get(key);
    if (v == nullptr || v->kind != json::Value::Kind::string) {
        return invalid("program field '" + std::string(key) + "' must be a string");
    }
    return v->text;
}

template <std::size_t N>
Result<std::array<std::int32_t, N>> get_ints(const json::Value& object, std::string_view key) {
    const auto* v = object.get(key);
    if (v == nullptr || v->kind != json::Value::Kind::array || v->items.size() != N) {
        return invalid("program field '" + std::string(key) + "' has the wrong length");
    }
    std::array<std::int32_t, N> out{};
    for (std::size_t i = 0; i < N; ++i) {
        if (v->items[i].kind != json::Value::Kind::number || !v->items[i].integer) {
            return invalid("program field '" + std::string(key) + "' must hold integers");
        }
        out[i] = static_cast<std::int32_t>(*v->items[i].integer);
    }
    return out;
}

// A float32 field whose JSON number must be exactly representable.
Result<float> get_exact_float(const json::Value& object, std::string_view key, std::string_view what) {
    const auto* v = object.get(key);
    if (v == nullptr || v->kind != json::Value::Kind::number) {
        return invalid(std::string(what) + " needs a numeric '" + std::string(key) + "'");
    }
    const auto f = static_cast<float>(v->number);
    if (static_cast<double>(f) != v->number) {
        return invalid(std::string(what) + " value is not exactly representable in float32");
    }
    return f;
}

Result<Op> op_from_name(std::string_view name) {
    static const std::pair<std::string_view, Op> table[] = {
        {"conv", Op::conv}, {"mul", Op::mul}, {"add", Op::add}, {"mul_scalar", Op::mul_scalar},
        {"sigmoid", Op::sigmoid}, {"slice_channels", Op::slice_channels},
        {"depth_to_space", Op::depth_to_space}, {"scale_channels", Op::scale_channels},
        {"clamp", Op::clamp}, {"concat", Op::concat}, {"crop", Op::crop},
        {"space_to_depth", Op::space_to_depth}, {"im2col", Op::im2col}};
    for (const auto& [text, op] : table) {
        if (text == name) return op;
    }
    return invalid("unsupported deterministic op '" + std::string(name) + "'");
}

class Tensors {
public:
    explicit Tensors(Program& program) : program_(program) {}
    std::size_t define(const std::string& name, std::int32_t channels) {
        const auto id = program_.tensor_names.size();
        program_.tensor_names.push_back(name);
        program_.tensor_channels.push_back(channels);
        ids_.emplace(name, id);
        return id;
    }
    Result<std::size_t> find(const std::string& name) const {
        auto it = ids_.find(name);
        if (it == ids_.end()) return invalid("program reads undefined tensor '" + name + "'");
        return it->second;
    }
    bool contains(const std::string& name) const { return ids_.count(name) != 0; }
    std::int32_t channels(std::size_t id) const { return program_.tensor_channels[id]; }

private:
    Program& program_;
    std::map<std::string, std::size_t, std::less<>> ids_;
};

bool binary_op(Op op) {
    return op == Op::mul || op == Op::add || op == Op::scale_channels || op == Op::concat || op == Op::crop;
}

Result<Node> parse_node(const json::Value& value, Tensors& tensors, std::size_t weight_count) {
    auto op_name = get_text(value, "op");
    if (!op_name) return op_name.error();
    auto op = op_from_name(op_name.value());
    if (!op) return op.error();
    Node node;
    node.op = op.value();
    if (binary_op(node.op)) {
        const auto* inputs = value.get("inputs");
        if (inputs == nullptr || inputs->items.size() != 2) return invalid("binary op needs two inputs");
        for (std::size_t i = 0; i < 2; ++i) {
            auto id = tensors.find(inputs->items[i].text);
            if (!id) return id.error();
            node.inputs[i] = id.value();
        }
        node.input_count = 2;
    } else {
        auto input = get_text(value, "input");
        if (!input) return input.error();
        auto id = tensors.find(input.value());
        if (!id) return id.error();
        node.inputs[0] = id.value();
    }

    std::int32_t channels = 0;  // 0: inherit the first input's channels
    switch (node.op) {
    case Op::conv: {
        auto in_channels = get_int(value, "in_channels");
        auto out_channels = get_int(value, "out_channels");
        auto kernel = get_ints<2>(value, "kernel");
        auto stride = get_ints<2>(value, "stride");
        auto pads = get_ints<4>(value, "pads");
        auto weight_offset = get_int(value, "weight_offset");
        auto bias_offset = get_int(value, "bias_offset");
        const auto* depthwise = value.get("depthwise");
        if (!in_channels) return in_channels.error();
        if (!out_channels) return out_channels.error();
        if (!kernel) return kernel.error();
        if (!stride) return stride.error();
        if (!pads) return pads.error();
        if (!weight_offset) return weight_offset.error();
        if (!bias_offset) return bias_offset.error();
        if (depthwise == nullptr || depthwise->kind != json::Value::Kind::boolean) {
            return invalid("conv needs a boolean 'depthwise'");
        }
        node.in_channels = static_cast<std::int32_t>(in_channels.value());
        node.out_channels = static_cast<std::int32_t>(out_channels.value());
        node.depthwise = depthwise->boolean;
        node.kernel = kernel.value();
        node.stride = stride.value();
        node.pads = pads.value();
        const bool bad_pad = std::any_of(node.pads.begin(), node.pads.end(), [](std::int32_t p) { return p < 0; });
        if (node.in_channels <= 0 || node.out_channels <= 0 || node.kernel[0] <= 0 || node.kernel[1] <= 0 ||
            node.stride[0] <= 0 || node.stride[1] <= 0 || bad_pad ||
            (node.depthwise && node.in_channels != node.out_channels) || weight_offset.value() < 0 ||
            bias_offset.value() < 0) {
            return invalid("conv has an invalid geometry");
        }
        node.weight_offset = static_cast<std::size_t>(weight_offset.value());
        node.bias_offset = static_cast<std::size_t>(bias_offset.value());
        const std::size_t per_output = static_cast<std::size_t>(node.depthwise ? 1 : node.in_channels) *
            static_cast<std::size_t>(node.kernel[0]) * static_cast<std::size_t>(node.kernel[1]);
        const std::size_t count = static_cast<std::size_t>(node.out_channels) * per_output;
        if (node.weight_offset > weight_count || count > weight_count - node.weight_offset ||
            node.bias_offset > weight_count ||
            static_cast<std::size_t>(node.out_channels) > weight_count - node.bias_offset) {
            return invalid("conv weights exceed the weights file");
        }
        channels = node.out_channels;
        break;
    }
    case Op::mul_scalar: {
        auto scalar = get_exact_float(value, "value", "mul_scalar");
        if (!scalar) return scalar.error();
        node.scalar = scalar.value();
        break;
    }
    case Op::slice_channels: {
        auto begin = get_int(value, "begin");
        auto end = get_int(value, "end");
        if (!begin) return begin.error();
        if (!end) return end.error();
        node.begin = static_cast<std::int32_t>(begin.value());
        node.end = static_cast<std::int32_t>(end.value());
        channels = node.end - node.begin;
        break;
    }
    case Op::depth_to_space:
    case Op::space_to_depth: {
        auto block = get_int(value, "block");
        if (!block) return block.error();
        node.block = static_cast<std::int32_t>(block.value());
        if (node.block <= 0 || node.block > 64) return invalid("block size must be in [1, 64]");
        if (node.op == Op::space_to_depth) channels = tensors.channels(node.inputs[0]) * node.block * node.block;
        break;
    }
    case Op::clamp: {
        const auto* lo = value.get("min");
        const auto* hi = value.get("max");
        if (lo == nullptr || hi == nullptr || lo->kind != json::Value::Kind::number ||
            hi->kind != json::Value::Kind::number) {
            return invalid("clamp needs numeric 'min' and 'max'");
        }
        node.minimum = static_cast<float>(lo->number);
        node.maximum = static_cast<float>(hi->number);
        if (static_cast<double>(node.minimum) != lo->number || static_cast<double>(node.maximum) != hi->number ||
            !(node.minimum <= node.maximum)) {
            return invalid("clamp bounds must be ordered float32 values");
        }
        break;
    }
    case Op::concat:
        channels = tensors.channels(node.inputs[0]) + tensors.channels(node.inputs[1]);
        break;
    case Op::im2col: {
        auto kernel = get_ints<2>(value, "kernel");
        auto stride = get_ints<2>(value, "stride");
        auto pads = get_ints<4>(value, "pads");
        if (!kernel) return kernel.error();
        if (!stride) return stride.error();
        if (!pads) return pads.error();
        node.kernel = kernel.value();
        node.stride = stride.value();
        node.pads = pads.value();
        const bool bad_pad = std::any_of(node.pads.begin(), node.pads.end(), [](std::int32_t p) { return p < 0; });
        if (node.kernel[0] <= 0 || node.kernel[1] <= 0 || node.kernel[0] * node.kernel[1] > 64 ||
            node.stride[0] <= 0 || node.stride[1] <= 0 || bad_pad) {
            return invalid("im2col has an invalid geometry");
        }
        channels = tensors.channels(node.inputs[0]) * node.kernel[0] * node.kernel[1];
        break;
    }
    case Op::crop: {
        auto axis = get_int(value, "axis");
        if (!axis) return axis.error();
        if (axis.value() != 2 && axis.value() != 3) return invalid("crop axis must be 2 or 3");
        node.axis = static_cast<std::int32_t>(axis.value());
        break;
    }
    case Op::mul:
    case Op::add:
    case Op::scale_channels:
    case Op::sigmoid:
        break;
    }

    if (const auto* integer = value.get("integer"); integer != nullptr) {
        auto weight_bits = get_int(*integer, "weight_bits");
        auto activation_bits = get_int(*integer, "activation_bits");
        if (!weight_bits) return weight_bits.error();
        if (!activation_bits) return activation_bits.error();
        node.weight_bits = static_cast<std::int32_t>(weight_bits.value());
        node.activation_bits = static_cast<std::int32_t>(activation_bits.value());
        const auto valid_bits = [](std::int32_t bits) { return bits == 8 || bits == 16; };
        if (node.op != Op::conv || !valid_bits(node.weight_bits) || !valid_bits(node.activation_bits)) {
            return invalid("invalid integer widths on a node");
        }
    }

    auto output = get_text(value, "output");
    if (!output) return output.error();
    if (tensors.contains(output.value())) return invalid("tensor '" + output.value() + "' is defined twice");
    node.output = tensors.define(output.value(), channels);
    return node;
}

Result<std::string> read_file(const std::string& path) {
    std::ifstream stream(path, std::ios::binary);
    if (!stream) return fail(Code::io_error, "cannot open " + path);
    std::ostringstream contents;
    contents << stream.rdbuf();
    if (!stream && !stream.eof()) return fail(Code::io_error, "cannot read " + path);
    return contents.str();
}

}  // namespace

bool is_integer_pointwise(const Node& node) {
    return node.op == Op::conv && !node.depthwise && node.kernel == std::array<std::int32_t, 2>{1, 1} &&
        node.stride == std::array<std::int32_t, 2>{1, 1} && node.pads == std::array<std::int32_t, 4>{0, 0, 0, 0};
}

float half_to_float(std::uint16_t half) {
    const std::uint32_t sign = static_cast<std::uint32_t>(half & 0x8000u) << 16;
    const std::uint32_t exponent = (half >> 10) & 0x1fu;
    std::uint32_t mantissa = half & 0x3ffu;
    std::uint32_t bits;
    if (exponent == 0x1fu) {
        bits = sign | 0x7f800000u | (mantissa << 13);
    } else if (exponent != 0) {
        bits = sign | ((exponent + 112u) << 23) | (mantissa << 13);
    } else if (mantissa == 0) {
        bits = sign;
    } else {
        // value = mantissa * 2^-24; normalise so the leading one is bit 10.
        int leading = 31 - __builtin_clz(mantissa);  // 0..9
        const std::uint32_t fraction = (mantissa << (10 - leading)) & 0x3ffu;
        bits = sign | (static_cast<std::uint32_t>(leading + 103) << 23) | (fraction << 13);
    }
    float value;
    std::memcpy(&value, &bits, 4);
    return value;
}

std::uint16_t float_to_half(float value) {
    std::uint32_t bits;
    std::memcpy(&bits, &value, 4);
    const std::uint32_t sign = (bits >> 16) & 0x8000u;
    const std::uint32_t magnitude = bits & 0x7fffffffu;
    if (magnitude >= 0x7f800000u) return static_cast<std::uint16_t>(sign | 0x7c00u | (magnitude > 0x7f800000u ? 0x200u : 0));
    if (magnitude >= 0x47800000u) return static_cast<std::uint16_t>(sign | 0x7c00u);  // >= 2^16: overflow
    const int exponent = static_cast<int>(magnitude >> 23) - 127;
    std::uint32_t significand = (magnitude & 0x7fffffu) | 0x800000u;
    if (exponent >= -14) {
        std::uint32_t out = (static_cast<std::uint32_t>(exponent + 15) << 10) | ((significand >> 13) & 0x3ffu);
        const std::uint32_t rest = significand & 0x1fffu;
        if (rest > 0x1000u || (rest == 0x1000u && (out & 1u))) ++out;  // a carry may reach infinity
        return static_cast<std::uint16_t>(sign | out);
    }
    if (exponent < -25) return static_cast<std::uint16_t>(sign);
    const std::uint32_t shift = static_cast<std::uint32_t>(-1 - exponent);  // 14..24 bits dropped
    std::uint32_t out = significand >> shift;
    const std::uint32_t rest = significand & ((1u << shift) - 1u);
    const std::uint32_t half = 1u << (shift - 1u);
    if (rest > half || (rest == half && (out & 1u))) ++out;
    return static_cast<std::uint16_t>(sign | out);
}

Result<Program> load_program_text(std::string_view text, const std::string& directory, const float* weights,
                                  std::size_t weight_count) {
    auto parsed = json::parse(text);
    if (!parsed) return parsed.error();
    const auto& root = parsed.value();
    auto format = get_text(root, "format");
    auto numerics = get_text(root, "numerics");
    auto version = get_int(root, "version");
    if (!format || format.value() != "nvcr.deterministic-program" || !version || version.value() != 1) {
        return invalid("not an NVCR deterministic program v1");
    }
    if (!numerics || numerics.value() != intconv_profile) return invalid("unsupported deterministic numerics");
    Program program;
    program.numerics = numerics.value();
    auto name = get_text(root, "name");
    if (!name) return name.error();
    program.name = name.value();

    const auto* weight_info = root.get("weights");
    if (weight_info == nullptr) return invalid("program has no weights");
    auto file = get_text(*weight_info, "file");
    auto count = get_int(*weight_info, "count");
    auto digest = get_text(*weight_info, "sha256");
    if (!file) return file.error();
    if (!count || count.value() < 0) return invalid("invalid weights count");
    if (!digest) return digest.error();
    if (file.value().find('/') != std::string::npos || file.value().find('\\') != std::string::npos) {
        return invalid("weights file must sit next to the program");
    }
    if (weights != nullptr) {
        if (weight_count != static_cast<std::size_t>(count.value())) {
            return invalid("in-memory weights do not match the declared count");
        }
        program.weights.assign(weights, weights + weight_count);
    } else {
        const std::string path = (directory.empty() ? std::string(".") : directory) + "/" + file.value();
        auto blob = read_file(path);
        if (!blob) return blob.error();
        if (sha256_hex(blob.value().data(), blob.value().size()) != digest.value()) {
            return fail(Code::digest_mismatch, "deterministic weights digest mismatch: " + path);
        }
        if (blob.value().size() != static_cast<std::size_t>(count.value()) * 2) {
            return invalid("weights file size does not match the declared count");
        }
        program.weights.resize(static_cast<std::size_t>(count.value()));
        for (std::size_t i = 0; i < program.weights.size(); ++i) {
            const auto lo = static_cast<unsigned char>(blob.value()[2 * i]);
            const auto hi = static_cast<unsigned char>(blob.value()[2 * i + 1]);
            program.weights[i] = half_to_float(static_cast<std::uint16_t>(lo | (hi << 8)));
        }
    }
    program.weights_sha256 = digest.value();

    Tensors tensors(program);
    const auto* inputs = root.get("inputs");
    const auto* outputs = root.get("outputs");
    const auto* nodes = root.get("nodes");
    if (inputs == nullptr || outputs == nullptr || nodes == nullptr) {
        return invalid("program needs inputs, outputs, and nodes");
    }
    for (const auto& input : inputs->items) {
        auto input_name = get_text(input, "name");
        auto channels = get_int(input, "channels");
        if (!input_name) return input_name.error();
        if (!channels || channels.value() <= 0) return invalid("input channels must be positive");
        program.inputs.push_back(tensors.define(input_name.value(), static_cast<std::int32_t>(channels.value())));
    }
    for (const auto& item : nodes->items) {
        auto node = parse_node(item, tensors, program.weights.size());
        if (!node) return node.error();
        auto& channels = program.tensor_channels[node.value().output];
        if (channels == 0) {
            const auto source = program.tensor_channels[node.value().inputs[0]];
            channels = node.value().op == Op::depth_to_space ? source / (node.value().block * node.value().block)
                                                            : source;
        }
        program.nodes.push_back(node.value());
    }
    for (const auto& output : outputs->items) {
        auto output_name = get_text(output, "name");
        if (!output_name) return output_name.error();
        auto id = tensors.find(output_name.value());
        if (!id) return id.error();
        program.outputs.push_back(id.value());
    }
    program.last_use.assign(program.tensor_names.size(), 0);
    for (std::size_t index = 0; index < program.nodes.size(); ++index) {
        const auto& node = program.nodes[index];
        for (std::size_t i = 0; i < node.input_count; ++i) program.last_use[node.inputs[i]] = index;
    }
    for (const auto id : program.outputs) program.last_use[id] = program.nodes.size();
    return program;
}

Result<Program> load_program_file(const std::string& path) {
    auto text = read_file(path);
    if (!text) return text.error();
    const auto slash = path.find_last_of('/');
    const std::string directory = slash == std::string::npos ? std::string(".") : path.substr(0, slash);
    return load_program_text(text.value(), directory, nullptr, 0);
}

Result<Extent> output_extent(const Program& program, const Node& node, const Extent* inputs,
                             std::size_t input_count) {
    const Extent& in = inputs[0];
    if (in.channels != program.tensor_channels[node.inputs[0]] || in.height <= 0 || in.width <= 0) {
        return invalid("tensor '" + program.tensor_names[node.inputs[0]] + "' has an unexpected shape");
    }
    const Extent* second = input_count > 1 ? &inputs[1] : nullptr;
    switch (node.op) {
    case Op::conv:
    case Op::im2col: {
        if (node.op == Op::conv && in.channels != node.in_channels) return invalid("conv input channel mismatch");
        const auto h = in.height + node.pads[0] + node.pads[2] - node.kernel[0];
        const auto w = in.width + node.pads[1] + node.pads[3] - node.kernel[1];
        if (h < 0 || w < 0) return invalid("input is smaller than its kernel");
        const auto c = node.op == Op::conv ? node.out_channels : in.channels * node.kernel[0] * node.kernel[1];
        return Extent{c, h / node.stride[0] + 1, w / node.stride[1] + 1};
    }
    case Op::mul:
    case Op::add:
        if (second == nullptr || second->channels != in.channels || second->height != in.height ||
            second->width != in.width) {
            return invalid("elementwise inputs differ in shape");
        }
        return in;
    case Op::scale_channels:
        if (second == nullptr || second->channels != in.channels || second->height != 1 || second->width != 1) {
            return invalid("scale_channels needs a [C, 1, 1] scale");
        }
        return in;
    case Op::concat:
        if (second == nullptr || second->height != in.height || second->width != in.width ||
            second->channels != program.tensor_channels[node.inputs[1]]) {
            return invalid("concat inputs differ in spatial shape");
        }
        return Extent{in.channels + second->channels, in.height, in.width};
    case Op::crop:
        if (second == nullptr || (node.axis == 2 ? second->height > in.height : second->width > in.width)) {
            return invalid("crop reference is larger than its input");
        }
        return node.axis == 2 ? Extent{in.channels, second->height, in.width}
                              : Extent{in.channels, in.height, second->width};
    case Op::space_to_depth:
        if (in.height % node.block != 0 || in.width % node.block != 0) {
            return invalid("space_to_depth input is not a multiple of its block");
        }
        return Extent{in.channels * node.block * node.block, in.height / node.block, in.width / node.block};
    case Op::mul_scalar:
    case Op::sigmoid:
    case Op::clamp:
        return in;
    case Op::slice_channels:
        if (node.begin < 0 || node.end <= node.begin || node.end > in.channels) {
            return invalid("channel slice is out of range");
        }
        return Extent{node.end - node.begin, in.height, in.width};
    case Op::depth_to_space:
        if (in.channels % (node.block * node.block) != 0) return invalid("depth_to_space channels are not divisible");
        return Extent{in.channels / (node.block * node.block), in.height * node.block, in.width * node.block};
    }
    return invalid("unknown op");
}

Result<std::vector<Extent>> infer_output_extents(const Program& program, const std::vector<Extent>& inputs) {
    if (inputs.size() != program.inputs.size()) return invalid(program.name + ": wrong number of inputs");
    std::vector<Extent> extents(program.tensor_names.size());
    std::vector<bool> known(program.tensor_names.size(), false);
    for (std::size_t slot = 0; slot < inputs.size(); ++slot) {
        extents[program.inputs[slot]] = inputs[slot];
        known[program.inputs[slot]] = true;
    }
    for (const auto& node : program.nodes) {
        Extent node_inputs[2];
        for (std::size_t i = 0; i < node.input_count; ++i) {
            if (!known[node.inputs[i]]) return invalid(program.name + ": tensor read before written");
            node_inputs[i] = extents[node.inputs[i]];
        }
        auto extent = output_extent(program, node, node_inputs, node.input_count);
        if (!extent) return extent.error();
        extents[node.output] = extent.value();
        known[node.output] = true;
    }
    std::vector<Extent> outputs;
    for (const auto id : program.outputs) {
        if (!known[id]) return invalid(program.name + ": output not produced");
        outputs.push_back(extents[id]);
    }
    return outputs;
}

IntegerWeights quantize_weights(const Program& program, const Node& node) {
    const auto rows = static_cast<std::size_t>(node.out_channels);
    const auto columns = static_cast<std::size_t>(node.in_channels);
    IntegerWeights out;
    out.values.assign(rows * columns, 0);
    out.scales.assign(rows, 1.0f);
    for (std::size_t row = 0; row < rows; ++row) {
        const float* w = program.weights.data() + node.weight_offset + row * columns;
        float maximum = 0.0f;
        // A NaN magnitude never replaces the running maximum (max(a, b) keeps a
        // unless a < b).
        for (std::size_t column = 0; column < columns; ++column) {
            const float magnitude = std::fabs(w[column]);
            if (maximum < magnitude) maximum = magnitude;
        }
        if (maximum == 0.0f) continue;
        const double limit = node.weight_bits == 16 ? 32767.0 : 127.0;
        const double scale = static_cast<double>(maximum) / limit;
        out.scales[row] = static_cast<float>(scale);
        for (std::size_t column = 0; column < columns; ++column) {
            double q = std::nearbyint(static_cast<double>(w[column]) / scale);
            if (q < -limit) q = -limit;
            else if (limit < q) q = limit;
            // A NaN quotient stores 0, as the reference's int16 conversion does on x86-64.
            out.values[row * columns + column] = q == q ? static_cast<std::int16_t>(q) : 0;
        }
    }
    return out;
}

}  // namespace nvcr_sm100
