#include "program.hpp"

#include "json.hpp"
#include "sha256.hpp"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <fstream>
#include <iterator>
#include <optional>
#include <sstream>
#include <unordered_map>

namespace nvcr_sm100 {
namespace {

Error invalid(const std::string& message) { return fail(Code::invalid_argument, message); }

// ------------------------------------------------------------ node schema
//
// A node is read in two passes. First every key its op's schema lists is
// fetched from the JSON object into a Fields record, checking only the JSON
// shape of each (an integer, a fixed-length integer array, a boolean, a number
// that is exactly a float32). Then the op's rule turns the record into the
// Node, refusing values the profile does not allow, and names the output's
// channel count. The node's inputs and output are resolved around the two
// passes against the tensors defined so far.

enum class Shape : std::uint8_t { integer, pair, quad, flag, exact_float, number };

enum Key : std::uint8_t {
    k_in_channels, k_out_channels, k_kernel, k_stride, k_pads, k_weight_offset, k_bias_offset, k_depthwise,
    k_value, k_begin, k_end, k_block, k_min, k_max, k_axis, key_count
};

constexpr struct {
    std::string_view json;
    Shape shape;
} keys[key_count] = {
    {"in_channels", Shape::integer}, {"out_channels", Shape::integer}, {"kernel", Shape::pair},
    {"stride", Shape::pair},         {"pads", Shape::quad},            {"weight_offset", Shape::integer},
    {"bias_offset", Shape::integer}, {"depthwise", Shape::flag},       {"value", Shape::exact_float},
    {"begin", Shape::integer},       {"end", Shape::integer},          {"block", Shape::integer},
    {"min", Shape::number},          {"max", Shape::number},           {"axis", Shape::integer},
};

// The values of one node's keys, by Key.
struct Fields {
    std::int64_t integer[key_count]{};
    std::array<std::int32_t, 4> list[key_count]{};
    bool flag[key_count]{};
    double number[key_count]{};
};

std::string quoted(Key key) { return "'" + std::string(keys[key].json) + "'"; }

// Fetches `key` from a node object into `fields`, checking its JSON shape.
std::optional<Error> fetch(const json::Value& object, Key key, std::string_view op, Fields& fields) {
    const json::Value* v = object.get(keys[key].json);
    const auto is_integer = [](const json::Value* x) {
        return x != nullptr && x->kind == json::Value::Kind::number && x->integer.has_value();
    };
    switch (keys[key].shape) {
    case Shape::integer:
        if (!is_integer(v)) return invalid(std::string(op) + " field " + quoted(key) + " is not an integer");
        fields.integer[key] = *v->integer;
        return std::nullopt;
    case Shape::pair:
    case Shape::quad: {
        const std::size_t length = keys[key].shape == Shape::pair ? 2 : 4;
        if (v == nullptr || v->kind != json::Value::Kind::array || v->items.size() != length) {
            return invalid(std::string(op) + " field " + quoted(key) + " is not a list of " +
                           std::to_string(length) + " values");
        }
        for (std::size_t i = 0; i < length; ++i) {
            if (!is_integer(&v->items[i])) {
                return invalid(std::string(op) + " field " + quoted(key) + " holds a non-integer");
            }
            fields.list[key][i] = static_cast<std::int32_t>(*v->items[i].integer);
        }
        return std::nullopt;
    }
    case Shape::flag:
        if (v == nullptr || v->kind != json::Value::Kind::boolean) {
            return invalid(std::string(op) + " field " + quoted(key) + " is not a boolean");
        }
        fields.flag[key] = v->boolean;
        return std::nullopt;
    case Shape::exact_float:
    case Shape::number:
        if (v == nullptr || v->kind != json::Value::Kind::number) {
            return invalid(std::string(op) + " field " + quoted(key) + " is not a number");
        }
        if (keys[key].shape == Shape::exact_float && static_cast<double>(static_cast<float>(v->number)) != v->number) {
            return invalid(std::string(op) + " field " + quoted(key) + " is not exactly a float32");
        }
        fields.number[key] = v->number;
        return std::nullopt;
    }
    return invalid("unknown field shape");
}

// Reading context of the op rules: the channels of the node's first input and
// second input (0 when unary), and the weights the file holds.
struct Context {
    std::int32_t first_channels;
    std::int32_t second_channels;
    std::size_t weight_count;
};

// An op rule fills the node's op-specific members from the fetched fields and
// returns the output's channel count, or refuses the node.
using Rule = Result<std::int32_t> (*)(const Fields&, const Context&, Node&);

bool any_negative(const std::array<std::int32_t, 4>& values) {
    return values[0] < 0 || values[1] < 0 || values[2] < 0 || values[3] < 0;
}

Result<std::int32_t> conv_rule(const Fields& f, const Context& context, Node& node) {
    const std::int64_t weight_offset = f.integer[k_weight_offset];
    const std::int64_t bias_offset = f.integer[k_bias_offset];
    node.in_channels = static_cast<std::int32_t>(f.integer[k_in_channels]);
    node.out_channels = static_cast<std::int32_t>(f.integer[k_out_channels]);
    node.depthwise = f.flag[k_depthwise];
    node.kernel = {f.list[k_kernel][0], f.list[k_kernel][1]};
    node.stride = {f.list[k_stride][0], f.list[k_stride][1]};
    node.pads = f.list[k_pads];
    const bool positive = node.in_channels > 0 && node.out_channels > 0 && node.kernel[0] > 0 && node.kernel[1] > 0 &&
        node.stride[0] > 0 && node.stride[1] > 0;
    if (!positive || any_negative(node.pads) || weight_offset < 0 || bias_offset < 0 ||
        (node.depthwise && node.in_channels != node.out_channels)) {
        return invalid("conv geometry or offsets out of range");
    }
    node.weight_offset = static_cast<std::size_t>(weight_offset);
    node.bias_offset = static_cast<std::size_t>(bias_offset);
    // [out][in or 1][kh][kw] weights from weight_offset, out_channels biases from bias_offset.
    const std::size_t fan_in = static_cast<std::size_t>(node.depthwise ? 1 : node.in_channels) *
        static_cast<std::size_t>(node.kernel[0]) * static_cast<std::size_t>(node.kernel[1]);
    const std::size_t total = context.weight_count;
    const auto fits = [total](std::size_t at, std::size_t count) { return at <= total && count <= total - at; };
    if (!fits(node.weight_offset, static_cast<std::size_t>(node.out_channels) * fan_in) ||
        !fits(node.bias_offset, static_cast<std::size_t>(node.out_channels))) {
        return invalid("conv reads past the end of the weights file");
    }
    return node.out_channels;
}

Result<std::int32_t> scalar_rule(const Fields& f, const Context& context, Node& node) {
    node.scalar = static_cast<float>(f.number[k_value]);
    return context.first_channels;
}

Result<std::int32_t> slice_rule(const Fields& f, const Context&, Node& node) {
    node.begin = static_cast<std::int32_t>(f.integer[k_begin]);
    node.end = static_cast<std::int32_t>(f.integer[k_end]);
    return node.end - node.begin;
}

Result<std::int32_t> block_rule(const Fields& f, const Context& context, Node& node) {
    node.block = static_cast<std::int32_t>(f.integer[k_block]);
    if (node.block < 1 || node.block > 64) return invalid("block must lie in 1..64");
    const std::int32_t area = node.block * node.block;
    return node.op == Op::space_to_depth ? context.first_channels * area : context.first_channels / area;
}

Result<std::int32_t> clamp_rule(const Fields& f, const Context& context, Node& node) {
    node.minimum = static_cast<float>(f.number[k_min]);
    node.maximum = static_cast<float>(f.number[k_max]);
    const bool exact = static_cast<double>(node.minimum) == f.number[k_min] &&
        static_cast<double>(node.maximum) == f.number[k_max];
    if (!exact || !(node.minimum <= node.maximum)) return invalid("clamp needs ordered, exactly float32 bounds");
    return context.first_channels;
}

Result<std::int32_t> im2col_rule(const Fields& f, const Context& context, Node& node) {
    node.kernel = {f.list[k_kernel][0], f.list[k_kernel][1]};
    node.stride = {f.list[k_stride][0], f.list[k_stride][1]};
    node.pads = f.list[k_pads];
    const std::int32_t taps = node.kernel[0] * node.kernel[1];
    if (node.kernel[0] < 1 || node.kernel[1] < 1 || taps > 64 || node.stride[0] < 1 || node.stride[1] < 1 ||
        any_negative(node.pads)) {
        return invalid("im2col geometry out of range");
    }
    return context.first_channels * taps;
}

Result<std::int32_t> crop_rule(const Fields& f, const Context& context, Node& node) {
    if (f.integer[k_axis] != 2 && f.integer[k_axis] != 3) return invalid("crop axis is neither 2 nor 3");
    node.axis = static_cast<std::int32_t>(f.integer[k_axis]);
    return context.first_channels;
}

Result<std::int32_t> concat_rule(const Fields&, const Context& context, Node&) {
    return context.first_channels + context.second_channels;
}

Result<std::int32_t> same_rule(const Fields&, const Context& context, Node&) { return context.first_channels; }

struct OpSchema {
    std::string_view name;
    Op op;
    bool binary;
    std::uint32_t keys;  // bit k: Key k is required
    Rule rule;
};

constexpr std::uint32_t bits() { return 0; }
template <typename... Rest>
constexpr std::uint32_t bits(Key first, Rest... rest) {
    return (1u << first) | bits(rest...);
}

constexpr OpSchema schemas[] = {
    {"conv", Op::conv, false,
     bits(k_in_channels, k_out_channels, k_kernel, k_stride, k_pads, k_weight_offset, k_bias_offset, k_depthwise),
     conv_rule},
    {"mul", Op::mul, true, 0, same_rule},
    {"add", Op::add, true, 0, same_rule},
    {"mul_scalar", Op::mul_scalar, false, bits(k_value), scalar_rule},
    {"sigmoid", Op::sigmoid, false, 0, same_rule},
    {"slice_channels", Op::slice_channels, false, bits(k_begin, k_end), slice_rule},
    {"depth_to_space", Op::depth_to_space, false, bits(k_block), block_rule},
    {"scale_channels", Op::scale_channels, true, 0, same_rule},
    {"clamp", Op::clamp, false, bits(k_min, k_max), clamp_rule},
    {"concat", Op::concat, true, 0, concat_rule},
    {"crop", Op::crop, true, bits(k_axis), crop_rule},
    {"space_to_depth", Op::space_to_depth, false, bits(k_block), block_rule},
    {"im2col", Op::im2col, false, bits(k_kernel, k_stride, k_pads), im2col_rule},
};

// Names to tensor ids while a program is read; also owns the growing Program.
class ProgramBuilder {
public:
    Program program;

    std::size_t add_tensor(const std::string& name, std::int32_t channels) {
        const std::size_t id = program.tensor_names.size();
        program.tensor_names.push_back(name);
        program.tensor_channels.push_back(channels);
        by_name_[name] = id;
        return id;
    }
    std::optional<std::size_t> lookup(const std::string& name) const {
        const auto found = by_name_.find(name);
        return found == by_name_.end() ? std::nullopt : std::optional<std::size_t>(found->second);
    }
    Result<std::size_t> existing(const std::string& name) const {
        if (auto id = lookup(name)) return *id;
        return invalid("no tensor named '" + name + "' is defined before this use");
    }

    // One node object: schema lookup, inputs, fields, rule, widths, output.
    std::optional<Error> read_node(const json::Value& object) {
        const json::Value* op_value = object.get("op");
        if (op_value == nullptr || op_value->kind != json::Value::Kind::string) {
            return invalid("node without a string 'op'");
        }
        const OpSchema* schema = nullptr;
        for (const auto& candidate : schemas) {
            if (candidate.name == op_value->text) schema = &candidate;
        }
        if (schema == nullptr) return invalid("op '" + op_value->text + "' is not part of nvcr.intconv.v1");
        Node node;
        node.op = schema->op;
        node.input_count = schema->binary ? 2 : 1;
        if (schema->binary) {
            const json::Value* list = object.get("inputs");
            if (list == nullptr || list->items.size() != 2) return invalid(std::string(schema->name) + " takes two inputs");
            for (std::size_t i = 0; i < 2; ++i) {
                auto id = existing(list->items[i].text);
                if (!id) return id.error();
                node.inputs[i] = id.value();
            }
        } else {
            const json::Value* single = object.get("input");
            if (single == nullptr || single->kind != json::Value::Kind::string) {
                return invalid(std::string(schema->name) + " needs a string 'input'");
            }
            auto id = existing(single->text);
            if (!id) return id.error();
            node.inputs[0] = id.value();
        }
        Fields fields;
        for (int key = 0; key < key_count; ++key) {
            if ((schema->keys >> key) & 1u) {
                if (auto error = fetch(object, static_cast<Key>(key), schema->name, fields)) return error;
            }
        }
        const Context context{program.tensor_channels[node.inputs[0]],
                              schema->binary ? program.tensor_channels[node.inputs[1]] : 0,
                              program.weights.size()};
        auto channels = schema->rule(fields, context, node);
        if (!channels) return channels.error();
        if (const json::Value* widths = object.get("integer"); widths != nullptr) {
            std::int32_t chosen[2] = {0, 0};
            const std::string_view names[2] = {"weight_bits", "activation_bits"};
            for (int i = 0; i < 2; ++i) {
                const json::Value* v = widths->get(names[i]);
                if (v == nullptr || v->kind != json::Value::Kind::number || !v->integer) {
                    return invalid("integer width '" + std::string(names[i]) + "' is not an integer");
                }
                chosen[i] = static_cast<std::int32_t>(*v->integer);
            }
            const auto allowed = [](std::int32_t b) { return b == 8 || b == 16; };
            if (node.op != Op::conv || !allowed(chosen[0]) || !allowed(chosen[1])) {
                return invalid("integer widths must be 8 or 16 and belong to a conv");
            }
            node.weight_bits = chosen[0];
            node.activation_bits = chosen[1];
        }
        const json::Value* output = object.get("output");
        if (output == nullptr || output->kind != json::Value::Kind::string) {
            return invalid(std::string(schema->name) + " needs a string 'output'");
        }
        if (lookup(output->text)) return invalid("tensor '" + output->text + "' is written by two nodes");
        node.output = add_tensor(output->text, channels.value());
        program.nodes.push_back(node);
        return std::nullopt;
    }

private:
    std::unordered_map<std::string, std::size_t> by_name_;
};

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

namespace {

// A top-level string or integer member of the program document, or nothing.
const std::string* text_member(const json::Value& object, std::string_view key) {
    const json::Value* v = object.get(key);
    return v != nullptr && v->kind == json::Value::Kind::string ? &v->text : nullptr;
}
std::optional<std::int64_t> integer_member(const json::Value& object, std::string_view key) {
    const json::Value* v = object.get(key);
    if (v == nullptr || v->kind != json::Value::Kind::number || !v->integer) return std::nullopt;
    return v->integer;
}

// The weights block: in-memory values, or the FP16 file beside the program,
// which must hash to the declared SHA-256 and hold exactly `count` values.
std::optional<Error> read_weights(const json::Value& root, const std::string& directory, const float* weights,
                                  std::size_t weight_count, Program& program) {
    const json::Value* block = root.get("weights");
    if (block == nullptr) return invalid("the program declares no weights");
    const std::string* file = text_member(*block, "file");
    const auto count = integer_member(*block, "count");
    const std::string* digest = text_member(*block, "sha256");
    if (file == nullptr) return invalid("weights 'file' is not a string");
    if (!count || *count < 0) return invalid("weights 'count' is not a non-negative integer");
    if (digest == nullptr) return invalid("weights 'sha256' is not a string");
    if (file->find_first_of("/\\") != std::string::npos) return invalid("the weights file must sit beside the program");
    const auto declared = static_cast<std::size_t>(*count);
    if (weights != nullptr) {
        if (weight_count != declared) return invalid("in-memory weights disagree with the declared count");
        program.weights.assign(weights, weights + weight_count);
    } else {
        const std::string path = (directory.empty() ? std::string(".") : directory) + "/" + *file;
        auto blob = read_file(path);
        if (!blob) return blob.error();
        const std::string& bytes = blob.value();
        if (sha256_hex(bytes.data(), bytes.size()) != *digest) {
            return fail(Code::digest_mismatch, "weights file does not match its declared SHA-256: " + path);
        }
        if (bytes.size() != 2 * declared) return invalid("weights file length disagrees with the declared count");
        program.weights.resize(declared);
        for (std::size_t i = 0; i < declared; ++i) {
            const std::uint16_t bits = static_cast<std::uint16_t>(static_cast<unsigned char>(bytes[2 * i]) |
                                                                  (static_cast<unsigned char>(bytes[2 * i + 1]) << 8));
            program.weights[i] = half_to_float(bits);
        }
    }
    program.weights_sha256 = *digest;
    return std::nullopt;
}

}  // namespace

Result<Program> load_program_text(std::string_view text, const std::string& directory, const float* weights,
                                  std::size_t weight_count) {
    auto parsed = json::parse(text);
    if (!parsed) return parsed.error();
    const json::Value& root = parsed.value();

    // Header: format, version, profile, name.
    const std::string* format = text_member(root, "format");
    const auto version = integer_member(root, "version");
    if (format == nullptr || *format != "nvcr.deterministic-program" || version != std::optional<std::int64_t>(1)) {
        return invalid("the document is not an nvcr.deterministic-program of version 1");
    }
    const std::string* numerics = text_member(root, "numerics");
    if (numerics == nullptr || *numerics != intconv_profile) return invalid("the program's numerics is not nvcr.intconv.v1");
    const std::string* name = text_member(root, "name");
    if (name == nullptr) return invalid("the program's 'name' is not a string");

    ProgramBuilder builder;
    builder.program.numerics = *numerics;
    builder.program.name = *name;
    if (auto error = read_weights(root, directory, weights, weight_count, builder.program)) return *error;

    // Graph: inputs define tensors, nodes read defined tensors and define one
    // more each, outputs name defined tensors.
    const json::Value* inputs = root.get("inputs");
    const json::Value* nodes = root.get("nodes");
    const json::Value* outputs = root.get("outputs");
    if (inputs == nullptr || nodes == nullptr || outputs == nullptr) {
        return invalid("the program lacks 'inputs', 'nodes' or 'outputs'");
    }
    for (const json::Value& input : inputs->items) {
        const std::string* input_name = text_member(input, "name");
        if (input_name == nullptr) return invalid("an input's 'name' is not a string");
        const auto channels = integer_member(input, "channels");
        if (!channels || *channels <= 0) return invalid("an input's 'channels' is not a positive integer");
        builder.program.inputs.push_back(builder.add_tensor(*input_name, static_cast<std::int32_t>(*channels)));
    }
    for (const json::Value& node : nodes->items) {
        if (auto error = builder.read_node(node)) return *error;
    }
    for (const json::Value& output : outputs->items) {
        const std::string* output_name = text_member(output, "name");
        if (output_name == nullptr) return invalid("an output's 'name' is not a string");
        auto id = builder.existing(*output_name);
        if (!id) return id.error();
        builder.program.outputs.push_back(id.value());
    }

    // Liveness: the index of each tensor's last reading node; stage outputs
    // live to the end.
    Program& program = builder.program;
    program.last_use.assign(program.tensor_names.size(), 0);
    for (std::size_t index = 0; index < program.nodes.size(); ++index) {
        for (std::size_t i = 0; i < program.nodes[index].input_count; ++i) {
            program.last_use[program.nodes[index].inputs[i]] = index;
        }
    }
    for (const std::size_t id : program.outputs) program.last_use[id] = program.nodes.size();
    return std::move(builder.program);
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
