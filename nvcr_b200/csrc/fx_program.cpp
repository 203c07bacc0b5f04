#include "fx_program.hpp"

#include "json.hpp"
#include "sha256.hpp"

#include <climits>
#include <cstring>
#include <fstream>
#include <iterator>

namespace nvcr_sm100::fx {
namespace {

using json::Value;

Error invalid(const std::string& message) { return fail(Code::invalid_argument, "fx program: " + message); }

const Value* member(const Value& object, std::string_view key) {
    return object.kind == Value::Kind::object ? object.get(key) : nullptr;
}

const std::vector<Value>& items(const Value* value) {
    static const std::vector<Value> none;
    return value != nullptr && value->kind == Value::Kind::array ? value->items : none;
}

std::string text(const Value* value) {
    return value != nullptr && value->kind == Value::Kind::string ? value->text : std::string();
}

std::optional<std::int64_t> integer_of(const Value* value) {
    if (value == nullptr || value->kind != Value::Kind::number) return std::nullopt;
    return value->integer;
}

Result<std::int64_t> integer(const Value& object, std::string_view key) {
    const auto value = integer_of(member(object, key));
    if (!value) return invalid("field '" + std::string(key) + "' must be an integer");
    return *value;
}

Result<int> ranged(const Value& object, std::string_view key, std::int64_t lo, std::int64_t hi) {
    auto value = integer(object, key);
    if (!value) return value.error();
    if (value.value() < lo || value.value() > hi) return invalid("field '" + std::string(key) + "' out of range");
    return static_cast<int>(value.value());
}

// A [byte offset, element count] reference into the data file.
template <typename T>
Result<std::vector<T>> data_array(const Value& object, std::string_view key, const std::string& data) {
    const auto& pair = items(member(object, key));
    const auto offset = pair.size() == 2 ? integer_of(&pair[0]) : std::nullopt;
    const auto count = pair.size() == 2 ? integer_of(&pair[1]) : std::nullopt;
    if (!offset || !count) return invalid("field '" + std::string(key) + "' must be [offset, count]");
    if (*offset < 0 || *count < 0 || static_cast<std::uint64_t>(*offset) > data.size() ||
        static_cast<std::uint64_t>(*count) > (data.size() - static_cast<std::size_t>(*offset)) / sizeof(T)) {
        return invalid("field '" + std::string(key) + "' lies outside the data file");
    }
    std::vector<T> out(static_cast<std::size_t>(*count));
    if (!out.empty()) std::memcpy(out.data(), data.data() + *offset, out.size() * sizeof(T));
    return out;
}

template <typename T>
bool within(const std::vector<T>& values, std::int64_t lo, std::int64_t hi) {
    for (const auto v : values) {
        if (static_cast<std::int64_t>(v) < lo || static_cast<std::int64_t>(v) > hi) return false;
    }
    return true;
}

constexpr std::int64_t bias_bound = std::int64_t{1} << 52;
constexpr std::int64_t table_bound = std::int64_t{1} << 24;

constexpr std::pair<std::string_view, FxOp> op_table[] = {
    {"gemm", FxOp::gemm}, {"depthwise3x3", FxOp::depthwise3x3}, {"mul", FxOp::mul}, {"affine", FxOp::affine},
    {"add", FxOp::add}, {"sat_table", FxOp::sat_table}, {"delta", FxOp::delta}, {"clamp", FxOp::clamp},
    {"concat", FxOp::concat}, {"slice", FxOp::slice}, {"pixel_shuffle", FxOp::pixel_shuffle},
    {"pixel_unshuffle", FxOp::pixel_unshuffle}, {"im2col", FxOp::im2col}, {"param_row", FxOp::param_row},
    {"crop_like", FxOp::crop_like},
};

std::size_t required_inputs(FxOp op) {
    switch (op) {
    case FxOp::mul:
    case FxOp::add:
    case FxOp::concat:
    case FxOp::crop_like:
        return 2;
    default:
        return 1;
    }
}

Result<FxNode> parse_node(const Value& entry, const FxProgram& program, const std::string& data) {
    FxNode node;
    const std::string name = text(member(entry, "op"));
    bool known = false;
    for (const auto& [label, op] : op_table) {
        if (label == name && member(entry, "op") != nullptr) {
            node.op = op;
            known = true;
        }
    }
    if (!known) return invalid("unknown op");
    const auto* inputs = member(entry, "inputs");
    if (inputs == nullptr) return invalid("node without inputs");
    for (const auto& input : items(inputs)) {
        const auto id = integer_of(&input);
        if (!id || *id < 0 || static_cast<std::uint64_t>(*id) >= program.tensor_names.size()) {
            return invalid("node input out of range");
        }
        node.inputs.push_back(static_cast<std::uint32_t>(*id));
    }
    const std::size_t residuals = node.op == FxOp::gemm ? 2 : 0;
    if (node.inputs.size() < required_inputs(node.op) || node.inputs.size() > required_inputs(node.op) + residuals) {
        return invalid("wrong number of node inputs");
    }
    auto output = ranged(entry, "output", 0, static_cast<std::int64_t>(program.tensor_names.size()) - 1);
    if (!output) return output.error();
    node.output = static_cast<std::uint32_t>(output.value());
    const auto table_ok = [&](int index) {
        return index >= -1 && index < static_cast<int>(program.delta_tables.size());
    };
    const auto channels_of = [&](std::uint32_t id) { return program.tensor_channels[id]; };

    switch (node.op) {
    case FxOp::gemm: {
        auto in = ranged(entry, "in_channels", 1, 1 << 20);
        auto out = ranged(entry, "out_channels", 1, 1 << 20);
        auto group = ranged(entry, "group", 1, 4);
        auto input_shift = ranged(entry, "input_shift", 0, 30);
        auto table = ranged(entry, "delta_table", -1, 1 << 20);
        for (const auto* field : {&in, &out, &group, &input_shift, &table}) {
            if (!*field) return field->error();
        }
        auto weights = data_array<std::int16_t>(entry, "weights", data);
        if (!weights) return weights.error();
        auto bias = data_array<std::int64_t>(entry, "bias", data);
        if (!bias) return bias.error();
        auto shifts = data_array<std::int32_t>(entry, "shift", data);
        if (!shifts) return shifts.error();
        node.in_channels = in.value();
        node.out_channels = out.value();
        node.group = group.value();
        node.input_shift = input_shift.value();
        node.delta_table = table.value();
        node.gemm_weights = std::move(weights.value());
        node.bias = std::move(bias.value());
        node.shifts = std::move(shifts.value());
        const auto rows = static_cast<std::size_t>(node.out_channels);
        if (node.group == 3 || node.out_channels % node.group != 0 || !table_ok(node.delta_table) ||
            node.gemm_weights.size() != rows * static_cast<std::size_t>(node.in_channels) ||
            node.bias.size() != rows || node.shifts.size() != rows) {
            return invalid("gemm parameters do not match its shape");
        }
        if (!within(node.gemm_weights, -digit2_max, digit2_max) || !within(node.bias, -bias_bound, bias_bound) ||
            !within(node.shifts, 1, 31)) {
            return invalid("gemm weights, bias or shifts exceed the profile's bounds");
        }
        break;
    }
    case FxOp::depthwise3x3: {
        auto weights = data_array<std::int32_t>(entry, "weights", data);
        if (!weights) return weights.error();
        auto bias = data_array<std::int64_t>(entry, "bias", data);
        if (!bias) return bias.error();
        auto shifts = data_array<std::int32_t>(entry, "shift", data);
        if (!shifts) return shifts.error();
        node.depthwise_weights = std::move(weights.value());
        node.bias = std::move(bias.value());
        node.shifts = std::move(shifts.value());
        const auto channels = static_cast<std::size_t>(channels_of(node.inputs[0]));
        if (node.depthwise_weights.size() != channels * 9 || node.bias.size() != channels ||
            node.shifts.size() != channels || !within(node.depthwise_weights, -table_bound, table_bound) ||
            !within(node.bias, -bias_bound, bias_bound) || !within(node.shifts, 0, 31)) {
            return invalid("depthwise parameters exceed the profile's bounds");
        }
        break;
    }
    case FxOp::mul: {
        auto shift = ranged(entry, "shift", 0, 31);
        if (!shift) return shift.error();
        node.shift = shift.value();
        const auto factor = channels_of(node.inputs[1]);
        if (factor != 1 && factor != channels_of(node.inputs[0])) return invalid("mul factor channels");
        break;
    }
    case FxOp::param_row: {
        auto rows = data_array<std::int64_t>(entry, "rows", data);
        if (!rows) return rows.error();
        node.rows = std::move(rows.value());
        const auto channels = static_cast<std::size_t>(channels_of(node.output));
        if (channels_of(node.inputs[0]) != 1 || node.rows.empty() || node.rows.size() % channels != 0 ||
            !within(node.rows, -table_bound, table_bound)) {
            return invalid("param_row table does not match its output or exceeds 2^24");
        }
        break;
    }
    case FxOp::affine: {
        auto alpha = integer(entry, "alpha");
        if (!alpha) return alpha.error();
        auto beta = integer(entry, "beta");
        if (!beta) return beta.error();
        auto shift = ranged(entry, "shift", 0, 31);
        if (!shift) return shift.error();
        node.alpha = alpha.value();
        node.beta = beta.value();
        node.shift = shift.value();
        if (node.alpha < -table_bound || node.alpha > table_bound || node.beta < -bias_bound || node.beta > bias_bound) {
            return invalid("affine parameters exceed the profile's bounds");
        }
        break;
    }
    case FxOp::sat_table: {
        auto table = data_array<std::int32_t>(entry, "table", data);
        if (!table) return table.error();
        auto top = integer(entry, "top");
        if (!top) return top.error();
        node.table = std::move(table.value());
        node.hi = top.value();
        if (node.table.empty() || node.table.size() % 2 != 0 || node.hi < INT32_MIN || node.hi > INT32_MAX) {
            return invalid("sat_table needs an even, non-empty table");
        }
        break;
    }
    case FxOp::delta: {
        auto table = ranged(entry, "delta_table", 0, 1 << 20);
        if (!table) return table.error();
        node.delta_table = table.value();
        if (!table_ok(node.delta_table)) return invalid("delta table out of range");
        break;
    }
    case FxOp::clamp: {
        auto lo = integer(entry, "lo");
        if (!lo) return lo.error();
        auto hi = integer(entry, "hi");
        if (!hi) return hi.error();
        node.lo = lo.value();
        node.hi = hi.value();
        if (node.lo > node.hi || node.lo < INT32_MIN || node.hi > INT32_MAX) return invalid("clamp bounds invalid");
        break;
    }
    case FxOp::slice: {
        auto begin = ranged(entry, "begin", 0, 1 << 20);
        if (!begin) return begin.error();
        auto end = ranged(entry, "end", 1, 1 << 20);
        if (!end) return end.error();
        node.begin = begin.value();
        node.end = end.value();
        if (node.begin >= node.end || node.end > channels_of(node.inputs[0])) return invalid("slice range invalid");
        break;
    }
    case FxOp::pixel_shuffle:
    case FxOp::pixel_unshuffle: {
        auto factor = ranged(entry, "factor", 2, 16);
        if (!factor) return factor.error();
        node.factor = factor.value();
        break;
    }
    case FxOp::im2col: {
        auto kernel = ranged(entry, "kernel", 2, 3);
        if (!kernel) return kernel.error();
        auto stride = ranged(entry, "stride", 1, 2);
        if (!stride) return stride.error();
        node.kernel = kernel.value();
        node.stride = stride.value();
        if (node.kernel == 2 && node.stride != 2) return invalid("im2col 2x2 needs stride 2");
        break;
    }
    case FxOp::add:
    case FxOp::concat:
    case FxOp::crop_like:
        break;
    }
    return node;
}

// Reads a whole file; `missing` is the code for a file that cannot be opened.
Result<std::string> read_bytes(const std::string& path, Code missing) {
    std::ifstream stream(path, std::ios::binary);
    if (!stream) return fail(missing, "cannot open " + path);
    std::string bytes{std::istreambuf_iterator<char>(stream), std::istreambuf_iterator<char>()};
    if (stream.bad()) return fail(Code::io_error, "cannot read " + path);
    return bytes;
}

std::string join(const std::string& directory, std::string_view file) {
    if (directory.empty()) return std::string(file);
    return directory.back() == '/' ? directory + std::string(file) : directory + "/" + std::string(file);
}

}  // namespace

const char* op_name(FxOp op) noexcept {
    for (const auto& [label, value] : op_table) {
        if (value == op) return label.data();
    }
    return "?";
}

Result<std::string> fx_program_digest(const std::string& directory, std::string_view stage) {
    auto document = read_bytes(join(directory, std::string(stage) + ".fxprog.json"), Code::io_error);
    if (!document) return document.error();
    return sha256_hex(document.value().data(), document.value().size());
}

Result<FxProgram> load_fx_program(const std::string& directory, std::string_view stage) {
    const std::string program_path = join(directory, std::string(stage) + ".fxprog.json");
    auto document = read_bytes(program_path, Code::missing_artifact);
    if (!document) return document.error();
    auto parsed = json::parse(document.value());
    if (!parsed) return fail(parsed.error().code, program_path + ": " + parsed.error().message);
    const Value& root = parsed.value();
    const auto* data_info = member(root, "data");
    if (member(root, "format") == nullptr || text(member(root, "format")) != "nvcr.fx-program.v1" ||
        member(root, "profile") == nullptr || text(member(root, "profile")) != "nvcr.fx.v1" || data_info == nullptr) {
        return invalid("not an nvcr.fx-program.v1 program for nvcr.fx.v1");
    }
    const auto* file = member(*data_info, "file");
    const auto* sha = member(*data_info, "sha256");
    if (file == nullptr || sha == nullptr || text(file).find('/') != std::string::npos) {
        return invalid("data file reference invalid");
    }
    const std::string data_path = join(directory, text(file));
    auto data = read_bytes(data_path, Code::io_error);
    if (!data) return data.error();
    if (sha256_hex(data.value().data(), data.value().size()) != text(sha)) {
        return fail(Code::digest_mismatch, "fx program data digest mismatch: " + data_path);
    }

    FxProgram program;
    program.name = std::string(stage);
    program.digest_hex = sha256_hex(document.value().data(), document.value().size());
    auto fa = ranged(root, "fa", 0, 24);
    if (!fa) return fa.error();
    program.fa = fa.value();
    const auto& tensors = items(member(root, "tensors"));
    if (tensors.empty()) return invalid("program without tensors");
    for (const auto& tensor : tensors) {
        const auto* name = member(tensor, "name");
        auto channels = ranged(tensor, "channels", 1, 1 << 20);
        if (name == nullptr || !channels) return invalid("tensor needs a name and channels");
        program.tensor_names.push_back(text(name));
        program.tensor_channels.push_back(channels.value());
    }
    for (const std::string_view key : {"inputs", "outputs"}) {
        const auto& list = items(member(root, key));
        if (list.empty()) return invalid(std::string(key) + " missing");
        for (const auto& entry : list) {
            const auto id = integer_of(&entry);
            if (!id || *id < 0 || static_cast<std::uint64_t>(*id) >= program.tensor_names.size()) {
                return invalid(std::string(key) + " out of range");
            }
            (key == "inputs" ? program.inputs : program.outputs).push_back(static_cast<std::uint32_t>(*id));
        }
    }
    for (const auto& entry : items(member(root, "delta_tables"))) {
        auto h = integer(entry, "h");
        auto shift = ranged(entry, "shift", 0, 30);
        auto dc = data_array<std::int16_t>(entry, "dc", data.value());
        if (!h || !shift || !dc) return invalid("delta table needs h, shift and dc");
        if (h.value() < 0 || h.value() > stored_max ||
            dc.value().size() != static_cast<std::size_t>(((2 * h.value()) >> shift.value()) + 1)) {
            return invalid("delta table size does not match h and shift");
        }
        program.delta_tables.push_back({h.value(), shift.value(), std::move(dc.value())});
    }
    const auto& nodes = items(member(root, "nodes"));
    if (nodes.empty()) return invalid("program without nodes");
    for (const auto& entry : nodes) {
        auto node = parse_node(entry, program, data.value());
        if (!node) return node.error();
        program.nodes.push_back(std::move(node.value()));
    }
    return program;
}

}  // namespace nvcr_sm100::fx
