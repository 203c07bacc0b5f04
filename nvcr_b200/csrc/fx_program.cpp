#include "fx_program.hpp"

#include "json.hpp"
#include "sha256.hpp"

#include <climits>
#include <cstring>
#include <fstream>
#include <iterator>
#include <optional>
#include <utility>

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

// Reads one node object. Every accessor records the first refusal it meets
// and returns a neutral value after it, so a node is read straight through and
// the recorded refusal (if any) is reported at the end; each op's reading is
// one short function over the accessors, followed by its shape rule.
class NodeReader {
public:
    NodeReader(const Value& entry, const FxProgram& program, const std::string& data)
        : entry_(entry), program_(program), data_(data) {}

    std::int64_t any_integer(std::string_view key) {
        const auto value = integer_of(member(entry_, key));
        if (!value) refuse("field '" + std::string(key) + "' must be an integer");
        return value.value_or(0);
    }
    int bounded(std::string_view key, std::int64_t lo, std::int64_t hi) {
        const std::int64_t value = any_integer(key);
        if (ok() && (value < lo || value > hi)) refuse("field '" + std::string(key) + "' out of range");
        return ok() ? static_cast<int>(value) : 0;
    }
    // A [byte offset, element count] reference into the data file.
    template <typename T>
    std::vector<T> array(std::string_view key) {
        const auto& pair = items(member(entry_, key));
        const auto offset = pair.size() == 2 ? integer_of(&pair[0]) : std::nullopt;
        const auto count = pair.size() == 2 ? integer_of(&pair[1]) : std::nullopt;
        if (!offset || !count) {
            refuse("field '" + std::string(key) + "' must be [offset, count]");
            return {};
        }
        const std::uint64_t size = data_.size();
        const bool inside = *offset >= 0 && *count >= 0 && static_cast<std::uint64_t>(*offset) <= size &&
            static_cast<std::uint64_t>(*count) <= (size - static_cast<std::uint64_t>(*offset)) / sizeof(T);
        if (!inside) {
            refuse("field '" + std::string(key) + "' lies outside the data file");
            return {};
        }
        std::vector<T> values(static_cast<std::size_t>(*count));
        if (!values.empty() && ok()) std::memcpy(values.data(), data_.data() + *offset, values.size() * sizeof(T));
        return values;
    }
    std::int32_t channels(std::uint32_t id) const { return program_.tensor_channels[id]; }
    bool table_exists(int index) const { return index >= -1 && index < static_cast<int>(program_.delta_tables.size()); }
    void require(bool condition, const char* message) {
        if (!condition) refuse(message);
    }
    void refuse(const std::string& message) {
        if (!error_) error_ = invalid(message);
    }
    bool ok() const { return !error_.has_value(); }
    const std::optional<Error>& error() const { return error_; }
    const Value& entry() const { return entry_; }
    std::size_t tensor_count() const { return program_.tensor_names.size(); }

private:
    const Value& entry_;
    const FxProgram& program_;
    const std::string& data_;
    std::optional<Error> error_;
};

template <typename T>
bool within(const std::vector<T>& values, std::int64_t lo, std::int64_t hi) {
    for (const auto v : values) {
        if (static_cast<std::int64_t>(v) < lo || static_cast<std::int64_t>(v) > hi) return false;
    }
    return true;
}

constexpr std::int64_t bias_bound = std::int64_t{1} << 52;
constexpr std::int64_t table_bound = std::int64_t{1} << 24;

// Op-specific reading: fields and arrays in a fixed order, then the rule the
// profile sets on them.
void read_gemm(NodeReader& r, FxNode& n) {
    n.in_channels = r.bounded("in_channels", 1, 1 << 20);
    n.out_channels = r.bounded("out_channels", 1, 1 << 20);
    n.group = r.bounded("group", 1, 4);
    n.input_shift = r.bounded("input_shift", 0, 30);
    n.delta_table = r.bounded("delta_table", -1, 1 << 20);
    n.gemm_weights = r.array<std::int16_t>("weights");
    n.bias = r.array<std::int64_t>("bias");
    n.shifts = r.array<std::int32_t>("shift");
    if (!r.ok()) return;
    const auto rows = static_cast<std::size_t>(n.out_channels);
    r.require(n.group != 3 && n.out_channels % n.group == 0 && r.table_exists(n.delta_table) &&
                  n.gemm_weights.size() == rows * static_cast<std::size_t>(n.in_channels) && n.bias.size() == rows &&
                  n.shifts.size() == rows,
              "gemm parameters do not match its shape");
    r.require(within(n.gemm_weights, -digit2_max, digit2_max) && within(n.bias, -bias_bound, bias_bound) &&
                  within(n.shifts, 1, 31),
              "gemm weights, bias or shifts exceed the profile's bounds");
}

void read_depthwise(NodeReader& r, FxNode& n) {
    n.depthwise_weights = r.array<std::int32_t>("weights");
    n.bias = r.array<std::int64_t>("bias");
    n.shifts = r.array<std::int32_t>("shift");
    if (!r.ok()) return;
    const auto c = static_cast<std::size_t>(r.channels(n.inputs[0]));
    r.require(n.depthwise_weights.size() == 9 * c && n.bias.size() == c && n.shifts.size() == c &&
                  within(n.depthwise_weights, -table_bound, table_bound) && within(n.bias, -bias_bound, bias_bound) &&
                  within(n.shifts, 0, 31),
              "depthwise parameters exceed the profile's bounds");
}

void read_mul(NodeReader& r, FxNode& n) {
    n.shift = r.bounded("shift", 0, 31);
    if (!r.ok()) return;
    const std::int32_t factor = r.channels(n.inputs[1]);
    r.require(factor == 1 || factor == r.channels(n.inputs[0]), "mul factor channels");
}

void read_param_row(NodeReader& r, FxNode& n) {
    n.rows = r.array<std::int64_t>("rows");
    if (!r.ok()) return;
    const auto c = static_cast<std::size_t>(r.channels(n.output));
    r.require(r.channels(n.inputs[0]) == 1 && !n.rows.empty() && n.rows.size() % c == 0 &&
                  within(n.rows, -table_bound, table_bound),
              "param_row table does not match its output or exceeds 2^24");
}

void read_affine(NodeReader& r, FxNode& n) {
    n.alpha = r.any_integer("alpha");
    n.beta = r.any_integer("beta");
    n.shift = r.bounded("shift", 0, 31);
    if (!r.ok()) return;
    r.require(n.alpha >= -table_bound && n.alpha <= table_bound && n.beta >= -bias_bound && n.beta <= bias_bound,
              "affine parameters exceed the profile's bounds");
}

void read_sat_table(NodeReader& r, FxNode& n) {
    n.table = r.array<std::int32_t>("table");
    n.hi = r.any_integer("top");
    if (!r.ok()) return;
    r.require(!n.table.empty() && n.table.size() % 2 == 0 && n.hi >= INT32_MIN && n.hi <= INT32_MAX,
              "sat_table needs an even, non-empty table");
}

void read_delta(NodeReader& r, FxNode& n) {
    n.delta_table = r.bounded("delta_table", 0, 1 << 20);
    if (r.ok()) r.require(r.table_exists(n.delta_table), "delta table out of range");
}

void read_clamp(NodeReader& r, FxNode& n) {
    n.lo = r.any_integer("lo");
    n.hi = r.any_integer("hi");
    if (r.ok()) r.require(n.lo <= n.hi && n.lo >= INT32_MIN && n.hi <= INT32_MAX, "clamp bounds invalid");
}

void read_slice(NodeReader& r, FxNode& n) {
    n.begin = r.bounded("begin", 0, 1 << 20);
    n.end = r.bounded("end", 1, 1 << 20);
    if (r.ok()) r.require(n.begin < n.end && n.end <= r.channels(n.inputs[0]), "slice range invalid");
}

void read_shuffle(NodeReader& r, FxNode& n) { n.factor = r.bounded("factor", 2, 16); }

void read_im2col(NodeReader& r, FxNode& n) {
    n.kernel = r.bounded("kernel", 2, 3);
    n.stride = r.bounded("stride", 1, 2);
    if (r.ok()) r.require(n.kernel != 2 || n.stride == 2, "im2col 2x2 needs stride 2");
}

void read_nothing(NodeReader&, FxNode&) {}

struct OpEntry {
    std::string_view name;
    FxOp op;
    std::size_t inputs;     // tensors the op reads
    std::size_t optional;   // further inputs it may read (gemm: up to two residuals)
    void (*read)(NodeReader&, FxNode&);
};

constexpr OpEntry op_entries[] = {
    {"gemm", FxOp::gemm, 1, 2, read_gemm},
    {"depthwise3x3", FxOp::depthwise3x3, 1, 0, read_depthwise},
    {"mul", FxOp::mul, 2, 0, read_mul},
    {"affine", FxOp::affine, 1, 0, read_affine},
    {"add", FxOp::add, 2, 0, read_nothing},
    {"sat_table", FxOp::sat_table, 1, 0, read_sat_table},
    {"delta", FxOp::delta, 1, 0, read_delta},
    {"clamp", FxOp::clamp, 1, 0, read_clamp},
    {"concat", FxOp::concat, 2, 0, read_nothing},
    {"slice", FxOp::slice, 1, 0, read_slice},
    {"pixel_shuffle", FxOp::pixel_shuffle, 1, 0, read_shuffle},
    {"pixel_unshuffle", FxOp::pixel_unshuffle, 1, 0, read_shuffle},
    {"im2col", FxOp::im2col, 1, 0, read_im2col},
    {"param_row", FxOp::param_row, 1, 0, read_param_row},
    {"crop_like", FxOp::crop_like, 2, 0, read_nothing},
};

Result<FxNode> read_node(const Value& entry, const FxProgram& program, const std::string& data) {
    const Value* op_value = member(entry, "op");
    const OpEntry* kind = nullptr;
    for (const auto& candidate : op_entries) {
        if (op_value != nullptr && candidate.name == text(op_value)) kind = &candidate;
    }
    if (kind == nullptr) return invalid("unknown op");
    NodeReader reader(entry, program, data);
    FxNode node;
    node.op = kind->op;
    const Value* inputs = member(entry, "inputs");
    if (inputs == nullptr) return invalid("node without inputs");
    for (const Value& input : items(inputs)) {
        const auto id = integer_of(&input);
        if (!id || *id < 0 || static_cast<std::uint64_t>(*id) >= program.tensor_names.size()) {
            return invalid("node input out of range");
        }
        node.inputs.push_back(static_cast<std::uint32_t>(*id));
    }
    if (node.inputs.size() < kind->inputs || node.inputs.size() > kind->inputs + kind->optional) {
        return invalid("wrong number of node inputs");
    }
    node.output = static_cast<std::uint32_t>(
        reader.bounded("output", 0, static_cast<std::int64_t>(program.tensor_names.size()) - 1));
    if (reader.ok()) kind->read(reader, node);
    if (reader.error()) return *reader.error();
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
    for (const auto& entry : op_entries) {
        if (entry.op == op) return entry.name.data();
    }
    return "?";
}

Result<std::string> fx_program_digest(const std::string& directory, std::string_view stage) {
    auto document = read_bytes(join(directory, std::string(stage) + ".fxprog.json"), Code::io_error);
    if (!document) return document.error();
    return sha256_hex(document.value().data(), document.value().size());
}

Result<FxProgram> load_fx_program(const std::string& directory, std::string_view stage) {
    // The two files: the program (missing_artifact when absent), then the data
    // file it names (io_error when unreadable), pinned by its SHA-256.
    const std::string program_path = join(directory, std::string(stage) + ".fxprog.json");
    auto document = read_bytes(program_path, Code::missing_artifact);
    if (!document) return document.error();
    auto parsed = json::parse(document.value());
    if (!parsed) return fail(parsed.error().code, program_path + ": " + parsed.error().message);
    const Value& root = parsed.value();
    const Value* format = member(root, "format");
    const Value* profile = member(root, "profile");
    const Value* data_info = member(root, "data");
    const bool identified = format != nullptr && text(format) == "nvcr.fx-program.v1" && profile != nullptr &&
        text(profile) == "nvcr.fx.v1" && data_info != nullptr;
    if (!identified) return invalid("not an nvcr.fx-program.v1 program for nvcr.fx.v1");
    const Value* file = member(*data_info, "file");
    const Value* pinned = member(*data_info, "sha256");
    if (file == nullptr || pinned == nullptr || text(file).find('/') != std::string::npos) {
        return invalid("data file reference invalid");
    }
    const std::string data_path = join(directory, text(file));
    auto data = read_bytes(data_path, Code::io_error);
    if (!data) return data.error();
    const std::string& bytes = data.value();
    if (sha256_hex(bytes.data(), bytes.size()) != text(pinned)) {
        return fail(Code::digest_mismatch, "fx program data digest mismatch: " + data_path);
    }

    FxProgram program;
    program.name = std::string(stage);
    program.digest_hex = sha256_hex(document.value().data(), document.value().size());
    NodeReader top(root, program, bytes);
    program.fa = top.bounded("fa", 0, 24);
    if (top.error()) return *top.error();

    // Tensors (name and channel count), then the input and output id lists.
    const auto& tensors = items(member(root, "tensors"));
    if (tensors.empty()) return invalid("program without tensors");
    for (const Value& tensor : tensors) {
        NodeReader entry(tensor, program, bytes);
        const int channels = entry.bounded("channels", 1, 1 << 20);
        if (member(tensor, "name") == nullptr || entry.error()) return invalid("tensor needs a name and channels");
        program.tensor_names.push_back(text(member(tensor, "name")));
        program.tensor_channels.push_back(channels);
    }
    for (auto [key, ids] : {std::pair<std::string_view, std::vector<std::uint32_t>*>{"inputs", &program.inputs},
                            std::pair<std::string_view, std::vector<std::uint32_t>*>{"outputs", &program.outputs}}) {
        const auto& list = items(member(root, key));
        if (list.empty()) return invalid(std::string(key) + " missing");
        for (const Value& id : list) {
            const auto value = integer_of(&id);
            if (!value || *value < 0 || static_cast<std::uint64_t>(*value) >= program.tensor_names.size()) {
                return invalid(std::string(key) + " out of range");
            }
            ids->push_back(static_cast<std::uint32_t>(*value));
        }
    }

    // Delta tables: h, shift and ((2h) >> shift) + 1 offsets each.
    for (const Value& table : items(member(root, "delta_tables"))) {
        NodeReader entry(table, program, bytes);
        DeltaTable delta;
        delta.h = entry.any_integer("h");
        delta.shift = entry.bounded("shift", 0, 30);
        delta.dc = entry.array<std::int16_t>("dc");
        if (entry.error()) return invalid("delta table needs h, shift and dc");
        const bool sized = delta.h >= 0 && delta.h <= stored_max &&
            delta.dc.size() == static_cast<std::size_t>(((2 * delta.h) >> delta.shift) + 1);
        if (!sized) return invalid("delta table size does not match h and shift");
        program.delta_tables.push_back(std::move(delta));
    }

    const auto& nodes = items(member(root, "nodes"));
    if (nodes.empty()) return invalid("program without nodes");
    for (const Value& entry : nodes) {
        auto node = read_node(entry, program, bytes);
        if (!node) return node.error();
        program.nodes.push_back(std::move(node.value()));
    }
    return program;
}

}  // namespace nvcr_sm100::fx
