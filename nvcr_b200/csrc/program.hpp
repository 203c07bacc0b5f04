#pragma once

// nvcr.intconv.v1 programs on the host: the same model as the reference
// (src/deterministic/program.hpp:57-136) so that a program means the same thing
// to both executors, plus its loader, shape inference and weight quantiser.

#include "status.hpp"

#include <array>
#include <cstddef>
#include <cstdint>
#include <string>
#include <string_view>
#include <vector>

namespace nvcr_sm100 {

inline constexpr std::string_view intconv_profile = "nvcr.intconv.v1";

// Op kinds in the reference's order (program.hpp:57-71).
enum class Op : std::uint8_t {
    conv,
    mul,
    add,
    mul_scalar,
    sigmoid,
    slice_channels,
    depth_to_space,
    scale_channels,
    clamp,
    concat,
    crop,
    space_to_depth,
    im2col,
};

struct Node {
    Op op{Op::conv};
    std::array<std::size_t, 2> inputs{};
    std::size_t input_count{1};
    std::size_t output{0};
    std::int32_t in_channels{0};
    std::int32_t out_channels{0};
    bool depthwise{false};
    std::array<std::int32_t, 2> kernel{1, 1};
    std::array<std::int32_t, 2> stride{1, 1};
    std::array<std::int32_t, 4> pads{0, 0, 0, 0};  // top, left, bottom, right
    std::size_t weight_offset{0};
    std::size_t bias_offset{0};
    float scalar{0.0f};
    std::int32_t begin{0};
    std::int32_t end{0};
    std::int32_t block{1};
    std::int32_t axis{2};  // crop: 2 = height, 3 = width
    float minimum{0.0f};
    float maximum{0.0f};
    std::int32_t weight_bits{16};
    std::int32_t activation_bits{16};
};

struct Program {
    std::string name;
    std::string numerics;
    std::string weights_sha256;
    std::vector<std::string> tensor_names;
    std::vector<std::int32_t> tensor_channels;
    std::vector<std::size_t> inputs;
    std::vector<std::size_t> outputs;
    std::vector<Node> nodes;
    std::vector<float> weights;        // FP16 on disk, widened exactly
    std::vector<std::size_t> last_use;  // last reading node; outputs: nodes.size()
};

struct Extent {
    std::int32_t channels{0};
    std::int32_t height{0};
    std::int32_t width{0};
    [[nodiscard]] std::size_t count() const {
        return static_cast<std::size_t>(channels) * static_cast<std::size_t>(height) *
            static_cast<std::size_t>(width);
    }
    bool operator==(const Extent&) const = default;
};

// A dense 1x1 stride-1 unpadded conv runs in exact integer arithmetic.
bool is_integer_pointwise(const Node& node);

// Loads <path> (.detprog.json) and the .detw beside it, checking format,
// version, profile, weight digest and every node (program.cpp:537-626).
Result<Program> load_program_file(const std::string& path);

// Loads a program from JSON text. When `weights` is not null the FP32 values
// are used as the program's weights (the in-memory program form) instead of
// reading the .detw file named in the JSON, which is then not required.
Result<Program> load_program_text(std::string_view json, const std::string& directory,
                                  const float* weights, std::size_t weight_count);

// Output extent of one node for its input extents (program.cpp:628-700).
Result<Extent> output_extent(const Program& program, const Node& node, const Extent* inputs,
                             std::size_t input_count);

// Output extents of the whole program (normative_stage.cpp:42-65).
Result<std::vector<Extent>> infer_output_extents(const Program& program, const std::vector<Extent>& inputs);

// Per-output-channel weight quantisation (program.cpp:509-535).
struct IntegerWeights {
    std::vector<std::int16_t> values;  // [out][in]
    std::vector<float> scales;
};
IntegerWeights quantize_weights(const Program& program, const Node& node);

// Exact IEEE binary16 <-> binary32 on the host.
float half_to_float(std::uint16_t half);
std::uint16_t float_to_half(float value);

}  // namespace nvcr_sm100
