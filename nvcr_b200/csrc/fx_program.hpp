#pragma once

// nvcr.fx.v1 stage programs (format nvcr.fx-program.v1): <stage>.fxprog.json
// plus the little-endian data file it pins by SHA-256 (<stage>.fxw). Loading
// applies the profile's load-time refusals (weight, bias, shift and table
// bounds; every tensor and data reference in range), in the order the
// reference's loader checks them (src/deterministic/fx_program.cpp:398-466,
// parse_node at :86-250), so a program is refused with the same error code.
//
// The arrays keep the element types of the data file (gemm weights int16,
// biases int64, shifts int32, depthwise weights int32, tables int16/int32):
// they are the forms a device executor uploads as they are.

#include "status.hpp"

#include <cstdint>
#include <string>
#include <string_view>
#include <vector>

namespace nvcr_sm100::fx {

inline constexpr std::int64_t digit2_max = 32639;                    // two balanced int8 digits
inline constexpr std::int64_t stored_max = std::int64_t{1} << 30;    // |stored value| bound
inline constexpr std::int64_t gemm_limit = (std::int64_t{1} << 29) - 1;

// In the reference's Op order (fx_program.hpp:20-36).
enum class FxOp : std::uint8_t {
    gemm,
    depthwise3x3,
    mul,
    affine,
    add,
    sat_table,
    delta,
    clamp,
    concat,
    slice,
    pixel_shuffle,
    pixel_unshuffle,
    im2col,
    param_row,
    crop_like,
};

const char* op_name(FxOp op) noexcept;

// act(r) = max(r, 0) + dc[(r + h) >> shift] on [-h, h], max(r, 0) outside.
struct DeltaTable {
    std::int64_t h{0};
    int shift{0};
    std::vector<std::int16_t> dc;  // ((2h) >> shift) + 1 entries
};

struct FxNode {
    FxOp op{FxOp::add};
    std::vector<std::uint32_t> inputs;  // tensor ids; gemm: x, then 0..2 residuals
    std::uint32_t output{0};
    // gemm
    std::int32_t in_channels{0};
    std::int32_t out_channels{0};  // before grouping
    int group{1};
    int input_shift{0};
    std::vector<std::int16_t> gemm_weights;  // [out][in], |w| <= digit2_max
    // gemm and depthwise3x3
    std::vector<std::int64_t> bias;
    std::vector<std::int32_t> shifts;
    std::vector<std::int32_t> depthwise_weights;  // [channels][3][3]
    int delta_table{-1};                          // gemm (optional), delta
    std::vector<std::int64_t> rows;               // param_row: [qp][channels]
    std::vector<std::int32_t> table;              // sat_table: 2n entries
    std::int64_t alpha{0};                        // affine
    std::int64_t beta{0};                         // affine
    std::int64_t lo{0};                           // clamp; sat_table's top is kept in hi
    std::int64_t hi{0};
    int shift{0};                                 // mul, affine
    int begin{0};                                 // slice
    int end{0};
    int factor{1};                                // pixel_shuffle, pixel_unshuffle
    int kernel{3};                                // im2col: 3 or 2
    int stride{1};                                // im2col: 1 or 2
};

struct FxProgram {
    std::string name;
    int fa{14};
    std::vector<std::string> tensor_names;
    std::vector<std::int32_t> tensor_channels;
    std::vector<std::uint32_t> inputs;
    std::vector<std::uint32_t> outputs;
    std::vector<DeltaTable> delta_tables;
    std::vector<FxNode> nodes;
    std::string digest_hex;  // SHA-256 of <stage>.fxprog.json: the program's identity
};

// Loads <directory>/<stage>.fxprog.json and its data file with the profile's
// load-time checks. Errors: missing_artifact (no program file), io_error (no
// data file), digest_mismatch (data file SHA-256), invalid_argument (anything
// else the loader refuses).
Result<FxProgram> load_fx_program(const std::string& directory, std::string_view stage);

// Lowercase hex SHA-256 of <directory>/<stage>.fxprog.json.
Result<std::string> fx_program_digest(const std::string& directory, std::string_view stage);

}  // namespace nvcr_sm100::fx
