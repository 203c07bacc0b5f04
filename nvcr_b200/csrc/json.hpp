#pragma once

// A small JSON reader for program metadata (RFC 8259). Numbers keep a double
// and, when the token is a plain integer that fits, an exact int64: program
// fields such as channel counts must be integers, scalars must be exact
// float32 values, and the loader tells the two apart the way the reference's
// program loader does.

#include "status.hpp"

#include <cstdint>
#include <map>
#include <optional>
#include <string>
#include <string_view>
#include <vector>

namespace nvcr_sm100::json {

struct Value {
    enum class Kind { null, boolean, number, string, array, object };
    Kind kind{Kind::null};
    bool boolean{false};
    double number{0.0};
    std::optional<std::int64_t> integer;
    std::string text;
    std::vector<Value> items;
    std::map<std::string, Value, std::less<>> members;

    [[nodiscard]] const Value* get(std::string_view key) const;
};

Result<Value> parse(std::string_view document);

}  // namespace nvcr_sm100::json
