#pragma once

// Error vocabulary of the sm_100a executor. The numeric values are the
// reference's ErrorCode order (include/nvcr/common/error.hpp:11-34), so a
// status crossing the C ABI maps 1:1 onto the reference's Result errors.

#include <string>
#include <utility>
#include <variant>

namespace nvcr_sm100 {

enum class Code : int {
    ok = -1,  // not a reference code: success across the C ABI is 0 (see capi.cpp)
    invalid_argument = 0,
    invalid_state,
    io_error,
    malformed_bitstream,
    resource_exhausted,
    dependency_unavailable,
    backend_error,
    not_implemented,
    internal_error,
    try_again,
    end_of_stream,
    missing_artifact,
    missing_codec,
    missing_provider,
    missing_model_set,
    incompatible_target,
    incompatible_precision,
    incompatible_version,
    digest_mismatch,
    license_restricted,
};

struct Error {
    Code code{Code::internal_error};
    std::string message;
};

// Minimal result type: a value or an Error.
template <typename T>
class Result {
public:
    Result(T value) : storage_(std::move(value)) {}
    Result(Error error) : storage_(std::move(error)) {}
    [[nodiscard]] bool ok() const noexcept { return std::holds_alternative<T>(storage_); }
    explicit operator bool() const noexcept { return ok(); }
    T& value() & { return std::get<T>(storage_); }
    const T& value() const& { return std::get<T>(storage_); }
    T&& value() && { return std::get<T>(std::move(storage_)); }
    const Error& error() const& { return std::get<Error>(storage_); }

private:
    std::variant<T, Error> storage_;
};

struct Ok {};
using Status = Result<Ok>;

inline Error fail(Code code, std::string message) { return Error{code, std::move(message)}; }

}  // namespace nvcr_sm100
