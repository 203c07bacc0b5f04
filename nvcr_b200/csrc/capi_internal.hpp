#pragma once

// Shared by the translation units that implement include/nvcr_sm100.h.

#include "executor.hpp"

#include <memory>
#include <string>

struct nvcr_sm100_executor {
    std::unique_ptr<nvcr_sm100::Executor> executor;
};

namespace nvcr_sm100 {

// Records `error` for nvcr_sm100_last_error() on this thread; returns 1 + its code.
int report_error(const Error& error);
// Clears the thread's last error; returns NVCR_SM100_OK.
int report_ok();

}  // namespace nvcr_sm100
