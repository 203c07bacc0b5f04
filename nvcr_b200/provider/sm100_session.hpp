#pragma once

// The sm_100a execution provider on the reference's provider-session boundary
// (include/nvcr/provider/experimental/session.hpp:132-166). It claims exactly
// one numerics profile, nvcr.intconv.v1, and reaches the GPU only through the
// C ABI of libnvcr_sm100 (include/nvcr_sm100.h): the stage program is loaded
// and digest-checked by nvcr_sm100_load_normative, and a submission runs
// nvcr_sm100_run_half on the session's stream.
//
// This is reference-side code: it compiles against the reference's headers
// (nvcr/provider/experimental/session.hpp, nvcr/runtime/registry.hpp,
// nvcr/common/error.hpp) and is what a maintainer adds as src/provider/sm100.
//
// Behaviour, as the reference's exact-stage providers:
//  * supports_numerics_profile: true for nvcr.intconv.v1 on an sm_100 device;
//  * load_stage: a native stage (empty profile) or any other profile is refused
//    with incompatible_precision (an exact stage never runs natively); the
//    program is loaded from artifact.path / artifact.component_id and must
//    hash to artifact.expected_digest (digest_mismatch otherwise,
//    missing_artifact when absent);
//  * submit: FP16 batch-1 NCHW tensors in buffers of this session, read for
//    stage inputs and write (or read_write) for outputs, named as the
//    program's; device buffers run asynchronously on the session's stream,
//    host and pinned-host buffers are copied through device memory; the
//    completion is an event on the stream.

#include "nvcr/provider/experimental/session.hpp"

#include <memory>

namespace nvcr::provider::sm100 {

// A new session on the current CUDA device with its own stream.
Result<std::shared_ptr<experimental::IProviderSession>> create_session();

// Adds the provider to the reference's registry (Registry::register_provider)
// with create_session as its session factory.
void register_provider();

// The device address of a provider_device buffer made by one of these
// sessions (for codec-side kernels that fill or read it on the device), or
// null for any other buffer.
void* device_address(const experimental::IProviderBuffer& buffer) noexcept;

}  // namespace nvcr::provider::sm100
