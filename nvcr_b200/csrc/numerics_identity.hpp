#pragma once

// The numerics-identity payload a stream carries to name the numerics profile
// and the exact programs of its normative stages (reference
// include/nvcr/bitstream/numerics_identity.hpp, src/bitstream/numerics_identity.cpp).
// Version 1 payload: u8 profile length, the profile id bytes, then the 32-byte
// program-set digest: SHA-256 over, per normative stage in the codec's order,
// u8 stage-id length, the stage id bytes and the stage program's 32-byte
// SHA-256. Ids are 1..128 bytes of 0x21..0x7e; 1..64 stages, ids unique.

#include "status.hpp"

#include <array>
#include <cstdint>
#include <string>
#include <vector>

namespace nvcr_sm100 {

struct StageDigest {
    std::string stage_id;
    std::array<std::uint8_t, 32> program_digest{};
};

struct NumericsIdentity {
    std::string profile;
    std::array<std::uint8_t, 32> program_set_digest{};
};

// invalid_argument for a bad profile or stage id, a duplicate stage, or a stage
// count outside 1..64.
Result<NumericsIdentity> make_numerics_identity(const std::string& profile, const std::vector<StageDigest>& stages);
Result<std::vector<std::uint8_t>> serialize_numerics_identity(const NumericsIdentity& identity);
// malformed_bitstream for a truncated payload, trailing bytes or a bad profile id.
Result<NumericsIdentity> parse_numerics_identity(const std::uint8_t* bytes, std::size_t size);

}  // namespace nvcr_sm100
