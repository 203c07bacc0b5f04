#include "numerics_identity.hpp"

#include "sha256.hpp"

#include <set>

namespace nvcr_sm100 {
namespace {

constexpr std::size_t id_limit = 128;
constexpr std::size_t stage_limit = 64;

// 1..128 bytes, each a printable ASCII character other than space.
bool printable_id(const std::string& id) {
    if (id.empty() || id.size() > id_limit) return false;
    for (const char c : id) {
        const auto byte = static_cast<unsigned char>(c);
        if (byte <= 0x20u || byte >= 0x7fu) return false;
    }
    return true;
}

}  // namespace

Result<NumericsIdentity> make_numerics_identity(const std::string& profile, const std::vector<StageDigest>& stages) {
    if (!printable_id(profile)) return fail(Code::invalid_argument, "numerics profile id is invalid");
    if (stages.empty() || stages.size() > stage_limit) {
        return fail(Code::invalid_argument, "numerics identity must cover 1 to 64 normative stages");
    }
    std::set<std::string> ids;
    Sha256 hash;
    for (const auto& stage : stages) {
        if (!printable_id(stage.stage_id)) return fail(Code::invalid_argument, "normative stage id is invalid");
        if (!ids.insert(stage.stage_id).second) return fail(Code::invalid_argument, "normative stage listed twice");
        const auto length = static_cast<std::uint8_t>(stage.stage_id.size());
        hash.update(&length, 1);
        hash.update(stage.stage_id.data(), stage.stage_id.size());
        hash.update(stage.program_digest.data(), stage.program_digest.size());
    }
    NumericsIdentity identity;
    identity.profile = profile;
    identity.program_set_digest = hash.finish();
    return identity;
}

Result<std::vector<std::uint8_t>> serialize_numerics_identity(const NumericsIdentity& identity) {
    if (!printable_id(identity.profile)) return fail(Code::invalid_argument, "numerics profile id is invalid");
    std::vector<std::uint8_t> bytes;
    bytes.reserve(1 + identity.profile.size() + identity.program_set_digest.size());
    bytes.push_back(static_cast<std::uint8_t>(identity.profile.size()));
    bytes.insert(bytes.end(), identity.profile.begin(), identity.profile.end());
    bytes.insert(bytes.end(), identity.program_set_digest.begin(), identity.program_set_digest.end());
    return bytes;
}

Result<NumericsIdentity> parse_numerics_identity(const std::uint8_t* bytes, std::size_t size) {
    constexpr std::size_t digest_size = 32;
    if (size == 0 || bytes == nullptr) return fail(Code::malformed_bitstream, "numerics identity is truncated");
    const std::size_t length = bytes[0];
    if (size < 1 + length + digest_size) return fail(Code::malformed_bitstream, "numerics identity is truncated");
    if (size > 1 + length + digest_size) {
        return fail(Code::malformed_bitstream, "numerics identity has trailing bytes");
    }
    NumericsIdentity identity;
    identity.profile.assign(reinterpret_cast<const char*>(bytes + 1), length);
    if (!printable_id(identity.profile)) {
        return fail(Code::malformed_bitstream, "numerics identity contains an invalid profile id");
    }
    for (std::size_t i = 0; i < digest_size; ++i) identity.program_set_digest[i] = bytes[1 + length + i];
    return identity;
}

}  // namespace nvcr_sm100
