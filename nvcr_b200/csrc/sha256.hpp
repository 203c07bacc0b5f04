#pragma once

// SHA-256 (FIPS 180-4). Program files pin their weights by the digest of the
// .detw bytes, and normative stage descriptors pin the program JSON the same
// way, so the loader needs it on the host.

#include <array>
#include <cstddef>
#include <cstdint>
#include <string>
#include <string_view>

namespace nvcr_sm100 {

class Sha256 {
public:
    Sha256();
    void update(const void* data, std::size_t size);
    std::array<std::uint8_t, 32> finish();

private:
    void block(const std::uint8_t* chunk);
    std::array<std::uint32_t, 8> state_{};
    std::array<std::uint8_t, 64> pending_{};
    std::size_t pending_size_{0};
    std::uint64_t total_{0};
};

std::string to_hex(const std::uint8_t* bytes, std::size_t size);
std::string sha256_hex(const void* data, std::size_t size);

}  // namespace nvcr_sm100
