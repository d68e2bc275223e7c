// Packed argument serialisation for invoke messages.
//
// Parity with the reference's ArgumentSerializer
// (include/kiwi/invoke/internal/serializer.hip.hpp:40-89 of AMDResearch/kiwi):
// arguments are laid out back to back, little-endian, with no padding, so the
// message is exactly sum(sizeof(Args)) bytes.  Only trivially copyable
// arguments are allowed.
#pragma once

#include <cstring>
#include <tuple>
#include <type_traits>

#include "kiwi/common.hpp"

namespace kiwi::invoke {

template <typename... Args>
struct ArgPack {
    static_assert((std::is_trivially_copyable_v<Args> && ...),
                  "invoke arguments must be trivially copyable");
    static constexpr uint32_t total_bytes = (0u + ... + static_cast<uint32_t>(sizeof(Args)));

    KIWI_HD static void serialize(uint8_t* dst, const Args&... args) {
        uint32_t off = 0;
        ((memcpy(dst + off, &args, sizeof(Args)), off += sizeof(Args)), ...);
        (void)off;
        (void)dst;
    }

    static std::tuple<Args...> deserialize(const uint8_t* src) {
        std::tuple<Args...> out;
        uint32_t off = 0;
        std::apply([&](auto&... a) { ((std::memcpy(&a, src + off, sizeof(a)), off += sizeof(a)), ...); },
                   out);
        return out;
    }
};

}  // namespace kiwi::invoke
