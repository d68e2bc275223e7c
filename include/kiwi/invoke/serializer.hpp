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

template <typename T, uint32_t N>
KIWI_HD void put_word(uint64_t (&w)[N], uint32_t& off, const T& v) {
    uint64_t u = 0;
    if constexpr (sizeof(T) == 1) {
        uint8_t t;
        memcpy(&t, &v, 1);
        u = t;
    } else if constexpr (sizeof(T) == 2) {
        uint16_t t;
        memcpy(&t, &v, 2);
        u = t;
    } else if constexpr (sizeof(T) == 4) {
        uint32_t t;
        memcpy(&t, &v, 4);
        u = t;
    } else if constexpr (sizeof(T) == 8) {
        memcpy(&u, &v, 8);
    }
    if constexpr (sizeof(T) == 1 || sizeof(T) == 2 || sizeof(T) == 4 || sizeof(T) == 8) {
        const uint32_t word = off / 8, shift = 8 * (off % 8);
        if (shift == 0) {
            w[word] |= u;
            off += sizeof(T);
            return;
        }
        w[word] |= u << shift;
        if (shift + 8 * sizeof(T) > 64) w[word + 1] |= u >> (64 - shift);
    } else if constexpr (sizeof(T) % 8 == 0 && alignof(T) >= 8) {
        // 8-byte-aligned structs (descriptors): word by word.
        if (off % 8 == 0) {
            for (uint32_t i = 0; i < sizeof(T) / 8; ++i) {
                uint64_t t;
                memcpy(&t, reinterpret_cast<const char*>(&v) + 8 * i, 8);
                w[off / 8 + i] = t;
            }
        } else {
            for (uint32_t i = 0; i < sizeof(T) / 8; ++i) {
                uint64_t t;
                memcpy(&t, reinterpret_cast<const char*>(&v) + 8 * i, 8);
                const uint32_t o = off + 8 * i, shift = 8 * (o % 8);
                w[o / 8] |= t << shift;
                w[o / 8 + 1] |= t >> (64 - shift);
            }
        }
    } else {
        // Other sizes: byte by byte (constant offsets; still register resident when unrolled).
        const uint8_t* b = reinterpret_cast<const uint8_t*>(&v);
        for (uint32_t i = 0; i < sizeof(T); ++i) {
            const uint32_t o = off + i;
            w[o / 8] |= static_cast<uint64_t>(b[i]) << (8 * (o % 8));
        }
    }
    off += sizeof(T);
}

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

    static constexpr uint32_t kWords = (total_bytes + 7) / 8 > 0 ? (total_bytes + 7) / 8 : 1;

    /// Register-friendly serialisation into 64-bit words: every argument of
    /// 1, 2, 4 or 8 bytes is placed with shifts at its constant offset, so no
    /// byte array (and no local memory) is needed on the device.  The byte
    /// image equals serialize()'s (little-endian, packed).
    KIWI_HD static void pack_words(uint64_t (&w)[kWords], const Args&... args) {
        for (uint32_t i = 0; i < kWords; ++i) w[i] = 0;
        uint32_t off = 0;
        (put_word(w, off, args), ...);
        (void)off;
    }

    static std::tuple<Args...> deserialize(const uint8_t* src) {
        std::tuple<Args...> out;
        uint32_t off = 0;
        std::apply([&](auto&... a) { ((std::memcpy(&a, src + off, sizeof(a)), off += sizeof(a)), ...); },
                   out);
        return out;
    }
};

/// Fixed-size word image of a packed argument list (what a device invoke sends).
template <uint32_t N>
struct alignas(8) PackedWords {
    uint64_t w[N];
};

}  // namespace kiwi::invoke
