// kiwi::invoke::PrintFormat: a native callback body that prints a kernel's
// invoke arguments with a printf-style format, so a kernel can log through the
// invoke queue without device printf's buffer limits or a Python callback.
//
// Parity: the reference's print example extension, whose one C++ callback
// prints the (int32_t, float, uint64_t) a Triton or FlyDSL kernel invokes it
// with (AMDResearch/kiwi examples/common/kiwi_print_ext.hip.cpp:22-47,
// examples/triton/triton_print_example.py).  Here the callback is generic: the
// argument layout is a Python-struct-style code string (the device serialises
// arguments little-endian and packed), and the format is checked against it
// once, at registration.
//
//   PrintFormat pf("step=%d value=%.2f tag=0x%llx", "ifQ");
//   ctx.register_raw_callback([pf](const uint8_t* p, uint32_t n) { pf.print(p, n, stdout); },
//                             pf.payload_bytes());
//
// Conversions: d i u x X o c take integer codes (b B h H i I l L q Q, l/L are 4
// bytes as in Python's standard sizes); e E f F g G a A take f or d.  Flags,
// width and precision are kept; length modifiers written by the user are
// replaced by the argument's own; `*` widths, %s, %p and %n are rejected.
// %d / %i of an unsigned 64-bit value past INT64_MAX prints the value through
// %u, where the + and space flags have no effect.
#pragma once

#include <climits>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "kiwi/common.hpp"

namespace kiwi::invoke {

class PrintFormat {
public:
    PrintFormat(const std::string& fmt, const std::string& codes) {
        size_t ci = 0;
        std::string c = codes;
        if (!c.empty() && (c[0] == '<' || c[0] == '=')) c.erase(0, 1);
        std::string literal;
        uint32_t off = 0;
        for (size_t i = 0; i < fmt.size(); ++i) {
            if (fmt[i] != '%') {
                literal += fmt[i];
                continue;
            }
            if (i + 1 < fmt.size() && fmt[i + 1] == '%') {
                literal += "%%";
                ++i;
                continue;
            }
            // flags, width, precision, length, conversion
            size_t j = i + 1;
            std::string spec = "%";
            while (j < fmt.size() && std::strchr("-+ #0", fmt[j])) spec += fmt[j++];
            while (j < fmt.size() && fmt[j] >= '0' && fmt[j] <= '9') spec += fmt[j++];
            if (j < fmt.size() && fmt[j] == '.') {
                spec += fmt[j++];
                while (j < fmt.size() && fmt[j] >= '0' && fmt[j] <= '9') spec += fmt[j++];
            }
            while (j < fmt.size() && std::strchr("hlLqjzt", fmt[j])) ++j;  // the argument decides the length
            if (j >= fmt.size()) throw kiwi::error("print format: incomplete conversion at the end of \"" + fmt + "\"");
            const char conv = fmt[j];
            if (ci >= c.size()) throw kiwi::error("print format: more conversions than argument codes");
            const char code = c[ci++];
            const uint32_t size = code_size(code);
            const bool is_float = code == 'f' || code == 'd';
            if (std::strchr("diuxXoc", conv)) {
                if (is_float) throw kiwi::error(std::string("print format: %") + conv + " needs an integer code, got " + code);
                spec += conv == 'c' ? "" : "ll";
            } else if (std::strchr("eEfFgGaA", conv)) {
                if (!is_float) throw kiwi::error(std::string("print format: %") + conv + " needs f or d, got " + code);
            } else {
                throw kiwi::error(std::string("print format: conversion %") + conv + " is not supported");
            }
            // An unsigned 64-bit value past INT64_MAX prints through the %u form
            // of the same spec (its value, not a negative reinterpretation).
            const std::string spec_u = (conv == 'd' || conv == 'i') ? literal + spec + 'u' : std::string();
            spec += conv;
            pieces_.push_back({literal + spec, spec_u, code, conv, off});
            literal.clear();
            off += size;
            i = j;
        }
        if (ci != c.size()) throw kiwi::error("print format: more argument codes than conversions");
        tail_ = literal;
        bytes_ = off;
    }

    /// Bytes of the packed argument image the callback expects.
    uint32_t payload_bytes() const { return bytes_; }

    /// The formatted text of one payload (no newline added).
    std::string format(const uint8_t* p, uint32_t n) const {
        if (n != bytes_) throw kiwi::error("print: payload of " + std::to_string(n) + " bytes, expected " +
                                           std::to_string(bytes_));
        std::string out;
        char buf[512];
        for (const Piece& pc : pieces_) {
            int w = 0;
            if (pc.code == 'f' || pc.code == 'd') {
                double v = 0;
                if (pc.code == 'f') {
                    float f;
                    std::memcpy(&f, p + pc.offset, 4);
                    v = f;
                } else {
                    std::memcpy(&v, p + pc.offset, 8);
                }
                w = std::snprintf(buf, sizeof(buf), pc.spec.c_str(), v);
            } else if (pc.conv == 'c') {
                w = std::snprintf(buf, sizeof(buf), pc.spec.c_str(), static_cast<int>(read_int(p, pc)));
            } else if (is_signed(pc.code)) {
                w = std::snprintf(buf, sizeof(buf), pc.spec.c_str(), static_cast<long long>(read_int(p, pc)));
            } else {
                const unsigned long long v = read_uint(p, pc);
                const bool signed_conv = pc.conv == 'd' || pc.conv == 'i';
                if (signed_conv && v <= static_cast<unsigned long long>(INT64_MAX)) {
                    w = std::snprintf(buf, sizeof(buf), pc.spec.c_str(), static_cast<long long>(v));
                } else {
                    w = std::snprintf(buf, sizeof(buf), (signed_conv ? pc.spec_u : pc.spec).c_str(), v);
                }
            }
            if (w > 0) out.append(buf, static_cast<size_t>(w) < sizeof(buf) ? static_cast<size_t>(w) : sizeof(buf) - 1);
        }
        if (!tail_.empty()) {
            const int w = std::snprintf(buf, sizeof(buf), tail_.c_str(), 0);  // only %% remain in the tail
            if (w > 0) out.append(buf, static_cast<size_t>(w) < sizeof(buf) ? static_cast<size_t>(w) : sizeof(buf) - 1);
        }
        return out;
    }

    /// Formats and writes one line to `f` (serialised across progress threads).
    void print(const uint8_t* p, uint32_t n, std::FILE* f) const {
        std::string s = format(p, n);
        s += '\n';
        static std::mutex mu;
        std::lock_guard<std::mutex> g(mu);
        std::fwrite(s.data(), 1, s.size(), f);
        std::fflush(f);
    }

private:
    struct Piece {
        std::string spec;    // literal text before the conversion + the conversion itself
        std::string spec_u;  // the same with %u, for %d / %i of unsigned values past INT64_MAX
        char code;
        char conv;
        uint32_t offset;
    };

    static uint32_t code_size(char code) {
        switch (code) {
            case 'b': case 'B': return 1;
            case 'h': case 'H': return 2;
            case 'i': case 'I': case 'l': case 'L': case 'f': return 4;
            case 'q': case 'Q': case 'd': return 8;
            default: throw kiwi::error(std::string("print format: unsupported argument code '") + code + "'");
        }
    }
    static bool is_signed(char code) { return code == 'b' || code == 'h' || code == 'i' || code == 'l' || code == 'q'; }

    // Each branch widens to int64_t on its own: a shared conditional type
    // would turn a negative narrow value into a large unsigned one first.
    static int64_t read_int(const uint8_t* p, const Piece& pc) {
        const bool sgn = is_signed(pc.code);
        switch (code_size(pc.code)) {
            case 1: {
                int8_t v;
                std::memcpy(&v, p + pc.offset, 1);
                return sgn ? static_cast<int64_t>(v) : static_cast<int64_t>(static_cast<uint8_t>(v));
            }
            case 2: {
                int16_t v;
                std::memcpy(&v, p + pc.offset, 2);
                return sgn ? static_cast<int64_t>(v) : static_cast<int64_t>(static_cast<uint16_t>(v));
            }
            case 4: {
                int32_t v;
                std::memcpy(&v, p + pc.offset, 4);
                return sgn ? static_cast<int64_t>(v) : static_cast<int64_t>(static_cast<uint32_t>(v));
            }
            default: {
                int64_t v;
                std::memcpy(&v, p + pc.offset, 8);
                return v;
            }
        }
    }
    static uint64_t read_uint(const uint8_t* p, const Piece& pc) {
        uint64_t v = 0;
        std::memcpy(&v, p + pc.offset, code_size(pc.code));  // little-endian, zero-extended
        return v;
    }

    std::vector<Piece> pieces_;
    std::string tail_;
    uint32_t bytes_ = 0;
};

}  // namespace kiwi::invoke
