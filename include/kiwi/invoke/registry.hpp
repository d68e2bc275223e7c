// Host callback registry: type-erased callbacks addressed by an 8-bit id.
//
// Parity with the reference (AMDResearch/kiwi):
//   CallbackRegistry  include/kiwi/invoke/internal/callback_registry.hpp:15-54 (<= 256 ids)
//   CallbackWrapper   include/kiwi/invoke/internal/callback_wrapper.hpp:17-64 (size check)
//   Dispatcher        include/kiwi/invoke/internal/dispatcher.hpp:18-47
// Added here: RawCallback, which receives the payload bytes as they are (used
// by the Python frontend, whose callbacks declare a struct format string).
#pragma once

#include <functional>
#include <memory>
#include <vector>

#include "kiwi/invoke/serializer.hpp"
#include "kiwi/queue/wire.hpp"

namespace kiwi::invoke {

class invoke_error : public kiwi::error {
public:
    using kiwi::error::error;
};

inline constexpr uint32_t kMaxCallbacks = 256;

class CallbackBase {
public:
    virtual ~CallbackBase() = default;
    /// Payload bytes the callback expects; kAnySize for raw callbacks.
    virtual uint32_t arg_bytes() const = 0;
    virtual void call(const uint8_t* args, uint32_t bytes) = 0;
    static constexpr uint32_t kAnySize = 0xffffffffu;
};

template <typename... Args>
class TypedCallback final : public CallbackBase {
public:
    explicit TypedCallback(std::function<void(Args...)> fn) : fn_(std::move(fn)) {}
    uint32_t arg_bytes() const override { return ArgPack<Args...>::total_bytes; }
    void call(const uint8_t* args, uint32_t bytes) override {
        if (bytes != ArgPack<Args...>::total_bytes) {
            throw invoke_error("kiwi::invoke: callback expects " +
                               std::to_string(ArgPack<Args...>::total_bytes) +
                               " argument bytes, message carries " + std::to_string(bytes));
        }
        std::apply(fn_, ArgPack<Args...>::deserialize(args));
    }

private:
    std::function<void(Args...)> fn_;
};

class RawCallback final : public CallbackBase {
public:
    using Fn = std::function<void(const uint8_t*, uint32_t)>;
    RawCallback(Fn fn, uint32_t expected_bytes) : fn_(std::move(fn)), expected_(expected_bytes) {}
    uint32_t arg_bytes() const override { return expected_; }
    void call(const uint8_t* args, uint32_t bytes) override {
        if (expected_ != kAnySize && bytes != expected_) {
            throw invoke_error("kiwi::invoke: raw callback expects " + std::to_string(expected_) +
                               " bytes, message carries " + std::to_string(bytes));
        }
        fn_(args, bytes);
    }

private:
    Fn fn_;
    uint32_t expected_;
};

class CallbackRegistry {
public:
    uint8_t add(std::unique_ptr<CallbackBase> cb) {
        if (callbacks_.size() >= kMaxCallbacks) {
            throw invoke_error("kiwi::invoke: callback registry is full (256 callbacks)");
        }
        callbacks_.push_back(std::move(cb));
        return static_cast<uint8_t>(callbacks_.size() - 1);
    }

    CallbackBase& get(uint32_t id) {
        if (id >= callbacks_.size()) {
            throw invoke_error("kiwi::invoke: message for unregistered callback id " +
                               std::to_string(id));
        }
        return *callbacks_[id];
    }

    size_t size() const { return callbacks_.size(); }

private:
    std::vector<std::unique_ptr<CallbackBase>> callbacks_;
};

}  // namespace kiwi::invoke
