// Host-side stress of kiwi::queue and kiwi::invoke, compiled with
// -fsanitize=thread and with -fsanitize=address,undefined by
// tests/test_sanitizers_host.py (CPU only, no GPU).
//
// Each case runs real producer and consumer threads over the host-only rings
// (plain memory instead of mapped pinned memory, same code paths):
//   spsc_d2h  - a producer thread and the consumer over an 8-line ring, so
//               every message wraps and the producer waits for credit;
//   mpsc      - four CPU stand-ins for the device producers (fetch-add line
//               claims, credit waits, out-of-order completion) and the host
//               consumer: every message once, each producer's in its order;
//   spsc_h2d  - the host producer of an H2D ring and a CPU stand-in for the
//               device consumer that publishes its position;
//   mpmc_push - four threads claim slots of one MPMC H2D ring concurrently;
//   mpmc      - three producers and two CPU stand-in consumers (the device
//               consumers' claim / tag / ack protocol) through a 16-slot MPMC
//               ring: every message arrives exactly once, payload intact;
//   invoke    - four producer threads (one per endpoint) feed an invoke
//               Context served by two progress threads, then stop() drains;
//   print     - the native print formatter over many formats and payloads,
//               from two threads at once (buffer and integer handling);
//   fuzz      - the host reader over random ring contents in which about
//               half the words carry the right lap tag: every pop returns,
//               consumes a whole message or throws queue_error, and never
//               reads outside the ring (ASan) or its output buffer;
//   fuzz_invoke - random callback ids (some unregistered) and payload sizes
//               (mostly wrong) through an invoke Context: every message
//               either runs its callback or raises invoke_error once, and
//               progress continues after each error;
//   fds       - four "ranks" (threads) exchange pipe descriptors with
//               SCM_RIGHTS over abstract sockets, then a broadcast; every
//               received descriptor must reach its sender's pipe.
// Exit status 0 and no sanitizer report mean the case passed.
#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <thread>
#include <vector>

#include "kiwi/invoke/invoke.hpp"
#include "kiwi/invoke/printer.hpp"
#include "kiwi/invoke/progress.hpp"
#include "kiwi/p2p/heap.hpp"
#include "kiwi/queue/queue.hpp"

#include <unistd.h>

using namespace kiwi;
using namespace kiwi::queue;

namespace {

int fail(const char* what, long a, long b) {
    std::fprintf(stderr, "FAIL %s: %ld vs %ld\n", what, a, b);
    return 1;
}

void fill(uint8_t* p, uint32_t n, uint32_t seed) {
    for (uint32_t i = 0; i < n; ++i) p[i] = static_cast<uint8_t>(seed * 31u + i);
}

bool check(const uint8_t* p, uint32_t n, uint32_t seed) {
    for (uint32_t i = 0; i < n; ++i) {
        if (p[i] != static_cast<uint8_t>(seed * 31u + i)) return false;
    }
    return true;
}

int spsc_d2h() {
    SPSCD2HQueue q(8, MemKind::kHost);
    RingWriter w = q.host_writer();
    const uint32_t n = 20000;
    std::thread producer([&] {
        alignas(16) uint8_t buf[kMaxMessageBytes];
        for (uint32_t i = 0; i < n; ++i) {
            const uint32_t bytes = (i * 7) % 121;
            fill(buf, bytes, i);
            while (!w.try_push(buf, bytes, i)) std::this_thread::yield();
        }
    });
    alignas(16) uint8_t buf[kMaxMessageBytes];
    for (uint32_t got = 0; got < n;) {
        uint32_t meta = 0, bytes = 0;
        if (!q.try_pop(buf, &meta, &bytes)) {
            std::this_thread::yield();
            continue;
        }
        if (meta != got) return fail("spsc_d2h order", meta, got);
        if (bytes != (got * 7) % 121 || !check(buf, bytes, got)) return fail("spsc_d2h payload", got, bytes);
        ++got;
    }
    producer.join();
    return 0;
}

int mpsc_d2h() {
    MPSCD2HQueue q(16, MemKind::kHost);
    const uint32_t producers = 4, per = 5000, total = producers * per;
    std::atomic<int> bad{0};
    std::vector<std::thread> ts;
    for (uint32_t p = 0; p < producers; ++p) {
        ts.emplace_back([&, p] {
            uint8_t msg[kMaxMessageBytes];
            try {
                for (uint32_t i = 0; i < per; ++i) {
                    const uint32_t bytes = 8 + (i * 13 + p * 5) % 200;  // 1 to 4 lines
                    std::memcpy(msg, &i, 4);
                    std::memcpy(msg + 4, &p, 4);
                    fill(msg + 8, bytes - 8, p * per + i);
                    q.host_push(msg, bytes, p, 60.0);
                }
            } catch (const std::exception& e) {
                std::fprintf(stderr, "producer %u: %s\n", p, e.what());
                bad.store(1);
            }
        });
    }
    std::vector<uint32_t> next(producers, 0);
    alignas(16) uint8_t buf[kMaxMessageBytes];
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::seconds(120);
    for (uint32_t got = 0; got < total && !bad.load();) {
        uint32_t meta = 0, bytes = 0;
        if (!q.try_pop(buf, &meta, &bytes)) {
            if (std::chrono::steady_clock::now() > deadline) return fail("mpsc stalled", got, total);
            std::this_thread::yield();
            continue;
        }
        uint32_t i, p;
        std::memcpy(&i, buf, 4);
        std::memcpy(&p, buf + 4, 4);
        if (p != meta || p >= producers || i != next[p] || bytes != 8 + (i * 13 + p * 5) % 200 ||
            !check(buf + 8, bytes - 8, p * per + i)) {
            bad.store(1);
            break;
        }
        ++next[p];
        ++got;
    }
    for (auto& t : ts) t.join();
    return bad.load() ? fail("mpsc order or payload", 1, 0) : 0;
}

int spsc_h2d() {
    SPSCH2DQueue q(16, MemKind::kHost);
    const uint32_t n = 20000;
    std::atomic<int> bad{0};
    std::thread consumer([&] {
        RingReader r(q.ring_host(), q.capacity(), q.consumer_pos_host());
        alignas(16) uint8_t buf[kMaxMessageBytes];
        for (uint32_t got = 0; got < n;) {
            uint32_t meta = 0, bytes = 0;
            if (!r.try_pop(buf, &meta, &bytes)) {
                std::this_thread::yield();
                continue;
            }
            if (meta != got || bytes != (got * 5) % 97 || !check(buf, bytes, got)) bad.store(1);
            ++got;
        }
    });
    alignas(16) uint8_t buf[kMaxMessageBytes];
    for (uint32_t i = 0; i < n; ++i) {
        const uint32_t bytes = (i * 5) % 97;
        fill(buf, bytes, i);
        while (!q.try_push(buf, bytes, i)) std::this_thread::yield();
    }
    consumer.join();
    return bad.load() ? fail("spsc_h2d payload", 1, 0) : 0;
}

int mpmc_push() {
    MPMCH2DQueue q(64, 2, MemKind::kHost);
    std::atomic<int> pushed{0};
    std::vector<std::thread> ts;
    for (int t = 0; t < 4; ++t) {
        ts.emplace_back([&, t] {
            uint64_t v = static_cast<uint64_t>(t);
            for (int i = 0; i < 16; ++i) {
                if (q.try_push(&v, sizeof(v), static_cast<uint32_t>(t))) pushed.fetch_add(1);
            }
        });
    }
    for (auto& th : ts) th.join();
    // 64 free slots, 64 attempts: every push lands in its own slot.
    if (pushed.load() != 64) return fail("mpmc_push count", pushed.load(), 64);
    if (q.producer_position() != 64) return fail("mpmc_push head", static_cast<long>(q.producer_position()), 64);
    return 0;
}

int mpmc_full() {
    MPMCH2DQueue q(16, 2, MemKind::kHost);
    const uint32_t producers = 3, per = 4000, total = producers * per;
    std::atomic<uint32_t> got{0};
    std::atomic<int> bad{0};
    std::vector<std::vector<uint64_t>> seen(2);
    std::vector<std::thread> ts;
    for (uint32_t p = 0; p < producers; ++p) {
        ts.emplace_back([&, p] {
            uint8_t msg[56];
            for (uint32_t i = 0; i < per; ++i) {
                const uint32_t bytes = 8 + (i * 7 + p) % 49;  // 8 .. 56
                std::memcpy(msg, &p, 4);
                std::memcpy(msg + 4, &i, 4);
                fill(msg + 8, bytes - 8, p * per + i);
                while (!q.try_push(msg, bytes, p)) std::this_thread::yield();
            }
        });
    }
    for (int c = 0; c < 2; ++c) {
        ts.emplace_back([&, c] {
            uint8_t buf[64];
            while (got.load() < total) {
                uint32_t meta = 0, bytes = 0;
                if (!q.host_try_pop(buf, &meta, &bytes)) {
                    std::this_thread::yield();
                    continue;
                }
                got.fetch_add(1);
                uint32_t p, i;
                std::memcpy(&p, buf, 4);
                std::memcpy(&i, buf + 4, 4);
                if (p != meta || p >= producers || i >= per || bytes != 8 + (i * 7 + p) % 49 ||
                    !check(buf + 8, bytes - 8, p * per + i)) {
                    bad.store(1);
                }
                seen[c].push_back(static_cast<uint64_t>(p) * per + i);
            }
        });
    }
    for (auto& t : ts) t.join();
    if (bad.load()) return fail("mpmc payload", 1, 0);
    std::vector<uint64_t> all(seen[0]);
    all.insert(all.end(), seen[1].begin(), seen[1].end());
    std::sort(all.begin(), all.end());
    if (all.size() != total) return fail("mpmc count", static_cast<long>(all.size()), total);
    for (uint32_t k = 0; k < total; ++k) {
        if (all[k] != k) return fail("mpmc exactly once", static_cast<long>(all[k]), k);
    }
    return 0;
}

int invoke_threads() {
    invoke::Context<SPSCD2HQueue> ctx(4, 16, MemKind::kHost);
    std::atomic<uint64_t> sum{0};
    std::atomic<uint32_t> calls{0};
    const uint8_t cb = ctx.register_callback(std::function<void(uint32_t, uint64_t)>([&](uint32_t ep, uint64_t v) {
        sum.fetch_add(v + ep, std::memory_order_relaxed);
        calls.fetch_add(1, std::memory_order_relaxed);
    }));
    invoke::ProgressThreads<SPSCD2HQueue> threads(ctx);
    threads.start(2);
    const uint32_t per = 3000;
    std::vector<std::thread> producers;
    for (uint32_t ep = 0; ep < 4; ++ep) {
        producers.emplace_back([&, ep] {
            RingWriter w = ctx.raw_queue(ep)->host_writer_any();
            for (uint32_t i = 0; i < per; ++i) {
                uint8_t msg[12];  // the serializer's packed image of (uint32_t, uint64_t)
                const uint64_t v = i;
                std::memcpy(msg, &ep, 4);
                std::memcpy(msg + 4, &v, 8);
                while (!w.try_push(msg, sizeof(msg), cb)) std::this_thread::yield();
            }
        });
    }
    for (auto& p : producers) p.join();
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::seconds(60);
    while (calls.load() < 4 * per && std::chrono::steady_clock::now() < deadline) std::this_thread::yield();
    threads.stop();
    threads.rethrow_if_failed();
    if (calls.load() != 4 * per) return fail("invoke calls", calls.load(), 4 * per);
    const uint64_t want = 4ull * per * (per - 1) / 2 + per * (0 + 1 + 2 + 3);
    if (sum.load() != want) return fail("invoke sum", static_cast<long>(sum.load()), static_cast<long>(want));
    const auto st = threads.stats();
    if (st.callbacks != 4ull * per) return fail("invoke stats", static_cast<long>(st.callbacks), 4 * per);
    return 0;
}

int invoke_active_prefix() {
    // Producers push to every endpoint while a controller grows and shrinks the
    // active prefix; every message must still run exactly once (a dropped
    // endpoint keeps its messages until the prefix covers it again or stop()).
    invoke::Context<SPSCD2HQueue> ctx(8, 16, MemKind::kHost);
    std::vector<std::atomic<uint32_t>> next(8);
    for (auto& n : next) n.store(0);
    std::atomic<int> bad{0};
    const uint8_t cb = ctx.register_callback(std::function<void(uint32_t, uint32_t)>([&](uint32_t ep, uint32_t i) {
        if (ep >= 8 || next[ep].fetch_add(1, std::memory_order_relaxed) != i) bad.store(1);
    }));
    invoke::ProgressThreads<SPSCD2HQueue> threads(ctx);
    threads.start(3);
    const uint32_t per = 2000;
    std::atomic<bool> done{false};
    std::thread controller([&] {
        const size_t cycle[] = {2, 8, 1, 5, 0, 3};
        for (size_t k = 0; !done.load(); ++k) {
            const uint32_t gen = threads.set_active_endpoints(cycle[k % 6]);
            while (!threads.active_applied(gen) && !done.load()) std::this_thread::yield();
        }
        threads.set_active_endpoints(0);
    });
    std::vector<std::thread> producers;
    for (uint32_t ep = 0; ep < 8; ++ep) {
        producers.emplace_back([&, ep] {
            RingWriter w = ctx.raw_queue(ep)->host_writer_any();
            for (uint32_t i = 0; i < per; ++i) {
                uint8_t msg[8];
                std::memcpy(msg, &ep, 4);
                std::memcpy(msg + 4, &i, 4);
                while (!w.try_push(msg, sizeof(msg), cb)) std::this_thread::yield();
            }
        });
    }
    for (auto& p : producers) p.join();
    done.store(true);
    controller.join();
    threads.stop();
    threads.rethrow_if_failed();
    if (bad.load()) return fail("active prefix order", 1, 0);
    for (uint32_t ep = 0; ep < 8; ++ep) {
        if (next[ep].load() != per) return fail("active prefix count", next[ep].load(), per);
    }
    return 0;
}

int print_formats() {
    struct F {
        const char* fmt;
        const char* codes;
    } formats[] = {{"step=%d value=%.2f tag=0x%llx", "ifQ"}, {"%-12u|%+08.3e|%c", "IdB"},
                   {"%llu %lld %x %o", "QqHb"}, {"%%%5.1g%% of %hhd", "fb"}, {"plain text", ""},
                   {"%300.200f", "d"}};
    std::atomic<int> bad{0};
    auto work = [&](uint64_t seed) {
        uint8_t payload[64];
        for (int it = 0; it < 2000; ++it) {
            for (const auto& f : formats) {
                kiwi::invoke::PrintFormat pf(f.fmt, f.codes);
                for (uint32_t i = 0; i < pf.payload_bytes(); ++i) {
                    seed = seed * 6364136223846793005ull + 1442695040888963407ull;
                    payload[i] = static_cast<uint8_t>(seed >> 56);
                }
                if (pf.payload_bytes() >= 8 && std::strcmp(f.codes, "d") == 0) {
                    const double v = 1e300;  // the widest %f output
                    std::memcpy(payload, &v, 8);
                }
                const std::string out = pf.format(payload, pf.payload_bytes());
                if (out.size() > 4096) bad.store(1);
            }
        }
    };
    std::thread t1(work, 1), t2(work, 2);
    t1.join();
    t2.join();
    return bad.load() ? fail("print length", 1, 0) : 0;
}

int fuzz_reader() {
    uint64_t seed = 0x2545F4914F6CDD1Dull;
    auto rnd = [&] {
        seed ^= seed << 13;
        seed ^= seed >> 7;
        seed ^= seed << 17;
        return seed;
    };
    uint64_t pops = 0, errors = 0;
    for (int round = 0; round < 4000; ++round) {
        const uint64_t cap = 1ull << (rnd() % 8);  // 1 .. 128 lines
        SPSCD2HQueue q(cap, MemKind::kHost);
        Chunk* ring = q.ring_host();
        const uint32_t log2cap = static_cast<uint32_t>(__builtin_ctzll(cap));
        for (uint64_t line = 0; line < cap; ++line) {
            const uint32_t tag = lap_tag(line, log2cap);
            for (uint32_t c = 0; c < kChunksPerLine; ++c) {
                uint32_t w[4];
                if (c == 0 && (rnd() & 1)) {
                    // a well-formed header: metadata and a length, half of them short,
                    // the rest up to 1.2x the maximum
                    const uint32_t len = (rnd() & 1) ? static_cast<uint32_t>(rnd() % 64)
                                                     : static_cast<uint32_t>(rnd() % (kMaxMessageBytes + kMaxMessageBytes / 5));
                    const uint64_t h0 = pack_half(static_cast<uint32_t>(rnd()), tag), h1 = pack_half(len, tag);
                    std::memcpy(w, &h0, 8);
                    std::memcpy(w + 2, &h1, 8);
                } else {
                    for (auto& x : w) {
                        const uint32_t data = static_cast<uint32_t>(rnd());
                        x = (rnd() % 10) ? tagged_word(data, tag) : static_cast<uint32_t>(rnd());
                    }
                }
                std::memcpy(&ring[line * kChunksPerLine + c], w, sizeof(w));
            }
        }
        alignas(16) uint8_t out[kMaxMessageBytes + 64];
        for (int k = 0; k < 64; ++k) {
            uint32_t meta = 0, bytes = 0;
            try {
                if (!q.try_pop(out, &meta, &bytes)) break;
                if (bytes > kMaxMessageBytes) return fail("fuzz length", bytes, kMaxMessageBytes);
                ++pops;
            } catch (const queue_error&) {
                ++errors;
                break;
            }
        }
    }
    std::printf("fuzz: %llu pops, %llu rejected rings\n", static_cast<unsigned long long>(pops),
                static_cast<unsigned long long>(errors));
    return 0;
}

int fuzz_invoke() {
    invoke::Context<SPSCD2HQueue> ctx(1, 64, MemKind::kHost);
    std::atomic<uint64_t> called{0};
    ctx.register_callback(std::function<void(uint32_t)>([&](uint32_t) { called.fetch_add(1); }));
    ctx.register_callback(std::function<void(uint64_t, float, uint8_t)>(
        [&](uint64_t, float, uint8_t) { called.fetch_add(1); }));
    ctx.register_raw_callback([&](const uint8_t*, uint32_t) { called.fetch_add(1); },
                              invoke::CallbackBase::kAnySize);
    RingWriter w = ctx.raw_queue(0)->host_writer_any();
    uint64_t seed = 88172645463325252ull, errors = 0, sent = 0;
    auto rnd = [&] {
        seed ^= seed << 13;
        seed ^= seed >> 7;
        seed ^= seed << 17;
        return seed;
    };
    auto drain_once = [&]() -> size_t {
        try {
            return ctx.progress(0);
        } catch (const std::exception&) {
            ++errors;
            return 1;
        }
    };
    uint8_t payload[128];
    for (int i = 0; i < 20000; ++i) {
        for (auto& b : payload) b = static_cast<uint8_t>(rnd());
        const uint32_t bytes = static_cast<uint32_t>(rnd() % 97);
        const uint32_t meta = static_cast<uint32_t>(rnd() % 6);  // ids 3..5 are not registered
        while (!w.try_push(payload, bytes, meta)) drain_once();
        ++sent;
    }
    while (drain_once() != 0) {
    }
    if (called.load() + errors != sent) {
        return fail("invoke fuzz accounting", static_cast<long>(called.load() + errors), static_cast<long>(sent));
    }
    std::printf("fuzz_invoke: %llu calls, %llu rejected\n", static_cast<unsigned long long>(called.load()),
                static_cast<unsigned long long>(errors));
    return 0;
}

int fd_exchange() {
    const int world = 4;
    int pipes[world][2];
    for (auto& p : pipes) {
        if (pipe(p) != 0) return fail("pipe", 0, 0);
    }
    const std::string job = "stress" + std::to_string(getpid());
    std::vector<std::vector<int>> got(world);
    std::vector<int> bcast(world, -1);
    std::atomic<int> bad{0};
    std::vector<std::thread> ts;
    for (int r = 0; r < world; ++r) {
        ts.emplace_back([&, r] {
            try {
                got[r] = kiwi::p2p::exchange_fds(job, r, world, pipes[r][1], 20.0);
                bcast[r] = kiwi::p2p::broadcast_fd(job + "b", r, world, 0, r == 0 ? pipes[0][1] : -1, 20.0);
            } catch (const std::exception& e) {
                std::fprintf(stderr, "rank %d: %s\n", r, e.what());
                bad.store(1);
            }
        });
    }
    for (auto& t : ts) t.join();
    if (bad.load()) return fail("fd exchange threw", 1, 0);
    // rank r writes (r, q) through its copy of q's descriptor; q's pipe must hold it.
    for (int r = 0; r < world; ++r) {
        if (static_cast<int>(got[r].size()) != world) return fail("fd count", static_cast<long>(got[r].size()), world);
        for (int q = 0; q < world; ++q) {
            const uint8_t msg[2] = {static_cast<uint8_t>(r), static_cast<uint8_t>(q)};
            if (write(got[r][q], msg, 2) != 2) return fail("write", r, q);
        }
    }
    for (int q = 0; q < world; ++q) {
        uint8_t buf[2 * world];
        ssize_t n = 0;
        while (n < 2 * world) {
            const ssize_t k = read(pipes[q][0], buf + n, sizeof(buf) - n);
            if (k <= 0) return fail("read", q, static_cast<long>(k));
            n += k;
        }
        for (int i = 0; i < world; ++i) {
            if (buf[2 * i + 1] != q) return fail("fd routed to the wrong pipe", buf[2 * i + 1], q);
        }
    }
    for (int r = 0; r < world; ++r) {
        const uint8_t m = 0xB0;
        if (write(bcast[r], &m, 1) != 1) return fail("broadcast write", r, 0);
    }
    uint8_t b[world];
    ssize_t n = 0;
    while (n < world) {
        const ssize_t k = read(pipes[0][0], b + n, sizeof(b) - n);
        if (k <= 0) return fail("broadcast read", static_cast<long>(k), 0);
        n += k;
    }
    for (int r = 0; r < world; ++r) {
        for (int q = 0; q < world; ++q) close(got[r][q]);
        close(bcast[r]);
        close(pipes[r][0]);
        close(pipes[r][1]);
    }
    return 0;
}

}  // namespace

int main(int argc, char** argv) {
    struct Case {
        const char* name;
        int (*fn)();
    } cases[] = {{"spsc_d2h", spsc_d2h}, {"mpsc", mpsc_d2h}, {"spsc_h2d", spsc_h2d}, {"mpmc_push", mpmc_push}, {"mpmc", mpmc_full},
                 {"invoke", invoke_threads}, {"invoke_active", invoke_active_prefix},
                 {"print", print_formats}, {"fuzz", fuzz_reader}, {"fuzz_invoke", fuzz_invoke},
                 {"fds", fd_exchange}};
    int rc = 0;
    for (const auto& c : cases) {
        if (argc > 1 && std::strcmp(argv[1], c.name) != 0) continue;
        const int r = c.fn();
        std::printf("%s %s\n", c.name, r ? "FAIL" : "ok");
        rc |= r;
    }
    return rc;
}
