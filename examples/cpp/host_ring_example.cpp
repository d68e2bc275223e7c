// Host-only use of a kiwi::queue ring: a producer thread and a consumer
// thread exchange messages through the same wire format the GPU writes
// (no GPU needed).  `make -C examples && examples/build/host_ring_example`
#include <cstdio>
#include <cstring>
#include <thread>

#include "kiwi/queue/queue.hpp"

int main() {
    using namespace kiwi::queue;
    SPSCD2HQueue q(64, MemKind::kHost);
    RingWriter w = q.host_writer();
    const int n = 100000;
    std::thread producer([&] {
        for (int i = 0; i < n; ++i) {
            uint64_t v = static_cast<uint64_t>(i) * 3;
            while (!w.try_push(&v, sizeof(v), static_cast<uint32_t>(i))) {
            }
        }
    });
    uint64_t sum = 0;
    alignas(16) uint8_t buf[kMaxMessageBytes];
    for (int got = 0; got < n;) {
        uint32_t meta, bytes;
        if (q.try_pop(buf, &meta, &bytes)) {
            uint64_t v;
            std::memcpy(&v, buf, 8);
            sum += v;
            ++got;
        }
    }
    producer.join();
    std::printf("received %d messages, sum %llu (expected %llu)\n", n, static_cast<unsigned long long>(sum),
                static_cast<unsigned long long>(3ull * n * (n - 1) / 2));
    return sum == 3ull * n * (n - 1) / 2 ? 0 : 1;
}
