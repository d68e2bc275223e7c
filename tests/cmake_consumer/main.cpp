// Host-only use of the installed libraries: the EP heap layout and B200 launch
// table, the allocation-free GEMM's limits and the topology helpers.  Prints
// one line the test parses; runs without a GPU.
#include <cstdio>

#include "kiwi/ep/config.hpp"
#include "kiwi/ep/tuning.hpp"
#include "kiwi/gemm/noalloc.h"
#include "kiwi/topology.hpp"

int main() {
    kiwi::ep::EpConfig c{};
    c.world = 8;
    c.rank = 0;
    c.hidden = 7168;
    c.num_experts = 256;
    c.topk = 8;
    c.max_tokens = 4096;
    c.quant = static_cast<int32_t>(kiwi::ep::Quant::kFp8);
    c = kiwi::ep::finalize(c);
    const kiwi::ep::EpTuning t = kiwi::ep::tune(c, 148, "");
    const auto cpus = kiwi::topology::parse_cpulist("0-3,8");
    std::printf("experts_per_rank=%d heap_bytes=%llu recv_blocks=%d m64=%d max_groups=%d cpus=%zu\n",
                c.experts_per_rank, static_cast<unsigned long long>(c.heap_bytes), t.recv_blocks,
                t.gemm_m64_tails ? 1 : 0, kiwi_noalloc_max_groups(), cpus.size());
    return 0;
}
