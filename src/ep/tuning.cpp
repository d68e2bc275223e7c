#include "kiwi/ep/tuning.hpp"

#include <cctype>
#include <cstdlib>
#include <sstream>

namespace kiwi::ep {

namespace {

struct Entry {
    int32_t max_tokens_upto;  // applies when c.max_tokens <= this
    int32_t recv_per_sm;
    int32_t combine_per_sm;
    const char* source;
};

// Measured on B200 (8-GPU HGX, NVLink 5 / NVSwitch), hidden 7168, top-8,
// FP8 dispatch: latency mode (128 tokens per rank) is bound by the expert
// weight stream, so its side kernels only need a couple of blocks per SM;
// throughput mode (4096 tokens per rank) keeps 8 blocks per SM of 8 warps in
// the memory-bound receive copy and the combine reduce (recv_copy 0.67 and
// combine reduce 0.94 of measured HBM bandwidth in the ncu capture of one
// EP8 rank's shape).
constexpr Entry kB200[] = {
    {256, 4, 4, "b200: latency mode (<= 256 tokens per rank)"},
    {1 << 30, 8, 8, "b200: throughput mode"},
};

bool parse_bool(const std::string& v) {
    if (v == "1" || v == "true" || v == "on") return true;
    if (v == "0" || v == "false" || v == "off") return false;
    throw kiwi::error("KIWI_EP_TUNING: expected a boolean, got '" + v + "'");
}

/// A block count: the whole value must be a decimal integer in [0, 2^20].
int parse_blocks(const std::string& v) {
    if (v.empty() || !(std::isdigit(static_cast<unsigned char>(v[0])) || v[0] == '-')) {
        throw kiwi::error("KIWI_EP_TUNING: expected a number, got '" + v + "'");
    }
    size_t used = 0;
    const long n = std::stol(v, &used, 10);  // invalid_argument / out_of_range handled by the caller
    if (used != v.size()) throw kiwi::error("KIWI_EP_TUNING: trailing characters in '" + v + "'");
    if (n < 0 || n > (1L << 20)) throw kiwi::error("KIWI_EP_TUNING: block count " + v + " outside [0, 2^20]");
    return static_cast<int>(n);
}

}  // namespace

EpTuning tune(const EpConfig& c, int sms, const char* env) {
    if (sms < 1) sms = 1;
    const Entry* e = &kB200[0];
    for (const Entry& x : kB200) {
        if (c.max_tokens <= x.max_tokens_upto) {
            e = &x;
            break;
        }
    }
    EpTuning t;
    t.dispatch_blocks = 0;
    t.recv_blocks = e->recv_per_sm * sms;
    t.combine_blocks = e->combine_per_sm * sms;
    // GEMM2 + NVLink combine fused: 993 us vs 1479 us unfused at EP8 (4096
    // tokens per rank); 4.53 vs 4.87 ms per step at N=1.
    t.fused_combine = true;
    // Gathering GEMM1: 2605 us vs 1483 us TMA-fed (+105 us receive copy) at
    // one EP8 rank's shape.
    t.gather_a = false;
    // 2-SM tiles (cta_group::2, 256 x 256): a third less L2 -> shared-memory
    // traffic per MMA; at one EP8 rank's GEMM1 shape 82 % tensor-pipe activity
    // vs 72 % and 12 % fewer SM cycles (ncu).  Under the power cap that turned
    // into a lower clock rather than a shorter step unless experts get many
    // rows (see kPairMinRows), so the 2-SM kernels run only from kPairMinRows
    // rows per local expert and the split variant is opt-in.
    t.gemm_pair = false;
    t.gemm_pair_auto = true;
    t.gemm_split = false;
    t.gemm2_pair = false;
    // M = 64 MMAs on tiles with at most 64 rows of their expert left: same
    // result bit for bit; one B200 under the power cap, 5.42 -> 5.22 ms per
    // step at 128 rows per expert, 7.84 -> 7.70 at 256, 12.99 -> 12.87 at 512,
    // no change at 1024 (less tensor energy on padding rows, higher clock).
    t.gemm_m64_tails = true;
    t.source = e->source;
    const char* ov = env ? env : std::getenv("KIWI_EP_TUNING");
    if (ov && *ov) {
        std::stringstream ss(ov);
        std::string item;
        while (std::getline(ss, item, ',')) {
            if (item.empty()) continue;
            const auto eq = item.find('=');
            if (eq == std::string::npos) throw kiwi::error("KIWI_EP_TUNING: expected key=value, got '" + item + "'");
            const std::string k = item.substr(0, eq), v = item.substr(eq + 1);
            try {
                if (k == "dispatch_blocks") t.dispatch_blocks = parse_blocks(v);
                else if (k == "recv_blocks") t.recv_blocks = parse_blocks(v);
                else if (k == "combine_blocks") t.combine_blocks = parse_blocks(v);
                else if (k == "fused_combine") t.fused_combine = parse_bool(v);
                else if (k == "gather_a") t.gather_a = parse_bool(v);
                else if (k == "gemm_pair") t.gemm_pair = parse_bool(v);
                else if (k == "gemm_pair_auto") t.gemm_pair_auto = parse_bool(v);
                else if (k == "gemm_split") t.gemm_split = parse_bool(v);
                else if (k == "gemm2_pair") t.gemm2_pair = parse_bool(v);
                else if (k == "gemm_m64_tails") t.gemm_m64_tails = parse_bool(v);
                else throw kiwi::error("KIWI_EP_TUNING: unknown key '" + k + "'");
            } catch (const std::invalid_argument&) {
                throw kiwi::error("KIWI_EP_TUNING: bad number in '" + item + "'");
            } catch (const std::out_of_range&) {
                throw kiwi::error("KIWI_EP_TUNING: number out of range in '" + item + "'");
            }
        }
        if (t.dispatch_blocks < 0 || t.recv_blocks < 1 || t.combine_blocks < 1) {
            throw kiwi::error("KIWI_EP_TUNING: block counts must be positive");
        }
        t.source += " + KIWI_EP_TUNING";
    }
    return t;
}

}  // namespace kiwi::ep
