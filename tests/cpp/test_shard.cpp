// The tensor-parallel split of a layer (csrc/shard.h), checked on the host for every tp the engine
// runs (1, 2, 4, 8) and every layer kind of the 31B target, the E2B-shaped drafter and the test
// models:
//   - the ranks' q heads and FFN rows tile the layer exactly once, in rank order;
//   - every local q head reads the KV head it reads unsplit (global head h / gqa), through the
//     local GQA ratio qh_l / kvh_l, so a KV head is held by exactly the ranks whose q heads need
//     it (replicated when tp exceeds the KV head count, as the 31B's 4 global KV heads are at 8);
//   - the o and down K-splits (qh_l * head_dim, F_l) are whole 64-groups;
//   - a split the engine cannot make (q heads or FFN width not divisible) is refused.
#include <cstdio>
#include <stdexcept>
#include <vector>

#include "shard.h"

using namespace g4b;

static int failures = 0;
#define CHECK(c)                                                                   \
    do {                                                                           \
        if (!(c)) {                                                                \
            std::fprintf(stderr, "CHECK failed: %s (line %d)\n", #c, __LINE__);   \
            ++failures;                                                            \
        }                                                                          \
    } while (0)

struct Kind {
    const char* name;
    LayerGeometry g;
    int ffn;
};

static void check_kind(const Kind& k, int tp) {
    const int Q = (int)k.g.q_heads, KV = (int)k.g.kv_heads, gqa = Q / KV;
    std::vector<int> q_owner(Q, -1), f_owner(k.ffn, -1), kv_holders(KV, 0);
    for (int r = 0; r < tp; ++r) {
        const Shard s = make_shard(k.g, k.ffn, r, tp);
        CHECK(s.qh_l * tp == Q && s.q0 == r * s.qh_l);
        CHECK(s.F_l * tp == k.ffn && s.f0 == r * s.F_l && s.F_l % 64 == 0);
        CHECK((s.qh_l * (int)k.g.head_dim) % 64 == 0);
        CHECK(s.kvh_l >= 1 && s.qh_l % s.kvh_l == 0);
        for (int h = s.q0; h < s.q0 + s.qh_l; ++h) {
            CHECK(q_owner[h] == -1);
            q_owner[h] = r;
            // local q head (h - q0) reads local KV head (h - q0) / (qh_l / kvh_l)
            CHECK(s.kv0 + (h - s.q0) / (s.qh_l / s.kvh_l) == h / gqa);
        }
        for (int kv = s.kv0; kv < s.kv0 + s.kvh_l; ++kv) {
            CHECK(kv >= 0 && kv < KV);
            if (kv >= 0 && kv < KV) ++kv_holders[kv];
        }
        for (int f = s.f0; f < s.f0 + s.F_l; ++f) {
            CHECK(f_owner[f] == -1);
            f_owner[f] = r;
        }
    }
    for (int h = 0; h < Q; ++h) CHECK(q_owner[h] >= 0);
    for (int f = 0; f < k.ffn; ++f) CHECK(f_owner[f] >= 0);
    // A KV head is held by as many ranks as split its gqa query heads (1 when tp <= KV).
    const int expect = tp > KV ? tp / KV : 1;
    for (int kv = 0; kv < KV; ++kv) CHECK(kv_holders[kv] == expect);
}

static bool refused(const LayerGeometry& g, int ffn, int tp) {
    try {
        make_shard(g, ffn, 0, tp);
    } catch (const std::runtime_error&) {
        return true;
    }
    return false;
}

int main() {
    const Kind kinds[] = {
        {"31B sliding", {256, 32, 16, false}, 21504},
        {"31B global", {512, 32, 4, true}, 21504},
        {"E2B-shaped drafter", {256, 8, 1, false}, 6144},
        {"config-0 target", {64, 4, 1, false}, 1024},
        {"TP test target", {64, 8, 8, false}, 1024},
    };
    const int tps[] = {1, 2, 4, 8};
    for (const Kind& k : kinds)
        for (int tp : tps)
            if (k.g.q_heads % tp == 0 && (k.ffn / tp) % 64 == 0) check_kind(k, tp);
    // The 31B at tp = 8: one global KV head per rank, each held by two ranks.
    const Shard s = make_shard({512, 32, 4, true}, 21504, 5, 8);
    CHECK(s.qh_l == 4 && s.q0 == 20 && s.kvh_l == 1 && s.kv0 == 2 && s.F_l == 2688 && s.f0 == 13440);
    CHECK(refused({64, 4, 1, false}, 1024, 8));   // 4 q heads over 8 ranks
    CHECK(refused({256, 32, 16, false}, 1000, 2)); // FFN width not divisible
    CHECK(refused({256, 32, 16, false}, 21504, 64)); // 336 rows per rank: not whole 64-groups
    if (failures) {
        std::fprintf(stderr, "%d check(s) failed\n", failures);
        return 1;
    }
    std::printf("shard plan: all checks passed\n");
    return 0;
}
