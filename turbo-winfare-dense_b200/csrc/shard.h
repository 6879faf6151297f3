// How one layer is split across tensor-parallel ranks (host-only; no CUDA).
//
// Rank r of tp holds q heads [q0, q0 + qh_l), the KV heads those q heads read
// [kv0, kv0 + kvh_l) (a KV head is replicated when fewer KV heads than ranks remain, as the
// global layers' 4 KV heads are at tp = 8), and FFN rows [f0, f0 + F_l). The o and down
// projections are split along their K dimension the same way, so each rank's partial sums
// cover its own heads and FFN rows; the ranks' partials add up to the full product.
#pragma once

#include <stdexcept>

#include "format.h"

namespace g4b {

struct Shard {
    int q0, qh_l, kv0, kvh_l, f0, F_l;
};

inline Shard make_shard(const LayerGeometry& g, int F, int rank, int tp) {
    Shard s;
    if (g.q_heads % tp) throw std::runtime_error("q_heads must divide by the tensor-parallel size");
    if (F % tp || (F / tp) % 64) throw std::runtime_error("FFN width / tp must be a multiple of 64");
    s.qh_l = g.q_heads / tp;
    s.q0 = rank * s.qh_l;
    const int gqa = g.q_heads / g.kv_heads;
    s.kv0 = s.q0 / gqa;
    s.kvh_l = (s.q0 + s.qh_l - 1) / gqa + 1 - s.kv0;
    if (s.qh_l % s.kvh_l) throw std::runtime_error("uneven GQA split across ranks");
    s.F_l = F / tp;
    s.f0 = rank * s.F_l;
    return s;
}

}  // namespace g4b
