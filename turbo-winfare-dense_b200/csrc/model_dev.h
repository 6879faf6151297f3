// Device-side descriptors shared by the forward-pass kernels and their host launchers.
#pragma once
#include <cuda_fp16.h>
#include <cstdint>

#include "passrows.h"
#include "vgemm.h"

namespace g4b {

// Per-pass inputs that change between graph replays: the position of the batch's first row
// and its token ids. Kernels read them from device memory so one captured graph serves every
// position.
struct StepParams {
    int base_pos;
    int draft_step;  // drafter chaining: index of the next draft written to the chain list
    int aux;         // MTP drafter: row of the target's normed hidden states a round starts from
    uint32_t tokens[kPrefillRows];  // a verify pass uses the first 16, a prefill chunk up to 128
};

// A GEMM output as its consumers see it: split-K partial slots (part.part != nullptr), summed
// by the consumer in slot order, or a dense fp32 [M][ld] matrix (a GEMM that finished its own
// sum, e.g. ahead of a tensor-parallel all-reduce).
struct GemmOut {
    PartView part;
    const float* y;
    int ld;
};

#ifdef __CUDACC__
// Slot 0 of row m in row group crg (slot s is 4096 floats further) and the slot count: the
// CTAs whose unit ranges [c*T/G, (c+1)*T/G) meet the group's units.
__device__ __forceinline__ const float* slot_base(const PartView& v, int m, int crg) {
    return v.part + ((size_t)crg * v.max_slots * 16 + m) * 256;
}
__device__ __forceinline__ int slot_count(const PartView& v, int crg) {
    const int T = v.n_crg * v.ktiles;
    return vgemm_cta_of_unit32((crg + 1) * v.ktiles - 1, T, v.grid) - vgemm_cta_of_unit32(crg * v.ktiles, T, v.grid) + 1;
}
// out[j] = sum over s < ns, in slot order, of p[s * 4096 + j * stride]. The loads of a batch
// (B slots x NE elements) are all issued before any is added: a few memory round trips in
// total rather than one per slot.
template <int NE, int B>
__device__ __forceinline__ void slot_sums(const float* p, int stride, int ns, float (&out)[NE]) {
#pragma unroll
    for (int j = 0; j < NE; ++j) out[j] = 0.f;
    for (int s0 = 0; s0 < ns; s0 += B) {
        float v[B][NE];
#pragma unroll
        for (int k = 0; k < B; ++k)
#pragma unroll
            for (int j = 0; j < NE; ++j)
                if (s0 + k < ns) v[k][j] = __ldcg(p + (size_t)(s0 + k) * 4096 + j * stride);
#pragma unroll
        for (int k = 0; k < B; ++k)
#pragma unroll
            for (int j = 0; j < NE; ++j)
                if (s0 + k < ns) out[j] += v[k][j];
    }
}
// Per-element variant: element j has its own slot-0 pointer p[j] and slot count ns[j]
// (elements may sit in different row groups); nsmax = max ns[j]. Same slot order.
template <int NE, int B>
__device__ __forceinline__ void slot_sums_each(const float* const (&p)[NE], const int (&ns)[NE], int nsmax,
                                               float (&out)[NE]) {
#pragma unroll
    for (int j = 0; j < NE; ++j) out[j] = 0.f;
    for (int s0 = 0; s0 < nsmax; s0 += B) {
        float v[B][NE];
#pragma unroll
        for (int k = 0; k < B; ++k)
#pragma unroll
            for (int j = 0; j < NE; ++j)
                if (s0 + k < ns[j]) v[k][j] = __ldcg(p[j] + (size_t)(s0 + k) * 4096);
#pragma unroll
        for (int k = 0; k < B; ++k)
#pragma unroll
            for (int j = 0; j < NE; ++j)
                if (s0 + k < ns[j]) out[j] += v[k][j];
    }
}
// Columns n, n+1 (n even) of row m of a split-K output, summed over the slots [lo, hi) of their
// row group in slot order.
__device__ __forceinline__ float2 slot_pair_range(const PartView& v, int m, int n, int lo, int hi) {
    const float2* p = reinterpret_cast<const float2*>(slot_base(v, m, n >> 8) + (n & 255));
    float2 s = make_float2(0.f, 0.f);
    for (int s0 = lo; s0 < hi; s0 += 16) {
        float2 t[16];
#pragma unroll
        for (int k = 0; k < 16; ++k)
            if (s0 + k < hi) t[k] = __ldcg(p + (size_t)(s0 + k) * 2048);
#pragma unroll
        for (int k = 0; k < 16; ++k)
            if (s0 + k < hi) {
                s.x += t[k].x;
                s.y += t[k].y;
            }
    }
    return s;
}
// Column pairs (na, na+1) and (nb, nb+1) of row m, the slot loads of both in flight together
// (each pair still summed in its own slot order).
__device__ __forceinline__ void gemm_out_two_pairs(const GemmOut& o, int m, int na, int nb, float2& a, float2& b) {
    if (!o.part.part) {
        a = *reinterpret_cast<const float2*>(o.y + (size_t)m * o.ld + na);
        b = *reinterpret_cast<const float2*>(o.y + (size_t)m * o.ld + nb);
        return;
    }
    const float2* pa = reinterpret_cast<const float2*>(slot_base(o.part, m, na >> 8) + (na & 255));
    const float2* pb = reinterpret_cast<const float2*>(slot_base(o.part, m, nb >> 8) + (nb & 255));
    const int nsa = slot_count(o.part, na >> 8), nsb = slot_count(o.part, nb >> 8);
    a = b = make_float2(0.f, 0.f);
    for (int s0 = 0; s0 < max(nsa, nsb); s0 += 16) {
        float2 ta[16], tb[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            if (s0 + k < nsa) ta[k] = __ldcg(pa + (size_t)(s0 + k) * 2048);
            if (s0 + k < nsb) tb[k] = __ldcg(pb + (size_t)(s0 + k) * 2048);
        }
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            if (s0 + k < nsa) {
                a.x += ta[k].x;
                a.y += ta[k].y;
            }
            if (s0 + k < nsb) {
                b.x += tb[k].x;
                b.y += tb[k].y;
            }
        }
    }
}
// Columns n, n+1 (n even) of row m.
__device__ __forceinline__ float2 gemm_out_pair(const GemmOut& o, int m, int n) {
    if (!o.part.part) return *reinterpret_cast<const float2*>(o.y + (size_t)m * o.ld + n);
    return slot_pair_range(o.part, m, n, 0, slot_count(o.part, n >> 8));
}
#endif

struct QkvEpiArgs {
    GemmOut qkv;            // rows: [q: qh*hd][k: kvh*hd][v: kvh*hd if has_v]
    const StepParams* sp;
    int M, qh, kvh, hd, has_v, rotated;
    float theta;
    const uint16_t* q_norm;  // bf16 [hd]
    const uint16_t* k_norm;  // bf16 [hd]
    float* q_out;            // [M][qh][hd]
    uint16_t* k_ring;        // [cap][kvh][hd] FP16 (or bf16 when kv_bf16) bit patterns
    uint16_t* v_ring;
    int cap;
    int kv_bf16;             // 1: round K/V through bf16 instead of FP16 (long-context mode)
    int pos_offset;          // rotary position = base_pos + row + pos_offset
};

// Tensor-parallel sum of one step's dense partial outputs over peer memory (NVLink). Every rank
// writes its partial [M][ld] into its own buffer y[rank] and, once the consuming kernel starts
// (so the partial is complete), publishes epoch = seq * 256 + step + 1 in its flag word; each
// consumer waits (bounded) for every rank's flag and adds the ranks' partials in rank order,
// so all ranks compute identical sums. Two buffer/flag parities alternate between the o and the
// down projection, so a buffer is rewritten only after every rank has consumed it.
constexpr int kMaxTp = 8;
struct TpGather {
    const float* y[kMaxTp];        // each rank's partial buffer for this step (peer-mapped)
    const unsigned* flag[kMaxTp];  // each rank's flag word for this step's parity (peer-mapped)
    unsigned* own_flag;            // this rank's flag word
    const unsigned* seq;           // passes completed on this rank (advanced by head_finalize)
    int n, rank, step;             // ranks (1: no gather), this rank, step index within a pass
    int* err;                      // set to 3 if a peer's flag never arrived
    // Verify rows (M <= 16) whose GEMM left split-K slots: each norm-epilogue thread stores its
    // columns' sums, each value paired with the step's epoch in one 8-byte word, into every peer's
    // receive area; readers poll their own words until the epochs match (no fences or flags).
    uint2* push_dst[kMaxTp];       // rank r's receive words for data from this rank ([16][d], peer-mapped)
    const uint2* recv;             // this rank's receive words for the parity: [source rank][16][d]
};

struct AttnArgs {
    const float* q;          // [M][qh][hd]
    const uint16_t* k_ring;
    const uint16_t* v_ring;
    const StepParams* sp;
    int M, qh, kvh, hd, cap, window;  // window 0: full attention
    int kv_bf16;
    float scale;
};

// A TMA tensor map (CUtensorMap) of one layer's K or V ring, [cap][kvh][hd] bf16, read in boxes
// of 128 positions x 64 dims with 128-byte swizzle.
struct alignas(64) KvTmap {
    unsigned char bytes[128];
};

// Long-context attention (attn_lc.cu): one CTA per (key split, query-head group, KV head).
struct AttnLcParams {
    const float* q;          // [M][qh][512]
    const StepParams* sp;
    float* part;             // [kvh][G][S][N][512] unnormalised partial outputs
    float2* ml;              // [kvh][G][S][N] {max, sum} per row
    int* err;
    int M, qh, kvh;
    int G, S, N, hpg;        // head groups per KV head, key splits, rows per CTA (padded), heads per group
    int BM, mb;              // position blocks (prefill chunks) and positions per block
    float scale;
};

}  // namespace g4b
