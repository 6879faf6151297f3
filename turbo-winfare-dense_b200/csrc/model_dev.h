// Device-side descriptors shared by the forward-pass kernels and their host launchers.
#pragma once
#include <cuda_fp16.h>
#include <cstdint>

#include "vgemm.h"

namespace g4b {

// Per-pass inputs that change between graph replays: the position of the batch's first row
// and its token ids. Kernels read them from device memory so one captured graph serves every
// position.
struct StepParams {
    int base_pos;
    int draft_step;  // drafter chaining: index of the next draft written to the chain list
    uint32_t tokens[16];
};

// A GEMM output as its consumers see it: split-K slots (part.part != nullptr) or a plain
// fp32 [M][ld] matrix (after a tensor-parallel all-reduce).
struct GemmOut {
    PartView part;
    const float* y;
    int ld;
};

#ifdef __CUDACC__
__device__ __forceinline__ float gemm_out_get(const GemmOut& o, int m, int n) {
    return o.part.part ? vgemm_part_get(o.part, m, n) : o.y[(size_t)m * o.ld + n];
}
// Columns n and n+1 (n even): one slot lookup, 8-byte loads, loads batched across slots.
__device__ __forceinline__ float2 gemm_out_pair(const GemmOut& o, int m, int n) {
    if (!o.part.part) return *reinterpret_cast<const float2*>(o.y + (size_t)m * o.ld + n);
    const SlotRow r = vgemm_slot_row(o.part, m, n >> 8);
    const float2* p = reinterpret_cast<const float2*>(r.p + (n & 255));
    float2 s = make_float2(0.f, 0.f);
    int i = 0;
    for (; i + 8 <= r.ns; i += 8) {
        float2 t[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) t[j] = __ldcg(p + (size_t)(i + j) * 2048);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            s.x += t[j].x;
            s.y += t[j].y;
        }
    }
    for (; i < r.ns; ++i) {
        const float2 t = __ldcg(p + (size_t)i * 2048);
        s.x += t.x;
        s.y += t.y;
    }
    return s;
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

}  // namespace g4b
