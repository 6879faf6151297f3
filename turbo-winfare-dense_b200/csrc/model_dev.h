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
    int nsplit;
    float* o_part;           // [nsplit][M*qh][hd] unnormalised
    float2* ml_part;         // [nsplit][M*qh] {running max, running sum}
};

}  // namespace g4b
