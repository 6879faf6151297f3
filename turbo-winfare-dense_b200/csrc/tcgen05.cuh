// Thin inline-PTX wrappers for the sm_100a 5th-generation tensor core (tcgen05): tensor-memory
// allocation, the MMA with its accumulator in tensor memory (TMEM), completion tracking through
// mbarriers, and TMEM <-> register moves. Only the forms the prefill GEMM and the long-context
// attention use are wrapped: cta_group::1, kind::f16 (fp16 or bf16 inputs, fp32 accumulate), B
// from shared memory, A from shared (K- or MN-major) or tensor memory.
//
// TMEM addresses are (lane << 16) | column. A warp may only touch the 32 lanes of its
// quadrant, lanes 32 * (warp % 4) .. +31.
#pragma once
#include <cstdint>

#include "tma.cuh"

namespace g4b {
namespace tc {

// Allocates `ncols` TMEM columns (a power of two >= 32) for this CTA; the base address is
// written to shared memory at `slot`. Warp-collective.
__device__ __forceinline__ void alloc(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

// Frees what alloc() took. Warp-collective, by the warp that allocated.
__device__ __forceinline__ void dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void fence_before_sync() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[tmem] * B[smem desc]^T, issued by one thread. `accumulate` = 0 overwrites D.
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, issued by one thread.
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrives once on `bar` when every tcgen05 operation this thread issued before has completed.
__device__ __forceinline__ void commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 16 consecutive 32-bit columns of this thread's lane. Warp-collective; follow with wait_ld().
__device__ __forceinline__ void ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
// 8 consecutive 32-bit columns of this thread's lane. Warp-collective; follow with wait_ld().
__device__ __forceinline__ void ld8(uint32_t taddr, float (&v)[8]) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr)
                 : "memory");
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 consecutive 32-bit columns of this thread's lane. Warp-collective; follow with wait_st().
__device__ __forceinline__ void st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
        "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
        "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
// 16 consecutive 32-bit columns of this thread's lane. Warp-collective; follow with wait_st().
__device__ __forceinline__ void st16(uint32_t taddr, const float (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
        "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
        "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
        "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
        "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
        : "memory");
}
__device__ __forceinline__ void wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor of a K-major operand tile in the canonical 128-byte-swizzled
// layout: rows of 64 fp16 (128 B) stored consecutively, 16-byte chunk c of row r at chunk
// position c ^ (r % 8), 8-row atoms 1024 B apart. `addr` is the shared-memory byte address of
// the first row, advanced by 32 B per 16-wide K slice; the tile itself is 1024-byte aligned.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t addr) {
    return (uint64_t)((addr & 0x3FFFFu) >> 4)  // start address, 16-byte units
           | ((uint64_t)1 << 16)               // leading byte offset (unused for swizzled K-major)
           | ((uint64_t)(1024 >> 4) << 32)     // stride byte offset: 8-row atom pitch
           | ((uint64_t)1 << 46)               // descriptor version for sm_100
           | ((uint64_t)2 << 61);              // 128-byte swizzle
}

// Shared-memory matrix descriptor of an MN-major operand tile in the 128-byte-swizzled layout:
// each 128-byte row holds 64 consecutive M (or N) elements of one K index, rows of consecutive K
// are 128 B apart (swizzled as above), the next 8 K rows `sbo` bytes on and the next 64 M
// elements `lbo` bytes on. `addr` is the first row's address (1024-byte aligned atom).
__device__ __forceinline__ uint64_t desc_sw128_mn(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr & 0x3FFFFu) >> 4)  // start address, 16-byte units
           | ((uint64_t)(lbo >> 4) << 16)       // leading byte offset: next 64 M elements
           | ((uint64_t)(sbo >> 4) << 32)       // stride byte offset: next 8 K rows
           | ((uint64_t)1 << 46)               // descriptor version for sm_100
           | ((uint64_t)2 << 61);              // 128-byte swizzle
}

// Instruction descriptor for kind::f16 with bf16 A and B, fp32 D, M x N; a_mn: A is MN-major.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, bool a_mn) {
    return (1u << 4)                        // D format: f32
           | (1u << 7) | (1u << 10)         // A, B format: bf16
           | ((a_mn ? 1u : 0u) << 15)       // A major-ness (0: K-major)
           | ((uint32_t)(N >> 3) << 17)     // N / 8
           | ((uint32_t)(M >> 4) << 24);    // M / 16
}

// Instruction descriptor for kind::f16: fp16 A and B (both K-major), fp32 D, M x N.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
    return (1u << 4)                        // D format: f32
           | (0u << 7) | (0u << 10)         // A, B format: f16
           | ((uint32_t)(N >> 3) << 17)     // N / 8
           | ((uint32_t)(M >> 4) << 24);    // M / 16
}

}  // namespace tc
}  // namespace g4b
