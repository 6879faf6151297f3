// Producer side of the activation layouts (see common.cuh). Every kernel that feeds a GEMM
// (input norm, post-attention norm, GeGLU, attention output, final norm) ends by calling
// bfrag_store_group (verify rows) or wide_store_group (prefill rows), so activations are
// converted once and the GEMM streams ready-made tensor-core operands.
#pragma once
#include "common.cuh"

namespace g4b {

// Wide layout (prefill rows): one (row m, 64-group gi) held by a warp, lane l owning columns
// 2l and 2l+1, scaled by the row's 1/E (wide_row_scale), split into hi/lo fp16 tiles, plus the
// group's Y record. Lane l's columns sit in 16-byte chunk l/4 of row m, stored at chunk
// position (l/4) ^ (m % 8) of the row's 128 bytes. The caller writes erow[m] = E once. All 32
// lanes must call it.
__device__ __forceinline__ void wide_store_group(const BFragView& v, int m, int gi, float x0, float x1,
                                                 float inv_e) {
    const int lane = threadIdx.x & 31;
    const float s0 = x0 * inv_e, s1 = x1 * inv_e;
    const __half h0 = __float2half_rn(s0), h1 = __float2half_rn(s1);
    const __half l0 = __float2half_rn(s0 - __half2float(h0));
    const __half l1 = __float2half_rn(s1 - __half2float(h1));
    const float y = warp_sum((__half2float(h0) + __half2float(l0)) + (__half2float(h1) + __half2float(l1)));
    auto pk = [](__half a, __half b) { return (uint32_t)__half_as_ushort(a) | ((uint32_t)__half_as_ushort(b) << 16); };
    char* hi = reinterpret_cast<char*>(v.frag) + (size_t)gi * kWideTileBytes;
    const uint32_t off = (uint32_t)m * 128 + ((((uint32_t)lane >> 2) ^ ((uint32_t)m & 7)) << 4) + (lane & 3) * 4;
    *reinterpret_cast<uint32_t*>(hi + off) = pk(h0, h1);
    *reinterpret_cast<uint32_t*>(hi + v.lo_off + off) = pk(l0, l1);
    if (lane == 0) v.ysum[(size_t)gi * kPrefillRows + m] = y * 5.9604644775390625e-08f;  // 2^-24
}

// Digit modes (M = 5..16): the (row m, group gi) held by a warp as three 8-bit digit planes.
// Lane l's values sit at k = 2l and 2l+1 of the group: k32 step l/16, fragment thread
// t = (l%16)/4, byte i = l%4, register b0 (even k) or b1 (odd k). Bytes meet in `stage`
// (192 bytes), then 24 lanes write one uint2 each.
__device__ __forceinline__ void digits_store_group(const BFragView& v, int M, int m, int gi, float x0, float x1,
                                                   __half* stage) {
    const int lane = threadIdx.x & 31;
    const int nt_count = bmode_for(M).nt;
    const float amax = warp_max(fmaxf(fabsf(x0), fabsf(x1)));
    int e = 0;
    frexpf(amax, &e);  // |x| < 2^e
    const float inv = ldexpf(1.0f, 22 - e);
    const int v0 = __float2int_rn(x0 * inv), v1 = __float2int_rn(x1 * inv);  // |v| < 2^22
    unsigned char* st = reinterpret_cast<unsigned char*>(stage);
    // byte index: ((d * 2 + kk_sub) * 2 + par) * 16 + t * 4 + i
    const int kk_sub = lane >> 4, t = (lane >> 2) & 3, i = lane & 3;
    int r0 = v0, r1 = v1;
#pragma unroll
    for (int d = 0; d < 3; ++d) {
        const int d0 = (int)(signed char)(r0 & 0xFF), d1 = (int)(signed char)(r1 & 0xFF);
        st[((d * 2 + kk_sub) * 2 + 0) * 16 + t * 4 + i] = (unsigned char)d0;
        st[((d * 2 + kk_sub) * 2 + 1) * 16 + t * 4 + i] = (unsigned char)d1;
        r0 = (r0 - d0) >> 8;
        r1 = (r1 - d1) >> 8;
    }
    const int ysum = warp_sum_int(v0 + v1);
    __syncwarp();
    if (lane < 24) {
        const int d = lane >> 3, ks = (lane >> 2) & 1, tt = lane & 3;
        const uint32_t* w = reinterpret_cast<const uint32_t*>(st);
        const uint2 val = make_uint2(w[((d * 2 + ks) * 2 + 0) * 4 + tt], w[((d * 2 + ks) * 2 + 1) * 4 + tt]);
        int nt, col;
        digit_col(nt_count, m, d, nt, col);
        const int kk = 2 * (gi & 1) + ks;  // k32 step within the 128-wide k-tile
        uint2* frag = reinterpret_cast<uint2*>(v.frag);
        frag[(((size_t)(gi >> 1) * 4 + kk) * nt_count + nt) * 32 + col * 4 + tt] = val;
    } else if (lane == 24) {
        v.gsum[(size_t)gi * kMaxM + m] = make_float2(ldexpf(1.0f, e - 22), (float)ysum);
    }
    __syncwarp();
}

// Converts one (row m, 64-group gi) held by a warp -- lane l owns columns 2l and 2l+1 of
// the group -- into B operands of an M <= 16-row batch (fp16 fragments for M <= 4, integer
// digits above) and the group's {E, Y} record. `stage` is 128 halves of per-warp shared
// scratch. All 32 lanes must call it.
__device__ __forceinline__ void bfrag_store_group(const BFragView& v, int M, int m, int gi,
                                                  float x0, float x1, __half* stage) {
    const int lane = threadIdx.x & 31;
    const BMode md = bmode_for(M);
    if (md.nt) {
        digits_store_group(v, M, m, gi, x0, x1, stage);
        return;
    }
    const float amax = warp_max(fmaxf(fabsf(x0), fabsf(x1)));
    int e = 0;
    frexpf(amax, &e);  // amax = f * 2^e, f in [0.5, 1)
    const float E = ldexpf(1.0f, e - 11);
    const float invE = ldexpf(1.0f, 11 - e);
    const float s0 = x0 * invE, s1 = x1 * invE;
    const __half h0 = __float2half_rn(s0), h1 = __float2half_rn(s1);
    const __half l0 = __float2half_rn(s0 - __half2float(h0));
    const __half l1 = __float2half_rn(s1 - __half2float(h1));
    const float y = warp_sum((__half2float(h0) + __half2float(l0)) + (__half2float(h1) + __half2float(l1)));
    stage[2 * lane] = h0;
    stage[2 * lane + 1] = h1;
    stage[64 + 2 * lane] = l0;
    stage[64 + 2 * lane + 1] = l1;
    __syncwarp();
    if (lane < 16) {
        const int kb = lane >> 3, part = (lane >> 2) & 1, t = lane & 3;
        const __half* src = stage + part * 64 + kb * 32 + 8 * t;
        int tile, n;
        if (md.packed) { tile = 0; n = m + 4 * part; }
        else if (md.nb == 2) { tile = part; n = m; }
        else { tile = 2 * (m >> 3) + part; n = m & 7; }
        const __half sixteenth = __float2half(0.0625f);
        auto pk = [](__half a, __half b) {
            return (uint32_t)__half_as_ushort(a) | ((uint32_t)__half_as_ushort(b) << 16);
        };
        uint4 o;
        o.x = pk(src[0], src[4]);
        o.y = pk(__hmul(src[1], sixteenth), __hmul(src[5], sixteenth));
        o.z = pk(src[2], src[6]);
        o.w = pk(__hmul(src[3], sixteenth), __hmul(src[7], sixteenth));
        v.frag[((size_t)(gi * 2 + kb) * md.nb + tile) * 32 + n * 4 + t] = o;
    } else if (lane == 16) {
        const float Y = y * 5.9604644775390625e-08f;  // 2^-24
        if (md.packed) {
            v.gsum[(size_t)gi * 8 + m] = make_float2(E, Y);
            v.gsum[(size_t)gi * 8 + m + 4] = make_float2(E, 0.0f);
        } else {
            v.gsum[((size_t)gi * md.nacc + (m >> 3)) * 8 + (m & 7)] = make_float2(E, Y);
        }
    }
    __syncwarp();
}

}  // namespace g4b
