// qdot.cuh — the q8_0 dot product on the CUDA cores, shared by the matvec and the attention's fused o-projection:
// packed f32x2 arithmetic, 16 int8 quants · 16 f32 activations, and the lane-blocked activation layout in shared
// memory that lets a warp's 16-byte weight reads and its activation reads both run without bank conflicts.
#pragma once

#include "common.cuh"

namespace ocr {

// ---- packed f32x2 arithmetic (sm_100): two lanes of f32 per instruction ------------------------------------------
__device__ __forceinline__ uint64_t pk2(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ float2 upk2(uint64_t v) {
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
    return r;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// 16 int8 quants (one 16-B load) · 16 activations (8 f32 pairs): each byte, biased to q + 128, is placed in the
// mantissa of 2^23 by one byte permute and 2^23 + 128 is subtracted pairwise (exact: integers below 2^24); the pairs
// then multiply-accumulate packed, two accumulators deep. Returns the f32 dot.
__device__ __forceinline__ float dot16x2(const uint4 w, const uint64_t* xp) {
    const uint64_t bias = pk2(-8388736.0f, -8388736.0f);
    const uint32_t wv[4] = {w.x ^ 0x80808080u, w.y ^ 0x80808080u, w.z ^ 0x80808080u, w.w ^ 0x80808080u};
    uint64_t a0 = 0, a1 = 0;  // +0.0f pairs
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const uint32_t u = wv[k];
        const uint64_t p01 = add2(pk2(__int_as_float(__byte_perm(u, 0x4B000000u, 0x7440)),
                                      __int_as_float(__byte_perm(u, 0x4B000000u, 0x7441))), bias);
        const uint64_t p23 = add2(pk2(__int_as_float(__byte_perm(u, 0x4B000000u, 0x7442)),
                                      __int_as_float(__byte_perm(u, 0x4B000000u, 0x7443))), bias);
        a0 = fma2(p01, xp[2 * k], a0);
        a1 = fma2(p23, xp[2 * k + 1], a1);
    }
    const float2 s = upk2(add2(a0, a1));
    return s.x + s.y;
}

// the smem float index of x[s][c] in the lane-blocked layout
__device__ __forceinline__ int xs_index(int s, int nch, int c) {
    const int i = c >> 9, w = c & 511, l = w >> 4, j = w & 15;
    return ((((s * nch + i) * 4 + (j >> 2)) * 32 + l) << 2) + (j & 3);
}

// this lane's share of row · x over the row's 16-column pieces l8, l8 + 8, … (8 lanes per row, so a quarter-warp
// reads 128 contiguous bytes of one row): `row` in the row layout (ncol quants, then the f16 block scales), x staged
// lane-blocked as f32 pairs (`ap`)
__device__ __forceinline__ float row_dot8(const uint8_t* row, int ncol, const uint64_t* ap, int l8) {
    float acc = 0.0f;
    for (int pc = l8; pc < ncol / 16; pc += 8) {
        const uint4 wq = *reinterpret_cast<const uint4*>(row + pc * 16);
        const float dsc = __half2float(reinterpret_cast<const __half*>(row + ncol)[pc >> 1]);
        uint64_t xp[8];
        const int xb = ((pc >> 5) * 128 + (pc & 31)) * 2;  // in f32 pairs
#pragma unroll
        for (int jj = 0; jj < 4; jj++) {
            xp[2 * jj] = ap[xb + jj * 64];
            xp[2 * jj + 1] = ap[xb + jj * 64 + 1];
        }
        acc = fmaf(dot16x2(wq, xp), dsc, acc);
    }
    return acc;
}

// row_dot8 for a row of exactly 128·NPC columns: the lane's NPC pieces unrolled, no trip count
template <int NPC>
__device__ __forceinline__ float row_dot8c(const uint8_t* row, const uint64_t* ap, int l8) {
    constexpr int ncol = NPC * 128;
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < NPC; i++) {
        const int pc = l8 + 8 * i;
        const uint4 wq = *reinterpret_cast<const uint4*>(row + pc * 16);
        const float dsc = __half2float(reinterpret_cast<const __half*>(row + ncol)[pc >> 1]);
        uint64_t xp[8];
        const int xb = ((pc >> 5) * 128 + (pc & 31)) * 2;  // in f32 pairs
#pragma unroll
        for (int jj = 0; jj < 4; jj++) {
            xp[2 * jj] = ap[xb + jj * 64];
            xp[2 * jj + 1] = ap[xb + jj * 64 + 1];
        }
        acc = fmaf(dot16x2(wq, xp), dsc, acc);
    }
    return acc;
}

}  // namespace ocr
