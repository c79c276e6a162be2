// Per-unit integer dot products of ggml weight blocks against Q8_0
// activations (dp4a). A "unit" is 32 weight elements: one Q8_0 / Q4_0 block
// or one Q4_K sub-block. The same routines feed the decode GEMV and the
// block-sum probe used for bit-exact checking.
#pragma once

#include "common.cuh"

namespace fbk {

// Weight integers of one unit packed 4 per 32-bit word (dp4a operands) plus
// its float scale terms.
struct Unit {
    uint32_t q[8];
    float s0;  // Q8_0/Q4_0: d; Q4_K: d*sc
    float s1;  // Q4_K: dmin*m (unused otherwise)
};

template <int WT>
__device__ __forceinline__ int unit_stride_bytes();
template <>
__device__ __forceinline__ int unit_stride_bytes<WT_Q8_0>() { return Q8_0_BYTES; }
template <>
__device__ __forceinline__ int unit_stride_bytes<WT_Q4_0>() { return Q4_0_BYTES; }

// `row` points at the first byte of a weight row (2-byte aligned); u is the
// unit index within the row.
template <int WT>
__device__ __forceinline__ void load_unit(const uint8_t *row, int u, Unit &U) {
    if constexpr (WT == WT_Q8_0) {
        const uint8_t *blk = row + Q8_0_BYTES * u;
        U.s0 = f16_bits_to_f32(ld_u16(blk));
        U.s1 = 0.0f;
        ld_words_a2<8>(blk + 2, U.q);
    } else if constexpr (WT == WT_Q4_0) {
        const uint8_t *blk = row + Q4_0_BYTES * u;
        U.s0 = f16_bits_to_f32(ld_u16(blk));
        U.s1 = 0.0f;
        uint32_t w[4];
        ld_words_a2<4>(blk + 2, w);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            U.q[i] = w[i] & 0x0f0f0f0fu;            // elements 4i..4i+3 (low nibbles)
            U.q[4 + i] = (w[i] >> 4) & 0x0f0f0f0fu;  // elements 16+4i.. (high nibbles)
        }
    } else {  // Q4_K: sub-block j of super-block u/8
        const int j = u & 7;
        const uint8_t *sb = row + Q4_K_BYTES * (u >> 3);
        const float d = f16_bits_to_f32(ld_u16(sb));
        const float dmin = f16_bits_to_f32(ld_u16(sb + 2));
        int sc, m;
        q4k_scale_min(j, sb + 4, sc, m);
        U.s0 = d * (float)sc;
        U.s1 = dmin * (float)m;
        uint32_t w[8];
        ld_words_a2<8>(sb + 16 + 32 * (j >> 1), w);
        const uint32_t sh = 4u * (uint32_t)(j & 1);
#pragma unroll
        for (int i = 0; i < 8; i++) U.q[i] = (w[i] >> sh) & 0x0f0f0f0fu;
    }
}

// Integer block sum: Q8_0 sum q_w*q_x; Q4_0 sum (nibble-8)*q_x; Q4_K sum nibble*q_x.
template <int WT>
__device__ __forceinline__ int unit_sumi(const Unit &U, const int4 x0, const int4 x1, int xsum) {
    int s = 0;
    s = __dp4a((int)U.q[0], x0.x, s);
    s = __dp4a((int)U.q[1], x0.y, s);
    s = __dp4a((int)U.q[2], x0.z, s);
    s = __dp4a((int)U.q[3], x0.w, s);
    s = __dp4a((int)U.q[4], x1.x, s);
    s = __dp4a((int)U.q[5], x1.y, s);
    s = __dp4a((int)U.q[6], x1.z, s);
    s = __dp4a((int)U.q[7], x1.w, s);
    if constexpr (WT == WT_Q4_0) s -= 8 * xsum;
    return s;
}

// Contribution of one unit to y: Q8_0/Q4_0 d_w*d_x*sumi;
// Q4_K d_x*(d*sc*sumi - dmin*m*xsum).
template <int WT>
__device__ __forceinline__ float unit_scale(const Unit &U, int sumi, float dx, int xsum) {
    if constexpr (WT == WT_Q4_K)
        return dx * (U.s0 * (float)sumi - U.s1 * (float)xsum);
    else
        return (U.s0 * dx) * (float)sumi;
}

}  // namespace fbk
