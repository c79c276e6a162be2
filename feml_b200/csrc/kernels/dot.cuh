// Integer dot products of ggml weight blocks against Q8_0 activations
// (dp4a), shared by the decode GEMV and the block-sum probe used for
// bit-exact checking.
//
// Work is done in 64-element pairs so that every shared-memory load is
// aligned:
//  - Q8_0 / Q4_0: two consecutive 32-element blocks (68 / 36 bytes, 4-byte
//    aligned when the row is). The odd block's integers are word aligned; the
//    even block's start 2 bytes into a word, so they are multiplied against a
//    copy of the activations shifted by 2 bytes with zeros at both ends (the
//    zero lanes cancel the f16 scale bytes that share those words).
//  - Q4_K: the two sub-blocks 2g, 2g+1 of a super-block, which share 32
//    nibble bytes (low nibbles: sub-block 2g, high: 2g+1). High nibbles are
//    used in place, as 16*h bytes in an unsigned x signed dp4a, and the sum is
//    divided by 16 (exact: every term is a multiple of 16).
#pragma once

#include "common.cuh"

namespace fbk {

__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
    return __dp4a((int)a, (int)b, c);
}
// unsigned bytes of a times signed bytes of b
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Shifted activation words of one even block, as the pair kernels read them
// (12 words, 16-byte aligned):
//   Q8_0: words 0..8  = bytes [0, 0, x0 .. x31, 0, 0]
//   Q4_0: words 0..4  = bytes [0, 0, x0 .. x15, 0, 0]
//         words 5..9  = bytes [0, 0, x16 .. x31, 0, 0]
constexpr int kShiftWords = 12;

// Builds the shifted words from the block's 8 packed activation words.
template <int WT>
__device__ __forceinline__ void make_shifted(const uint32_t (&w)[8], uint32_t (&s)[kShiftWords]) {
#pragma unroll
    for (int i = 0; i < kShiftWords; i++) s[i] = 0;
    if constexpr (WT == WT_Q8_0) {
#pragma unroll
        for (int k = 0; k <= 8; k++) s[k] = __funnelshift_r(k > 0 ? w[k - 1] : 0u, k < 8 ? w[k] : 0u, 16);
    } else {
#pragma unroll
        for (int k = 0; k <= 4; k++) {
            s[k] = __funnelshift_r(k > 0 ? w[k - 1] : 0u, k < 4 ? w[k] : 0u, 16);
            s[5 + k] = __funnelshift_r(k > 0 ? w[3 + k] : 0u, k < 4 ? w[4 + k] : 0u, 16);
        }
    }
}

// The activation words one block pair of Q8_0 / Q4_0 weights is dotted with:
// the even block's shifted words (e0, e1, e2: words 0..9; Q8_0 uses 0..8) and
// the odd block's 8 packed words (o0, o1). Held in registers by callers that
// reuse one pair's activations across many weight rows.
struct XFrag {
    uint4 e0, e1;
    uint2 e2;
    uint4 o0, o1;
};

// `xe` the even block's shifted words (16-byte aligned), `xo` the odd block's
// 8 words (16-byte aligned).
__device__ __forceinline__ XFrag load_xfrag(const uint32_t *xe, const uint32_t *xo) {
    XFrag f;
    f.e0 = *reinterpret_cast<const uint4 *>(xe);
    f.e1 = *reinterpret_cast<const uint4 *>(xe + 4);
    f.e2 = *reinterpret_cast<const uint2 *>(xe + 8);
    f.o0 = *reinterpret_cast<const uint4 *>(xo);
    f.o1 = *reinterpret_cast<const uint4 *>(xo + 4);
    return f;
}

// Block-pair integer sums. `wp` is the pair's first byte (4-byte aligned);
// `x` the pair's activation words; xsum_* the activation block sums (Q4_0
// offset). Returns sums s0 (even block), s1 (odd block) and the blocks' f16
// scales as f32.
template <int WT>
__device__ __forceinline__ void pair_dot_frag(const uint32_t *wp, const XFrag &x, int xsum0, int xsum1, int &s0,
                                              int &s1, float &d0, float &d1) {
    if constexpr (WT == WT_Q8_0) {
        uint32_t w[17];
#pragma unroll
        for (int i = 0; i < 17; i++) w[i] = wp[i];
        // four independent chains (even lo/hi, odd lo/hi) for ILP
        int a0 = 0, a1 = 0, b0 = 0, b1 = 0;
        a0 = dp4a_ss(w[0], x.e0.x, a0);
        a1 = dp4a_ss(w[1], x.e0.y, a1);
        b0 = dp4a_ss(w[9], x.o0.x, b0);
        b1 = dp4a_ss(w[10], x.o0.y, b1);
        a0 = dp4a_ss(w[2], x.e0.z, a0);
        a1 = dp4a_ss(w[3], x.e0.w, a1);
        b0 = dp4a_ss(w[11], x.o0.z, b0);
        b1 = dp4a_ss(w[12], x.o0.w, b1);
        a0 = dp4a_ss(w[4], x.e1.x, a0);
        a1 = dp4a_ss(w[5], x.e1.y, a1);
        b0 = dp4a_ss(w[13], x.o1.x, b0);
        b1 = dp4a_ss(w[14], x.o1.y, b1);
        a0 = dp4a_ss(w[6], x.e1.z, a0);
        a1 = dp4a_ss(w[7], x.e1.w, a1);
        b0 = dp4a_ss(w[15], x.o1.z, b0);
        b1 = dp4a_ss(w[16], x.o1.w, b1);
        a0 = dp4a_ss(w[8], x.e2.x, a0);
        s0 = a0 + a1;
        s1 = b0 + b1;
        d0 = f16_bits_to_f32((uint16_t)(w[0] & 0xffffu));
        d1 = f16_bits_to_f32((uint16_t)(w[8] >> 16));
    } else {  // Q4_0: 36 bytes
        uint32_t w[9];
#pragma unroll
        for (int i = 0; i < 9; i++) w[i] = wp[i];
        const uint32_t lo = 0x0f0f0f0fu, hi = 0xf0f0f0f0u;
        // even block: low nibbles vs shifted x0..15 (words 0..4), high vs x16..31 (words 5..9)
        int el = 0, eh = 0;
        el = dp4a_ss(w[0] & lo, x.e0.x, el);
        el = dp4a_ss(w[1] & lo, x.e0.y, el);
        el = dp4a_ss(w[2] & lo, x.e0.z, el);
        el = dp4a_ss(w[3] & lo, x.e0.w, el);
        el = dp4a_ss(w[4] & lo, x.e1.x, el);
        eh = dp4a_us(w[0] & hi, x.e1.y, eh);
        eh = dp4a_us(w[1] & hi, x.e1.z, eh);
        eh = dp4a_us(w[2] & hi, x.e1.w, eh);
        eh = dp4a_us(w[3] & hi, x.e2.x, eh);
        eh = dp4a_us(w[4] & hi, x.e2.y, eh);
        // odd block: words 5..8
        int ol = 0, oh = 0;
        ol = dp4a_ss(w[5] & lo, x.o0.x, ol);
        ol = dp4a_ss(w[6] & lo, x.o0.y, ol);
        ol = dp4a_ss(w[7] & lo, x.o0.z, ol);
        ol = dp4a_ss(w[8] & lo, x.o0.w, ol);
        oh = dp4a_us(w[5] & hi, x.o1.x, oh);
        oh = dp4a_us(w[6] & hi, x.o1.y, oh);
        oh = dp4a_us(w[7] & hi, x.o1.z, oh);
        oh = dp4a_us(w[8] & hi, x.o1.w, oh);
        s0 = el + (eh >> 4) - 8 * xsum0;
        s1 = ol + (oh >> 4) - 8 * xsum1;
        d0 = f16_bits_to_f32((uint16_t)(w[0] & 0xffffu));
        d1 = f16_bits_to_f32((uint16_t)(w[4] >> 16));
    }
}

// pair_dot_frag with the activation words read from shared memory.
template <int WT>
__device__ __forceinline__ void pair_dot(const uint32_t *wp, const uint32_t *xe, const uint32_t *xo, int xsum0,
                                         int xsum1, int &s0, int &s1, float &d0, float &d1) {
    pair_dot_frag<WT>(wp, load_xfrag(xe, xo), xsum0, xsum1, s0, s1, d0, d1);
}

// One even block with no odd partner (odd block count): Q8_0 / Q4_0 sums
// against the shifted activations (the bytes after the block meet the zero
// padding).
template <int WT>
__device__ __forceinline__ int single_even_dot(const uint32_t *wp, const uint32_t *xe, int xsum, float &d) {
    int s = 0;
    if constexpr (WT == WT_Q8_0) {
#pragma unroll
        for (int i = 0; i < 9; i++) s = dp4a_ss(wp[i], xe[i], s);
    } else {
        int l = 0, h = 0;
#pragma unroll
        for (int i = 0; i < 5; i++) {
            l = dp4a_ss(wp[i] & 0x0f0f0f0fu, xe[i], l);
            h = dp4a_us(wp[i] & 0xf0f0f0f0u, xe[5 + i], h);
        }
        s = l + (h >> 4) - 8 * xsum;
    }
    d = f16_bits_to_f32((uint16_t)(wp[0] & 0xffffu));
    return s;
}

// One Q4_K sub-block pair g (0..3) of a super-block, weight side: the 32
// nibble bytes the two sub-blocks share and their scale terms d*sc, dmin*m.
struct Q4kPair {
    uint4 q0, q1;
    float dsc0, dmm0, dsc1, dmm1;
};

// Integer sums of a pair against activation words a0, a1 (sub-block 2g, 32
// int8) and b0, b1 (sub-block 2g+1): s0 from the low nibbles, s1 from the
// high ones.
__device__ __forceinline__ void q4k_pair_sums(const uint4 q0, const uint4 q1, const uint4 a0, const uint4 a1,
                                              const uint4 b0, const uint4 b1, int &s0, int &s1) {
    const uint32_t lo = 0x0f0f0f0fu, hi = 0xf0f0f0f0u;
    int l0 = 0, l1 = 0, u0 = 0, u1 = 0;  // independent chains for ILP
    l0 = dp4a_ss(q0.x & lo, a0.x, l0);
    l1 = dp4a_ss(q0.y & lo, a0.y, l1);
    u0 = dp4a_us(q0.x & hi, b0.x, u0);
    u1 = dp4a_us(q0.y & hi, b0.y, u1);
    l0 = dp4a_ss(q0.z & lo, a0.z, l0);
    l1 = dp4a_ss(q0.w & lo, a0.w, l1);
    u0 = dp4a_us(q0.z & hi, b0.z, u0);
    u1 = dp4a_us(q0.w & hi, b0.w, u1);
    l0 = dp4a_ss(q1.x & lo, a1.x, l0);
    l1 = dp4a_ss(q1.y & lo, a1.y, l1);
    u0 = dp4a_us(q1.x & hi, b1.x, u0);
    u1 = dp4a_us(q1.y & hi, b1.y, u1);
    l0 = dp4a_ss(q1.z & lo, a1.z, l0);
    l1 = dp4a_ss(q1.w & lo, a1.w, l1);
    u0 = dp4a_us(q1.z & hi, b1.z, u0);
    u1 = dp4a_us(q1.w & hi, b1.w, u1);
    const int l = l0 + l1, u = u0 + u1;
    s0 = l;
    s1 = u >> 4;
}

// Scale terms of sub-blocks 2g, 2g+1 from the super-block's first 16 bytes
// `h` (f16 d, f16 dmin, 12 bytes of packed 6-bit scales and mins).
__device__ __forceinline__ void q4k_pair_scales(const uint4 h, int g, float &dsc0, float &dmm0, float &dsc1,
                                                float &dmm1) {
    // 6-bit (scale, min) pairs j0 = 2g, j1 = 2g+1 (public ggml get_scale_min_k4
    // layout) from scale bytes 0..11 = words h.y, h.z, h.w
    auto byte = [&](int j) -> int {
        const uint32_t w = (j >> 2) == 0 ? h.y : ((j >> 2) == 1 ? h.z : h.w);
        return (int)((w >> (8 * (j & 3))) & 0xffu);
    };
    int sc0, m0, sc1, m1;
    const int j0 = 2 * g, j1 = 2 * g + 1;
    if (g < 2) {
        sc0 = byte(j0) & 63;
        m0 = byte(j0 + 4) & 63;
        sc1 = byte(j1) & 63;
        m1 = byte(j1 + 4) & 63;
    } else {
        sc0 = (byte(j0 + 4) & 0x0f) | ((byte(j0 - 4) >> 6) << 4);
        m0 = (byte(j0 + 4) >> 4) | ((byte(j0) >> 6) << 4);
        sc1 = (byte(j1 + 4) & 0x0f) | ((byte(j1 - 4) >> 6) << 4);
        m1 = (byte(j1 + 4) >> 4) | ((byte(j1) >> 6) << 4);
    }
    const float d = f16_bits_to_f32((uint16_t)(h.x & 0xffffu));
    const float dmin = f16_bits_to_f32((uint16_t)(h.x >> 16));
    dsc0 = d * (float)sc0;
    dmm0 = dmin * (float)m0;
    dsc1 = d * (float)sc1;
    dmm1 = dmin * (float)m1;
}

// The weight side of pair g of the super-block at `sb` (16-byte aligned).
__device__ __forceinline__ Q4kPair q4k_pair_load(const uint8_t *sb, int g) {
    Q4kPair w;
    const uint4 h = *reinterpret_cast<const uint4 *>(sb);
    w.q0 = *reinterpret_cast<const uint4 *>(sb + 16 + 32 * g);
    w.q1 = *reinterpret_cast<const uint4 *>(sb + 32 + 32 * g);
    q4k_pair_scales(h, g, w.dsc0, w.dmm0, w.dsc1, w.dmm1);
    return w;
}

// Q4_K sub-block pair g (0..3) of the super-block at `sb` (16-byte aligned):
// integer sums s0 (sub-block 2g, low nibbles), s1 (sub-block 2g+1, high
// nibbles) and the scale terms d*sc, dmin*m of both.
// Activation words by value: a0, a1 = sub-block 2g (32 int8), b0, b1 =
// sub-block 2g+1.
__device__ __forceinline__ void q4k_pair_dot_x(const uint8_t *sb, int g, const uint4 a0, const uint4 a1,
                                               const uint4 b0, const uint4 b1, int &s0, int &s1, float &dsc0,
                                               float &dmm0, float &dsc1, float &dmm1) {
    const Q4kPair w = q4k_pair_load(sb, g);
    q4k_pair_sums(w.q0, w.q1, a0, a1, b0, b1, s0, s1);
    dsc0 = w.dsc0;
    dmm0 = w.dmm0;
    dsc1 = w.dsc1;
    dmm1 = w.dmm1;
}

// Q5_K sub-block pair g of the super-block at `sb` (16-byte aligned; d, dmin
// and the 12 scale bytes as in Q4_K, then qh[32], then the nibbles): value
// = nibble + 16 * fifth bit, the fifth bit of element l of sub-block j being
// bit j of qh[l]. Integer sums s0 (sub-block 2g), s1 (2g+1) and scale terms.
__device__ __forceinline__ void q5k_pair_dot(const uint8_t *sb, int g, const uint32_t *xa, const uint32_t *xb,
                                             int &s0, int &s1, float &dsc0, float &dmm0, float &dsc1, float &dmm1) {
    const uint4 h = *reinterpret_cast<const uint4 *>(sb);
    const uint4 qh0 = *reinterpret_cast<const uint4 *>(sb + 16), qh1 = *reinterpret_cast<const uint4 *>(sb + 32);
    const uint4 q0 = *reinterpret_cast<const uint4 *>(sb + 48 + 32 * g);
    const uint4 q1 = *reinterpret_cast<const uint4 *>(sb + 64 + 32 * g);
    const uint4 a0 = *reinterpret_cast<const uint4 *>(xa), a1 = *reinterpret_cast<const uint4 *>(xa + 4);
    const uint4 b0 = *reinterpret_cast<const uint4 *>(xb), b1 = *reinterpret_cast<const uint4 *>(xb + 4);
    q4k_pair_sums(q0, q1, a0, a1, b0, b1, s0, s1);
    const uint32_t m = 0x01010101u;
    const int ea = 2 * g, eb = 2 * g + 1;  // bit of qh for sub-blocks 2g and 2g+1
    int h0 = 0, h1 = 0;
    h0 = dp4a_us((qh0.x >> ea) & m, a0.x, h0);
    h1 = dp4a_us((qh0.x >> eb) & m, b0.x, h1);
    h0 = dp4a_us((qh0.y >> ea) & m, a0.y, h0);
    h1 = dp4a_us((qh0.y >> eb) & m, b0.y, h1);
    h0 = dp4a_us((qh0.z >> ea) & m, a0.z, h0);
    h1 = dp4a_us((qh0.z >> eb) & m, b0.z, h1);
    h0 = dp4a_us((qh0.w >> ea) & m, a0.w, h0);
    h1 = dp4a_us((qh0.w >> eb) & m, b0.w, h1);
    h0 = dp4a_us((qh1.x >> ea) & m, a1.x, h0);
    h1 = dp4a_us((qh1.x >> eb) & m, b1.x, h1);
    h0 = dp4a_us((qh1.y >> ea) & m, a1.y, h0);
    h1 = dp4a_us((qh1.y >> eb) & m, b1.y, h1);
    h0 = dp4a_us((qh1.z >> ea) & m, a1.z, h0);
    h1 = dp4a_us((qh1.z >> eb) & m, b1.z, h1);
    h0 = dp4a_us((qh1.w >> ea) & m, a1.w, h0);
    h1 = dp4a_us((qh1.w >> eb) & m, b1.w, h1);
    s0 += 16 * h0;
    s1 += 16 * h1;
    q4k_pair_scales(h, g, dsc0, dmm0, dsc1, dmm1);
}

// Q6_K sub-block pair g (0..3) of the super-block at `sb` (2-byte aligned:
// 210-byte super-blocks): ql[128] low 4 bits, qh[64] top 2 bits, int8
// scales[16] (one per 16 elements), f16 d at byte 208; value =
// d * scale * (q - 32). Pair g is half h = g / 2, quarters t = 2 (g % 2) and
// t + 1: the nibbles of ql[64h + l] (sub-block 2g) and ql[64h + 32 + l]
// (sub-block 2g+1), low for even g and high for odd g; their top bits are
// bits 2t.. and 2t+2.. of qh[32h + l]; their scales are bytes 8h + 2t ..
// 8h + 2t + 3. Returns s0, s1 = sum over each sub-block's two 16-element
// groups of scale * sum((q - 32) * x), and d.
__device__ __forceinline__ void q6k_pair_dot(const uint8_t *sb, int g, const uint32_t *xa, const uint32_t *xb,
                                             int &s0, int &s1, float &d) {
    const int h = g >> 1, t = 2 * (g & 1);
    uint32_t ql[16], qh[8], scw[1];
    ld_words_a2<16>(sb + 64 * h, ql);
    ld_words_a2<8>(sb + 128 + 32 * h, qh);
    ld_words_a2<1>(sb + 192 + 8 * h + 2 * t, scw);
    d = f16_bits_to_f32(ld_u16(sb + 208));
    const int nsh = (g & 1) ? 4 : 0;
    const uint32_t m4 = 0x0f0f0f0fu, m2 = 0x03030303u, ones = 0x01010101u;
    int sum[2];
#pragma unroll
    for (int j = 0; j < 2; j++) {  // sub-block 2g + j
        const uint4 xl = *reinterpret_cast<const uint4 *>(j ? xb : xa);
        const uint4 xh = *reinterpret_cast<const uint4 *>((j ? xb : xa) + 4);
        const uint32_t xw[8] = {xl.x, xl.y, xl.z, xl.w, xh.x, xh.y, xh.z, xh.w};
        const int hs = 2 * (t + j);
        int acc = 0;
#pragma unroll
        for (int grp = 0; grp < 2; grp++) {
            int u = 0, hi = 0, xs = 0;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int w = 4 * grp + i;
                u = dp4a_us((ql[8 * j + w] >> nsh) & m4, xw[w], u);
                hi = dp4a_us((qh[w] >> hs) & m2, xw[w], hi);
                xs = dp4a_ss(ones, xw[w], xs);
            }
            const int sc = (int)(int8_t)((scw[0] >> (8 * (2 * j + grp))) & 0xffu);
            acc += sc * (u + 16 * hi - 32 * xs);
        }
        sum[j] = acc;
    }
    s0 = sum[0];
    s1 = sum[1];
}

// The same with the activation words read from `xa` / `xb` (16-byte aligned).
__device__ __forceinline__ void q4k_pair_dot(const uint8_t *sb, int g, const uint32_t *xa, const uint32_t *xb,
                                             int &s0, int &s1, float &dsc0, float &dmm0, float &dsc1, float &dmm1) {
    q4k_pair_dot_x(sb, g, *reinterpret_cast<const uint4 *>(xa), *reinterpret_cast<const uint4 *>(xa + 4),
                   *reinterpret_cast<const uint4 *>(xb), *reinterpret_cast<const uint4 *>(xb + 4), s0, s1, dsc0,
                   dmm0, dsc1, dmm1);
}

}  // namespace fbk
