// Quantized mul_mat for larger N (prefill, MoE experts):
//   y[n][m] = sum_b scale(m, b, n) * sumi(m, b, n)
// sumi = int32 dot product of a 32-element weight block with the matching
// Q8_0 activation block, computed by int8 tensor-core MMA (m16n8k32, whose K
// is exactly one ggml block); the per-block scale is applied to the int32
// tile in registers (Q8_0/Q4_0: d_w*d_x; Q4_K: d_x*(d*sc*sumi - dmin*m*sum_x)).
//
// Layout: a CTA owns a BM x 64 output tile and walks K in 256-element chunks
// (8 blocks, one Q4_K super-block). Raw weight rows and planar activation
// rows are copied with 16-byte cp.async into a two-stage ring; each chunk's
// weight bytes are unpacked to a plain int8 tile (Q4_0 nibbles re-centred by
// -8) plus per-row block scales before the MMAs. Optional column grouping
// (mul_mat_id) maps a column tile to (expert, slot list) through the routing
// tables, gathering activation columns and scattering output columns.
//
// Requirements: K % 256 == 0, weight base and row stride 16-byte aligned.
#include <cuda_runtime.h>

#include <algorithm>

#include "../host_common.h"
#include "common.cuh"
#include "dot.cuh"
#include "kernels.h"

namespace fbk {

namespace {

constexpr int BN = 64;
constexpr int KC = 256;          // elements per chunk
constexpr int NBC = KC / QK;     // blocks per chunk
constexpr int XS = KC + 16;      // int8 tile row stride (bank-conflict padding)
constexpr int THREADS = 256;

template <int WT>
struct QF;
template <>
struct QF<WT_Q8_0> {
    static constexpr int kChunkBytes = NBC * Q8_0_BYTES;  // 272
};
template <>
struct QF<WT_Q4_0> {
    static constexpr int kChunkBytes = NBC * Q4_0_BYTES;  // 144
};
template <>
struct QF<WT_Q4_K> {
    static constexpr int kChunkBytes = Q4_K_BYTES;  // 144
};

struct GemmQParams {
    const uint8_t *w;
    uint64_t w_nb1;
    Q8Planar xq;
    int K, M, N;
    uint8_t *y;
    uint64_t y_nb1;
    GroupMap g;
    bool grouped;
    // split-K: CTA z of gridDim.z walks chunks [z*split_chunks, ...) and
    // writes its partial tile to partial[z][n][m] (reduced afterwards)
    int split_chunks;
    float *partial;
};

template <int WT, int BM>
struct Smem {
    static constexpr int CHB = QF<WT>::kChunkBytes;
    static constexpr uint32_t wraw = 0;                                   // [2][BM][CHB]
    static constexpr uint32_t xq = wraw + 2 * BM * CHB;                   // [2][BN][XS]
    static constexpr uint32_t xd = xq + 2 * BN * XS;                      // [2][BN][8] f32
    static constexpr uint32_t xs = xd + 2 * BN * NBC * 4;                 // [2][BN][8] i32
    static constexpr uint32_t a = xs + 2 * BN * NBC * 4;                  // [BM][XS] i8
    static constexpr uint32_t sa = a + BM * XS;                           // [BM][8] f32
    static constexpr uint32_t sb = sa + BM * NBC * 4;                     // [BM][8] f32
    static constexpr uint32_t csrc = sb + BM * NBC * 4;                   // [BN] i32
    static constexpr uint32_t cdst = csrc + BN * 4;                       // [BN] u64
    static constexpr uint32_t total = cdst + BN * 8;
};

__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gsrc, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem_dst)), "l"(gsrc),
                 "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void mma_s8(int (&c)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]), "r"(0), "r"(0), "r"(0), "r"(0));
}

template <int WT, int BM>
__global__ void __launch_bounds__(THREADS) gemm_q_kernel(const GemmQParams p) {
    using S = Smem<WT, BM>;
    constexpr int CHB = S::CHB;
    constexpr int WARPS_M = BM / 32;
    constexpr int WARPS_N = 8 / WARPS_M;
    constexpr int WN = BN / WARPS_N;
    constexpr int NT = WN / 8;
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t *wraw = smem + S::wraw;
    int8_t *xq = reinterpret_cast<int8_t *>(smem + S::xq);
    float *xd = reinterpret_cast<float *>(smem + S::xd);
    int32_t *xs = reinterpret_cast<int32_t *>(smem + S::xs);
    int8_t *At = reinterpret_cast<int8_t *>(smem + S::a);
    float *sa = reinterpret_cast<float *>(smem + S::sa);
    float *sb = reinterpret_cast<float *>(smem + S::sb);
    int32_t *csrc = reinterpret_cast<int32_t *>(smem + S::csrc);
    uint64_t *cdst = reinterpret_cast<uint64_t *>(smem + S::cdst);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int m0 = blockIdx.x * BM;
    const int K = p.K, nblk = K / QK, nchunks = K / KC;

    // column tile -> (weights, activation column, output offset)
    const uint8_t *w = p.w;
    int tile_e = 0;
    if (p.grouped) {
        while (tile_e < p.g.n_groups && p.g.tile_start[tile_e + 1] <= (int)blockIdx.y) tile_e++;
        if (tile_e >= p.g.n_groups) return;  // uniform: no columns for this tile
        w += (uint64_t)tile_e * p.g.w_group_stride;
    }
    if (tid < BN) {
        int src = -1;
        uint64_t dst = 0;
        if (!p.grouped) {
            const int n = blockIdx.y * BN + tid;
            if (n < p.N) {
                src = n;
                dst = (uint64_t)n * p.y_nb1;
            }
        } else {
            const int j = ((int)blockIdx.y - p.g.tile_start[tile_e]) * BN + tid;
            if (j < p.g.counts[tile_e]) {
                const int slot = p.g.rows[p.g.offsets[tile_e] + j];
                const int tok = slot / p.g.n_selected, s = slot % p.g.n_selected;
                src = tok;
                dst = (uint64_t)s * p.g.dst_nb1 + (uint64_t)tok * p.g.dst_nb2;
            }
        }
        csrc[tid] = src;
        cdst[tid] = dst;
    }
    __syncthreads();

    auto load_stage = [&](int st, int c) {
        uint8_t *wr = wraw + st * BM * CHB;
        constexpr int PR = CHB / 16;
        for (int i = tid; i < BM * PR; i += THREADS) {
            const int r = i / PR, pc = i % PR;
            const bool ok = m0 + r < p.M;
            const uint8_t *src = ok ? w + (uint64_t)(m0 + r) * p.w_nb1 + (uint64_t)c * CHB + pc * 16 : w;
            cp_async16(wr + r * CHB + pc * 16, src, ok);
        }
        int8_t *xr = xq + st * BN * XS;
        for (int i = tid; i < BN * (KC / 16); i += THREADS) {
            const int col = i / (KC / 16), pc = i % (KC / 16);
            const int s = csrc[col];
            const int8_t *src = s >= 0 ? p.xq.qs + (uint64_t)s * K + (uint64_t)c * KC + pc * 16 : p.xq.qs;
            cp_async16(xr + col * XS + pc * 16, src, s >= 0);
        }
        for (int i = tid; i < BN * 4; i += THREADS) {  // 2 x 16 B of d and 2 x 16 B of sum per column
            const int col = i / 4, part = i % 4;
            const int s = csrc[col];
            const uint64_t eoff = (uint64_t)(s >= 0 ? s : 0) * nblk + (uint64_t)c * NBC + (part & 1) * 4;
            if (part < 2)
                cp_async16(xd + (st * BN + col) * NBC + (part & 1) * 4, p.xq.d + eoff, s >= 0);
            else
                cp_async16(xs + (st * BN + col) * NBC + (part & 1) * 4, p.xq.sum + eoff, s >= 0);
        }
    };

    const int wm = warp % WARPS_M, wn = warp / WARPS_M;
    const int g = lane >> 2, t4 = lane & 3;
    float acc[2][NT][4];
#pragma unroll
    for (int i = 0; i < 2; i++)
#pragma unroll
        for (int j = 0; j < NT; j++)
#pragma unroll
            for (int k = 0; k < 4; k++) acc[i][j][k] = 0.0f;

    const int c_begin = p.partial ? (int)blockIdx.z * p.split_chunks : 0;
    const int c_end = p.partial ? min(nchunks, c_begin + p.split_chunks) : nchunks;
    load_stage(0, c_begin);
    cp_async_commit();
    for (int c = c_begin; c < c_end; c++) {
        const int st = (c - c_begin) & 1;
        if (c + 1 < c_end) {
            load_stage(st ^ 1, c + 1);
            cp_async_commit();
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();

        // unpack the chunk's weights into At / sa / sb
        const uint8_t *wr = wraw + st * BM * CHB;
        for (int i = tid; i < BM * (KC / 4); i += THREADS) {
            const int r = i / (KC / 4), wi = i % (KC / 4);
            const int b = wi / 8, e = (wi % 8) * 4;
            const uint8_t *row = wr + r * CHB;
            uint32_t v;
            if constexpr (WT == WT_Q8_0) {
                uint32_t t1[1];
                ld_words_a2<1>(row + Q8_0_BYTES * b + 2 + e, t1);
                v = t1[0];
            } else if constexpr (WT == WT_Q4_0) {
                uint32_t t1[1];
                ld_words_a2<1>(row + Q4_0_BYTES * b + 2 + (e & 15), t1);
                v = __vsub4((e < 16 ? t1[0] : t1[0] >> 4) & 0x0f0f0f0fu, 0x08080808u);
            } else {
                const uint32_t raw = *reinterpret_cast<const uint32_t *>(row + 16 + 32 * (b >> 1) + e);
                v = (raw >> (4 * (b & 1))) & 0x0f0f0f0fu;
            }
            *reinterpret_cast<uint32_t *>(At + r * XS + wi * 4) = v;
        }
        for (int i = tid; i < BM * NBC; i += THREADS) {
            const int r = i / NBC, b = i % NBC;
            const uint8_t *row = wr + r * CHB;
            if constexpr (WT == WT_Q8_0) {
                sa[i] = f16_bits_to_f32(ld_u16(row + Q8_0_BYTES * b));
            } else if constexpr (WT == WT_Q4_0) {
                sa[i] = f16_bits_to_f32(ld_u16(row + Q4_0_BYTES * b));
            } else {
                int sc, m;
                q4k_scale_min(b, row + 4, sc, m);
                sa[i] = f16_bits_to_f32(ld_u16(row)) * (float)sc;
                sb[i] = f16_bits_to_f32(ld_u16(row + 2)) * (float)m;
            }
        }
        __syncthreads();

        const int8_t *xr = xq + st * BN * XS;
        const float *xdr = xd + st * BN * NBC;
        const int32_t *xsr = xs + st * BN * NBC;
#pragma unroll
        for (int kb = 0; kb < NBC; kb++) {
            uint32_t a[2][4];
#pragma unroll
            for (int mt = 0; mt < 2; mt++) {
                const int r0 = wm * 32 + mt * 16 + g;
                const int8_t *pa = At + r0 * XS + kb * QK + t4 * 4;
                a[mt][0] = *reinterpret_cast<const uint32_t *>(pa);
                a[mt][1] = *reinterpret_cast<const uint32_t *>(pa + 8 * XS);
                a[mt][2] = *reinterpret_cast<const uint32_t *>(pa + 16);
                a[mt][3] = *reinterpret_cast<const uint32_t *>(pa + 8 * XS + 16);
            }
            float rs[2][2], rm[2][2];
#pragma unroll
            for (int mt = 0; mt < 2; mt++)
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    const int r = wm * 32 + mt * 16 + g + 8 * h;
                    rs[mt][h] = sa[r * NBC + kb];
                    rm[mt][h] = WT == WT_Q4_K ? sb[r * NBC + kb] : 0.0f;
                }
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                const int col = wn * WN + nt * 8 + g;
                const int8_t *pb = xr + col * XS + kb * QK + t4 * 4;
                const uint32_t bfr[2] = {*reinterpret_cast<const uint32_t *>(pb),
                                         *reinterpret_cast<const uint32_t *>(pb + 16)};
                const int c0 = wn * WN + nt * 8 + t4 * 2;
                const float cd0 = xdr[c0 * NBC + kb], cd1 = xdr[(c0 + 1) * NBC + kb];
                const float cs0 = WT == WT_Q4_K ? (float)xsr[c0 * NBC + kb] : 0.0f;
                const float cs1 = WT == WT_Q4_K ? (float)xsr[(c0 + 1) * NBC + kb] : 0.0f;
#pragma unroll
                for (int mt = 0; mt < 2; mt++) {
                    int cc[4];
                    mma_s8(cc, a[mt], bfr);
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const int h = i >> 1;
                        const float cd = (i & 1) ? cd1 : cd0;
                        if constexpr (WT == WT_Q4_K) {
                            const float cs = (i & 1) ? cs1 : cs0;
                            acc[mt][nt][i] += cd * (rs[mt][h] * (float)cc[i] - rm[mt][h] * cs);
                        } else {
                            acc[mt][nt][i] += (rs[mt][h] * cd) * (float)cc[i];
                        }
                    }
                }
            }
        }
        __syncthreads();
    }

#pragma unroll
    for (int mt = 0; mt < 2; mt++)
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int r = m0 + wm * 32 + mt * 16 + g + 8 * (i >> 1);
                const int col = wn * WN + nt * 8 + t4 * 2 + (i & 1);
                if (r < p.M && csrc[col] >= 0) {
                    if (p.partial)
                        p.partial[((uint64_t)blockIdx.z * p.N + csrc[col]) * p.M + r] = acc[mt][nt][i];
                    else
                        reinterpret_cast<float *>(p.y + cdst[col])[r] = acc[mt][nt][i];
                }
            }
}

template <int WT, int BM>
int launch_bm(const GemmQParams &p, int tiles_n, cudaStream_t s) {
    using S = Smem<WT, BM>;
    auto kern = gemm_q_kernel<WT, BM>;
    static DeviceFlags smem_set;
    const int rc = raise_smem_limit((const void *)kern, (int)S::total, smem_set, "gemm_q");
    if (rc) return rc;
    cudaError_t e;
    const int splits = p.partial ? (p.K / KC + p.split_chunks - 1) / p.split_chunks : 1;
    dim3 grid((p.M + BM - 1) / BM, tiles_n, splits);
    kern<<<grid, THREADS, S::total, s>>>(p);
    e = cudaGetLastError();
    if (e != cudaSuccess) return fb::set_error(FB_ERR_CUDA, "gemm_q launch: %s", cudaGetErrorString(e));
    return FB_OK;
}

// y[n][m] = sum over z in order of partial[z][n][m] (deterministic).
__global__ void split_reduce_kernel(const float *__restrict__ partial, int splits, int M, int N, uint8_t *y,
                                    uint64_t y_nb1) {
    const int64_t total = (int64_t)M * N;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        float acc = partial[i];
        for (int z = 1; z < splits; z++) acc += partial[(int64_t)z * total + i];
        const int n = (int)(i / M), m = (int)(i % M);
        reinterpret_cast<float *>(y + (uint64_t)n * y_nb1)[m] = acc;
    }
}

template <int WT>
int launch_wt(const GemmQParams &p, int tiles_n, cudaStream_t s) {
    const int64_t sms = sm_count();
    if (p.partial) return launch_bm<WT, 128>(p, tiles_n, s);
    const int64_t t128 = (int64_t)((p.M + 127) / 128) * tiles_n;
    const int64_t t64 = (int64_t)((p.M + 63) / 64) * tiles_n;
    if (t128 >= 2 * sms) return launch_bm<WT, 128>(p, tiles_n, s);
    if (t64 >= sms) return launch_bm<WT, 64>(p, tiles_n, s);
    return launch_bm<WT, 32>(p, tiles_n, s);
}

// One thread per (m, n, 64-element pair): the pair routines of the decode
// GEMV, on copies of the pair's bytes in an aligned local buffer (so nothing
// is read past the tensors' ends).
template <int WT>
__global__ void block_dots_kernel(const uint8_t *w, uint64_t w_nb1, const uint8_t *xq, int K, int M, int N,
                                  int32_t *out) {
    const int nblk = K / QK, npair = (nblk + 1) / 2;
    const int64_t total = (int64_t)M * N * npair;
    const uint64_t xrow = (uint64_t)nblk * Q8_0_BYTES;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int pr = (int)(i % npair);
        const int64_t mn = i / npair;
        const int n = (int)(mn % N), m = (int)(mn / N);
        const int b0 = 2 * pr;
        const bool single = b0 + 1 >= nblk;
        // activation blocks b0, b0+1 as packed words, their sums, the shifted form
        __align__(16) uint32_t xw[2][8];
        int xs[2] = {0, 0};
        for (int k = 0; k < 2; k++) {
            const int b = b0 + k;
            for (int l = 0; l < 8; l++) xw[k][l] = 0;
            if (b >= nblk) continue;
            const uint8_t *xb = xq + (uint64_t)n * xrow + (uint64_t)b * Q8_0_BYTES + 2;
            for (int l = 0; l < 32; l++) {
                xw[k][l / 4] |= (uint32_t)xb[l] << (8 * (l % 4));
                xs[k] += (int8_t)xb[l];
            }
        }
        const uint8_t *row = w + (uint64_t)m * w_nb1;
        int s0 = 0, s1 = 0;
        if constexpr (WT == WT_Q4_K) {
            __align__(16) uint8_t sbuf[Q4_K_BYTES];
            const uint8_t *sbp = row + (uint64_t)(b0 / 8) * Q4_K_BYTES;
            for (int l = 0; l < Q4_K_BYTES; l++) sbuf[l] = sbp[l];
            float a, b, c, d;
            q4k_pair_dot(sbuf, (b0 % 8) / 2, xw[0], xw[1], s0, s1, a, b, c, d);
        } else {
            constexpr int UBY = WT == WT_Q8_0 ? Q8_0_BYTES : Q4_0_BYTES;
            __align__(16) uint32_t wbuf[(2 * UBY + 4 + 3) / 4];
            uint8_t *wb8 = reinterpret_cast<uint8_t *>(wbuf);
            const uint8_t *up = row + (uint64_t)b0 * UBY;
            const int nb = single ? UBY : 2 * UBY;
            for (int l = 0; l < (int)sizeof(wbuf); l++) wb8[l] = l < nb ? up[l] : 0;
            __align__(16) uint32_t sh[kShiftWords];
            make_shifted<WT>(xw[0], sh);
            float d0, d1;
            if (single)
                s0 = single_even_dot<WT>(wbuf, sh, xs[0], d0);
            else
                pair_dot<WT>(wbuf, sh, xw[1], xs[0], xs[1], s0, s1, d0, d1);
        }
        int32_t *o = out + ((int64_t)m * N + n) * nblk + b0;
        o[0] = s0;
        if (!single) o[1] = s1;
    }
}

}  // namespace

int gemm_q_block_n() { return BN; }

// Split-K plan of the ungrouped GEMM: used when the BM = 128 tile grid would
// leave most SMs idle; every split walks at least two chunks.
int gemm_q_splits(int64_t K, int64_t M, int64_t N) {
    const int64_t nchunks = K / KC;
    const int64_t tiles = ((M + 127) / 128) * ((N + BN - 1) / BN);
    const int64_t sms = sm_count();
    if (nchunks < 4 || tiles >= sms) return 1;
    int64_t splits = std::min<int64_t>({(2 * sms + tiles - 1) / tiles, nchunks / 2, 16});
    if (splits < 2) return 1;
    const int64_t per = (nchunks + splits - 1) / splits;
    return (int)((nchunks + per - 1) / per);
}

uint64_t gemm_q_split_bytes(int64_t K, int64_t M, int64_t N) {
    const int sp = gemm_q_splits(K, M, N);
    return sp > 1 ? (uint64_t)sp * (uint64_t)M * (uint64_t)N * 4 : 0;
}

bool gemm_q_supported(int32_t wtype, int64_t K, const void *w, uint64_t w_nb1) {
    if (wtype != WT_Q8_0 && wtype != WT_Q4_0 && wtype != WT_Q4_K) return false;
    if (K <= 0 || K % KC) return false;
    return ((reinterpret_cast<uintptr_t>(w) | w_nb1) & 15) == 0;
}

int launch_gemm_q(int32_t wtype, const void *w, uint64_t w_nb1, const Q8Planar &xq, int64_t K, int64_t M, int64_t N,
                  void *y, uint64_t y_nb1, const GroupMap *groups, cudaStream_t s, void *split_ws) {
    if (!gemm_q_supported(wtype, K, w, w_nb1))
        return fb::set_error(FB_ERR_UNSUPPORTED, "gemm_q: needs K %% 256 == 0 and 16-byte aligned weight rows");
    if (K > INT32_MAX || M > INT32_MAX || N > INT32_MAX) return fb::set_error(FB_ERR_UNSUPPORTED, "gemm_q: too large");
    if ((reinterpret_cast<uintptr_t>(y) | y_nb1) & 3) return fb::set_error(FB_ERR_INVALID, "gemm_q: output alignment");
    GemmQParams p{};
    p.w = static_cast<const uint8_t *>(w);
    p.w_nb1 = w_nb1;
    p.xq = xq;
    p.K = (int)K;
    p.M = (int)M;
    p.N = (int)N;
    p.y = static_cast<uint8_t *>(y);
    p.y_nb1 = y_nb1;
    int tiles_n;
    if (groups) {
        if ((groups->dst_nb1 | groups->dst_nb2) & 3 || (groups->w_group_stride & 15))
            return fb::set_error(FB_ERR_INVALID, "gemm_q: grouped strides misaligned");
        p.g = *groups;
        p.grouped = true;
        tiles_n = groups->max_tiles;
    } else {
        p.grouped = false;
        tiles_n = (int)((N + BN - 1) / BN);
    }
    if (M == 0 || tiles_n == 0) return FB_OK;
    if (tiles_n > 65535) return fb::set_error(FB_ERR_UNSUPPORTED, "gemm_q: too many column tiles");
    const int splits = groups ? 1 : gemm_q_splits(K, M, N);
    if (splits > 1 && split_ws) {
        const int nchunks = (int)(K / KC);
        p.split_chunks = (nchunks + splits - 1) / splits;
        p.partial = static_cast<float *>(split_ws);
    }
    int rc;
    switch (wtype) {
    case WT_Q8_0: rc = launch_wt<WT_Q8_0>(p, tiles_n, s); break;
    case WT_Q4_0: rc = launch_wt<WT_Q4_0>(p, tiles_n, s); break;
    default: rc = launch_wt<WT_Q4_K>(p, tiles_n, s); break;
    }
    if (rc || !p.partial) return rc;
    const int64_t total = M * N;
    const int blocks = (int)std::min<int64_t>((total + 255) / 256, 4 * sm_count());
    split_reduce_kernel<<<blocks, 256, 0, s>>>(p.partial, splits, (int)M, (int)N, static_cast<uint8_t *>(y), y_nb1);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fb::set_error(FB_ERR_CUDA, "gemm_q split reduce launch: %s", cudaGetErrorString(e));
    return FB_OK;
}

int launch_block_dots(int32_t wtype, const void *w, uint64_t w_nb1, const void *xq, int64_t K, int64_t M, int64_t N,
                      int32_t *out, cudaStream_t s) {
    if (K % (wtype == WT_Q4_K ? QKK : QK)) return fb::set_error(FB_ERR_SHAPE, "block_dots: K not a block multiple");
    if (M * N * (K / QK) == 0) return FB_OK;
    const int64_t total = M * N * ((K / QK + 1) / 2);
    const int grid = (int)std::min<int64_t>((total + 255) / 256, (int64_t)sm_count() * 32);
    const auto *wb = static_cast<const uint8_t *>(w);
    const auto *xb = static_cast<const uint8_t *>(xq);
    switch (wtype) {
    case WT_Q8_0: block_dots_kernel<WT_Q8_0><<<grid, 256, 0, s>>>(wb, w_nb1, xb, (int)K, (int)M, (int)N, out); break;
    case WT_Q4_0: block_dots_kernel<WT_Q4_0><<<grid, 256, 0, s>>>(wb, w_nb1, xb, (int)K, (int)M, (int)N, out); break;
    case WT_Q4_K: block_dots_kernel<WT_Q4_K><<<grid, 256, 0, s>>>(wb, w_nb1, xb, (int)K, (int)M, (int)N, out); break;
    default: return fb::set_error(FB_ERR_UNSUPPORTED, "block_dots: dtype %d", wtype);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fb::set_error(FB_ERR_CUDA, "block_dots launch: %s", cudaGetErrorString(e));
    return FB_OK;
}

}  // namespace fbk
