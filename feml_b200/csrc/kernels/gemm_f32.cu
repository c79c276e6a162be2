// F32 mul_mat (feml-cpu/src/ops/mul_mat.rs:14-58 semantics):
//   y[n][m] = sum_k W[m][k] * X[n][k]   (both operands K-contiguous)
// SIMT FP32 with FMA. Each CTA owns a 32x32 output tile; its 16 warps form
// four K-slices that each accumulate a partial tile, then the partials are
// added in slice order in shared memory, so the result does not depend on
// scheduling. Optional column grouping (mul_mat_id with F32 experts) reuses
// the routing tables of the quantized path.
#include <cuda_runtime.h>

#include "../host_common.h"
#include "common.cuh"
#include "kernels.h"

namespace fbk {

namespace {

constexpr int BM = 32, BN = 32, BK = 32;
constexpr int SLICES = 4, SLICE_THREADS = 128;
constexpr int THREADS = SLICES * SLICE_THREADS;

struct F32Params {
    const uint8_t *w;
    uint64_t w_nb1;
    const uint8_t *x;
    uint64_t x_nb1;
    uint8_t *y;
    uint64_t y_nb1;
    int K, M, N;
    GroupMap g;
    bool grouped;
};

__global__ void __launch_bounds__(THREADS) gemm_f32_kernel(const F32Params p) {
    // operand tiles during the K loop; the same bytes hold the partial tiles
    // for the final reduction
    constexpr int kTileFloats = SLICES * BK * (BM + 4) + SLICES * BK * (BN + 4);
    constexpr int kRedFloats = SLICES * BN * (BM + 1);
    __shared__ __align__(16) float buf[kTileFloats > kRedFloats ? kTileFloats : kRedFloats];
    auto As = reinterpret_cast<float(*)[BK][BM + 4]>(buf);
    auto Bs = reinterpret_cast<float(*)[BK][BN + 4]>(buf + SLICES * BK * (BM + 4));
    auto Red = reinterpret_cast<float(*)[BN][BM + 1]>(buf);
    __shared__ int col_src[BN];     // activation column per tile column (-1 = none)
    __shared__ uint64_t col_dst[BN];  // output byte offset per tile column

    const int slice = threadIdx.x / SLICE_THREADS;
    const int t = threadIdx.x % SLICE_THREADS;
    const int m0 = blockIdx.x * BM;

    const uint8_t *w = p.w;
    if (threadIdx.x < BN) {
        const int c = threadIdx.x;
        int src = -1;
        uint64_t dst = 0;
        if (!p.grouped) {
            const int n = blockIdx.y * BN + c;
            if (n < p.N) {
                src = n;
                dst = (uint64_t)n * p.y_nb1;
            }
        } else {
            const int tile = blockIdx.y;
            int e = 0;
            while (e < p.g.n_groups && p.g.tile_start[e + 1] <= tile) e++;
            if (e < p.g.n_groups) {
                const int j = (tile - p.g.tile_start[e]) * BN + c;
                if (j < p.g.counts[e]) {
                    const int slot = p.g.rows[p.g.offsets[e] + j];
                    const int tok = slot / p.g.n_selected, s = slot % p.g.n_selected;
                    src = tok;
                    dst = (uint64_t)s * p.g.dst_nb1 + (uint64_t)tok * p.g.dst_nb2;
                }
            }
        }
        col_src[c] = src;
        col_dst[c] = dst;
    }
    if (p.grouped) {
        const int tile = blockIdx.y;
        int e = 0;
        while (e < p.g.n_groups && p.g.tile_start[e + 1] <= tile) e++;
        if (e >= p.g.n_groups) return;  // uniform across the CTA
        w += (uint64_t)e * p.g.w_group_stride;
    }
    __syncthreads();

    // this slice's K range
    const int kper = (p.K + SLICES - 1) / SLICES;
    const int kb = slice * kper;
    const int ke = min(p.K, kb + kper);
    const int trips = (kper + BK - 1) / BK;

    const int tm = (t % 8) * 4;   // 4 rows
    const int tn = (t / 8) * 2;   // 2 cols
    float acc[4][2] = {};

    for (int it = 0; it < trips; it++) {
        const int k0 = kb + it * BK;
        // load A: BM rows x BK k, lane -> k (coalesced)
        for (int i = t; i < BM * BK; i += SLICE_THREADS) {
            const int kk = i % BK, mm = i / BK;
            const int m = m0 + mm, k = k0 + kk;
            float v = 0.0f;
            if (m < p.M && k < ke) v = reinterpret_cast<const float *>(w + (uint64_t)m * p.w_nb1)[k];
            As[slice][kk][mm] = v;
        }
        for (int i = t; i < BN * BK; i += SLICE_THREADS) {
            const int kk = i % BK, nn = i / BK;
            const int src = col_src[nn], k = k0 + kk;
            float v = 0.0f;
            if (src >= 0 && k < ke) v = reinterpret_cast<const float *>(p.x + (uint64_t)src * p.x_nb1)[k];
            Bs[slice][kk][nn] = v;
        }
        __syncthreads();
#pragma unroll 8
        for (int kk = 0; kk < BK; kk++) {
            const float4 a = *reinterpret_cast<const float4 *>(&As[slice][kk][tm]);
            const float2 b = *reinterpret_cast<const float2 *>(&Bs[slice][kk][tn]);
            acc[0][0] = fmaf(a.x, b.x, acc[0][0]);
            acc[1][0] = fmaf(a.y, b.x, acc[1][0]);
            acc[2][0] = fmaf(a.z, b.x, acc[2][0]);
            acc[3][0] = fmaf(a.w, b.x, acc[3][0]);
            acc[0][1] = fmaf(a.x, b.y, acc[0][1]);
            acc[1][1] = fmaf(a.y, b.y, acc[1][1]);
            acc[2][1] = fmaf(a.z, b.y, acc[2][1]);
            acc[3][1] = fmaf(a.w, b.y, acc[3][1]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 2; j++) Red[slice][tn + j][tm + i] = acc[i][j];
    __syncthreads();
    for (int i = threadIdx.x; i < BM * BN; i += THREADS) {
        const int mm = i % BM, nn = i / BM;
        const int m = m0 + mm;
        if (m >= p.M || col_src[nn] < 0) continue;
        float v = Red[0][nn][mm];
#pragma unroll
        for (int s = 1; s < SLICES; s++) v += Red[s][nn][mm];
        reinterpret_cast<float *>(p.y + col_dst[nn])[m] = v;
    }
}

}  // namespace

static int launch_f32(const F32Params &p, int tiles_n, cudaStream_t s) {
    if (p.M == 0 || tiles_n == 0) return FB_OK;
    dim3 grid((p.M + BM - 1) / BM, tiles_n);
    gemm_f32_kernel<<<grid, THREADS, 0, s>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fb::set_error(FB_ERR_CUDA, "gemm_f32 launch: %s", cudaGetErrorString(e));
    return FB_OK;
}

int launch_gemm_f32(const void *w, uint64_t w_nb1, const void *x, uint64_t x_nb1, void *y, uint64_t y_nb1, int64_t K,
                    int64_t M, int64_t N, cudaStream_t s) {
    if ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) | w_nb1 |
         x_nb1 | y_nb1) & 3)
        return fb::set_error(FB_ERR_INVALID, "mul_mat f32: operands must be 4-byte aligned");
    if (K > INT32_MAX || M > INT32_MAX || N > INT32_MAX)
        return fb::set_error(FB_ERR_UNSUPPORTED, "mul_mat f32: dimension too large");
    if (N == 0 || M == 0) return FB_OK;
    F32Params p{};
    p.w = static_cast<const uint8_t *>(w);
    p.w_nb1 = w_nb1;
    p.x = static_cast<const uint8_t *>(x);
    p.x_nb1 = x_nb1;
    p.y = static_cast<uint8_t *>(y);
    p.y_nb1 = y_nb1;
    p.K = (int)K;
    p.M = (int)M;
    p.N = (int)N;
    p.grouped = false;
    return launch_f32(p, (int)((N + BN - 1) / BN), s);
}

int launch_gemm_f32_grouped(const void *w, uint64_t w_nb1, const void *x, uint64_t x_nb1, int64_t K, int64_t M,
                            void *dst, const GroupMap &g, cudaStream_t s) {
    if ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(dst) | w_nb1 |
         x_nb1 | g.dst_nb1 | g.dst_nb2 | g.w_group_stride) & 3)
        return fb::set_error(FB_ERR_INVALID, "mul_mat_id f32: operands must be 4-byte aligned");
    F32Params p{};
    p.w = static_cast<const uint8_t *>(w);
    p.w_nb1 = w_nb1;
    p.x = static_cast<const uint8_t *>(x);
    p.x_nb1 = x_nb1;
    p.y = static_cast<uint8_t *>(dst);
    p.y_nb1 = 0;
    p.K = (int)K;
    p.M = (int)M;
    p.N = 0;
    p.g = g;
    p.grouped = true;
    return launch_f32(p, g.max_tiles, s);
}

int gemm_f32_block_n() { return BN; }

}  // namespace fbk
