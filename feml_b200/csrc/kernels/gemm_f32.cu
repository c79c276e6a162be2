// F32 mul_mat with the reference's rounding, bit for bit
// (feml-cpu/src/ops/mul_mat.rs:36-57, and feml-cuda's kernel_mul_mat built
// with fmad=false, feml-cuda/src/backend.rs:42-49):
//   acc = 0; for k in 0..K: acc = acc + round(a[k, m] * b[k, n])
// Every output is one sequential chain in k with the product and the sum
// rounded separately (__fmul_rn / __fadd_rn: no contraction, no reordering),
// so results equal the reference CPU backend exactly.
//
// Tiling: a CTA owns a 32x32 output tile; each of its 128 threads owns a
// 4 (rows) x 2 (columns) micro-tile, i.e. 8 independent chains (the ILP that
// hides the add latency). K is walked in 32-wide slabs staged through a
// two-stage cp.async ring; the weight slab is stored k-major so a thread
// reads its 4 rows with one 16-byte load. Optional column grouping
// (mul_mat_id with F32 experts) reuses the routing tables.
#include <cuda_runtime.h>

#include "../host_common.h"
#include "common.cuh"
#include "kernels.h"

namespace fbk {

namespace {

constexpr int BM = 32, BN = 32, BK = 32;
constexpr int THREADS = 128;
constexpr int AS = BM + 4;  // k-major row strides (floats)
constexpr int BS = BN + 4;

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

__device__ __forceinline__ void cp_async4(float *smem_dst, const float *gsrc, bool valid) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(smem_dst)), "l"(gsrc),
                 "r"(valid ? 4 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__global__ void __launch_bounds__(THREADS) gemm_f32_exact_kernel(const F32Params p) {
    __shared__ __align__(16) float As[2][BK][AS];
    __shared__ __align__(16) float Bs[2][BK][BS];
    __shared__ int col_src[BN];
    __shared__ uint64_t col_dst[BN];

    const int tid = threadIdx.x;
    const int m0 = blockIdx.x * BM;
    const uint8_t *w = p.w;
    int e = 0;
    if (p.grouped) {
        while (e < p.g.n_groups && p.g.tile_start[e + 1] <= (int)blockIdx.y) e++;
        if (e >= p.g.n_groups) return;  // uniform across the CTA
        w += (uint64_t)e * p.g.w_group_stride;
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
            const int j = ((int)blockIdx.y - p.g.tile_start[e]) * BN + tid;
            if (j < p.g.counts[e]) {
                const int slot = p.g.rows[p.g.offsets[e] + j];
                const int tok = slot / p.g.n_selected, s = slot % p.g.n_selected;
                src = tok;
                dst = (uint64_t)s * p.g.dst_nb1 + (uint64_t)tok * p.g.dst_nb2;
            }
        }
        col_src[tid] = src;
        col_dst[tid] = dst;
    }
    __syncthreads();

    // per-thread load coordinates: element i = tid + 128*j of a 32x32 slab,
    // k = i % 32 (coalesced along k), row/col = i / 32
    auto load = [&](int st, int k0) {
#pragma unroll
        for (int j = 0; j < (BM * BK) / THREADS; j++) {
            const int i = tid + THREADS * j;
            const int kk = i % BK, r = i / BK;
            const int k = k0 + kk, m = m0 + r;
            const bool ok = k < p.K && m < p.M;
            const float *src = ok ? reinterpret_cast<const float *>(w + (uint64_t)m * p.w_nb1) + k
                                  : reinterpret_cast<const float *>(w);
            cp_async4(&As[st][kk][r], src, ok);
        }
#pragma unroll
        for (int j = 0; j < (BN * BK) / THREADS; j++) {
            const int i = tid + THREADS * j;
            const int kk = i % BK, c = i / BK;
            const int k = k0 + kk, s = col_src[c];
            const bool ok = k < p.K && s >= 0;
            const float *src = ok ? reinterpret_cast<const float *>(p.x + (uint64_t)s * p.x_nb1) + k
                                  : reinterpret_cast<const float *>(p.x);
            cp_async4(&Bs[st][kk][c], src, ok);
        }
    };

    const int tm = (tid % 8) * 4;  // rows tm..tm+3
    const int tn = (tid / 8) * 2;  // cols tn, tn+1
    float acc[4][2];
#pragma unroll
    for (int i = 0; i < 4; i++) acc[i][0] = acc[i][1] = 0.0f;

    const int nslab = (p.K + BK - 1) / BK;
    load(0, 0);
    cp_commit();
    for (int sl = 0; sl < nslab; sl++) {
        const int st = sl & 1;
        if (sl + 1 < nslab) {
            load(st ^ 1, (sl + 1) * BK);
            cp_commit();
            cp_wait<1>();
        } else {
            cp_wait<0>();
        }
        __syncthreads();
        const int kn = min(BK, p.K - sl * BK);  // zero-filled tail must not add (-0 + 0 != -0)
#pragma unroll 8
        for (int kk = 0; kk < kn; kk++) {
            const float4 a = *reinterpret_cast<const float4 *>(&As[st][kk][tm]);
            const float2 b = *reinterpret_cast<const float2 *>(&Bs[st][kk][tn]);
            acc[0][0] = __fadd_rn(acc[0][0], __fmul_rn(a.x, b.x));
            acc[1][0] = __fadd_rn(acc[1][0], __fmul_rn(a.y, b.x));
            acc[2][0] = __fadd_rn(acc[2][0], __fmul_rn(a.z, b.x));
            acc[3][0] = __fadd_rn(acc[3][0], __fmul_rn(a.w, b.x));
            acc[0][1] = __fadd_rn(acc[0][1], __fmul_rn(a.x, b.y));
            acc[1][1] = __fadd_rn(acc[1][1], __fmul_rn(a.y, b.y));
            acc[2][1] = __fadd_rn(acc[2][1], __fmul_rn(a.z, b.y));
            acc[3][1] = __fadd_rn(acc[3][1], __fmul_rn(a.w, b.y));
        }
        __syncthreads();
    }
#pragma unroll
    for (int j = 0; j < 2; j++) {
        const int c = tn + j;
        if (col_src[c] < 0) continue;
        float *yc = reinterpret_cast<float *>(p.y + col_dst[c]);
#pragma unroll
        for (int i = 0; i < 4; i++)
            if (m0 + tm + i < p.M) yc[m0 + tm + i] = acc[i][j];
    }
}

int launch_f32(const F32Params &p, int tiles_n, cudaStream_t s) {
    if (p.M == 0 || tiles_n == 0) return FB_OK;
    if (tiles_n > 65535) return fb::set_error(FB_ERR_UNSUPPORTED, "mul_mat f32: too many column tiles");
    dim3 grid((p.M + BM - 1) / BM, tiles_n);
    gemm_f32_exact_kernel<<<grid, THREADS, 0, s>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fb::set_error(FB_ERR_CUDA, "gemm_f32 launch: %s", cudaGetErrorString(e));
    return FB_OK;
}

}  // namespace

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
