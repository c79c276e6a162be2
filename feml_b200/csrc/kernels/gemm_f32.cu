// F32 mul_mat with the reference's rounding, bit for bit
// (feml-cpu/src/ops/mul_mat.rs:36-57, and feml-cuda's kernel_mul_mat built
// with fmad=false, feml-cuda/src/backend.rs:42-49):
//   acc = 0; for k in 0..K: acc = acc + round(a[k, m] * b[k, n])
// Every output is one sequential chain in k with the product and the sum
// rounded separately (__fmul_rn / __fadd_rn: no contraction, no reordering),
// so results equal the reference CPU backend exactly.
//
// Two kernels share that arithmetic:
//  - gemm_f32_pipe_kernel (16-byte aligned operands, K % 4 == 0, ungrouped):
//    a CTA owns 4*W rows x 32 columns (W <= 8 compute warps, two per SM
//    sub-partition, W even). One producer thread streams 128-wide k chunks into a
//    4-stage shared-memory ring as 2D TMA boxes (32 k x the CTA's rows, 32 k
//    x its 32 columns; 128-byte swizzle), 8 tensor copies per chunk: with
//    one bulk copy per 512-byte row segment (64 per chunk) the copies, not
//    the arithmetic, set the pace (110 us against 88 us for 4096 x 4096 weights x 32 columns). A compute
//    warp owns 4 rows x 32 columns; each lane a 2-row x 2-column micro-tile
//    (4 chains), reading 4 k values of each of its rows and columns with
//    16-byte shared loads two steps ahead of the arithmetic: 4 loads per 16
//    multiply-adds, conflict-free through the swizzle. Two warps per SM
//    sub-partition hide each other's latencies better than one warp with
//    twice the chains (84 against 88 us at that size, identical outputs). The sequential chains
//    leave the kernel bound by FP32 issue, not by HBM: a lane's two columns
//    of a row take their adds in one packed f32x2 instruction (two
//    independent round-to-nearest adds, so the bits are unchanged), three
//    FP32 instructions per two multiply-adds instead of four (82.9 -> 76.7 us
//    at that size).
//  - gemm_f32_exact_kernel (everything else, and mul_mat_id with F32
//    experts): a CTA owns a 32x32 output tile; each of its 128 threads owns a
//    4 (rows) x 2 (columns) micro-tile, i.e. 8 independent chains. K is walked
//    in 32-wide slabs staged through a two-stage cp.async ring; the weight
//    slab is stored k-major so a thread reads its 4 rows with one 16-byte
//    load. Optional column grouping (mul_mat_id) reuses the routing tables.
#include <cuda_runtime.h>

#include <algorithm>

#include "../host_common.h"
#include "common.cuh"
#include "kernels.h"
#include "tmap.h"

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
// 16-byte shared-memory load at a shared-window address. Volatile, so it
// stays after the mbarrier wait that makes the data visible.
__device__ __forceinline__ float4 lds_f4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
    return v;
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Two independent round-to-nearest FP32 adds in one packed instruction (sm_100).
__device__ __forceinline__ void add2_rn(float &a0, float &a1, float p0, float p1) {
    asm("{\n\t.reg .b64 ta, tp;\n\tmov.b64 ta, {%0, %1};\n\tmov.b64 tp, {%2, %3};\n\t"
        "add.rn.f32x2 ta, ta, tp;\n\tmov.b64 {%0, %1}, ta;\n\t}"
        : "+f"(a0), "+f"(a1)
        : "f"(p0), "f"(p1));
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
            add2_rn(acc[0][0], acc[0][1], __fmul_rn(a.x, b.x), __fmul_rn(a.x, b.y));
            add2_rn(acc[1][0], acc[1][1], __fmul_rn(a.y, b.x), __fmul_rn(a.y, b.y));
            add2_rn(acc[2][0], acc[2][1], __fmul_rn(a.z, b.x), __fmul_rn(a.z, b.y));
            add2_rn(acc[3][0], acc[3][1], __fmul_rn(a.w, b.x), __fmul_rn(a.w, b.y));
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

// ---- pipelined path ---------------------------------------------------------
// A warp owns 4 rows x 32 columns: lane l takes columns l%16 and l%16 + 16
// and rows 2*(l/16), 2*(l/16)+1 of the warp's rows (4 chains).
constexpr int kLaneRows = 2;
constexpr int kWarpRows = 2 * kLaneRows;
constexpr int kMaxWarps = 8;          // compute warps per CTA
constexpr int kChunk = 128;           // k values per stage (four 32-wide boxes)
constexpr int kBoxK = 32;             // k values per 128-byte swizzled box row
constexpr int kPipeStages = 4;
constexpr int kPipeCols = 32;         // columns per CTA
constexpr uint32_t kPipeBarBytes = 128;

struct F32PipeParams {
    uint8_t *y;
    uint64_t y_nb1;
    int K, M, N;
    int warps;  // compute warps; the CTA owns kWarpRows * warps rows
    int32_t *status;
    bool y_vec16;
};

// A stage: 4 weight boxes [bm rows][128 B] then 4 activation boxes
// [32 columns][128 B], each 1024-byte aligned (bm is a multiple of 8).
__host__ __device__ inline uint32_t pipe_stage_bytes(int warps) {
    return (uint32_t)(kChunk / kBoxK) * (uint32_t)(kWarpRows * warps + kPipeCols) * 128u;
}
__host__ __device__ inline uint32_t pipe_smem_bytes(int warps) {
    return kPipeBarBytes + 1024u + kPipeStages * pipe_stage_bytes(warps);  // + 1024: alignment slack
}

__global__ void __launch_bounds__((kMaxWarps + 1) * 32, 1)
    gemm_f32_pipe_kernel(const __grid_constant__ CUtensorMap tmw, const __grid_constant__ CUtensorMap tmx,
                         const F32PipeParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + kPipeStages;
    const uint32_t smem_base = smem_u32(smem);
    const uint32_t stages = (smem_base + kPipeBarBytes + 1023u) & ~1023u;  // shared-window address
    const uint32_t stage_bytes = pipe_stage_bytes(p.warps);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int bm = kWarpRows * p.warps;
    const int m0 = blockIdx.x * bm, n0 = blockIdx.y * kPipeCols;
    const int rows = min(bm, p.M - m0), cols = min(kPipeCols, p.N - n0);
    const int nchunks = (p.K + kChunk - 1) / kChunk;
    const uint32_t wbox = (uint32_t)bm * 128u;        // one weight box
    const uint32_t wbytes = (kChunk / kBoxK) * wbox;  // weight part of a stage

    if (threadIdx.x == 0) {
        for (int st = 0; st < kPipeStages; st++) {
            mbar_init(&full[st], 1);
            mbar_init(&empty[st], (uint32_t)p.warps);
        }
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == p.warps) {
        // Producer (one lane): chunk c goes to stage c % 4 once the compute
        // warps have released that stage's previous chunk; one swizzled box
        // per 32 k values of the weight rows and of the activation columns
        // (rows, columns and k past the matrix read as zeros and are not used).
        if (lane != 0) return;
        int c = 0;
        bool ok = true;
        for (; c < nchunks; c++) {
            const int st = c % kPipeStages;
            if (c >= kPipeStages && !mbar_wait_bounded(&empty[st], (uint32_t)(c / kPipeStages - 1) & 1u)) {
                ok = false;
                break;
            }
            const int k0 = c * kChunk;
            const int nb = (min(kChunk, p.K - k0) + kBoxK - 1) / kBoxK;
            const uint32_t sw = stages + (uint32_t)st * stage_bytes, sx = sw + wbytes;
            fence_proxy_async_smem();
            mbar_arrive_expect_tx(&full[st], (uint32_t)nb * (wbox + kPipeCols * 128u));
            for (int b = 0; b < nb; b++) {
                tma_load_2d(sw + (uint32_t)b * wbox, &tmw, k0 + b * kBoxK, m0, smem_u32(&full[st]));
                tma_load_2d(sx + (uint32_t)b * (kPipeCols * 128u), &tmx, k0 + b * kBoxK, n0, smem_u32(&full[st]));
            }
        }
        if (!ok) report_status(p.status, STATUS_TIMEOUT);
        // the CTA ends only after every copy it issued has landed (chunks
        // before c - 4 were released by the compute warps, so they had)
        for (int j = max(0, c - kPipeStages); j < c; j++)
            mbar_wait_bounded(&full[j % kPipeStages], (uint32_t)(j / kPipeStages) & 1u);
        return;
    }

    // Compute warps. Row y's 16-byte unit u of a box sits at
    // y * 128 + ((u ^ (y % 8)) * 16).
    const int cp = lane & 15;                           // columns cp and cp + 16
    const int r0 = warp * kWarpRows + kLaneRows * (lane >> 4);
    const uint32_t wrow = (uint32_t)r0 * 128u;
    const uint32_t wsw = (uint32_t)(r0 & 7);            // (r0 + r) % 8 == wsw + r (r0 even, r < 2)
    const uint32_t xrow = (uint32_t)cp * 128u;          // column cp + 16 is 2048 bytes on
    const uint32_t xsw = (uint32_t)((cp & 7) << 4);
    float acc[kLaneRows][2];
#pragma unroll
    for (int r = 0; r < kLaneRows; r++) acc[r][0] = acc[r][1] = 0.0f;
    struct Step {
        float4 xa, xb, w[kLaneRows];
    };
    // step t: k values 4t .. 4t+3 of the chunk = box t / 8, unit t % 8
    auto load = [&](uint32_t sw, uint32_t sx, int t) {
        Step v;
        const uint32_t u = (uint32_t)(t & 7) << 4;
        const uint32_t bw = sw + (uint32_t)(t >> 3) * wbox + wrow;
        const uint32_t bx = sx + (uint32_t)(t >> 3) * (kPipeCols * 128u) + xrow + (u ^ xsw);
        v.xa = lds_f4(bx);
        v.xb = lds_f4(bx + 16u * 128u);
#pragma unroll
        for (int r = 0; r < kLaneRows; r++) v.w[r] = lds_f4(bw + (uint32_t)r * 128u + (u ^ ((wsw + (uint32_t)r) << 4)));
        return v;
    };
    auto step = [&](const Step &v) {
#pragma unroll
        for (int r = 0; r < kLaneRows; r++) {
            add2_rn(acc[r][0], acc[r][1], __fmul_rn(v.w[r].x, v.xa.x), __fmul_rn(v.w[r].x, v.xb.x));
        }
#pragma unroll
        for (int r = 0; r < kLaneRows; r++) {
            add2_rn(acc[r][0], acc[r][1], __fmul_rn(v.w[r].y, v.xa.y), __fmul_rn(v.w[r].y, v.xb.y));
        }
#pragma unroll
        for (int r = 0; r < kLaneRows; r++) {
            add2_rn(acc[r][0], acc[r][1], __fmul_rn(v.w[r].z, v.xa.z), __fmul_rn(v.w[r].z, v.xb.z));
        }
#pragma unroll
        for (int r = 0; r < kLaneRows; r++) {
            add2_rn(acc[r][0], acc[r][1], __fmul_rn(v.w[r].w, v.xa.w), __fmul_rn(v.w[r].w, v.xb.w));
        }
    };

    bool ok = true;
    for (int c = 0; c < nchunks; c++) {
        const int st = c % kPipeStages;
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(&full[st], (uint32_t)(c / kPipeStages) & 1u))) {
            ok = false;
            break;
        }
        const uint32_t sw = stages + (uint32_t)st * stage_bytes, sx = sw + wbytes;
        const int nsteps = min(kChunk, p.K - c * kChunk) >> 2;  // 4 k values per step
        // shared loads two steps ahead of the arithmetic (steps past the
        // chunk reload its last step instead of reading beyond it)
        Step s0 = load(sw, sx, 0), s1 = load(sw, sx, min(1, nsteps - 1));
#pragma unroll 2
        for (int t = 0; t < nsteps; t += 2) {
            const Step n0v = load(sw, sx, min(t + 2, nsteps - 1));
            const Step n1v = load(sw, sx, min(t + 3, nsteps - 1));
            step(s0);
            if (t + 1 < nsteps) step(s1);
            s0 = n0v;
            s1 = n1v;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
    }
    if (!ok) {
        if (lane == 0) report_status(p.status, STATUS_TIMEOUT);
        return;
    }
#pragma unroll
    for (int j = 0; j < 2; j++) {
        const int col = cp + 16 * j;
        if (col >= cols || r0 >= rows) continue;
        float *yc = reinterpret_cast<float *>(p.y + (uint64_t)(n0 + col) * p.y_nb1);
        const int m = m0 + r0;  // even
        if (p.y_vec16 && r0 + 2 <= rows) {
            *reinterpret_cast<float2 *>(yc + m) = make_float2(acc[0][j], acc[1][j]);
        } else {
#pragma unroll
            for (int r = 0; r < kLaneRows; r++)
                if (r0 + r < rows) yc[m + r] = acc[r][j];
        }
    }
}

// Compute warps per CTA: enough row tiles times column tiles to cover the
// SMs once where the matrix allows (one warp per SM sub-partition at most).
int pipe_warps(int64_t M, int64_t N) {
    const int64_t col_tiles = (N + kPipeCols - 1) / kPipeCols;
    const int64_t sms = sm_count();
    const int64_t rows_per_cta = (M * col_tiles + sms - 1) / sms;
    const int64_t w = std::min<int64_t>(kMaxWarps, std::max<int64_t>(1, (rows_per_cta + kWarpRows - 1) / kWarpRows));
    return (int)((w + 1) / 2 * 2);  // boxes of a multiple of 8 rows keep the 1024-byte swizzle alignment
}

int launch_f32_pipe(const void *w, uint64_t w_nb1, const void *x, uint64_t x_nb1, const F32PipeParams &p,
                    cudaStream_t s) {
    const int bm = kWarpRows * p.warps;
    CUtensorMap tmw, tmx;
    int rc = encode_tensor_map_2d_sw128(&tmw, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, w, (uint64_t)p.K, (uint64_t)p.M, w_nb1,
                                        kBoxK, (uint32_t)bm);
    if (rc) return rc;
    rc = encode_tensor_map_2d_sw128(&tmx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, x, (uint64_t)p.K, (uint64_t)p.N, x_nb1,
                                    kBoxK, kPipeCols);
    if (rc) return rc;
    static DeviceFlags smem_set;
    rc = raise_smem_limit((const void *)gemm_f32_pipe_kernel, (int)pipe_smem_bytes(kMaxWarps), smem_set, "gemm_f32");
    if (rc) return rc;
    cudaError_t e;
    dim3 grid((unsigned)((p.M + bm - 1) / bm), (unsigned)((p.N + kPipeCols - 1) / kPipeCols));
    gemm_f32_pipe_kernel<<<grid, (p.warps + 1) * 32, pipe_smem_bytes(p.warps), s>>>(tmw, tmx, p);
    e = cudaGetLastError();
    if (e != cudaSuccess) return fb::set_error(FB_ERR_CUDA, "gemm_f32 launch: %s", cudaGetErrorString(e));
    return FB_OK;
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
                    int64_t M, int64_t N, int32_t *status, cudaStream_t s) {
    if ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) | w_nb1 |
         x_nb1 | y_nb1) & 3)
        return fb::set_error(FB_ERR_INVALID, "mul_mat f32: operands must be 4-byte aligned");
    if (K > INT32_MAX || M > INT32_MAX || N > INT32_MAX)
        return fb::set_error(FB_ERR_UNSUPPORTED, "mul_mat f32: dimension too large");
    if (N == 0 || M == 0) return FB_OK;
    const bool aligned16 =
        ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(x) | w_nb1 | x_nb1) & 15) == 0;
    if (aligned16 && K > 0 && K % 4 == 0 && (N + kPipeCols - 1) / kPipeCols <= 65535) {
        F32PipeParams q{};
        q.y = static_cast<uint8_t *>(y);
        q.y_nb1 = y_nb1;
        q.K = (int)K;
        q.M = (int)M;
        q.N = (int)N;
        q.warps = pipe_warps(M, N);
        q.status = status;
        q.y_vec16 = ((reinterpret_cast<uintptr_t>(y) | y_nb1) & 15) == 0;
        return launch_f32_pipe(w, w_nb1, x, x_nb1, q, s);
    }
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
