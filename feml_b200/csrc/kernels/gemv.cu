// Decode-path mul_mat for quantized weights and small N (1..4 columns):
//   y[m, n] = sum_b scale(m, b, n) * sumi(m, b, n)
// with sumi the int32 dot product of one 32-element weight block and the
// matching Q8_0 activation block (dp4a), scale = d_w * d_x (Q8_0, Q4_0) or
// d_x * (d*sc, dmin*m terms) for Q4_K sub-blocks.
//
// B200 mapping. The kernel is HBM-bound (weights are read once), so it is
// built to keep as many weight bytes in flight as possible:
//  - one CTA per SM, each owning a contiguous range of weight rows;
//  - every warp owns its rows and a private ring of shared-memory stages;
//    lane 0 streams row chunks with cp.async.bulk (TMA, evict-first L2 policy)
//    completing on per-stage mbarriers, and re-arms a stage as soon as the
//    warp has consumed it, so a warp has `nstage` chunks in flight at once;
//  - activations are quantized to Q8_0 into shared memory by the CTA itself
//    while the first weight chunks are in flight (no workspace), or read from
//    a planar buffer written by a preceding quantize kernel launched with
//    programmatic dependent launch, so the weight stream starts before the
//    activation quantizer finishes;
//  - ggml blocks keep their 2-byte alignment in shared memory; 32-bit words
//    are assembled with funnel shifts. Row chunks whose global address is not
//    16-byte aligned are copied in their aligned interior by TMA and their
//    ragged head/tail bytes by plain loads.
#include <cuda_runtime.h>

#include <algorithm>

#include "../host_common.h"
#include "common.cuh"
#include "dot.cuh"
#include "kernels.h"

namespace fbk {

namespace {

constexpr int kGemvWarps = 8;
constexpr int kGemvThreads = kGemvWarps * 32;
constexpr int kMaxCols = 4;
constexpr int kSmemLimit = 227 * 1024;
constexpr int kFusedMaxElems = 16384;  // N*K up to which each CTA quantizes x itself

template <int WT>
struct Fmt;
template <>
struct Fmt<WT_Q8_0> {
    static constexpr int kUnitBytes = Q8_0_BYTES;  // one 32-element block
};
template <>
struct Fmt<WT_Q4_0> {
    static constexpr int kUnitBytes = Q4_0_BYTES;
};
template <>
struct Fmt<WT_Q4_K> {
    static constexpr int kUnitBytes = Q4_K_BYTES / 8;  // one 32-element sub-block
};

struct GemvParams {
    const uint8_t *w;
    uint64_t w_nb1;
    const uint8_t *x;
    uint64_t x_nb1;
    uint8_t *y;
    uint64_t y_nb1;
    int K;
    int M;
    int nchunks;      // chunks per row
    int chunk_units;  // 32-element units per chunk (multiple of 8)
    int nstage;       // ring stages per warp
    uint32_t stage_bytes;
    Q8Planar xq;  // xq.qs == nullptr: quantize in-kernel
    int32_t *status;
};

__host__ __device__ inline uint32_t align16(uint32_t v) { return (v + 15u) & ~15u; }

struct SmemLayout {
    uint32_t bars, qs, d, sum, ring, total;
};

__host__ __device__ inline SmemLayout smem_layout(int K, int ncols, int nstage, uint32_t stage_bytes) {
    SmemLayout L;
    const uint32_t nblk = (uint32_t)K / QK;
    L.bars = 0;
    L.qs = align16(kGemvWarps * nstage * 8);
    L.d = L.qs + align16((uint32_t)ncols * K);
    L.sum = L.d + align16(ncols * nblk * 4);
    L.ring = (L.sum + align16(ncols * nblk * 4) + 127u) & ~127u;
    L.total = L.ring + (uint32_t)kGemvWarps * nstage * stage_bytes;
    return L;
}

// One 32-element unit against NC activation columns, accumulated into acc[n].
template <int WT, int NC>
__device__ __forceinline__ void dot_unit(const uint8_t *p0, int u, int b, const int8_t *sq, const float *sd,
                                         const int32_t *ss, int K, int nblk, float (&acc)[kMaxCols]) {
    Unit U;
    load_unit<WT>(p0, u, U);
#pragma unroll
    for (int n = 0; n < NC; n++) {
        const int4 *xv = reinterpret_cast<const int4 *>(sq + n * K + b * QK);
        const int xsum = ss[n * nblk + b];
        const int s = unit_sumi<WT>(U, xv[0], xv[1], xsum);
        acc[n] += unit_scale<WT>(U, s, sd[n * nblk + b], xsum);
    }
}

template <int WT, int NC>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_kernel(const GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int UB = Fmt<WT>::kUnitBytes;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int K = p.K, nblk = K / QK;
    const SmemLayout L = smem_layout(K, NC, p.nstage, p.stage_bytes);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bars) + warp * p.nstage;
    int8_t *sq = reinterpret_cast<int8_t *>(smem + L.qs);
    float *sd = reinterpret_cast<float *>(smem + L.d);
    int32_t *ss = reinterpret_cast<int32_t *>(smem + L.sum);
    uint8_t *ring = smem + L.ring + (uint32_t)warp * p.nstage * p.stage_bytes;

    const int r_begin = (int)((int64_t)blockIdx.x * p.M / gridDim.x);
    const int r_end = (int)((int64_t)(blockIdx.x + 1) * p.M / gridDim.x);
    const int cta_rows = r_end - r_begin;
    const int my_rows = cta_rows > warp ? (cta_rows - warp + kGemvWarps - 1) / kGemvWarps : 0;
    const int n_items = my_rows * p.nchunks;
    const uint32_t chunk_bytes = (uint32_t)p.chunk_units * UB;
    const uint32_t row_units = (uint32_t)nblk;

    // Item i of this warp = (row, chunk); its global byte range.
    auto item_range = [&](int i, uintptr_t &start, uint32_t &len, int &row, int &c) {
        row = r_begin + warp + (i / p.nchunks) * kGemvWarps;
        c = i % p.nchunks;
        const uint32_t u0 = (uint32_t)c * p.chunk_units;
        const uint32_t nu = min((uint32_t)p.chunk_units, row_units - u0);
        start = reinterpret_cast<uintptr_t>(p.w + (uint64_t)row * p.w_nb1 + (uint64_t)c * chunk_bytes);
        len = nu * UB;
    };

    const uint64_t policy = policy_evict_first();
    auto issue = [&](int i) {  // lane 0 only
        uintptr_t start;
        uint32_t len;
        int row, c;
        item_range(i, start, len, row, c);
        const uintptr_t base = start & ~uintptr_t(15);
        const uintptr_t a = (start + 15) & ~uintptr_t(15);
        const uintptr_t e = (start + len) & ~uintptr_t(15);
        uint64_t *bar = &bars[i % p.nstage];
        uint8_t *dst = ring + (uint32_t)(i % p.nstage) * p.stage_bytes;
        if (e > a) {
            mbar_arrive_expect_tx(bar, (uint32_t)(e - a));
            bulk_g2s_evict_first(dst + (a - base), reinterpret_cast<const void *>(a), (uint32_t)(e - a), bar, policy);
        } else {
            mbar_arrive(bar);
        }
    };

    if (lane == 0) {
        for (int s = 0; s < p.nstage; s++) mbar_init(&bars[s], 1);
        fence_barrier_init();
    }
    __syncwarp();
    int issued = 0;
    if (lane == 0)
        for (; issued < min(p.nstage, n_items); issued++) issue(issued);
    issued = __shfl_sync(0xffffffffu, issued, 0);

    // Activations -> Q8_0 in shared memory (overlaps the weight stream). Every
    // thread issues all its float4 loads first (one L2 round trip in total),
    // then 8-lane groups quantize one 32-element block each.
    if (p.xq.qs == nullptr) {
        constexpr int kBatch = 8;  // float4 loads in flight per thread
        const int nq = NC * K / 4;  // float4 quads; a block is 8 consecutive quads
        for (int base = 0; base < nq; base += kGemvThreads * kBatch) {  // uniform trip count
            const int q0 = base + (int)threadIdx.x;
            float4 v[kBatch];
#pragma unroll
            for (int j = 0; j < kBatch; j++) {
                const int q = q0 + j * kGemvThreads;
                if (q < nq) {
                    const int n = q / (K / 4), e = (q % (K / 4)) * 4;
                    const float *xr = reinterpret_cast<const float *>(p.x + (uint64_t)n * p.x_nb1);
                    v[j] = make_float4(xr[e], xr[e + 1], xr[e + 2], xr[e + 3]);
                } else {
                    v[j] = make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
#pragma unroll
            for (int j = 0; j < kBatch; j++) {
                // every lane takes part in the group shuffles (padding quads are
                // zeros); nq is a multiple of 8, so a group is valid or not as a whole
                const int q = q0 + j * kGemvThreads;
                uint16_t dbits;
                int qsum;
                const uint32_t packed = quantize_q8_0_quad(v[j], dbits, qsum);
                if (q < nq) {
                    const int n = q / (K / 4), e = (q % (K / 4)) * 4;
                    *reinterpret_cast<uint32_t *>(sq + n * K + e) = packed;
                    if ((threadIdx.x & 7u) == 0) {
                        const int b = e / QK;
                        sd[n * nblk + b] = f16_bits_to_f32(dbits);
                        ss[n * nblk + b] = qsum;
                    }
                }
            }
        }
    } else {
        grid_dependency_wait();
        const int4 *src = reinterpret_cast<const int4 *>(p.xq.qs);
        int4 *dst = reinterpret_cast<int4 *>(sq);
        for (int t = threadIdx.x; t < NC * K / 16; t += kGemvThreads) dst[t] = src[t];
        for (int t = threadIdx.x; t < NC * nblk; t += kGemvThreads) {
            sd[t] = p.xq.d[t];
            ss[t] = p.xq.sum[t];
        }
    }
    __syncthreads();

    float acc[kMaxCols];
#pragma unroll
    for (int n = 0; n < kMaxCols; n++) acc[n] = 0.0f;

    for (int i = 0; i < n_items; i++) {
        const int stage = i % p.nstage;
        const bool ok = mbar_wait_bounded(&bars[stage], (uint32_t)(i / p.nstage) & 1u);
        if (!__all_sync(0xffffffffu, ok)) {
            if (lane == 0) {
                report_status(p.status, STATUS_TIMEOUT);
                for (int j = i; j < issued; j++) mbar_wait_bounded(&bars[j % p.nstage], (uint32_t)(j / p.nstage) & 1u);
            }
            __syncwarp();
            return;
        }
        uintptr_t start;
        uint32_t len;
        int row, c;
        item_range(i, start, len, row, c);
        uint8_t *buf = ring + (uint32_t)stage * p.stage_bytes;
        const uintptr_t base = start & ~uintptr_t(15);
        const uintptr_t a = (start + 15) & ~uintptr_t(15);
        const uintptr_t e = (start + len) & ~uintptr_t(15);
        if (a != start || e != start + len) {  // ragged edges: plain byte loads
            const uint8_t *g = reinterpret_cast<const uint8_t *>(base);
            if (e > a) {
                for (uintptr_t t = start + lane; t < a; t += 32) buf[t - base] = g[t - base];
                for (uintptr_t t = e + lane; t < start + len; t += 32) buf[t - base] = g[t - base];
            } else {
                for (uintptr_t t = start + lane; t < start + len; t += 32) buf[t - base] = g[t - base];
            }
            __syncwarp();
        }
        const uint8_t *p0 = buf + (start - base);
        const int u0 = c * p.chunk_units;
        const int nu = (int)(len / UB);
        for (int u = lane; u < nu; u += 32) dot_unit<WT, NC>(p0, u, u0 + u, sq, sd, ss, K, nblk, acc);
        __syncwarp();
        if (lane == 0 && issued < n_items) {
            fence_proxy_async_smem();
            issue(issued);
        }
        issued = min(issued + 1, n_items);
        if (c == p.nchunks - 1) {
#pragma unroll
            for (int n = 0; n < NC; n++) {
                const float v = warp_sum(acc[n]);
                if (lane == 0) reinterpret_cast<float *>(p.y + (uint64_t)n * p.y_nb1)[row] = v;
                acc[n] = 0.0f;
            }
        }
    }
}

template <int WT, int NC>
int launch_typed(const GemvParams &p, int grid, uint32_t smem, cudaStream_t s, bool pdl) {
    auto kern = gemv_kernel<WT, NC>;
    static int smem_set[64] = {0};  // per device: largest dynamic smem size already granted
    int dev = 0;
    cudaGetDevice(&dev);
    cudaError_t e = cudaSuccess;
    if (dev < 0 || dev >= 64 || smem_set[dev] < (int)smem) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
        if (e != cudaSuccess) return fb::set_error(FB_ERR_CUDA, "gemv: smem attribute: %s", cudaGetErrorString(e));
        if (dev >= 0 && dev < 64) smem_set[dev] = kSmemLimit;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kGemvThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    e = cudaLaunchKernelEx(&cfg, kern, p);
    if (e != cudaSuccess) return fb::set_error(FB_ERR_CUDA, "gemv launch: %s", cudaGetErrorString(e));
    return FB_OK;
}

template <int WT>
int launch_cols(int ncols, const GemvParams &p, int grid, uint32_t smem, cudaStream_t s, bool pdl) {
    switch (ncols) {
    case 1: return launch_typed<WT, 1>(p, grid, smem, s, pdl);
    case 2: return launch_typed<WT, 2>(p, grid, smem, s, pdl);
    case 3: return launch_typed<WT, 3>(p, grid, smem, s, pdl);
    default: return launch_typed<WT, 4>(p, grid, smem, s, pdl);
    }
}

}  // namespace

bool gemv_supported(int32_t wtype, int64_t K, int64_t N) {
    if (wtype != WT_Q8_0 && wtype != WT_Q4_0 && wtype != WT_Q4_K) return false;
    if (N < 1 || N > kMaxCols) return false;
    if (K % (wtype == WT_Q4_K ? QKK : QK)) return false;
    // activations + at least two minimal stages per warp must fit
    const uint32_t ub = wtype == WT_Q8_0 ? Q8_0_BYTES : Q4_0_BYTES;
    const SmemLayout L = smem_layout((int)K, (int)N, 2, align16(8 * ub + 32));
    return K <= (1 << 20) && L.total <= (uint32_t)kSmemLimit;
}

bool gemv_fused_ok(int64_t K, int64_t N) { return K * N <= kFusedMaxElems; }

int launch_gemv(int32_t wtype, const void *w, uint64_t w_nb1, const void *x, uint64_t x_nb1, void *y, uint64_t y_nb1,
                int64_t K, int64_t M, int64_t N, const Q8Planar *xq, int32_t *status, cudaStream_t s, bool pdl) {
    if (!gemv_supported(wtype, K, N)) return fb::set_error(FB_ERR_UNSUPPORTED, "gemv: unsupported shape");
    if (M == 0) return FB_OK;
    if ((reinterpret_cast<uintptr_t>(w) & 1) || (w_nb1 & 1))
        return fb::set_error(FB_ERR_INVALID, "gemv: weight rows must be 2-byte aligned");
    if (!xq && ((reinterpret_cast<uintptr_t>(x) & 3) || (x_nb1 & 3)))
        return fb::set_error(FB_ERR_INVALID, "gemv: activations must be 4-byte aligned");
    if ((reinterpret_cast<uintptr_t>(y) & 3) || (y_nb1 & 3))
        return fb::set_error(FB_ERR_INVALID, "gemv: output must be 4-byte aligned");
    if (M > INT32_MAX) return fb::set_error(FB_ERR_UNSUPPORTED, "gemv: M too large");

    const int nunits = (int)(K / QK);
    const uint32_t ub = wtype == WT_Q8_0 ? Q8_0_BYTES : (wtype == WT_Q4_0 ? Q4_0_BYTES : Q4_K_BYTES / 8);
    const int sms = sm_count();
    int grid = (int)std::min<int64_t>(sms, (M + kGemvWarps - 1) / kGemvWarps);
    grid = std::max(grid, 1);

    // Ring sizing: a few stages per warp, chunks as large as the budget allows.
    const SmemLayout base = smem_layout((int)K, (int)N, 4, 0);
    const uint32_t budget = (uint32_t)kSmemLimit - base.total - 256;
    int units_fit = (int)((budget / (kGemvWarps * 4) - 32) / ub);
    units_fit = std::max(8, units_fit / 8 * 8);
    int chunk_units = std::min(units_fit, (nunits + 7) / 8 * 8);
    chunk_units = std::min(chunk_units, 512);  // keep chunks at most ~17 KB
    const int nchunks0 = (nunits + chunk_units - 1) / chunk_units;
    chunk_units = ((nunits + nchunks0 - 1) / nchunks0 + 7) / 8 * 8;  // balance the chunks of a row
    const int nchunks = (nunits + chunk_units - 1) / chunk_units;
    const uint32_t stage_bytes = align16((uint32_t)chunk_units * ub + 32);
    int nstage = 4;
    while (nstage > 2 && smem_layout((int)K, (int)N, nstage, stage_bytes).total > (uint32_t)kSmemLimit) nstage--;
    const SmemLayout L = smem_layout((int)K, (int)N, nstage, stage_bytes);
    if (L.total > (uint32_t)kSmemLimit) return fb::set_error(FB_ERR_UNSUPPORTED, "gemv: shared memory budget exceeded");

    GemvParams p;
    p.w = static_cast<const uint8_t *>(w);
    p.w_nb1 = w_nb1;
    p.x = static_cast<const uint8_t *>(x);
    p.x_nb1 = x_nb1;
    p.y = static_cast<uint8_t *>(y);
    p.y_nb1 = y_nb1;
    p.K = (int)K;
    p.M = (int)M;
    p.nchunks = nchunks;
    p.chunk_units = chunk_units;
    p.nstage = nstage;
    p.stage_bytes = stage_bytes;
    p.xq = xq ? *xq : Q8Planar{nullptr, nullptr, nullptr};
    p.status = status;
    const bool use_pdl = pdl && xq != nullptr;
    switch (wtype) {
    case WT_Q8_0: return launch_cols<WT_Q8_0>((int)N, p, grid, L.total, s, use_pdl);
    case WT_Q4_0: return launch_cols<WT_Q4_0>((int)N, p, grid, L.total, s, use_pdl);
    default: return launch_cols<WT_Q4_K>((int)N, p, grid, L.total, s, use_pdl);
    }
}

}  // namespace fbk
