// Decode-path mul_mat for quantized weights and small N (1..8 columns):
//   y[m, n] = sum_b scale(m, b, n) * sumi(m, b, n)
// with sumi the int32 dot product of one 32-element weight block and the
// matching Q8_0 activation block (dp4a), scale = d_w * d_x (Q8_0, Q4_0) or
// d_x * (d*sc, dmin*m terms) for Q4_K sub-blocks.
//
// B200 mapping. The kernel is HBM-bound (weights are read once):
//  - one CTA per SM with at most 112 KB of shared memory, so the CTA of the
//    next launch fits beside it; launches are chained with programmatic
//    dependent launch (PDL): a CTA streams its weights before waiting for the
//    preceding grid, so the weight stream of launch i+1 overlaps launch i;
//    activations are read and outputs written only after that wait;
//  - every warp owns a contiguous share of the CTA's rows and a private ring of
//    shared-memory stages; lane 0 streams row chunks with cp.async.bulk (TMA,
//    L2 evict-first) completing on per-stage mbarriers (bounded waits) and
//    re-arms a stage as soon as the warp has consumed it;
//  - activations are quantized to Q8_0 into shared memory by the CTA (one
//    thread per 32-element block), or copied from a planar buffer written by a
//    preceding quantize kernel (large N*K);
//  - the dot products run on 64-element pairs with aligned shared-memory loads
//    (kernels/dot.cuh); for one column and rows of at most 128 blocks the
//    activation words of a lane's pairs stay in registers for all rows and a
//    warp takes its rows two at a time (the time after the dependency wait,
//    not HBM, bounds a small decode GEMV chained with PDL);
//  - rows whose bytes are not 4-byte (Q4_K: 16-byte) aligned are copied into
//    the stage with plain loads instead of TMA; rows that are aligned but not
//    16-byte aligned get their ragged head/tail bytes by plain loads.
#include <cuda_runtime.h>

#include <algorithm>

#include "../host_common.h"
#include "common.cuh"
#include "dot.cuh"
#include "kernels.h"
#include "tmap.h"

namespace fbk {

namespace {

constexpr int kGemvWarps = 8;
constexpr int kGemvThreads = kGemvWarps * 32;
constexpr int kMaxCols = 8;
constexpr int kSmemLimit = 227 * 1024;
constexpr int kFusedMaxElems = 16384;            // N*K up to which each CTA quantizes x itself
// per-CTA smem that leaves room for the next launch's CTA (2 x (112 + 1
// reserved) KB of the SM's 228 KB)
constexpr uint32_t kCoResidentCta = 112 * 1024;
constexpr uint32_t kCoResidentActs = 40 * 1024;  // activation bytes up to which that budget is used

template <int WT>
struct Fmt;
template <>
struct Fmt<WT_Q8_0> {
    static constexpr int kUnitBytes = Q8_0_BYTES;  // one 32-element block
    static constexpr bool kShifted = true;
};
template <>
struct Fmt<WT_Q4_0> {
    static constexpr int kUnitBytes = Q4_0_BYTES;
    static constexpr bool kShifted = true;
};
template <>
struct Fmt<WT_Q4_K> {
    static constexpr int kUnitBytes = Q4_K_BYTES / 8;  // one 32-element sub-block
    static constexpr bool kShifted = false;
};
template <>
struct Fmt<WT_Q5_K> {
    static constexpr int kUnitBytes = Q5_K_BYTES / 8;
    static constexpr bool kShifted = false;
};
template <>
struct Fmt<WT_Q6_K> {
    static constexpr int kUnitBytes = 0;  // 210-byte super-blocks: sizes are counted in super-blocks
    static constexpr bool kShifted = false;
};
// K-quants: chunks are whole 256-element super-blocks of this many bytes.
template <int WT>
constexpr int super_bytes() {
    return WT == WT_Q4_K ? Q4_K_BYTES : (WT == WT_Q5_K ? Q5_K_BYTES : (WT == WT_Q6_K ? Q6_K_BYTES : 0));
}

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
    Q8Planar xq;      // xq.qs == nullptr: quantize in-kernel
    int32_t *status;
    bool x_vec16;     // activation columns are 16-byte aligned
    bool copy_rows;   // rows not aligned for the pair loads: plain copies
    bool norm;        // rms-normalize each activation column before quantizing it
    float norm_eps;
    PeerOut peer;     // peer.n > 0: outputs go to every peer's buffer, then a signal
    EpiAct epi;       // fused bias / SiLU on every output
};

__host__ __device__ inline uint32_t align16(uint32_t v) { return (v + 15u) & ~15u; }

struct SmemLayout {
    uint32_t bars, qs, sx2, d, sum, ring, total;
};

__host__ __device__ inline SmemLayout smem_layout(int K, int ncols, bool shifted, int nstage, uint32_t stage_bytes) {
    SmemLayout L;
    const uint32_t nblk = (uint32_t)K / QK;
    L.bars = 0;
    L.qs = align16(kGemvWarps * nstage * 8);
    L.sx2 = L.qs + align16((uint32_t)ncols * K);
    const uint32_t nbp = (nblk + 1) & ~1u;  // per-column stride of d/sum, even so pairs load as float2/int2
    L.d = L.sx2 + (shifted ? (uint32_t)ncols * ((nblk + 1) / 2) * kShiftWords * 4 : 0u);
    L.sum = L.d + align16(ncols * nbp * 4);
    L.ring = (L.sum + align16(ncols * nbp * 4) + 127u) & ~127u;
    L.total = L.ring + (uint32_t)kGemvWarps * nstage * stage_bytes;
    return L;
}

// Quantize one 32-element activation block with 4 lanes (an aligned lane
// group), 8 elements per lane: the same operations as quantize_q8_0_quad
// (d = amax/127, id = 1/d, q = roundf(x*id)). Writes the block's packed
// integers, f16-rounded scale and integer sum, and for even blocks of Q8_0 /
// Q4_0 the shifted copy read by the pair kernels. All 32 lanes of the warp
// must call it (`valid` false for padding groups). The load is separate so a
// caller can issue the loads of several blocks before quantizing any.
__device__ __forceinline__ void load_block_quarter(const float *xb, bool vec, bool valid, float (&v)[8]) {
    const int t = threadIdx.x & 3;  // quarter of the block
    if (valid) {
        const float *xe = xb + 8 * t;
        if (vec) {
            const float4 a = __ldg(reinterpret_cast<const float4 *>(xe));
            const float4 b = __ldg(reinterpret_cast<const float4 *>(xe) + 1);
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
            v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        } else {
#pragma unroll
            for (int i = 0; i < 8; i++) v[i] = __ldg(xe + i);
        }
    } else {
#pragma unroll
        for (int i = 0; i < 8; i++) v[i] = 0.0f;
    }
}

template <int WT>
__device__ __forceinline__ void quantize_block_quarter(const float (&v)[8], bool valid, bool even, int8_t *sq_blk,
                                                       uint32_t *sx2_blk, float *sd_b, int32_t *ss_b) {
    const int t = threadIdx.x & 3;  // quarter of the block
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) amax = fmaxf(amax, fabsf(v[i]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __frcp_rn(d) : 0.0f;
    uint32_t w[2];
    int s = 0;
#pragma unroll
    for (int k = 0; k < 2; k++) {
        const int q0 = (int)roundf(__fmul_rn(v[4 * k], id));
        const int q1 = (int)roundf(__fmul_rn(v[4 * k + 1], id));
        const int q2 = (int)roundf(__fmul_rn(v[4 * k + 2], id));
        const int q3 = (int)roundf(__fmul_rn(v[4 * k + 3], id));
        s += q0 + q1 + q2 + q3;
        w[k] = (uint32_t)(q0 & 0xff) | ((uint32_t)(q1 & 0xff) << 8) | ((uint32_t)(q2 & 0xff) << 16) |
               ((uint32_t)(q3 & 0xff) << 24);
    }
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    // the word just before this lane's pair (lane t-1's second word)
    const uint32_t prev = __shfl_up_sync(0xffffffffu, w[1], 1);
    if (!valid) return;
    reinterpret_cast<uint2 *>(sq_blk)[t] = make_uint2(w[0], w[1]);
    if (t == 0) {
        *sd_b = f16_bits_to_f32(__half_as_ushort(__float2half_rn(d)));
        *ss_b = s;
    }
    if constexpr (WT == WT_Q8_0 || WT == WT_Q4_0) {
        if (even) {
            // byte stream shifted by 2 with zeros at the ends (see make_shifted)
            if constexpr (WT == WT_Q8_0) {
                const uint32_t pw = t == 0 ? 0u : prev;
                sx2_blk[2 * t] = __funnelshift_r(pw, w[0], 16);
                sx2_blk[2 * t + 1] = __funnelshift_r(w[0], w[1], 16);
                if (t == 3) sx2_blk[8] = w[1] >> 16;
            } else {
                // low nibble half: words 0..3 -> shifted words 0..4; high half: 4..7 -> 5..9
                const uint32_t pw = (t == 0 || t == 2) ? 0u : prev;
                const int o = t < 2 ? 2 * t : 5 + 2 * (t - 2);
                sx2_blk[o] = __funnelshift_r(pw, w[0], 16);
                sx2_blk[o + 1] = __funnelshift_r(w[0], w[1], 16);
                if (t == 1) sx2_blk[4] = w[1] >> 16;
                if (t == 3) sx2_blk[9] = w[1] >> 16;
            }
        }
    }
}

// XR > 0: every row is one chunk and a lane's XR block pairs (lane, lane+32,
// ...) are the same in every row, so their activation words stay in
// registers instead of being re-read from shared memory for every row (the
// shared-memory reads of a row then are its weights only). Register use is
// capped so the next launch's CTA still fits beside this one.
template <int WT, int NC, int XR>
__global__ void __launch_bounds__(kGemvThreads, XR > 0 ? 2 : 1) gemv_kernel(const GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int UB = Fmt<WT>::kUnitBytes;
    constexpr bool SH = Fmt<WT>::kShifted;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int K = p.K, nblk = K / QK, npair_blk = (nblk + 1) / 2, nbp = 2 * npair_blk;
    const SmemLayout L = smem_layout(K, NC, SH, p.nstage, p.stage_bytes);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bars) + warp * p.nstage;
    int8_t *sq = reinterpret_cast<int8_t *>(smem + L.qs);
    uint32_t *sx2 = reinterpret_cast<uint32_t *>(smem + L.sx2);
    float *sd = reinterpret_cast<float *>(smem + L.d);
    int32_t *ss = reinterpret_cast<int32_t *>(smem + L.sum);
    uint8_t *ring = smem + L.ring + (uint32_t)warp * p.nstage * p.stage_bytes;

    // rows of this CTA, then a contiguous share per warp
    const int r_begin = (int)((int64_t)blockIdx.x * p.M / gridDim.x);
    const int r_end = (int)((int64_t)(blockIdx.x + 1) * p.M / gridDim.x);
    const int cta_rows = r_end - r_begin;
    const int w_begin = r_begin + cta_rows * warp / kGemvWarps;
    const int w_end = r_begin + cta_rows * (warp + 1) / kGemvWarps;
    const int n_items = (w_end - w_begin) * p.nchunks;
    constexpr bool KQ = super_bytes<WT>() > 0;
    // bytes of `nu` 32-element units (whole super-blocks for K-quants)
    auto units_bytes = [](uint32_t nu) -> uint32_t { return KQ ? nu / 8 * super_bytes<WT>() : nu * UB; };
    const uint32_t chunk_bytes = units_bytes((uint32_t)p.chunk_units);

    auto item_range = [&](int i, uintptr_t &start, uint32_t &len, int &row, int &c) {
        row = w_begin + i / p.nchunks;
        c = i % p.nchunks;
        const uint32_t u0 = (uint32_t)c * p.chunk_units;
        const uint32_t nu = min((uint32_t)p.chunk_units, (uint32_t)nblk - u0);
        start = reinterpret_cast<uintptr_t>(p.w + (uint64_t)row * p.w_nb1 + (uint64_t)c * chunk_bytes);
        len = units_bytes(nu);
    };

    const uint64_t policy = policy_evict_first();
    auto issue = [&](int i) {  // lane 0 only
        uintptr_t start;
        uint32_t len;
        int row, c;
        item_range(i, start, len, row, c);
        uint64_t *bar = &bars[i % p.nstage];
        const uintptr_t base = start & ~uintptr_t(15);
        const uintptr_t a = (start + 15) & ~uintptr_t(15);
        const uintptr_t e = (start + len) & ~uintptr_t(15);
        if (!p.copy_rows && e > a) {
            uint8_t *dst = ring + (uint32_t)(i % p.nstage) * p.stage_bytes;
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
    // Weight prefetch: every ring stage is issued before the dependency wait
    // (weights are never written by the kernels this one waits for).
    int issued = 0;
    if (lane == 0) {
        for (; issued < min(p.nstage, n_items); issued++) issue(issued);
        // rows beyond the ring go to L2 now, so the refills after the wait hit L2
        if (!p.copy_rows)
            for (int i = issued; i < n_items; i++) {
                uintptr_t start;
                uint32_t len;
                int row, c;
                item_range(i, start, len, row, c);
                const uintptr_t a = (start + 15) & ~uintptr_t(15), e = (start + len) & ~uintptr_t(15);
                if (e > a) bulk_prefetch_l2(reinterpret_cast<const void *>(a), (uint32_t)(e - a));
            }
    }
    issued = __shfl_sync(0xffffffffu, issued, 0);

    grid_launch_dependents();
    grid_dependency_wait();

    // Activations -> Q8_0 in shared memory.
    if (p.xq.qs == nullptr) {
        // Fused rms_norm (a plan's rms_norm feeding this mul_mat): column n is
        // scaled by 1 / sqrt(sum(x^2) / K + eps) before it is quantized; the
        // warps' partial sums are added in warp order (deterministic). The
        // scale area `sd` (not yet written) holds the partials (launch_gemv
        // requires K >= 512, so it has room for 9 * NC floats); every thread
        // keeps the NC scales in registers before quantization writes `sd`.
        float nscale[kMaxCols];
#pragma unroll
        for (int n = 0; n < kMaxCols; n++) nscale[n] = 1.0f;
        if (p.norm) {
#pragma unroll
            for (int n = 0; n < NC; n++) {
                const float *xc = reinterpret_cast<const float *>(p.x + (uint64_t)n * p.x_nb1);
                float ssq = 0.0f;
                for (int k = threadIdx.x; k < K; k += kGemvThreads) {
                    const float v = __ldg(xc + k);
                    ssq = fmaf(v, v, ssq);
                }
                ssq = warp_sum(ssq);
                if (lane == 0) sd[warp * NC + n] = ssq;
            }
            __syncthreads();
            if (threadIdx.x < NC) {
                float t = 0.0f;
#pragma unroll
                for (int w = 0; w < kGemvWarps; w++) t += sd[w * NC + threadIdx.x];
                sd[kGemvWarps * NC + threadIdx.x] = 1.0f / sqrtf(t / (float)K + p.norm_eps);
            }
            __syncthreads();
#pragma unroll
            for (int n = 0; n < NC; n++) nscale[n] = sd[kGemvWarps * NC + n];
            __syncthreads();
        }
        auto normalize = [&](int n, float (&v)[8]) {
            if (p.norm) {
                float sc = nscale[0];
#pragma unroll
                for (int j = 1; j < NC; j++)
                    if (n == j) sc = nscale[j];
#pragma unroll
                for (int i = 0; i < 8; i++) v[i] *= sc;
            }
        };
        constexpr int kGroups = kGemvThreads / 4;  // 4 lanes per block
        auto block_of = [&](int base, bool &valid, int &n, int &b) {
            const int t = base + (int)(threadIdx.x >> 2);
            valid = t < NC * nblk;
            n = !valid ? 0 : (NC == 1 ? 0 : t / nblk);
            b = !valid ? 0 : t - n * nblk;
        };
        auto xptr = [&](int n, int b) {
            return reinterpret_cast<const float *>(p.x + (uint64_t)n * p.x_nb1) + b * QK;
        };
        if (NC * nblk <= 2 * kGroups) {
            // both blocks' loads in flight before either is quantized (this
            // phase sits between the dependency wait and the first dot product)
            bool v0, v1;
            int n0, b0, n1, b1;
            block_of(0, v0, n0, b0);
            block_of(kGroups, v1, n1, b1);
            float x0[8], x1[8];
            load_block_quarter(xptr(n0, b0), p.x_vec16, v0, x0);
            load_block_quarter(xptr(n1, b1), p.x_vec16, v1, x1);
            normalize(n0, x0);
            normalize(n1, x1);
            quantize_block_quarter<WT>(x0, v0, SH && !(b0 & 1), sq + n0 * K + b0 * QK,
                                       sx2 + (n0 * npair_blk + b0 / 2) * kShiftWords, sd + n0 * nbp + b0,
                                       ss + n0 * nbp + b0);
            quantize_block_quarter<WT>(x1, v1, SH && !(b1 & 1), sq + n1 * K + b1 * QK,
                                       sx2 + (n1 * npair_blk + b1 / 2) * kShiftWords, sd + n1 * nbp + b1,
                                       ss + n1 * nbp + b1);
        } else {
#pragma unroll 2
            for (int base = 0; base < NC * nblk; base += kGroups) {  // uniform trip count
                bool valid;
                int n, b;
                block_of(base, valid, n, b);
                float xv[8];
                load_block_quarter(xptr(n, b), p.x_vec16, valid, xv);
                normalize(n, xv);
                quantize_block_quarter<WT>(xv, valid, SH && !(b & 1), sq + n * K + b * QK,
                                           sx2 + (n * npair_blk + b / 2) * kShiftWords, sd + n * nbp + b,
                                           ss + n * nbp + b);
            }
        }
    } else {
        const int4 *src = reinterpret_cast<const int4 *>(p.xq.qs);
        int4 *dst = reinterpret_cast<int4 *>(sq);
        for (int t = threadIdx.x; t < NC * K / 16; t += kGemvThreads) dst[t] = src[t];
        for (int t = threadIdx.x; t < NC * nblk; t += kGemvThreads) {
            const int n = NC == 1 ? 0 : t / nblk;
            sd[t + n * (nbp - nblk)] = p.xq.d[t];
            ss[t + n * (nbp - nblk)] = p.xq.sum[t];
        }
        if constexpr (SH) {
            __syncthreads();
            for (int t = threadIdx.x; t < NC * npair_blk; t += kGemvThreads) {
                const int n = NC == 1 ? 0 : t / npair_blk;
                const int b = 2 * (t - n * npair_blk);
                const uint4 *q = reinterpret_cast<const uint4 *>(sq + n * K + b * QK);
                const uint4 q0 = q[0], q1 = q[1];
                const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
                uint32_t sh[kShiftWords];
                make_shifted<WT>(w, sh);
                uint4 *o = reinterpret_cast<uint4 *>(sx2 + t * kShiftWords);
                o[0] = make_uint4(sh[0], sh[1], sh[2], sh[3]);
                o[1] = make_uint4(sh[4], sh[5], sh[6], sh[7]);
                o[2] = make_uint4(sh[8], sh[9], sh[10], sh[11]);
            }
        }
    }
    __syncthreads();

    float acc[kMaxCols];
#pragma unroll
    for (int n = 0; n < kMaxCols; n++) acc[n] = 0.0f;

    constexpr int XRN = XR > 0 ? XR : 1;
    XFrag xf[XRN];
    int2 xsr[XRN];
    float2 dxr[XRN];
    if constexpr (XR > 0) {
#pragma unroll
        for (int j = 0; j < XR; j++) {
            const int pr = lane + 32 * j, b0 = 2 * pr;
            if (2 * pr + 1 < nblk) {
                xf[j] = load_xfrag(sx2 + (b0 / 2) * kShiftWords, reinterpret_cast<const uint32_t *>(sq + (b0 + 1) * QK));
                xsr[j] = *reinterpret_cast<const int2 *>(ss + b0);
                dxr[j] = *reinterpret_cast<const float2 *>(sd + b0);
            }
        }
    }

    // output row `row`, column n: this rank's buffer or every peer's
    auto store_row = [&](int n, int row, float v) {
        v = apply_act(v, p.epi, row);
        if (p.peer.n == 0) {
            reinterpret_cast<float *>(p.y + (uint64_t)n * p.y_nb1)[row] = v;
        } else {
            const int b = (int)((*p.peer.epoch + 1u) & 1u);
            for (int r = 0; r < p.peer.n; r++)  // NVLink stores into each rank's output
                reinterpret_cast<float *>(p.peer.y[b][r] + (uint64_t)n * p.y_nb1)[row] = v;
        }
    };

    if constexpr (XR > 0) {
        // Whole 16-byte-aligned rows, two at a time: the two rows' dot
        // products and warp reductions interleave, and both stages are
        // re-armed together.
        const int nu = nblk, np = nu / 2;
        for (int i = 0; i < n_items; i += 2) {
            const bool two = i + 1 < n_items;
            bool ok = mbar_wait_bounded(&bars[i % p.nstage], (uint32_t)(i / p.nstage) & 1u);
            if (two) ok = ok && mbar_wait_bounded(&bars[(i + 1) % p.nstage], (uint32_t)((i + 1) / p.nstage) & 1u);
            if (!__all_sync(0xffffffffu, ok)) {
                if (lane == 0) {
                    report_status(p.status, STATUS_TIMEOUT);
                    for (int j = i; j < issued; j++)
                        mbar_wait_bounded(&bars[j % p.nstage], (uint32_t)(j / p.nstage) & 1u);
                }
                __syncwarp();
                return;
            }
            const uint8_t *r0 = ring + (uint32_t)(i % p.nstage) * p.stage_bytes;
            const uint8_t *r1 = ring + (uint32_t)((i + 1) % p.nstage) * p.stage_bytes;
            float a0 = 0.0f, a1 = 0.0f;
#pragma unroll
            for (int j = 0; j < XR; j++) {
                const int pr = lane + 32 * j;
                if (pr < np) {
                    int s0, s1;
                    float d0, d1;
                    pair_dot_frag<WT>(reinterpret_cast<const uint32_t *>(r0 + 2 * UB * pr), xf[j], xsr[j].x,
                                      xsr[j].y, s0, s1, d0, d1);
                    a0 += (d0 * dxr[j].x) * (float)s0 + (d1 * dxr[j].y) * (float)s1;
                    if (two) {
                        pair_dot_frag<WT>(reinterpret_cast<const uint32_t *>(r1 + 2 * UB * pr), xf[j], xsr[j].x,
                                          xsr[j].y, s0, s1, d0, d1);
                        a1 += (d0 * dxr[j].x) * (float)s0 + (d1 * dxr[j].y) * (float)s1;
                    }
                }
            }
            if ((nu & 1) && lane == (np & 31)) {  // trailing unpaired block of an odd-length row
                const int b0 = 2 * np;
                const uint32_t *xe = sx2 + (b0 / 2) * kShiftWords;
                float d0;
                const int s0 = single_even_dot<WT>(reinterpret_cast<const uint32_t *>(r0 + 2 * UB * np), xe, ss[b0], d0);
                a0 += (d0 * sd[b0]) * (float)s0;
                if (two) {
                    const int s1 = single_even_dot<WT>(reinterpret_cast<const uint32_t *>(r1 + 2 * UB * np), xe,
                                                       ss[b0], d0);
                    a1 += (d0 * sd[b0]) * (float)s1;
                }
            }
            __syncwarp();
            if (lane == 0 && issued < n_items) {
                fence_proxy_async_smem();
                issue(issued);
                if (two && issued + 1 < n_items) issue(issued + 1);
            }
            issued = min(issued + (two ? 2 : 1), n_items);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {  // the two rows' butterflies interleaved
                a0 += __shfl_xor_sync(0xffffffffu, a0, o);
                a1 += __shfl_xor_sync(0xffffffffu, a1, o);
            }
            if (lane == 0) {
                store_row(0, w_begin + i, a0);
                if (two) store_row(0, w_begin + i + 1, a1);
            }
        }
    }

    for (int i = 0; i < (XR > 0 ? 0 : n_items); i++) {
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
        const uint8_t *p0;
        if (p.copy_rows) {  // 2-byte-aligned rows: plain copy to the aligned stage start
            const uint16_t *g = reinterpret_cast<const uint16_t *>(start);
            uint16_t *d = reinterpret_cast<uint16_t *>(buf);
            for (uint32_t t = lane; t < len / 2; t += 32) d[t] = g[t];
            __syncwarp();
            p0 = buf;
        } else {
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
            p0 = buf + (start - base);
        }
        const int u0 = c * p.chunk_units;
        const int nu = KQ ? (int)(len / super_bytes<WT>()) * 8 : (int)(len / UB);
        const int np = nu / 2;  // pairs in this chunk
        if constexpr (WT == WT_Q6_K) {
#pragma unroll 2
            for (int pr = lane; pr < np; pr += 32) {
                const int b0 = u0 + 2 * pr;  // sub-block index within the row
                const uint8_t *sb = p0 + Q6_K_BYTES * (pr >> 2);  // its super-block (2-byte aligned)
                const int g = pr & 3;
#pragma unroll
                for (int n = 0; n < NC; n++) {
                    const uint32_t *xa = reinterpret_cast<const uint32_t *>(sq + n * K + b0 * QK);
                    int s0, s1;
                    float d;
                    q6k_pair_dot(sb, g, xa, xa + 8, s0, s1, d);
                    const float2 dx = *reinterpret_cast<const float2 *>(sd + n * nbp + b0);
                    acc[n] += dx.x * (d * (float)s0) + dx.y * (d * (float)s1);
                }
            }
        } else if constexpr (WT == WT_Q4_K || WT == WT_Q5_K) {
#pragma unroll 2
            for (int pr = lane; pr < np; pr += 32) {
                const int b0 = u0 + 2 * pr;  // sub-block index within the row
                const uint8_t *sb = p0 + super_bytes<WT>() * (pr >> 2);  // its super-block
                const int g = pr & 3;
#pragma unroll
                for (int n = 0; n < NC; n++) {
                    const uint32_t *xa = reinterpret_cast<const uint32_t *>(sq + n * K + b0 * QK);
                    int s0, s1;
                    float dsc0, dmm0, dsc1, dmm1;
                    if constexpr (WT == WT_Q4_K)
                        q4k_pair_dot(sb, g, xa, xa + 8, s0, s1, dsc0, dmm0, dsc1, dmm1);
                    else
                        q5k_pair_dot(sb, g, xa, xa + 8, s0, s1, dsc0, dmm0, dsc1, dmm1);
                    const float2 dx = *reinterpret_cast<const float2 *>(sd + n * nbp + b0);
                    const int2 xs = *reinterpret_cast<const int2 *>(ss + n * nbp + b0);
                    acc[n] += dx.x * (dsc0 * (float)s0 - dmm0 * (float)xs.x) +
                              dx.y * (dsc1 * (float)s1 - dmm1 * (float)xs.y);
                }
            }
        } else {
#pragma unroll 2
            for (int pr = lane; pr < np; pr += 32) {
                const int b0 = u0 + 2 * pr;  // even block index within the row
                const uint32_t *wp = reinterpret_cast<const uint32_t *>(p0 + 2 * UB * pr);
#pragma unroll
                for (int n = 0; n < NC; n++) {
                    const uint32_t *xe = sx2 + (n * npair_blk + b0 / 2) * kShiftWords;
                    const uint32_t *xo = reinterpret_cast<const uint32_t *>(sq + n * K + (b0 + 1) * QK);
                    const int2 xs = *reinterpret_cast<const int2 *>(ss + n * nbp + b0);
                    int s0, s1;
                    float d0, d1;
                    pair_dot<WT>(wp, xe, xo, xs.x, xs.y, s0, s1, d0, d1);
                    const float2 dx = *reinterpret_cast<const float2 *>(sd + n * nbp + b0);
                    acc[n] += (d0 * dx.x) * (float)s0 + (d1 * dx.y) * (float)s1;
                }
            }
            if ((nu & 1) && lane == (np & 31)) {  // trailing unpaired block of an odd-length row
                const int b0 = u0 + 2 * np;
                const uint32_t *wp = reinterpret_cast<const uint32_t *>(p0 + 2 * UB * np);
#pragma unroll
                for (int n = 0; n < NC; n++) {
                    const uint32_t *xe = sx2 + (n * npair_blk + b0 / 2) * kShiftWords;
                    float d0;
                    const int s0 = single_even_dot<WT>(wp, xe, ss[n * nbp + b0], d0);
                    acc[n] += (d0 * sd[n * nbp + b0]) * (float)s0;
                }
            }
        }
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
                if (lane == 0) store_row(n, row, v);
                acc[n] = 0.0f;
            }
        }
    }
    if (p.peer.n > 0) {
        // Every warp publishes its stores (system scope) and counts itself
        // done; the last warp of the grid resets the counter and raises each
        // rank's flag by one. Ranks wait for `world` raises per step.
        __syncwarp();
        if (lane == 0) {
            __threadfence_system();
            const uint32_t prev = atomicAdd(p.peer.count, 1u);
            if (prev == gridDim.x * kGemvWarps - 1) {
                atomicExch(p.peer.count, 0u);
                __threadfence_system();
                for (int r = 0; r < p.peer.n; r++) atomicAdd_system(p.peer.flag[r], 1u);
            }
        }
    }
}

// ---- K-split decode GEMV for wide Q4_K rows, one column ---------------------
// Every warp of a CTA takes one eighth of K (a run of whole super-blocks) for
// all the CTA's rows, so a lane's activation words (one or two sub-block
// pairs of the warp's slice) are the same for the whole launch: the lane
// quantizes them itself, straight into registers, right after the dependency
// wait (no shared-memory activations and no CTA barrier before the rows).
// Boxes of kKsRows rows x the warp's slice come by 2D TMA into a per-warp
// ring; the eight slices' partial sums of a row meet in shared memory and are
// added in warp order.
constexpr int kKsRows = 4;    // rows per TMA box
constexpr int kKsStages = 2;  // ring stages per warp (Q4_K 14336 x 4096, one column: 3 stages 11.9 us, 2 stages 11.4 us)

struct KsParams {
    const float *x;
    uint8_t *y;
    int M;
    int nsb;             // super-blocks per row
    uint32_t box_bytes;  // bytes of one row of a box (the widest warp slice)
    uint32_t ring_off;   // shared-memory offset of the rings
    int32_t *status;
    bool x_vec16;
    PeerOut peer;        // peer.n > 0: outputs go to every peer's buffer, then a signal
    EpiAct epi;          // fused bias / SiLU on every output
};

// One 32-element activation block quantized by a single lane: the operations
// of quantize_block_quarter (d = amax/127 rounded to f16 for the scale,
// q = roundf(x * (1/d))), giving the packed int8 words, the scale and the
// integer sum.
__device__ __forceinline__ void quantize_block_lane(const float *xb, bool vec, uint4 &w0, uint4 &w1, float &dq,
                                                    int &sum) {
    float v[QK];
    if (vec) {
#pragma unroll
        for (int i = 0; i < QK / 4; i++) {
            const float4 a = __ldg(reinterpret_cast<const float4 *>(xb) + i);
            v[4 * i] = a.x, v[4 * i + 1] = a.y, v[4 * i + 2] = a.z, v[4 * i + 3] = a.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < QK; i++) v[i] = __ldg(xb + i);
    }
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < QK; i++) amax = fmaxf(amax, fabsf(v[i]));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __frcp_rn(d) : 0.0f;
    uint32_t w[8];
    int s = 0;
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const int q0 = (int)roundf(__fmul_rn(v[4 * k], id));
        const int q1 = (int)roundf(__fmul_rn(v[4 * k + 1], id));
        const int q2 = (int)roundf(__fmul_rn(v[4 * k + 2], id));
        const int q3 = (int)roundf(__fmul_rn(v[4 * k + 3], id));
        s += q0 + q1 + q2 + q3;
        w[k] = (uint32_t)(q0 & 0xff) | ((uint32_t)(q1 & 0xff) << 8) | ((uint32_t)(q2 & 0xff) << 16) |
               ((uint32_t)(q3 & 0xff) << 24);
    }
    w0 = make_uint4(w[0], w[1], w[2], w[3]);
    w1 = make_uint4(w[4], w[5], w[6], w[7]);
    dq = f16_bits_to_f32(__half_as_ushort(__float2half_rn(d)));
    sum = s;
}

// XP: sub-block pairs per lane (the widest warp slice has at most 32 * XP).
template <int XP>
__global__ void __launch_bounds__(kGemvThreads, 2) gemv_ks_kernel(const __grid_constant__ CUtensorMap tm,
                                                                  const KsParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r_begin = (int)((int64_t)blockIdx.x * p.M / gridDim.x);
    const int r_end = (int)((int64_t)(blockIdx.x + 1) * p.M / gridDim.x);
    const int rows = r_end - r_begin;
    const int n_items = (rows + kKsRows - 1) / kKsRows;
    const int sb0 = warp * p.nsb / kGemvWarps, sb1 = (warp + 1) * p.nsb / kGemvWarps;
    const int npairs = 4 * (sb1 - sb0);  // sub-block pairs of this warp's slice
    const uint32_t box_total = kKsRows * p.box_bytes;                  // bytes one box writes
    const uint32_t stage_bytes = (box_total + 127u) & ~127u;           // stages start 128-byte aligned
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem) + warp * kKsStages;
    float *part = reinterpret_cast<float *>(smem + 256);  // [rows][warp]
    uint8_t *ring = smem + p.ring_off + (uint32_t)warp * kKsStages * stage_bytes;

    auto issue = [&](int i) {  // lane 0 only
        uint64_t *bar = &bars[i % kKsStages];
        mbar_arrive_expect_tx(bar, box_total);
        tma_load_2d(smem_u32(ring + (uint32_t)(i % kKsStages) * stage_bytes), &tm, sb0 * (Q4_K_BYTES / 8),
                    r_begin + i * kKsRows, smem_u32(bar));
    };
    if (lane == 0) {
        for (int st = 0; st < kKsStages; st++) mbar_init(&bars[st], 1);
        fence_barrier_init();
    }
    __syncwarp();
    // weight boxes before the dependency wait (weights are never written by
    // the kernels this one waits for)
    int issued = 0;
    if (lane == 0)
        for (; issued < min(kKsStages, n_items); issued++) issue(issued);
    issued = __shfl_sync(0xffffffffu, issued, 0);

    grid_launch_dependents();
    grid_dependency_wait();

    uint4 xa0[XP], xa1[XP], xb0[XP], xb1[XP];
    float dxa[XP], dxb[XP];
    int sxa[XP], sxb[XP];
#pragma unroll
    for (int j = 0; j < XP; j++) {
        const int q = lane + 32 * j;
        if (q < npairs) {
            const float *xp = p.x + (size_t)(sb0 + q / 4) * QKK + (q % 4) * 2 * QK;
            quantize_block_lane(xp, p.x_vec16, xa0[j], xa1[j], dxa[j], sxa[j]);
            quantize_block_lane(xp + QK, p.x_vec16, xb0[j], xb1[j], dxb[j], sxb[j]);
        } else {
            xa0[j] = xa1[j] = xb0[j] = xb1[j] = make_uint4(0u, 0u, 0u, 0u);
            dxa[j] = dxb[j] = 0.0f;
            sxa[j] = sxb[j] = 0;
        }
    }

    // Up to kKsDefer boxes (all of a CTA's rows when it has at most 32): the
    // lane keeps its partial sum of every row in registers and the warp
    // reduces them once at the end with a transposing butterfly (31 shuffles,
    // lane l ends with row l), instead of a 5-level reduction after each box.
    constexpr int kKsDefer = 32 / kKsRows;
    if (n_items <= kKsDefer) {
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; j++) v[j] = 0.0f;
#pragma unroll
        for (int i = 0; i < kKsDefer; i++) {
            if (i >= n_items) break;
            const int stage = i % kKsStages;
            const bool ok = mbar_wait_bounded(&bars[stage], (uint32_t)(i / kKsStages) & 1u);
            if (!__all_sync(0xffffffffu, ok)) {
                if (lane == 0) {
                    report_status(p.status, STATUS_TIMEOUT);
                    for (int j = i; j < issued; j++)
                        mbar_wait_bounded(&bars[j % kKsStages], (uint32_t)(j / kKsStages) & 1u);
                }
                break;
            }
            const uint8_t *st = ring + (uint32_t)stage * stage_bytes;
#pragma unroll
            for (int r = 0; r < kKsRows; r++) {
#pragma unroll
                for (int j = 0; j < XP; j++) {
                    const int q = lane + 32 * j;
                    if (q < npairs) {
                        int s0, s1;
                        float dsc0, dmm0, dsc1, dmm1;
                        q4k_pair_dot_x(st + r * p.box_bytes + (q / 4) * Q4_K_BYTES, q % 4, xa0[j], xa1[j], xb0[j],
                                       xb1[j], s0, s1, dsc0, dmm0, dsc1, dmm1);
                        v[i * kKsRows + r] += dxa[j] * (dsc0 * (float)s0 - dmm0 * (float)sxa[j]) +
                                              dxb[j] * (dsc1 * (float)s1 - dmm1 * (float)sxb[j]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0 && issued < n_items) {
                fence_proxy_async_smem();
                issue(issued);
            }
            issued = min(issued + 1, n_items);
        }
#pragma unroll
        for (int o = 16, cnt = 16; o >= 1; o >>= 1, cnt >>= 1) {
            const bool upper = (lane & o) != 0;
#pragma unroll
            for (int j = 0; j < cnt; j++) {
                const float send = upper ? v[j] : v[j + cnt];
                const float keep = upper ? v[j + cnt] : v[j];
                v[j] = keep + __shfl_xor_sync(0xffffffffu, send, o);
            }
        }
        if (lane < rows) part[lane * kGemvWarps + warp] = v[0];
    } else
    for (int i = 0; i < n_items; i++) {
        const int stage = i % kKsStages;
        const bool ok = mbar_wait_bounded(&bars[stage], (uint32_t)(i / kKsStages) & 1u);
        if (!__all_sync(0xffffffffu, ok)) {
            if (lane == 0) {
                report_status(p.status, STATUS_TIMEOUT);
                for (int j = i; j < issued; j++)
                    mbar_wait_bounded(&bars[j % kKsStages], (uint32_t)(j / kKsStages) & 1u);
            }
            break;
        }
        const uint8_t *st = ring + (uint32_t)stage * stage_bytes;
        float a[kKsRows];
#pragma unroll
        for (int r = 0; r < kKsRows; r++) {
            a[r] = 0.0f;
#pragma unroll
            for (int j = 0; j < XP; j++) {
                const int q = lane + 32 * j;
                if (q < npairs) {
                    int s0, s1;
                    float dsc0, dmm0, dsc1, dmm1;
                    q4k_pair_dot_x(st + r * p.box_bytes + (q / 4) * Q4_K_BYTES, q % 4, xa0[j], xa1[j], xb0[j],
                                   xb1[j], s0, s1, dsc0, dmm0, dsc1, dmm1);
                    a[r] += dxa[j] * (dsc0 * (float)s0 - dmm0 * (float)sxa[j]) +
                            dxb[j] * (dsc1 * (float)s1 - dmm1 * (float)sxb[j]);
                }
            }
        }
        __syncwarp();
        if (lane == 0 && issued < n_items) {
            fence_proxy_async_smem();
            issue(issued);
        }
        issued = min(issued + 1, n_items);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int r = 0; r < kKsRows; r++) a[r] += __shfl_xor_sync(0xffffffffu, a[r], o);
        if (lane == 0) {
#pragma unroll
            for (int r = 0; r < kKsRows; r++) {
                const int row = i * kKsRows + r;
                if (row < rows) part[row * kGemvWarps + warp] = a[r];
            }
        }
    }
    __syncthreads();
    for (int t = threadIdx.x; t < rows; t += kGemvThreads) {
        float v = part[t * kGemvWarps];
#pragma unroll
        for (int w = 1; w < kGemvWarps; w++) v += part[t * kGemvWarps + w];
        v = apply_act(v, p.epi, r_begin + t);
        if (p.peer.n == 0) {
            reinterpret_cast<float *>(p.y)[r_begin + t] = v;
        } else {
            const int b = (int)((*p.peer.epoch + 1u) & 1u);
            for (int r = 0; r < p.peer.n; r++)  // NVLink stores into each rank's output
                reinterpret_cast<float *>(p.peer.y[b][r])[r_begin + t] = v;
        }
    }
    if (p.peer.n > 0) {
        // every thread publishes its stores (system scope), then the CTA
        // counts itself done; the grid's last CTA resets the counter and
        // raises each rank's flag by one (ranks wait for `world` raises)
        __threadfence_system();
        __syncthreads();
        if (threadIdx.x == 0) {
            if (atomicAdd(p.peer.count, 1u) == gridDim.x - 1) {
                atomicExch(p.peer.count, 0u);
                __threadfence_system();
                for (int r = 0; r < p.peer.n; r++) atomicAdd_system(p.peer.flag[r], 1u);
            }
        }
    }
}

// ---- K-split decode GEMV for wide Q4_K rows, 2..8 columns -------------------
// The same slices and 2D boxes as gemv_ks_kernel; the activations were
// quantized by a preceding kernel into planar form. After the
// programmatic-dependent-launch wait each warp copies the int8 words of its
// slice into shared memory, transposed to [column][16-byte quarter][pair] so
// that a lane's loads of its pair are conflict-free; block scales and sums
// are read through L1. A lane holds the weight words and scale terms of its
// sub-block pair for all rows of a box in registers and walks the columns.
// The box's kKsRows x NC partial sums (padded to 32) are reduced across the
// warp with a transposing butterfly (31 shuffles, lane l ends with value l)
// and meet the other slices in shared memory, added in warp order.
struct KsColsParams {
    Q8Planar xq;
    uint8_t *y;
    uint64_t y_nb1;
    int K;
    int M;
    int nsb;
    uint32_t box_bytes;
    uint32_t ring_off;
    uint32_t xs_off;  // shared-memory offset of the staged activations
    int32_t *status;
    EpiAct epi;       // fused bias / SiLU on every output
};

template <int NC>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_ks_cols_kernel(const __grid_constant__ CUtensorMap tm,
                                                                       const KsColsParams p) {
    static_assert(kKsRows * NC <= 32, "one reduced value per lane");
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r_begin = (int)((int64_t)blockIdx.x * p.M / gridDim.x);
    const int r_end = (int)((int64_t)(blockIdx.x + 1) * p.M / gridDim.x);
    const int rows = r_end - r_begin;
    const int n_items = (rows + kKsRows - 1) / kKsRows;
    const int sb0 = warp * p.nsb / kGemvWarps, sb1 = (warp + 1) * p.nsb / kGemvWarps;
    const int npairs = 4 * (sb1 - sb0);
    const uint32_t box_total = kKsRows * p.box_bytes;
    const uint32_t stage_bytes = (box_total + 127u) & ~127u;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem) + warp * kKsStages;
    float *part = reinterpret_cast<float *>(smem + 256);  // [rows][NC][warp]
    uint8_t *ring = smem + p.ring_off + (uint32_t)warp * kKsStages * stage_bytes;

    auto issue = [&](int i) {  // lane 0 only
        uint64_t *bar = &bars[i % kKsStages];
        mbar_arrive_expect_tx(bar, box_total);
        tma_load_2d(smem_u32(ring + (uint32_t)(i % kKsStages) * stage_bytes), &tm, sb0 * (Q4_K_BYTES / 8),
                    r_begin + i * kKsRows, smem_u32(bar));
    };
    if (lane == 0) {
        for (int st = 0; st < kKsStages; st++) mbar_init(&bars[st], 1);
        fence_barrier_init();
    }
    __syncwarp();
    int issued = 0;
    if (lane == 0)
        for (; issued < min(kKsStages, n_items); issued++) issue(issued);
    issued = __shfl_sync(0xffffffffu, issued, 0);

    grid_launch_dependents();
    grid_dependency_wait();

    const bool active = lane < npairs;
    const int g = lane & 3;                              // pair within the super-block
    const int b0 = (sb0 + (lane >> 2)) * 8 + 2 * g;      // its even sub-block in the row
    const int nblk = p.K / QK;
    // this warp's activation words: [n][quarter j][pair], 16 bytes each
    const int pmax = 4 * ((p.nsb + kGemvWarps - 1) / kGemvWarps);  // pairs of the widest slice
    uint4 *xs = reinterpret_cast<uint4 *>(smem + p.xs_off) + (size_t)warp * NC * 4 * pmax;
    if (active) {
#pragma unroll
        for (int n = 0; n < NC; n++) {
            const uint4 *src = reinterpret_cast<const uint4 *>(p.xq.qs + (size_t)n * p.K + (size_t)b0 * QK);
            uint4 v[4];
#pragma unroll
            for (int j = 0; j < 4; j++) v[j] = __ldg(src + j);
#pragma unroll
            for (int j = 0; j < 4; j++) xs[(n * 4 + j) * pmax + lane] = v[j];
        }
    }
    __syncwarp();
    for (int i = 0; i < n_items; i++) {
        const int stage = i % kKsStages;
        const bool ok = mbar_wait_bounded(&bars[stage], (uint32_t)(i / kKsStages) & 1u);
        if (!__all_sync(0xffffffffu, ok)) {
            if (lane == 0) {
                report_status(p.status, STATUS_TIMEOUT);
                for (int j = i; j < issued; j++)
                    mbar_wait_bounded(&bars[j % kKsStages], (uint32_t)(j / kKsStages) & 1u);
            }
            break;
        }
        const uint8_t *st = ring + (uint32_t)stage * stage_bytes;
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; j++) v[j] = 0.0f;
        if (active) {
            Q4kPair wr[kKsRows];
#pragma unroll
            for (int r = 0; r < kKsRows; r++) wr[r] = q4k_pair_load(st + r * p.box_bytes + (lane >> 2) * Q4_K_BYTES, g);
#pragma unroll
            for (int n = 0; n < NC; n++) {
                const uint4 *xa = xs + n * 4 * pmax + lane;
                const uint4 a0 = xa[0], a1 = xa[pmax], c0 = xa[2 * pmax], c1 = xa[3 * pmax];
                const float2 dx = __ldg(reinterpret_cast<const float2 *>(p.xq.d + (size_t)n * nblk + b0));
                const int2 sx = __ldg(reinterpret_cast<const int2 *>(p.xq.sum + (size_t)n * nblk + b0));
#pragma unroll
                for (int r = 0; r < kKsRows; r++) {
                    int s0, s1;
                    q4k_pair_sums(wr[r].q0, wr[r].q1, a0, a1, c0, c1, s0, s1);
                    v[r * NC + n] = dx.x * (wr[r].dsc0 * (float)s0 - wr[r].dmm0 * (float)sx.x) +
                                    dx.y * (wr[r].dsc1 * (float)s1 - wr[r].dmm1 * (float)sx.y);
                }
            }
        }
        __syncwarp();
        if (lane == 0 && issued < n_items) {
            fence_proxy_async_smem();
            issue(issued);
        }
        issued = min(issued + 1, n_items);
        // transposing butterfly: after the step with offset o a lane keeps the
        // half of its values selected by its lane bit o, plus its partner's
        // copy of that half; lane l ends with the warp's sum of value l
#pragma unroll
        for (int o = 16, cnt = 16; o >= 1; o >>= 1, cnt >>= 1) {
            const bool upper = (lane & o) != 0;
#pragma unroll
            for (int j = 0; j < cnt; j++) {
                const float send = upper ? v[j] : v[j + cnt];
                const float keep = upper ? v[j + cnt] : v[j];
                v[j] = keep + __shfl_xor_sync(0xffffffffu, send, o);
            }
        }
        const int r = lane / NC, n = lane % NC, row = i * kKsRows + r;
        if (r < kKsRows && row < rows) part[(row * NC + n) * kGemvWarps + warp] = v[0];
    }
    __syncthreads();
    for (int t = threadIdx.x; t < rows * NC; t += kGemvThreads) {
        float sum = part[t * kGemvWarps];
#pragma unroll
        for (int w = 1; w < kGemvWarps; w++) sum += part[t * kGemvWarps + w];
        const int row = t / NC, n = t % NC;
        reinterpret_cast<float *>(p.y + (uint64_t)n * p.y_nb1)[r_begin + row] = apply_act(sum, p.epi, r_begin + row);
    }
}

// Waits (one thread) until every rank has signalled this step: the flag
// reaches (epoch + 1) * n_ranks; then advances the epoch. The wait is
// bounded twice: by `timeout_ns` of the GPU's global timer and by a poll
// count (each poll sleeps at least 32 ns, so the count alone ends it within
// a few seconds). On expiry it raises STATUS_TIMEOUT and returns, leaving
// the context usable (the epoch stays, so later waits report too).
// Launched with programmatic dependent launch: it lets the next step's GEMV
// start streaming its weights right away, but reads the epoch only after the
// preceding grids (this step's GEMV, and through it the previous wait) have
// completed.
__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__global__ void peer_wait_kernel(const uint32_t *flag, uint32_t *epoch, int n_ranks, uint64_t timeout_ns,
                                 int32_t *status) {
    grid_launch_dependents();
    grid_dependency_wait();
    if (threadIdx.x != 0) return;
    const uint32_t e = *epoch;
    const uint32_t expected = (e + 1u) * (uint32_t)n_ranks;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t i = 0; i < (1u << 24); i++) {
        uint32_t v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
        if ((int32_t)(v - expected) >= 0) {
            *epoch = e + 1u;
            return;
        }
        if ((i & 15u) == 15u && global_timer_ns() - t0 > timeout_ns) break;
        __nanosleep(32);
    }
    report_status(status, STATUS_TIMEOUT);
}

template <int WT, int NC, int XR>
int launch_typed(const GemvParams &p, int grid, uint32_t smem, cudaStream_t s, bool pdl) {
    auto kern = gemv_kernel<WT, NC, XR>;
    static DeviceFlags smem_set;
    const int rc = raise_smem_limit((const void *)kern, kSmemLimit, smem_set, "gemv");
    if (rc) return rc;
    cudaError_t e;
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

// xr: activation pairs per lane held in registers (0: read from shared memory)
template <int WT>
int launch_cols(int ncols, int xr, const GemvParams &p, int grid, uint32_t smem, cudaStream_t s, bool pdl) {
    if constexpr (WT == WT_Q8_0 || WT == WT_Q4_0) {
        if (ncols == 1 && xr == 1) return launch_typed<WT, 1, 1>(p, grid, smem, s, pdl);
        if (ncols == 1 && xr == 2) return launch_typed<WT, 1, 2>(p, grid, smem, s, pdl);
    }
    switch (ncols) {
    case 1: return launch_typed<WT, 1, 0>(p, grid, smem, s, pdl);
    case 2: return launch_typed<WT, 2, 0>(p, grid, smem, s, pdl);
    case 3: return launch_typed<WT, 3, 0>(p, grid, smem, s, pdl);
    case 4: return launch_typed<WT, 4, 0>(p, grid, smem, s, pdl);
    case 5: return launch_typed<WT, 5, 0>(p, grid, smem, s, pdl);
    case 6: return launch_typed<WT, 6, 0>(p, grid, smem, s, pdl);
    case 7: return launch_typed<WT, 7, 0>(p, grid, smem, s, pdl);
    default: return launch_typed<WT, 8, 0>(p, grid, smem, s, pdl);
    }
}

bool shifted_of(int32_t wtype) { return wtype == WT_Q8_0 || wtype == WT_Q4_0; }
// bytes per 32-element unit, rounded up (Q6_K: 210 / 8 = 26.25), for budgets
uint32_t unit_bytes_of(int32_t wtype) {
    switch (wtype) {
    case WT_Q8_0: return Q8_0_BYTES;
    case WT_Q4_0: return Q4_0_BYTES;
    case WT_Q5_K: return Q5_K_BYTES / 8;
    case WT_Q6_K: return (Q6_K_BYTES + 7) / 8;
    default: return Q4_K_BYTES / 8;
    }
}
bool k_quant(int32_t wtype) { return wtype == WT_Q4_K || wtype == WT_Q5_K || wtype == WT_Q6_K; }
// exact bytes of `units` 32-element units (a multiple of 8 for K-quants)
uint32_t chunk_bytes_of(int32_t wtype, uint32_t units) {
    switch (wtype) {
    case WT_Q4_K: return units / 8 * Q4_K_BYTES;
    case WT_Q5_K: return units / 8 * Q5_K_BYTES;
    case WT_Q6_K: return units / 8 * Q6_K_BYTES;
    default: return units * unit_bytes_of(wtype);
    }
}

// The K-split path for one column of wide Q4_K rows; returns -1 (nothing
// launched) when the shape does not fit it.
int launch_gemv_ks(const void *w, uint64_t w_nb1, const void *x, void *y, int64_t K, int64_t M, int32_t *status,
                   cudaStream_t s, bool pdl, const PeerOut *peer, const EpiAct &epi) {
    const int nsb = (int)(K / QKK);
    const int widest = (nsb + kGemvWarps - 1) / kGemvWarps;  // super-blocks in the widest slice
    const uint32_t box_bytes = (uint32_t)widest * Q4_K_BYTES;
    // at least six super-blocks per warp (24 of 32 lanes busy); the box's
    // inner extent (8-byte elements) at most 256
    // at most 32 sub-block pairs per slice (one per lane)
    if (nsb < 6 * kGemvWarps || widest > 8 || M > INT32_MAX / 2) return -1;
    const int grid = std::max<int>(1, (int)std::min<int64_t>(sm_count(), (M + 1) / 2));
    const int64_t rows_max = (M + grid - 1) / grid + 1;
    const uint32_t ring_off = (uint32_t)((256 + rows_max * kGemvWarps * 4 + 127) / 128 * 128);
    const uint64_t stage_bytes = ((uint64_t)kKsRows * box_bytes + 127) / 128 * 128;
    const uint64_t smem = ring_off + (uint64_t)kGemvWarps * kKsStages * stage_bytes;
    if (smem > kCoResidentCta) return -1;
    CUtensorMap tm;
    int rc = encode_tensor_map_2d(&tm, CU_TENSOR_MAP_DATA_TYPE_UINT64, w, (uint64_t)nsb * Q4_K_BYTES / 8,
                                  (uint64_t)M, w_nb1, box_bytes / 8, kKsRows);
    if (rc) return rc;
    KsParams p;
    p.x = static_cast<const float *>(x);
    p.y = static_cast<uint8_t *>(y);
    p.M = (int)M;
    p.nsb = nsb;
    p.box_bytes = box_bytes;
    p.ring_off = ring_off;
    p.status = status;
    p.x_vec16 = (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    p.peer = peer ? *peer : PeerOut{};
    p.epi = epi;
    auto kern = gemv_ks_kernel<1>;
    static DeviceFlags smem_set;
    rc = raise_smem_limit((const void *)kern, (int)kCoResidentCta, smem_set, "gemv");
    if (rc) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kGemvThreads);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tm, p);
    if (e != cudaSuccess) return fb::set_error(FB_ERR_CUDA, "gemv launch: %s", cudaGetErrorString(e));
    return FB_OK;
}

// The K-split path for 2..8 columns of wide Q4_K rows over planar
// activations; returns -1 (nothing launched) when the shape does not fit it.
template <int NC>
int launch_ks_cols_typed(const CUtensorMap &tm, const KsColsParams &p, int grid, uint32_t smem, cudaStream_t s,
                         bool pdl) {
    auto kern = gemv_ks_cols_kernel<NC>;
    static DeviceFlags smem_set;
    const int rc = raise_smem_limit((const void *)kern, kSmemLimit, smem_set, "gemv");
    if (rc) return rc;
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
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tm, p);
    if (e != cudaSuccess) return fb::set_error(FB_ERR_CUDA, "gemv launch: %s", cudaGetErrorString(e));
    return FB_OK;
}

int launch_gemv_ks_cols(const void *w, uint64_t w_nb1, const Q8Planar &xq, void *y, uint64_t y_nb1, int64_t K,
                        int64_t M, int64_t N, int32_t *status, cudaStream_t s, bool pdl, const EpiAct &epi) {
    const int nsb = (int)(K / QKK);
    const int widest = (nsb + kGemvWarps - 1) / kGemvWarps;
    const uint32_t box_bytes = (uint32_t)widest * Q4_K_BYTES;
    if (N < 2 || N > kMaxCols || nsb < 6 * kGemvWarps || widest > 8 || M > INT32_MAX / 2) return -1;
    // planar activations: 16-byte rows of int8, 8-byte aligned scale pairs
    if (((reinterpret_cast<uintptr_t>(xq.qs) | (uint64_t)K) & 15) || ((reinterpret_cast<uintptr_t>(xq.d) |
                                                                         reinterpret_cast<uintptr_t>(xq.sum)) & 7))
        return -1;
    const int grid = std::max<int>(1, (int)std::min<int64_t>(sm_count(), (M + 1) / 2));
    const int64_t rows_max = (M + grid - 1) / grid + 1;
    const uint32_t ring_off = (uint32_t)((256 + rows_max * N * kGemvWarps * 4 + 127) / 128 * 128);
    const uint64_t stage_bytes = ((uint64_t)kKsRows * box_bytes + 127) / 128 * 128;
    const uint64_t xs_off = ring_off + (uint64_t)kGemvWarps * kKsStages * stage_bytes;
    const uint64_t smem = xs_off + (uint64_t)kGemvWarps * N * 4 * (4 * widest) * 16;
    if (smem > (uint64_t)kSmemLimit) return -1;
    CUtensorMap tm;
    int rc = encode_tensor_map_2d(&tm, CU_TENSOR_MAP_DATA_TYPE_UINT64, w, (uint64_t)nsb * Q4_K_BYTES / 8,
                                  (uint64_t)M, w_nb1, box_bytes / 8, kKsRows);
    if (rc) return rc;
    KsColsParams p;
    p.xq = xq;
    p.y = static_cast<uint8_t *>(y);
    p.y_nb1 = y_nb1;
    p.K = (int)K;
    p.M = (int)M;
    p.nsb = nsb;
    p.box_bytes = box_bytes;
    p.ring_off = ring_off;
    p.xs_off = (uint32_t)xs_off;
    p.status = status;
    p.epi = epi;
    switch (N) {
    case 2: return launch_ks_cols_typed<2>(tm, p, grid, (uint32_t)smem, s, pdl);
    case 3: return launch_ks_cols_typed<3>(tm, p, grid, (uint32_t)smem, s, pdl);
    case 4: return launch_ks_cols_typed<4>(tm, p, grid, (uint32_t)smem, s, pdl);
    case 5: return launch_ks_cols_typed<5>(tm, p, grid, (uint32_t)smem, s, pdl);
    case 6: return launch_ks_cols_typed<6>(tm, p, grid, (uint32_t)smem, s, pdl);
    case 7: return launch_ks_cols_typed<7>(tm, p, grid, (uint32_t)smem, s, pdl);
    default: return launch_ks_cols_typed<8>(tm, p, grid, (uint32_t)smem, s, pdl);
    }
}

}  // namespace

bool gemv_supported(int32_t wtype, int64_t K, int64_t N) {
    if (wtype != WT_Q8_0 && wtype != WT_Q4_0 && !k_quant(wtype)) return false;
    if (N < 1 || N > kMaxCols) return false;
    if (K % (k_quant(wtype) ? QKK : QK)) return false;
    // activations + two minimal stages per warp must fit
    const SmemLayout L = smem_layout((int)K, (int)N, shifted_of(wtype), 2, align16(chunk_bytes_of(wtype, 8) + 32));
    return K <= (1 << 20) && L.total <= (uint32_t)kSmemLimit;
}

bool gemv_fused_ok(int64_t K, int64_t N) { return K * N <= kFusedMaxElems; }

int gemv_max_cols() { return kMaxCols; }

int launch_peer_wait(const uint32_t *flag, uint32_t *epoch, int32_t n_ranks, int32_t *status, cudaStream_t s,
                     uint64_t timeout_us) {
    if (!flag || !epoch || ((reinterpret_cast<uintptr_t>(flag) | reinterpret_cast<uintptr_t>(epoch)) & 3))
        return fb::set_error(FB_ERR_INVALID, "peer_wait: bad flag or epoch");
    if (n_ranks < 1 || n_ranks > kMaxPeers) return fb::set_error(FB_ERR_INVALID, "peer_wait: %d ranks", n_ranks);
    if (timeout_us == 0 || timeout_us > 10000000ull)
        return fb::set_error(FB_ERR_INVALID, "peer_wait: timeout %llu us outside 1 us .. 10 s",
                             (unsigned long long)timeout_us);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(32);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, peer_wait_kernel, flag, epoch, (int)n_ranks, timeout_us * 1000ull, status);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return fb::set_error(FB_ERR_CUDA, "peer_wait launch: %s", cudaGetErrorString(e));
    return FB_OK;
}

int launch_gemv(int32_t wtype, const void *w, uint64_t w_nb1, const void *x, uint64_t x_nb1, void *y, uint64_t y_nb1,
                int64_t K, int64_t M, int64_t N, const Q8Planar *xq, int32_t *status, cudaStream_t s, bool pdl,
                const PeerOut *peer, const float *norm_eps, const EpiAct *epi) {
    const EpiAct ep = epi ? *epi : EpiAct{nullptr, 0};
    if (!gemv_supported(wtype, K, N)) return fb::set_error(FB_ERR_UNSUPPORTED, "gemv: unsupported shape");
    if (norm_eps && (xq || peer || K < 512 || !gemv_fused_ok(K, N)))
        return fb::set_error(FB_ERR_UNSUPPORTED, "gemv: fused rms_norm needs in-kernel activation quantization and K >= 512");
    if (M == 0) return FB_OK;
    if ((reinterpret_cast<uintptr_t>(w) & 1) || (w_nb1 & 1))
        return fb::set_error(FB_ERR_INVALID, "gemv: weight rows must be 2-byte aligned");
    if (!xq && ((reinterpret_cast<uintptr_t>(x) & 3) || (x_nb1 & 3)))
        return fb::set_error(FB_ERR_INVALID, "gemv: activations must be 4-byte aligned");
    if (peer) {
        if (peer->n < 1 || peer->n > kMaxPeers || !peer->count || !peer->epoch)
            return fb::set_error(FB_ERR_INVALID, "gemv: bad peer set");
        for (int r = 0; r < peer->n; r++)
            if (!peer->y[0][r] || !peer->y[1][r] || !peer->flag[r] ||
                ((reinterpret_cast<uintptr_t>(peer->y[0][r]) | reinterpret_cast<uintptr_t>(peer->y[1][r]) |
                  reinterpret_cast<uintptr_t>(peer->flag[r])) & 3))
                return fb::set_error(FB_ERR_INVALID, "gemv: peer %d pointers", r);
    } else if (!y) {
        return fb::set_error(FB_ERR_INVALID, "gemv: null output");
    }
    if ((reinterpret_cast<uintptr_t>(y) & 3) || (y_nb1 & 3))
        return fb::set_error(FB_ERR_INVALID, "gemv: output must be 4-byte aligned");
    if (M > INT32_MAX) return fb::set_error(FB_ERR_UNSUPPORTED, "gemv: M too large");

    const bool rows16 = ((reinterpret_cast<uintptr_t>(w) | w_nb1) & 15) == 0;
    if (wtype == WT_Q4_K && N == 1 && !xq && rows16 && !norm_eps) {
        const int rc = launch_gemv_ks(w, w_nb1, x, y, K, M, status, s, pdl, peer, ep);
        if (rc >= 0) return rc;  // launched, or an error; -1: not this path
    }
    if (wtype == WT_Q4_K && N > 1 && xq && !peer && rows16) {
        const int rc = launch_gemv_ks_cols(w, w_nb1, *xq, y, y_nb1, K, M, N, status, s, pdl, ep);
        if (rc >= 0) return rc;
    }

    const int nunits = (int)(K / QK);
    const uint32_t ub = unit_bytes_of(wtype);
    const bool sh = shifted_of(wtype);
    const int sms = sm_count();
    const int grid = std::max<int>(1, (int)std::min<int64_t>(sms, (M + 1) / 2));

    // Shared-memory budget: small activations leave room for the next
    // launch's CTA on the same SM; otherwise one large CTA.
    const SmemLayout base = smem_layout((int)K, (int)N, sh, 4, 0);
    const uint32_t cta_limit = base.total <= kCoResidentActs ? kCoResidentCta : (uint32_t)kSmemLimit;
    const uint32_t per_warp = (cta_limit - base.total - 256) / kGemvWarps;
    // chunks as large as two stages per warp allow (whole rows when they fit)
    int chunk_units = (int)((per_warp / 2 - 32) / ub) / 8 * 8;
    chunk_units = std::max(8, std::min({chunk_units, (nunits + 7) / 8 * 8, 512}));
    const int nchunks0 = (nunits + chunk_units - 1) / chunk_units;
    chunk_units = ((nunits + nchunks0 - 1) / nchunks0 + 7) / 8 * 8;  // balance the chunks of a row
    const int nchunks = (nunits + chunk_units - 1) / chunk_units;
    const uint32_t stage_bytes = align16(chunk_bytes_of(wtype, (uint32_t)chunk_units) + 32);
    int nstage = 4;
    while (nstage > 2 && smem_layout((int)K, (int)N, sh, nstage, stage_bytes).total > cta_limit) nstage--;
    const SmemLayout L = smem_layout((int)K, (int)N, sh, nstage, stage_bytes);
    if (L.total > (uint32_t)kSmemLimit) return fb::set_error(FB_ERR_UNSUPPORTED, "gemv: shared memory budget exceeded");

    const int align = wtype == WT_Q6_K ? 2 : (k_quant(wtype) ? 16 : 4);  // Q6_K super-blocks are 2-byte aligned
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
    p.x_vec16 = ((reinterpret_cast<uintptr_t>(x) | x_nb1) & 15) == 0;
    p.peer = peer ? *peer : PeerOut{};
    p.copy_rows = ((reinterpret_cast<uintptr_t>(w) | w_nb1) % align) != 0;
    p.norm = norm_eps != nullptr;
    p.norm_eps = norm_eps ? *norm_eps : 0.0f;
    p.epi = ep;
    // whole rows per chunk and at most two pairs per lane: activations in registers
    const int xr = (N == 1 && nchunks == 1 && rows16) ? (nunits <= 64 ? 1 : (nunits <= 128 ? 2 : 0)) : 0;
    switch (wtype) {
    case WT_Q8_0: return launch_cols<WT_Q8_0>((int)N, xr, p, grid, L.total, s, pdl);
    case WT_Q4_0: return launch_cols<WT_Q4_0>((int)N, xr, p, grid, L.total, s, pdl);
    case WT_Q5_K: return launch_cols<WT_Q5_K>((int)N, xr, p, grid, L.total, s, pdl);
    case WT_Q6_K: return launch_cols<WT_Q6_K>((int)N, xr, p, grid, L.total, s, pdl);
    default: return launch_cols<WT_Q4_K>((int)N, xr, p, grid, L.total, s, pdl);
    }
}

}  // namespace fbk
