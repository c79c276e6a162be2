// Quantized mul_mat on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Arithmetic. The reference result is the F32 mul_mat of the dequantized
// weights W[m,k] = dw[m,b] * qw[m,k] and the dequantized Q8_0 activations
// X[n,k] = dx[n,b] * qx[n,k] (b = k / 32; feml-cpu/src/ops/mul_mat.rs:36-57
// on dequantized operands). Per 32-element block b this kernel computes
//     T_b[m,n] = sum_{k in b} qw[m,k] * X[n,k]
// on the tensor core in f32 with f16 operands that are exact:
//   * qw is an integer in [-128, 127] (Q8_0) or [-8, 7] (Q4_0): exact in f16;
//   * X[n,k] (an f32 with at most 11 + 8 significant bits) is split into
//     X = hi + lo, hi = f16(X), lo = f16(X - hi), both exact in f16 for the
//     activation range after a per-row power-of-two normalisation;
// so T_b = qw.hi + qw.lo takes two MMAs of K = 32 (four of K = 16) into one
// TMEM accumulator slot, and the epilogue applies the row's block scale in
// FP32:  acc[m,n] += dw[m,b] * T_b[m,n]  (one FFMA per element and block).
// Products qw*hi and qw*lo are exact in f32; only the f32 sums round, so the
// result is within the path's tolerance of the reference (not bit-exact).
//
// Tiles and roles (one CTA of 512 threads per SM, BM = 128 rows, BN = 128
// columns, full K):
//   warp 0      TMA producer: raw weight chunks (8 blocks x 128 rows) into a
//               ring (2D tensor map over the ggml rows, no swizzle).
//   warp 1      TMA producer: activation panels [hi 32 | lo 32] per block,
//               128-byte swizzled, two blocks per stage.
//   warp 2      allocates TMEM (512 columns = 4 slots of 128) and issues the
//               MMAs from one thread (kind::f16, M = 128, N = 128, K = 16).
//   warps 4-7   converters: unpack each weight row's blocks into integer
//               f16 (bit tricks, no conversion instructions), store them in
//               the 128-byte swizzled K-major layout the MMA reads, and
//               publish the block scales.
//   warps 8-15  epilogue: per block, read the slot (tcgen05.ld 32x32b),
//               acc += dw * T, release the slot; finally store acc.
// Every barrier wait is bounded; on timeout the CTA raises STATUS_TIMEOUT,
// drains the copies and MMAs it issued and frees its TMEM before returning.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <mutex>

#include "../host_common.h"
#include "common.cuh"
#include "kernels.h"

namespace fbk {

namespace {

constexpr int TC_BM = 128;
constexpr int TC_BN = 128;
constexpr int TC_THREADS = 512;
constexpr int TC_SLOTS = 4;           // TMEM accumulator slots (one block each)
constexpr int TC_TMEM_COLS = 512;     // TC_SLOTS * TC_BN
constexpr int TC_NS = 8;              // block-scale ring (pairs)
constexpr int A_STAGE = TC_BM * 128;  // one pair of blocks: 128 rows x 64 f16
constexpr int B_PANEL = TC_BN * 128;  // one block: BN rows x [hi 32 | lo 32] f16
constexpr int B_STAGE = 2 * B_PANEL;

template <int WT>
struct TcCfg;
template <>
struct TcCfg<WT_Q8_0> {
    static constexpr int RAWB = 8 * Q8_0_BYTES;  // 272 bytes: 8 blocks of one row
    static constexpr int NR = 2, NA = 3, NB = 3;
};
template <>
struct TcCfg<WT_Q4_0> {
    static constexpr int RAWB = 8 * Q4_0_BYTES;  // 144
    static constexpr int NR = 2, NA = 4, NB = 3;
};

template <int WT>
struct TcLayout {
    using C = TcCfg<WT>;
    static constexpr int RAW_STAGE = TC_BM * C::RAWB;
    static constexpr int OFF_A = 0;
    static constexpr int OFF_B = OFF_A + C::NA * A_STAGE;
    static constexpr int OFF_RAW = OFF_B + C::NB * B_STAGE;
    static constexpr int OFF_SC = OFF_RAW + ((C::NR * RAW_STAGE + 1023) / 1024) * 1024;
    static constexpr int OFF_BAR = OFF_SC + TC_NS * 2 * TC_BM * 4;
    static constexpr int N_BARS = 2 * (C::NR + C::NA + C::NB + TC_SLOTS + TC_NS) + 1;
    static constexpr int OFF_MISC = OFF_BAR + N_BARS * 8;
    static constexpr int BYTES = OFF_MISC + 16 + 1024;  // + alignment slack
};

struct TcParams {
    int M, N, K;
    uint8_t *y;
    uint64_t y_nb1;
    const float *rscale;  // per activation row: 2^e undone in the epilogue
    int32_t *status;
    // grouped mode (mul_mat_id): activation rows are the routed slots in
    // expert order; column tile blockIdx.y belongs to the expert whose
    // tile_start range holds it, and weights come from that expert's plane
    bool grouped;
    GroupMap g;
};

// ---- tcgen05 / TMA primitives (inline PTX) -----------------------------------
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int c0, int c1, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *map, int c0, int c1, int c2,
                                            uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, f16 inputs, f32 accumulate.
__device__ __forceinline__ void tc_mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u)
        : "memory");
}

// 32 consecutive 32-bit TMEM columns of this warp's 32 lanes.
__device__ __forceinline__ void tc_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row atoms
// 1024 bytes apart (start address, LBO unused = 1, SBO = 1024, version 1,
// layout SWIZZLE_128B = 2).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor, kind::f16: D f32, A f16, B f16, both K-major, M, N.
__host__ __device__ constexpr uint32_t f16_idesc(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Bounded wait that also gives up when another role has aborted.
__device__ __forceinline__ bool tc_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
    for (uint32_t i = 0; i < kWaitLimit; i++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63u) == 63u && *abort_flag) return false;
    }
    *abort_flag = 1;
    return false;
}

// Warp-uniform form for roles that then run .sync.aligned instructions: lane
// 0 polls, the verdict is broadcast, and every lane re-reads the completed
// phase (acquire) before touching the data it guards.
__device__ __forceinline__ bool tc_wait_warp(uint64_t *bar, uint32_t parity, volatile int *abort_flag, int lane) {
    int ok = 0;
    if (lane == 0) ok = tc_wait(bar, parity, abort_flag) ? 1 : 0;
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (ok) mbar_try_wait(bar, parity);
    return ok != 0;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(0u), "r"(sel));
    return r;
}
__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }
__device__ __forceinline__ __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2 *>(&u); }

// 4 signed bytes -> 4 f16 integers (two half2 words), exact.
// (0x6400 | (b ^ 0x80)) is the f16 1024 + (b + 128); subtracting 1152 gives b.
__device__ __forceinline__ void q8_word_to_f16(uint32_t w, uint32_t &lo, uint32_t &hi) {
    const __half2 off = __half2half2(__ushort_as_half(0x6480));  // 1152
    const uint32_t a = (prmt(w, 0x4140) ^ 0x00800080u) | 0x64006400u;
    const uint32_t b = (prmt(w, 0x4342) ^ 0x00800080u) | 0x64006400u;
    lo = h2_bits(__hsub2(bits_h2(a), off));
    hi = h2_bits(__hsub2(bits_h2(b), off));
}

// 4 Q4_0 bytes -> low nibbles (elements j..j+3) and high nibbles (j+16..j+19)
// as f16 integers minus 8, exact. Low: 1024 + n - 1032; high: the nibble sits
// at bit 4, (1024 + 16 n) / 16 - 72 = n - 8.
__device__ __forceinline__ void q4_word_to_f16(uint32_t w, uint32_t (&lo)[2], uint32_t (&hi)[2]) {
    const __half2 off_lo = __half2half2(__ushort_as_half(0x6408));   // 1032
    const __half2 sc_hi = __half2half2(__ushort_as_half(0x2C00));    // 1/16
    const __half2 off_hi = __half2half2(__ushort_as_half(0xD480));   // -72
    const uint32_t a = prmt(w, 0x4140), b = prmt(w, 0x4342);
    lo[0] = h2_bits(__hsub2(bits_h2((a & 0x000F000Fu) | 0x64006400u), off_lo));
    lo[1] = h2_bits(__hsub2(bits_h2((b & 0x000F000Fu) | 0x64006400u), off_lo));
    hi[0] = h2_bits(__hfma2(bits_h2((a & 0x00F000F0u) | 0x64006400u), sc_hi, off_hi));
    hi[1] = h2_bits(__hfma2(bits_h2((b & 0x00F000F0u) | 0x64006400u), sc_hi, off_hi));
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

// Store the 32 f16 integers of one block (16 words, element order) of row
// `row` at block position j (0/1) of an A stage (128-byte swizzled rows).
__device__ __forceinline__ void store_a_block(uint32_t a_stage, int row, int j, const uint32_t (&v)[16]) {
    const uint32_t rbase = a_stage + (uint32_t)row * 128u;
#pragma unroll
    for (int q = 0; q < 4; q++) {
        const uint32_t chunk = (uint32_t)(4 * j + q) ^ (uint32_t)(row & 7);
        st_shared_v4(rbase + chunk * 16u, v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    }
}

// Convert block pair p (blocks 2p, 2p+1 of an 8-block raw row held in
// registers) into f16 integers; returns the two scales.
template <int WT>
__device__ __forceinline__ void convert_pair(const uint32_t *w, int p, uint32_t (&v0)[16], uint32_t (&v1)[16],
                                             float &d0, float &d1) {
    if constexpr (WT == WT_Q8_0) {
        // block 2p at byte 68p (word 17p): d in the low half, qs from byte 2
        const int b = 17 * p;
        d0 = f16_bits_to_f32((uint16_t)(w[b] & 0xFFFFu));
#pragma unroll
        for (int i = 0; i < 8; i++) q8_word_to_f16(__funnelshift_r(w[b + i], w[b + i + 1], 16), v0[2 * i], v0[2 * i + 1]);
        // block 2p+1 at byte 68p + 34: d in the high half of word 17p+8, qs word-aligned
        d1 = f16_bits_to_f32((uint16_t)(w[b + 8] >> 16));
#pragma unroll
        for (int i = 0; i < 8; i++) q8_word_to_f16(w[b + 9 + i], v1[2 * i], v1[2 * i + 1]);
    } else {
        // Q4_0: block 2p at byte 36p (word 9p), block 2p+1 at byte 36p + 18
        const int b = 9 * p;
        d0 = f16_bits_to_f32((uint16_t)(w[b] & 0xFFFFu));
#pragma unroll
        for (int i = 0; i < 4; i++) {
            uint32_t lo[2], hi[2];
            q4_word_to_f16(__funnelshift_r(w[b + i], w[b + i + 1], 16), lo, hi);
            v0[2 * i] = lo[0];
            v0[2 * i + 1] = lo[1];
            v0[8 + 2 * i] = hi[0];
            v0[8 + 2 * i + 1] = hi[1];
        }
        d1 = f16_bits_to_f32((uint16_t)(w[b + 4] >> 16));
#pragma unroll
        for (int i = 0; i < 4; i++) {
            uint32_t lo[2], hi[2];
            q4_word_to_f16(w[b + 5 + i], lo, hi);
            v1[2 * i] = lo[0];
            v1[2 * i + 1] = lo[1];
            v1[8 + 2 * i] = hi[0];
            v1[8 + 2 * i + 1] = hi[1];
        }
    }
}

template <int WT>
__global__ void __launch_bounds__(TC_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                   const TcParams p) {
    using C = TcCfg<WT>;
    using L = TcLayout<WT>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
    uint8_t *gbase = smem_raw + (sbase - smem_u32(smem_raw));

    uint64_t *bars = reinterpret_cast<uint64_t *>(gbase + L::OFF_BAR);
    uint64_t *raw_full = bars;
    uint64_t *raw_empty = raw_full + C::NR;
    uint64_t *a_full = raw_empty + C::NR;
    uint64_t *a_empty = a_full + C::NA;
    uint64_t *b_full = a_empty + C::NA;
    uint64_t *b_empty = b_full + C::NB;
    uint64_t *t_full = b_empty + C::NB;
    uint64_t *t_empty = t_full + TC_SLOTS;
    uint64_t *s_full = t_empty + TC_SLOTS;
    uint64_t *s_empty = s_full + TC_NS;
    uint64_t *mma_done = s_empty + TC_NS;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(gbase + L::OFF_MISC);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(gbase + L::OFF_MISC + 4);
    float *scales = reinterpret_cast<float *>(gbase + L::OFF_SC);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int m0 = blockIdx.x * TC_BM;
    // activation rows [xrow0, xrow0 + ncols) of this tile, weight plane `expert`
    int xrow0 = blockIdx.y * TC_BN, ncols = min(TC_BN, p.N - xrow0), expert = 0;
    if (p.grouped) {
        const int t = blockIdx.y;
        if (t >= p.g.tile_start[p.g.n_groups]) return;  // unused tile (uniform, before any set-up)
        while (p.g.tile_start[expert + 1] <= t) expert++;
        const int jt = t - p.g.tile_start[expert];
        xrow0 = p.g.offsets[expert] + jt * TC_BN;
        ncols = min(TC_BN, p.g.counts[expert] - jt * TC_BN);
    }
    const int nblk = p.K / QK, npairs = nblk / 2, nchunks = p.K / QKK;

    if (tid == 0) {
        for (int i = 0; i < C::NR; i++) {
            mbar_init(&raw_full[i], 1);
            mbar_init(&raw_empty[i], 128);
        }
        for (int i = 0; i < C::NA; i++) {
            mbar_init(&a_full[i], 128);
            mbar_init(&a_empty[i], 1);
        }
        for (int i = 0; i < C::NB; i++) {
            mbar_init(&b_full[i], 1);
            mbar_init(&b_empty[i], 1);
        }
        for (int i = 0; i < TC_SLOTS; i++) {
            mbar_init(&t_full[i], 1);
            mbar_init(&t_empty[i], 8);
        }
        for (int i = 0; i < TC_NS; i++) {
            mbar_init(&s_full[i], 128);
            mbar_init(&s_empty[i], 8);
        }
        mbar_init(mma_done, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 2) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TC_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---- raw weight chunks ------------------------------------------------
        if (lane == 0) {
            int armed[C::NR];
            for (int i = 0; i < C::NR; i++) armed[i] = -1;
            for (int c = 0; c < nchunks; c++) {
                const int s = c % C::NR;
                if (!tc_wait(&raw_empty[s], ((c / C::NR) & 1) ^ 1, abort_flag)) break;
                mbar_arrive_expect_tx(&raw_full[s], L::RAW_STAGE);
                const int x0 = WT == WT_Q8_0 ? c * (C::RAWB / 2) : c * C::RAWB;
                tma_load_3d(sbase + L::OFF_RAW + s * L::RAW_STAGE, &tm_w, x0, m0, expert, smem_u32(&raw_full[s]));
                armed[s] = (c / C::NR) & 1;
            }
            if (*abort_flag)  // let the copies in flight land before the CTA exits
                for (int i = 0; i < C::NR; i++)
                    if (armed[i] >= 0) mbar_wait_bounded(&raw_full[i], (uint32_t)armed[i]);
        }
    } else if (warp == 1) {
        // ---- activation panels ------------------------------------------------
        if (lane == 0) {
            int armed[C::NB];
            for (int i = 0; i < C::NB; i++) armed[i] = -1;
            for (int q = 0; q < npairs; q++) {
                const int s = q % C::NB;
                if (!tc_wait(&b_empty[s], ((q / C::NB) & 1) ^ 1, abort_flag)) break;
                mbar_arrive_expect_tx(&b_full[s], B_STAGE);
                const uint32_t dst = sbase + L::OFF_B + s * B_STAGE;
                tma_load_2d(dst, &tm_x, (2 * q) * 64, xrow0, smem_u32(&b_full[s]));
                tma_load_2d(dst + B_PANEL, &tm_x, (2 * q + 1) * 64, xrow0, smem_u32(&b_full[s]));
                armed[s] = (q / C::NB) & 1;
            }
            if (*abort_flag)
                for (int i = 0; i < C::NB; i++)
                    if (armed[i] >= 0) mbar_wait_bounded(&b_full[i], (uint32_t)armed[i]);
        }
    } else if (warp == 2) {
        // ---- MMA issue (one thread) ---------------------------------------------
        if (lane == 0) {
            constexpr uint32_t idesc = f16_idesc(TC_BM, TC_BN);
            bool ok = true;
            for (int q = 0; q < npairs && ok; q++) {
                const int sa = q % C::NA, sb = q % C::NB;
                if (!tc_wait(&a_full[sa], (q / C::NA) & 1, abort_flag) ||
                    !tc_wait(&b_full[sb], (q / C::NB) & 1, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t a_addr = sbase + L::OFF_A + sa * A_STAGE;
                const uint32_t b_addr = sbase + L::OFF_B + sb * B_STAGE;
                for (int j = 0; j < 2; j++) {
                    const int blk = 2 * q + j, slot = blk % TC_SLOTS;
                    if (!tc_wait(&t_empty[slot], ((blk / TC_SLOTS) & 1) ^ 1, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d = tmem + (uint32_t)(slot * TC_BN);
                    const uint32_t aj = a_addr + 64u * j, bj = b_addr + (uint32_t)B_PANEL * j;
                    tc_mma_f16(d, sw128_desc(aj), sw128_desc(bj), idesc, 0u);            // hi, k 0-15
                    tc_mma_f16(d, sw128_desc(aj + 32), sw128_desc(bj + 32), idesc, 1u);  // hi, k 16-31
                    tc_mma_f16(d, sw128_desc(aj), sw128_desc(bj + 64), idesc, 1u);       // lo, k 0-15
                    tc_mma_f16(d, sw128_desc(aj + 32), sw128_desc(bj + 96), idesc, 1u);  // lo, k 16-31
                    tc_commit(smem_u32(&t_full[slot]));
                }
                if (!ok) break;
                tc_commit(smem_u32(&a_empty[sa]));
                tc_commit(smem_u32(&b_empty[sb]));
            }
            // all issued MMAs complete before TMEM can be released
            tc_commit(smem_u32(mma_done));
            mbar_wait_bounded(mma_done, 0);
        }
    } else if (warp >= 4 && warp < 8) {
        // ---- converters: one weight row per thread ------------------------------
        const int row = tid - 128;
        constexpr int NW = C::RAWB / 4;
        for (int c = 0; c < nchunks; c++) {
            const int s = c % C::NR;
            if (!tc_wait_warp(&raw_full[s], (c / C::NR) & 1, abort_flag, lane)) break;
            uint32_t w[NW];
            const uint4 *src = reinterpret_cast<const uint4 *>(gbase + L::OFF_RAW + s * L::RAW_STAGE + row * C::RAWB);
#pragma unroll
            for (int i = 0; i < NW / 4; i++) {
                const uint4 v = src[i];
                w[4 * i] = v.x;
                w[4 * i + 1] = v.y;
                w[4 * i + 2] = v.z;
                w[4 * i + 3] = v.w;
            }
            mbar_arrive(&raw_empty[s]);
            bool ok = true;
#pragma unroll
            for (int pp = 0; pp < 4; pp++) {
                const int q = 4 * c + pp;
                const int sa = q % C::NA, ss = q % TC_NS;
                if (!tc_wait_warp(&a_empty[sa], ((q / C::NA) & 1) ^ 1, abort_flag, lane) ||
                    !tc_wait_warp(&s_empty[ss], ((q / TC_NS) & 1) ^ 1, abort_flag, lane)) {
                    ok = false;
                    break;
                }
                uint32_t v0[16], v1[16];
                float d0, d1;
                convert_pair<WT>(w, pp, v0, v1, d0, d1);
                const uint32_t a_addr = sbase + L::OFF_A + sa * A_STAGE;
                store_a_block(a_addr, row, 0, v0);
                store_a_block(a_addr, row, 1, v1);
                scales[(ss * 2 + 0) * TC_BM + row] = d0;
                scales[(ss * 2 + 1) * TC_BM + row] = d1;
                fence_proxy_async_smem();
                mbar_arrive(&a_full[sa]);
                mbar_arrive(&s_full[ss]);
            }
            if (!ok) break;
        }
    } else if (warp >= 8) {
        // ---- epilogue: warp w reads TMEM lanes 32*(w%4).., columns 64*h.. -------
        const int sub = warp & 3, h = (warp - 8) >> 2;
        const int row = 32 * sub + lane;
        float acc[64];
#pragma unroll
        for (int i = 0; i < 64; i++) acc[i] = 0.0f;
        bool ok = true;
        for (int q = 0; q < npairs && ok; q++) {
            const int ss = q % TC_NS;
            if (!tc_wait_warp(&s_full[ss], (q / TC_NS) & 1, abort_flag, lane)) {
                ok = false;
                break;
            }
#pragma unroll
            for (int j = 0; j < 2; j++) {
                const int blk = 2 * q + j, slot = blk % TC_SLOTS;
                if (!tc_wait_warp(&t_full[slot], (blk / TC_SLOTS) & 1, abort_flag, lane)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const float dw = scales[(ss * 2 + j) * TC_BM + row];
                const uint32_t taddr = tmem + ((uint32_t)(32 * sub) << 16) + (uint32_t)(slot * TC_BN + 64 * h);
#pragma unroll
                for (int cc = 0; cc < 2; cc++) {
                    uint32_t r[32];
                    tc_ld32(taddr + 32u * cc, r);
                    tc_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; i++) acc[32 * cc + i] = fmaf(__uint_as_float(r[i]), dw, acc[32 * cc + i]);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&t_empty[slot]);
            }
            __syncwarp();
            if (ok && lane == 0) mbar_arrive(&s_empty[ss]);
        }
        if (ok) {
            const int m = m0 + row;
            if (m < p.M) {
#pragma unroll
                for (int i = 0; i < 64; i++) {
                    const int c = 64 * h + i;
                    if (c < ncols) {
                        const int r = xrow0 + c;
                        uint64_t off;
                        if (p.grouped) {
                            const int slot = p.g.rows[r];
                            off = (uint64_t)(slot % p.g.n_selected) * p.g.dst_nb1 +
                                  (uint64_t)(slot / p.g.n_selected) * p.g.dst_nb2;
                        } else {
                            off = (uint64_t)r * p.y_nb1;
                        }
                        reinterpret_cast<float *>(p.y + off)[m] = acc[i] * p.rscale[r];
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (*abort_flag && tid == 0) report_status(p.status, STATUS_TIMEOUT);
    if (warp == 2) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TC_TMEM_COLS)
                     : "memory");
    }
}

// ---- activations: Q8_0 quantize, dequantize, split into f16 hi + lo ---------
// One CTA per activation row. The row is scaled by 2^-e (e >= 0, chosen so
// |X| stays below 2^14 and hi never overflows f16); rscale[n] = 2^e is
// multiplied back in the GEMM epilogue (exact: powers of two).
constexpr int HL_THREADS = 256;

// With `routed` (mul_mat_id), output row r is the activation of routed slot
// r (token rows[r] / n_selected) for the r < sum(counts) routed slots.
__global__ void __launch_bounds__(HL_THREADS) quantize_q8_hilo_kernel(const uint8_t *__restrict__ x, uint64_t x_nb1,
                                                                     int K, uint8_t *__restrict__ out,
                                                                     float *__restrict__ rscale, bool routed,
                                                                     GroupMap g) {
    __shared__ float red[HL_THREADS / 32];
    const int n = blockIdx.x, tid = threadIdx.x, lane = tid & 31;
    int src = n;
    if (routed) {
        if (g.n_groups == 0 || n >= g.offsets[g.n_groups - 1] + g.counts[g.n_groups - 1]) return;
        src = g.rows[n] / g.n_selected;
    }
    const float *xr = reinterpret_cast<const float *>(x + (uint64_t)src * x_nb1);
    float amax = 0.0f;
    for (int k = tid * 4; k < K; k += HL_THREADS * 4) {
        const float4 v = *reinterpret_cast<const float4 *>(xr + k);
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
    amax = warp_max(amax);
    if (lane == 0) red[tid >> 5] = amax;
    __syncthreads();
    amax = red[0];
#pragma unroll
    for (int i = 1; i < HL_THREADS / 32; i++) amax = fmaxf(amax, red[i]);
    // 2^-e with amax * 2^-e < 2^14 (the f16-rounded block scale can exceed amax by 2^-11)
    int e = 0;
    if (amax >= 16384.0f && amax <= 3.0e38f) e = min(126, (int)ceilf(log2f(amax / 16384.0f)) + 1);
    const float down = exp2f((float)-e);
    if (tid == 0) rscale[n] = exp2f((float)e);

    const int nblk = K / QK;
    uint16_t *orow = reinterpret_cast<uint16_t *>(out + (uint64_t)n * nblk * 128);
    // 8 lanes per block, 4 elements per lane; every lane of the warp calls the
    // quantize routine (uniform trip count)
    const int groups = (nblk + 31) / 32;  // 32 blocks per CTA pass
    for (int g = 0; g < groups; g++) {
        const int b = g * 32 + (tid >> 3);
        const int k = b * QK + (tid & 7) * 4;
        const bool valid = b < nblk;
        const float4 v = valid ? *reinterpret_cast<const float4 *>(xr + k) : make_float4(0.f, 0.f, 0.f, 0.f);
        uint16_t dbits;
        int qsum;
        const uint32_t q = quantize_q8_0_quad(v, dbits, qsum);
        if (!valid) continue;
        const float d = f16_bits_to_f32(dbits);
        uint16_t hi[4], lo[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int qi = (int)(int8_t)((q >> (8 * i)) & 0xFFu);
            const float xd = __fmul_rn(__fmul_rn(d, (float)qi), down);
            const __half hh = __float2half_rn(xd);
            hi[i] = __half_as_ushort(hh);
            lo[i] = __half_as_ushort(__float2half_rn(__fsub_rn(xd, __half2float(hh))));
        }
        uint16_t *ob = orow + b * 64 + (tid & 7) * 4;
        *reinterpret_cast<uint2 *>(ob) = make_uint2(hi[0] | ((uint32_t)hi[1] << 16), hi[2] | ((uint32_t)hi[3] << 16));
        *reinterpret_cast<uint2 *>(ob + 32) =
            make_uint2(lo[0] | ((uint32_t)lo[1] << 16), lo[2] | ((uint32_t)lo[3] << 16));
    }
}

// ---- host side ---------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static std::once_flag once;
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// Tiled tensor map of rank 2 (dim2 == 0) or 3; strides in bytes.
int encode_map(CUtensorMap *map, CUtensorMapDataType dt, const void *base, uint64_t dim0, uint64_t dim1,
               uint64_t dim2, uint64_t stride1, uint64_t stride2, uint32_t box0, uint32_t box1,
               CUtensorMapSwizzle swz) {
    auto fn = encode_fn();
    if (!fn) return fb::set_error(FB_ERR_CUDA, "gemm_tc: cuTensorMapEncodeTiled unavailable");
    const cuuint32_t rank = dim2 ? 3 : 2;
    const cuuint64_t dims[3] = {dim0, dim1, dim2 ? dim2 : 1};
    const cuuint64_t strides[2] = {stride1, stride2};
    const cuuint32_t box[3] = {box0, box1, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, dt, rank, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fb::set_error(FB_ERR_CUDA, "gemm_tc: tensor map encode failed (%d)", (int)r);
    return FB_OK;
}

// N: activation rows in the hi/lo buffer; n_planes / w_nb2: weight planes
// (experts) for the grouped mode (1 / unused otherwise).
template <int WT>
int launch_tc_typed(const void *w, uint64_t w_nb1, uint64_t w_nb2, int64_t n_planes, const void *xhl,
                    const float *rscale, int64_t K, int64_t M, int64_t N, void *y, uint64_t y_nb1,
                    const GroupMap *groups, int32_t *status, cudaStream_t s) {
    using C = TcCfg<WT>;
    using L = TcLayout<WT>;
    static_assert(L::BYTES <= 232448, "gemm_tc shared memory");
    CUtensorMap tw, tx;
    const uint64_t planes = (uint64_t)n_planes, pstride = n_planes > 1 ? w_nb2 : w_nb1 * (uint64_t)M;
    int rc;
    if (WT == WT_Q8_0)
        rc = encode_map(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT16, w, w_nb1 / 2, (uint64_t)M, planes, w_nb1, pstride,
                        C::RAWB / 2, TC_BM, CU_TENSOR_MAP_SWIZZLE_NONE);
    else
        rc = encode_map(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, w_nb1, (uint64_t)M, planes, w_nb1, pstride, C::RAWB,
                        TC_BM, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    const uint64_t nblk = (uint64_t)K / QK;
    rc = encode_map(&tx, CU_TENSOR_MAP_DATA_TYPE_UINT16, xhl, nblk * 64, (uint64_t)N, 0, nblk * 128, 0, 64, TC_BN,
                    CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<WT>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::BYTES);
        if (e != cudaSuccess) return fb::set_error(FB_ERR_CUDA, "gemm_tc smem attribute: %s", cudaGetErrorString(e));
        configured[dev] = 1;
    }
    TcParams p{};
    p.M = (int)M;
    p.N = (int)N;
    p.K = (int)K;
    p.y = static_cast<uint8_t *>(y);
    p.y_nb1 = y_nb1;
    p.rscale = rscale;
    p.status = status;
    p.grouped = groups != nullptr;
    if (groups) p.g = *groups;
    const unsigned tiles_n = groups ? (unsigned)groups->max_tiles : (unsigned)((N + TC_BN - 1) / TC_BN);
    if (tiles_n == 0 || M == 0) return FB_OK;
    if (tiles_n > 65535) return fb::set_error(FB_ERR_UNSUPPORTED, "gemm_tc: too many column tiles");
    dim3 grid((unsigned)((M + TC_BM - 1) / TC_BM), tiles_n);
    gemm_tc_kernel<WT><<<grid, TC_THREADS, L::BYTES, s>>>(tw, tx, p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fb::set_error(FB_ERR_CUDA, "gemm_tc launch: %s", cudaGetErrorString(e));
    return FB_OK;
}

}  // namespace

uint64_t xhilo_bytes(int64_t K, int64_t N) {
    const uint64_t a = ((uint64_t)N * (uint64_t)K * 4 + 255) & ~uint64_t(255);
    return a + (((uint64_t)N * 4 + 255) & ~uint64_t(255));
}

XHiLo xhilo_carve(void *base, int64_t K, int64_t N) {
    XHiLo r;
    r.x = base;
    r.rscale = reinterpret_cast<float *>(static_cast<uint8_t *>(base) +
                                         (((uint64_t)N * (uint64_t)K * 4 + 255) & ~uint64_t(255)));
    return r;
}

bool gemm_tc_supported(int32_t wtype, int64_t K, int64_t M, int64_t N, const void *w, uint64_t w_nb1) {
    if (wtype != WT_Q8_0 && wtype != WT_Q4_0) return false;
    if (K <= 0 || K % QKK || K > (1 << 24) || M <= 0 || N <= 0 || M > INT32_MAX || N > INT32_MAX) return false;
    if (((reinterpret_cast<uintptr_t>(w) | w_nb1) & 15) != 0) return false;
    return (N + TC_BN - 1) / TC_BN <= 65535;
}

int gemm_tc_block_n() { return TC_BN; }

int launch_quantize_q8_hilo(const void *x, uint64_t x_nb1, int64_t K, int64_t N, XHiLo out, const GroupMap *routed,
                            cudaStream_t s) {
    const int64_t rows = routed ? N * routed->n_selected : N;
    if (rows == 0) return FB_OK;
    if (K % QK || K <= 0 || K > INT32_MAX / 4 || rows > INT32_MAX)
        return fb::set_error(FB_ERR_UNSUPPORTED, "quantize_q8_hilo: unsupported shape");
    if ((reinterpret_cast<uintptr_t>(x) | x_nb1) & 15)
        return fb::set_error(FB_ERR_INVALID, "quantize_q8_hilo: activations must be 16-byte aligned");
    GroupMap g{};
    if (routed) g = *routed;
    quantize_q8_hilo_kernel<<<(unsigned)rows, HL_THREADS, 0, s>>>(static_cast<const uint8_t *>(x), x_nb1, (int)K,
                                                                 static_cast<uint8_t *>(out.x), out.rscale,
                                                                 routed != nullptr, g);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fb::set_error(FB_ERR_CUDA, "quantize_q8_hilo launch: %s", cudaGetErrorString(e));
    return FB_OK;
}

int launch_gemm_tc(int32_t wtype, const void *w, uint64_t w_nb1, const XHiLo &xhl, int64_t K, int64_t M, int64_t N,
                   void *y, uint64_t y_nb1, const GroupMap *groups, int32_t *status, cudaStream_t s) {
    const int64_t rows = groups ? N * groups->n_selected : N;
    if (!gemm_tc_supported(wtype, K, M, rows, w, w_nb1))
        return fb::set_error(FB_ERR_UNSUPPORTED, "gemm_tc: unsupported shape or alignment");
    const uint64_t w_nb2 = groups ? groups->w_group_stride : 0;
    const int64_t planes = groups ? groups->n_groups : 1;
    if (groups && (groups->n_groups < 1 || (w_nb2 & 15) || ((groups->dst_nb1 | groups->dst_nb2) & 3)))
        return fb::set_error(FB_ERR_INVALID, "gemm_tc: grouped strides");
    if ((reinterpret_cast<uintptr_t>(y) | y_nb1) & 3) return fb::set_error(FB_ERR_INVALID, "gemm_tc: output alignment");
    if (wtype == WT_Q8_0)
        return launch_tc_typed<WT_Q8_0>(w, w_nb1, w_nb2, planes, xhl.x, xhl.rscale, K, M, rows, y, y_nb1, groups,
                                        status, s);
    return launch_tc_typed<WT_Q4_0>(w, w_nb1, w_nb2, planes, xhl.x, xhl.rscale, K, M, rows, y, y_nb1, groups, status,
                                    s);
}

}  // namespace fbk
