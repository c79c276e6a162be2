// Quantized mul_mat on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// The reference result is the F32 mul_mat of the dequantized weights and the
// dequantized Q8_0 activations X[n,k] = dx[n,b] * qx[n,k] (b = k / 32;
// feml-cpu/src/ops/mul_mat.rs:36-57 on dequantized operands). Two kernels:
//
// gemm_tc3_kernel (Q8_0, Q4_0; further below): the dequantized weights and
// activations as exact hi + lo pairs of f16, three MMAs per K step, the f32
// accumulator in TMEM over the whole K range, read once per tile.
//
// gemm_tc_kernel (Q4_K, whose dequantized values d*sc*q - dmin*m do not fit
// two f16): per 32-element block b the tensor core computes the integer dot
// product
//     T_b[m,n] = sum_{k in b} qw[m,k] * qx[n,k]
// with f16 operands holding exact integers (qx in [-127, 127]; qw in
// [-128, 127] for Q8_0, [-8, 7] for Q4_0, [0, 15] for Q4_K) and an f32
// accumulator that represents every partial sum exactly (|T| < 2^19). The
// epilogue applies the block scales in FP32:
//     Q8_0 / Q4_0:  acc += T_b * (dw[m,b] * dx[n,b])
//     Q4_K:         acc += T_b * (d*sc[m,b] * dx[n,b]) - dmin*m[m,b] * (dx[n,b] * sum_k qx[n,k])
// so T is exact and only the scale products and the f32 sum round: results
// are within the path's tolerance of the reference, not bit-identical.
//
// Tiles and roles: one CTA of 768 threads per SM computes a 128 x 128
// output tile (rows m, activation rows n) over a K range (all of K, or a
// split-K slice written to a partial buffer and summed afterwards in a fixed
// order).
//   warp 0      TMA: raw weight rows, 8 blocks x 128 rows per chunk (tensor
//               map over the ggml rows; rank 3 for mul_mat_id experts).
//   warp 1      TMA: activation panels (128 rows x 64 f16 integers = two
//               blocks, 128-byte swizzle).
//   warp 3      stages the activation block scales of each pair (one pair
//               ahead) into the scale ring for the epilogue.
//   warp 2      allocates TMEM (2 slots of 2 x 128 f32 columns, one block
//               pair each) and issues the MMAs (kind::f16, M = 128, N = 128,
//               K = 16) from one thread, one commit per pair.
//   warps 4-7   converters: one weight row each; unpack blocks into integer
//               f16 (prmt/lop3 + one half2 add, no conversion instructions),
//               store them in the swizzled K-major layout the MMA reads,
//               publish the row's block scales.
//   warps 8-23  epilogue: 16 warps, each 32 lanes (rows) x 32 columns; per
//               block read the slot with tcgen05.ld 32x32b, apply the
//               scales, release the slot; store at the end.
// Every barrier wait is bounded; on timeout the CTA raises STATUS_TIMEOUT,
// lets the copies and MMAs it issued land and frees its TMEM before it
// returns.
#include <cuda.h>
#include <type_traits>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>

#include "../host_common.h"
#include "common.cuh"
#include "kernels.h"
#include "tmap.h"

namespace fbk {

namespace {

constexpr int TC_BM = 128;
constexpr int TC_BN = 128;
constexpr int TC_THREADS = 768;      // 4 helper warps, 4 converter warps, 16 epilogue warps
constexpr int TC_EPI_WARPS = 16;
constexpr int TC_PSLOTS = 2;           // TMEM accumulator slots, one block pair (2 x 128 columns) each
constexpr int TC_TMEM_COLS = 512;      // TC_PSLOTS * 2 * TC_BN f32 columns
constexpr int TC_ND = 8;               // pair-done barrier ring (one MMA commit per pair)
constexpr int TC_NS = 8;               // scale ring depth (block pairs)
constexpr int A_STAGE = TC_BM * 128;   // a block pair: 128 rows x 64 f16
constexpr int B_STAGE = TC_BN * 128;   // a block pair: 128 rows x 64 f16
constexpr int CHUNK_PAIRS = 4;         // 8 blocks per raw weight chunk

template <int WT>
struct TcCfg;
template <>
struct TcCfg<WT_Q8_0> {
    static constexpr int RAWB = 8 * Q8_0_BYTES;  // 272 bytes: 8 blocks of one row
    static constexpr int NR = 2, NA = 4, NB = 4, SCN = 2;
};
template <>
struct TcCfg<WT_Q4_0> {
    static constexpr int RAWB = 8 * Q4_0_BYTES;  // 144
    static constexpr int NR = 4, NA = 4, NB = 4, SCN = 2;
};
template <>
struct TcCfg<WT_Q4_K> {
    static constexpr int RAWB = Q4_K_BYTES;  // 144: one super-block
    static constexpr int NR = 3, NA = 4, NB = 4, SCN = 4;
};

// Scale ring entry (per block pair): SCN planes x 2 blocks x 128 floats.
// plane 0: weight scale per row (Q4_K: d*sc), plane 1: activation scale per
// column; Q4_K adds plane 2: dmin*m per row, plane 3: dx*sum(qx) per column.
template <int WT>
struct TcLayout {
    using C = TcCfg<WT>;
    static constexpr int RAW_STAGE = TC_BM * C::RAWB;
    static constexpr int OFF_A = 0;
    static constexpr int OFF_B = OFF_A + C::NA * A_STAGE;
    static constexpr int OFF_RAW = OFF_B + C::NB * B_STAGE;
    static constexpr int OFF_SC = OFF_RAW + ((C::NR * RAW_STAGE + 1023) / 1024) * 1024;
    static constexpr int SC_PAIR = C::SCN * 2 * 128;  // floats per ring entry
    static constexpr int OFF_BAR = OFF_SC + TC_NS * SC_PAIR * 4;
    static constexpr int N_BARS = 2 * C::NR + C::NA + C::NB + TC_PSLOTS + TC_ND + 2 * TC_NS + 1;
    static constexpr int OFF_MISC = OFF_BAR + N_BARS * 8;
    static constexpr int BYTES = OFF_MISC + 16 + 1024;  // + alignment slack
};

struct TcParams {
    int M, N, K;          // N: activation rows of the operand buffer
    int bw;               // ungrouped column-tile width (<= the kernel's tile width)
    uint8_t *y;
    uint64_t y_nb1;
    const float *dxT;     // [K/32][N] activation block scales
    const float *xsdT;    // [K/32][N] dx * sum(qx) (Q4_K)
    const float *xscale;  // [N] power of two per activation row (split-f16 kernel)
    int32_t *status;
    bool grouped;         // mul_mat_id: column tiles through the group map
    GroupMap g;
    int split_pairs;      // split-K: pairs per CTA along blockIdx.z (0: none)
    float *partial;       // [splits][N][M] when split
    // Tail split (ungrouped, 1D grid): work items [0, tail_full) are whole
    // tiles in (m-tile, n-tile) order; the rest split the last tail_rows
    // m-tile rows (every n-tile of them) tail_S ways in K, item
    // tail_full + t * tail_S + s being split s of tail tile t, written to
    // tail_partial[s][t][128 columns][128 rows]. tail_full < 0: off.
    int tail_full, tail_S, tail_tiles_n, tail_m0, tail_n, tail_split_pairs;
    float *tail_partial;
    // Grouped tail (mul_mat_id, 1D grid; gtail_sms > 0): the same split,
    // planned in the kernel from the routed column tile count (tail_plan);
    // partials in tail_partial as above.
    int gtail_sms;
    bool gtail_even;
    PeerOut peer;         // peer.n > 0 (grouped): outputs into every rank's buffer, then a signal
    EpiAct epi;           // fused bias / SiLU (ungrouped, not split)
};

// Peer mode: count this CTA done; the grid's last CTA raises every rank's
// flag by one (after a system-scope fence, so all CTAs' stores are visible).
__device__ __forceinline__ void peer_cta_done(const PeerOut &pe) {
    __threadfence_system();
    const uint32_t total = gridDim.x * gridDim.y * gridDim.z;
    if (atomicAdd(pe.count, 1u) == total - 1u) {
        atomicExch(pe.count, 0u);
        __threadfence_system();
        for (int r = 0; r < pe.n; r++) atomicAdd_system(pe.flag[r], 1u);
    }
}

// ---- TMA / tcgen05 primitives (inline PTX) -----------------------------------
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

// D[tmem] (+)= A[smem] * B[smem]^T, f16 operands, f32 accumulator.
__device__ __forceinline__ void tc_mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u)
        : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T: A read from tensor memory (lane = row,
// two f16 of K per 32-bit column), f16 operands, f32 accumulator.
__device__ __forceinline__ void tc_mma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u)
        : "memory");
}

// Store 32 consecutive 32-bit TMEM columns of this warp's 32 lanes.
__device__ __forceinline__ void tc_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
        "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
        "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Store 8 consecutive 32-bit TMEM columns of this warp's 32 lanes.
__device__ __forceinline__ void tc_st8(uint32_t taddr, const uint32_t (&r)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
                 "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
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

// 16 consecutive 32-bit TMEM columns of this warp's 32 lanes.
__device__ __forceinline__ void tc_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}

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

// Bounded wait that also gives up when another role has aborted. Roles off
// the MMA thread's critical path back off between polls (`sleep_ns`): a
// dozen warps polling mbarriers slow down everyone's barrier operations.
__device__ __forceinline__ bool tc_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag,
                                        uint32_t sleep_ns = 0) {
    for (uint32_t i = 0; i < kWaitLimit; i++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63u) == 63u && *abort_flag) return false;
        if (sleep_ns) __nanosleep(sleep_ns);
    }
    *abort_flag = 1;
    return false;
}

// Named barrier `id` of `nthreads` threads (whole warps) with an OR vote:
// every participant gets the OR of all votes. It orders memory among the
// participants like __syncthreads (no shared-memory traffic).
__device__ __forceinline__ bool named_bar_red_or(int id, int nthreads, bool vote) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred pv, pr;\n\t"
        "setp.ne.u32 pv, %1, 0;\n\t"
        "bar.red.or.pred pr, %2, %3, pv;\n\t"
        "selp.u32 %0, 1, 0, pr;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)vote), "r"(id), "r"(nthreads)
        : "memory");
    return r != 0;
}

// Warp-uniform form for roles that then run .sync.aligned instructions or
// read what the barrier guards: lane 0 polls, the verdict is broadcast, and
// every lane re-reads the completed phase (acquire).
__device__ __forceinline__ bool tc_wait_warp(uint64_t *bar, uint32_t parity, volatile int *abort_flag, int lane,
                                             uint32_t sleep_ns = 32) {
    int ok = 0;
    if (lane == 0) ok = tc_wait(bar, parity, abort_flag, sleep_ns) ? 1 : 0;
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (ok) mbar_try_wait(bar, parity);
    return ok != 0;
}

// Packed f32x2 arithmetic (sm_100): one instruction for two lanes' worth of
// FP32 work, halving the epilogue's issue slots.
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ uint64_t f2_pack_bits(uint32_t a, uint32_t b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(a), "r"(b));
    return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float &a, float &b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(0u), "r"(sel));
    return r;
}
__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }
__device__ __forceinline__ __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2 *>(&u); }

// 4 signed bytes -> 4 f16 integers (two half2 words), exact:
// (0x6400 | (b ^ 0x80)) is the f16 1024 + (b + 128); minus 1152 gives b.
__device__ __forceinline__ void q8_word_to_f16(uint32_t w, uint32_t &lo, uint32_t &hi) {
    const __half2 off = __half2half2(__ushort_as_half(0x6480));  // 1152
    lo = h2_bits(__hsub2(bits_h2((prmt(w, 0x4140) ^ 0x00800080u) | 0x64006400u), off));
    hi = h2_bits(__hsub2(bits_h2((prmt(w, 0x4342) ^ 0x00800080u) | 0x64006400u), off));
}

// 4 nibble bytes -> low nibbles (4 values) and high nibbles (4 values) as f16
// integers minus `bias` (8 for Q4_0, 0 for Q4_K), exact. Low: the f16
// 1024 + n minus (1024 + bias); high: the nibble sits at bit 4,
// (1024 + 16 n) / 16 - (64 + bias).
template <int BIAS>
__device__ __forceinline__ void nib_word_to_f16(uint32_t w, uint32_t (&lo)[2], uint32_t (&hi)[2]) {
    const __half2 off_lo = __half2half2(__ushort_as_half(BIAS == 8 ? 0x6408 : 0x6400));  // 1032 / 1024
    const __half2 sc_hi = __half2half2(__ushort_as_half(0x2C00));                        // 1/16
    const __half2 off_hi = __half2half2(__ushort_as_half(BIAS == 8 ? 0xD480 : 0xD400));  // -72 / -64
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

__device__ __forceinline__ uint32_t byte_of(const uint32_t *w, int k) { return (w[k >> 2] >> (8 * (k & 3))) & 0xFFu; }

// Q4_K super-block header (4 words: d, dmin as f16, then the 12 bytes of
// 6-bit scales and mins): the scale and min of sub-block j (0..7), in the
// ggml k-quant packing (j < 4: low 6 bits of bytes j and j + 4; j >= 4: a
// nibble of byte j + 4 with the top 2 bits of bytes j - 4 / j).
__device__ __forceinline__ void q4k_scale_min(const uint32_t *hdr, int j, int &sc, int &mn) {
    if (j < 4) {
        sc = (int)(byte_of(hdr, 4 + j) & 63u);
        mn = (int)(byte_of(hdr, 8 + j) & 63u);
    } else {
        sc = (int)((byte_of(hdr, 8 + j) & 0x0Fu) | ((byte_of(hdr, j) >> 6) << 4));
        mn = (int)((byte_of(hdr, 8 + j) >> 4) | ((byte_of(hdr, j + 4) >> 6) << 4));
    }
}

// Words of block pair p of a raw chunk row: Q8_0 17 (68 bytes at 68p, 4-byte
// aligned), Q4_0 9 (36 bytes at 36p), Q4_K 8 (the 32 nibble bytes at
// 16 + 32p; the super-block header comes separately).
template <int WT>
struct PairWords {
    static constexpr int N = WT == WT_Q8_0 ? 17 : (WT == WT_Q4_0 ? 9 : 8);
};

template <int WT>
__device__ __forceinline__ void load_pair_words(const uint8_t *row, int p, uint32_t (&w)[PairWords<WT>::N]) {
    if constexpr (WT == WT_Q4_K) {
        const uint4 *src = reinterpret_cast<const uint4 *>(row + 16 + 32 * p);
        const uint4 a = src[0], b = src[1];
        w[0] = a.x, w[1] = a.y, w[2] = a.z, w[3] = a.w;
        w[4] = b.x, w[5] = b.y, w[6] = b.z, w[7] = b.w;
    } else {
        constexpr int PB = WT == WT_Q8_0 ? 68 : 36;
        const uint32_t *src = reinterpret_cast<const uint32_t *>(row + PB * p);
#pragma unroll
        for (int i = 0; i < PairWords<WT>::N; i++) w[i] = src[i];
    }
}

// The same words through 16-byte loads (Q8_0 / Q4_0): rows of 272 / 144
// bytes are odd multiples of 16, so the 16-byte loads of 8 consecutive rows
// fall in 8 different bank groups (the 4-byte loads of 32 rows 272 bytes
// apart hit only 8 banks). Pair p starts p words into its first 16 bytes.
template <int WT>
__device__ __forceinline__ void load_pair_words_v(const uint8_t *row, int p, uint32_t (&w)[PairWords<WT>::N]) {
    static_assert(WT == WT_Q8_0 || WT == WT_Q4_0, "Q8_0 / Q4_0 rows");
    constexpr int PB = WT == WT_Q8_0 ? 68 : 36, NV = WT == WT_Q8_0 ? 5 : 3;
    const uint4 *src = reinterpret_cast<const uint4 *>(row + ((PB * p) & ~15));
    uint32_t u[4 * NV];
#pragma unroll
    for (int i = 0; i < NV; i++) {
        const uint4 v = src[i];
        u[4 * i] = v.x, u[4 * i + 1] = v.y, u[4 * i + 2] = v.z, u[4 * i + 3] = v.w;
    }
#pragma unroll
    for (int i = 0; i < PairWords<WT>::N; i++) w[i] = u[p + i];
}

// Convert one block pair (its words w; for Q4_K also the super-block header
// hdr and the pair index p) into f16 integers. Returns the pair's row scales
// (sc0, sc1) and, for Q4_K, the min scales (mn0, mn1).
template <int WT>
__device__ __forceinline__ void convert_pair(const uint32_t *w, const uint32_t *hdr, int p, uint32_t (&v0)[16],
                                             uint32_t (&v1)[16], float &sc0, float &sc1, float &mn0, float &mn1) {
    mn0 = mn1 = 0.0f;
    if constexpr (WT == WT_Q8_0) {
        // block 2p: d in the low half of word 0, qs from byte 2
        const int b = 0;
        sc0 = f16_bits_to_f32((uint16_t)(w[b] & 0xFFFFu));
#pragma unroll
        for (int i = 0; i < 8; i++) q8_word_to_f16(__funnelshift_r(w[b + i], w[b + i + 1], 16), v0[2 * i], v0[2 * i + 1]);
        // block 2p+1 at byte 68p + 34: d in the high half of word 17p+8
        sc1 = f16_bits_to_f32((uint16_t)(w[b + 8] >> 16));
#pragma unroll
        for (int i = 0; i < 8; i++) q8_word_to_f16(w[b + 9 + i], v1[2 * i], v1[2 * i + 1]);
    } else if constexpr (WT == WT_Q4_0) {
        // block 2p at word 0, block 2p+1 at byte 18
        const int b = 0;
        sc0 = f16_bits_to_f32((uint16_t)(w[b] & 0xFFFFu));
#pragma unroll
        for (int i = 0; i < 4; i++) {
            uint32_t lo[2], hi[2];
            nib_word_to_f16<8>(__funnelshift_r(w[b + i], w[b + i + 1], 16), lo, hi);
            v0[2 * i] = lo[0];
            v0[2 * i + 1] = lo[1];
            v0[8 + 2 * i] = hi[0];
            v0[8 + 2 * i + 1] = hi[1];
        }
        sc1 = f16_bits_to_f32((uint16_t)(w[b + 4] >> 16));
#pragma unroll
        for (int i = 0; i < 4; i++) {
            uint32_t lo[2], hi[2];
            nib_word_to_f16<8>(w[b + 5 + i], lo, hi);
            v1[2 * i] = lo[0];
            v1[2 * i + 1] = lo[1];
            v1[8 + 2 * i] = hi[0];
            v1[8 + 2 * i + 1] = hi[1];
        }
    } else {
        // Q4_K super-block: d (f16), dmin (f16), 12 bytes of 6-bit scales and
        // mins, 128 bytes of nibbles. Sub-blocks 2p and 2p+1 are the low and
        // high nibbles of bytes 16 + 32p .. 16 + 32p + 31.
        const float d = f16_bits_to_f32((uint16_t)(hdr[0] & 0xFFFFu));
        const float dmin = f16_bits_to_f32((uint16_t)(hdr[0] >> 16));
        int sc[2], mn[2];
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int j = 2 * p + h;
            if (j < 4) {
                sc[h] = (int)(byte_of(hdr, 4 + j) & 63u);
                mn[h] = (int)(byte_of(hdr, 8 + j) & 63u);
            } else {
                sc[h] = (int)((byte_of(hdr, 8 + j) & 0x0Fu) | ((byte_of(hdr, j) >> 6) << 4));
                mn[h] = (int)((byte_of(hdr, 8 + j) >> 4) | ((byte_of(hdr, j + 4) >> 6) << 4));
            }
        }
        sc0 = d * (float)sc[0];
        sc1 = d * (float)sc[1];
        mn0 = dmin * (float)mn[0];
        mn1 = dmin * (float)mn[1];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            uint32_t lo[2], hi[2];
            nib_word_to_f16<0>(w[i], lo, hi);
            v0[2 * i] = lo[0];
            v0[2 * i + 1] = lo[1];
            v1[2 * i] = hi[0];
            v1[2 * i + 1] = hi[1];
        }
    }
}

// One CTA's work: output rows [m0, m0 + 128) x activation rows [xrow0,
// xrow0 + ncols) (ncols <= bn, the kernel's tile width) of weight plane `expert`, over block pairs [pair0, pair0 +
// npairs) (chunks [chunk0, chunk0 + nchunks) of 4 pairs). tsplit >= 0: a
// tail-split CTA (split tsplit of tail tile ttile). unused: a grouped grid's
// spare tile (no work).
struct TileWork {
    int m0, xrow0, ncols, expert, tsplit, ttile, pair0, npairs, chunk0, nchunks;
    int tail_n;  // tail tiles (partial buffer index: split * tail_n + tile)
    bool unused;
};

// Tail split of a grid of tiles_m x tiles_n tiles over `nchunks` weight
// chunks, one CTA per SM on `sms` SMs: when the last wave is a few rows of
// tiles past a whole number of waves, the last `rows` m-tile rows (every
// n-tile of them, so every column of those rows is treated alike) are split
// `splits` ways in K so that their CTAs fill one wave, each doing 1/splits of
// the work, and the launch takes at least one wave less. `even`: slices of
// whole chunk pairs (Q4_K on the split-f16 kernel). Evaluated on the host
// for mul_mat and in the kernels for mul_mat_id, whose column tile count is
// known only on the device.
__host__ __device__ inline bool tail_plan(int64_t tiles_m, int64_t tiles_n, int64_t nchunks, int64_t sms, bool even,
                                          TailPlan *tp) {
    const int64_t tiles = tiles_m * tiles_n;
    if (tiles_n <= 0 || tiles <= sms || nchunks < 4) return false;
    const int64_t over = tiles % sms;
    if (over == 0) return false;
    const int64_t r = (over + tiles_n - 1) / tiles_n, n_tail = r * tiles_n;
    if (r >= tiles_m) return false;
    int64_t S = sms / n_tail;
    if (S > nchunks / 2) S = nchunks / 2;
    if (S > 8) S = 8;
    if (S < 2) return false;
    // whole waves before and after: the split CTAs add 1/S of a wave
    if ((tiles - n_tail + sms - 1) / sms >= (tiles + sms - 1) / sms) return false;
    int64_t per = (nchunks + S - 1) / S;
    if (even) per = (per + 1) / 2 * 2;
    tp->rows = (int)r;
    tp->splits = (int)((nchunks + per - 1) / per);
    tp->split_pairs = (int)(per * CHUNK_PAIRS);
    return tp->splits >= 2;
}

__device__ __forceinline__ TileWork decode_tile(const TcParams &p, int bn) {
    TileWork t;
    t.m0 = blockIdx.x * TC_BM;
    t.xrow0 = blockIdx.y * p.bw;
    t.ncols = min(p.bw, p.N - t.xrow0);
    t.expert = 0;
    t.tsplit = -1;
    t.ttile = 0;
    t.tail_n = p.tail_n;
    t.unused = false;
    int tail_pairs = p.tail_split_pairs;
    int tt = blockIdx.y;  // grouped: column tile over the experts' groups
    if (p.grouped && p.gtail_sms > 0) {
        // 1D grid: tiles in (m-tile, column tile) order over the column tile
        // count the routing wrote, then the tail split's work items; the
        // grid is sized for the largest count, the rest exit
        const int T = p.g.tile_start[p.g.n_groups];
        const int tiles_m = (p.M + TC_BM - 1) / TC_BM;
        TailPlan tp{};
        const bool on = tail_plan(tiles_m, T, p.K / QKK, p.gtail_sms, p.gtail_even, &tp);
        const int n_tail = on ? tp.rows * T : 0, full = tiles_m * T - n_tail;
        const int w = (int)blockIdx.x;
        int mt;
        if (w < full) {
            mt = w / T;
            tt = w % T;
        } else if (on && w < full + n_tail * tp.splits) {
            t.tsplit = (w - full) % tp.splits;
            t.ttile = (w - full) / tp.splits;
            mt = tiles_m - tp.rows + t.ttile / T;
            tt = t.ttile % T;
            t.tail_n = n_tail;
            tail_pairs = tp.split_pairs;
        } else {
            t.unused = true;
            t.npairs = t.nchunks = 0;
            return t;
        }
        t.m0 = mt * TC_BM;
    } else if (p.tail_full >= 0) {
        const int w = (int)blockIdx.x;
        int mt, nt;
        if (w < p.tail_full) {
            mt = w / p.tail_tiles_n;
            nt = w % p.tail_tiles_n;
        } else {
            t.tsplit = (w - p.tail_full) % p.tail_S;
            t.ttile = (w - p.tail_full) / p.tail_S;
            mt = p.tail_m0 + t.ttile / p.tail_tiles_n;
            nt = t.ttile % p.tail_tiles_n;
        }
        t.m0 = mt * TC_BM;
        t.xrow0 = nt * p.bw;
        t.ncols = min(p.bw, p.N - t.xrow0);
    }
    if (p.grouped) {
        if (tt >= p.g.tile_start[p.g.n_groups]) {
            t.unused = true;
            t.npairs = t.nchunks = 0;
            return t;
        }
        while (p.g.tile_start[t.expert + 1] <= tt) t.expert++;
        const int jt = tt - p.g.tile_start[t.expert];
        t.xrow0 = p.g.offsets[t.expert] + jt * bn;
        t.ncols = min(bn, p.g.counts[t.expert] - jt * bn);
    }
    // K range in block pairs (split-K: a slice per blockIdx.z); chunks of 4 pairs
    const int total_pairs = p.K / (2 * QK);
    t.pair0 = t.tsplit >= 0 ? t.tsplit * tail_pairs : (p.split_pairs ? (int)blockIdx.z * p.split_pairs : 0);
    t.npairs = t.tsplit >= 0    ? min(tail_pairs, total_pairs - t.pair0)
               : p.split_pairs ? min(p.split_pairs, total_pairs - t.pair0)
                               : total_pairs;
    t.chunk0 = t.pair0 / CHUNK_PAIRS;
    t.nchunks = t.npairs / CHUNK_PAIRS;
    return t;
}

template <int WT, bool PEER>
__global__ void __launch_bounds__(TC_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                   const TcParams p) {
    using C = TcCfg<WT>;
    using L = TcLayout<WT>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
    uint8_t *gbase = smem_raw + (sbase - smem_u32(smem_raw));

    const TileWork tw = decode_tile(p, TC_BN);
    if (tw.unused) {  // unused tile (uniform, before any set-up)
        if (PEER && threadIdx.x == 0) peer_cta_done(p.peer);
        return;
    }
    const int m0 = tw.m0, xrow0 = tw.xrow0, ncols = tw.ncols, expert = tw.expert;
    const int pair0 = tw.pair0, npairs = tw.npairs, chunk0 = tw.chunk0, nchunks = tw.nchunks;

    // Barriers. tcgen05.commit arrivals complete one after another (a few
    // hundred cycles each), so the MMA thread commits once per block pair:
    // pair_done[q % TC_ND] completes when pair q's MMAs have finished, which
    // at once frees its A and B stages and hands its TMEM slot to the
    // epilogue.
    uint64_t *bars = reinterpret_cast<uint64_t *>(gbase + L::OFF_BAR);
    uint64_t *raw_full = bars;
    uint64_t *raw_empty = raw_full + C::NR;
    uint64_t *a_full = raw_empty + C::NR;
    uint64_t *b_full = a_full + C::NA;
    uint64_t *t_empty = b_full + C::NB;
    uint64_t *pair_done = t_empty + TC_PSLOTS;
    uint64_t *s_full = pair_done + TC_ND;
    uint64_t *s_empty = s_full + TC_NS;
    uint64_t *mma_done = s_empty + TC_NS;
    // phase parity of pair_done for pair q
    auto done_parity = [](int q) { return (uint32_t)((q / TC_ND) & 1); };
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(gbase + L::OFF_MISC);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(gbase + L::OFF_MISC + 4);
    float *ring = reinterpret_cast<float *>(gbase + L::OFF_SC);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // epilogue warps with columns: a narrow tile (a group's or the matrix's
    // last columns) leaves whole column quarters empty, and their warps sit
    // the tile out instead of polling the pipeline's barriers
    const int epi_live = 4 * min(4, (ncols + 31) / 32);

    if (tid == 0) {
        for (int i = 0; i < C::NR; i++) {
            mbar_init(&raw_full[i], 1);
            mbar_init(&raw_empty[i], 128);
        }
        for (int i = 0; i < C::NA; i++) mbar_init(&a_full[i], 128);
        for (int i = 0; i < C::NB; i++) mbar_init(&b_full[i], 1);
        for (int i = 0; i < TC_PSLOTS; i++) mbar_init(&t_empty[i], epi_live);
        for (int i = 0; i < TC_ND; i++) mbar_init(&pair_done[i], 1);
        for (int i = 0; i < TC_NS; i++) {
            mbar_init(&s_full[i], 128 + 32);  // converter rows + the activation-scale warp
            mbar_init(&s_empty[i], epi_live);
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
                if (!tc_wait(&raw_empty[s], ((c / C::NR) & 1) ^ 1, abort_flag, 64)) break;
                mbar_arrive_expect_tx(&raw_full[s], L::RAW_STAGE);
                const int gc = chunk0 + c;
                const int x0 = WT == WT_Q8_0 ? gc * (C::RAWB / 2) : gc * C::RAWB;
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
                if (q >= C::NB &&
                    !tc_wait(&pair_done[(q - C::NB) % TC_ND], done_parity(q - C::NB), abort_flag, 64))
                    break;
                mbar_arrive_expect_tx(&b_full[s], B_STAGE);
                tma_load_2d(sbase + L::OFF_B + s * B_STAGE, &tm_x, (pair0 + q) * 64, xrow0, smem_u32(&b_full[s]));
                armed[s] = (q / C::NB) & 1;
            }
            if (*abort_flag)
                for (int i = 0; i < C::NB; i++)
                    if (armed[i] >= 0) mbar_wait_bounded(&b_full[i], (uint32_t)armed[i]);
        }
    } else if (warp == 3) {
        // ---- activation block scales into the scale ring (one pair ahead) -------
        // lane l stages columns 4l..4l+3 of both blocks of a pair
        constexpr int NP = C::SCN / 2;  // per-column planes: dx (+ dx*sum(qx) for Q4_K)
        auto load = [&](int q, float4 (&v)[NP][2]) {
#pragma unroll
            for (int j = 0; j < 2; j++) {
                const uint64_t base = (uint64_t)(2 * (pair0 + q) + j) * (uint64_t)p.N + xrow0;
#pragma unroll
                for (int pl = 0; pl < NP; pl++) {
                    const float *src = pl == 0 ? p.dxT : p.xsdT;
                    float t[4];
#pragma unroll
                    for (int i = 0; i < 4; i++) t[i] = (4 * lane + i < ncols) ? src[base + 4 * lane + i] : 0.0f;
                    v[pl][j] = make_float4(t[0], t[1], t[2], t[3]);
                }
            }
        };
        float4 cur[NP][2], nxt[NP][2];
        if (npairs > 0) load(0, cur);
        for (int q = 0; q < npairs; q++) {
            if (q + 1 < npairs) load(q + 1, nxt);
            const int ss = q % TC_NS;
            if (!tc_wait_warp(&s_empty[ss], ((q / TC_NS) & 1) ^ 1, abort_flag, lane)) break;
            float *e = ring + ss * L::SC_PAIR;
#pragma unroll
            for (int j = 0; j < 2; j++)
#pragma unroll
                for (int pl = 0; pl < NP; pl++)
                    *reinterpret_cast<float4 *>(e + ((1 + 2 * pl) * 2 + j) * 128 + 4 * lane) = cur[pl][j];
            mbar_arrive(&s_full[ss]);
#pragma unroll
            for (int j = 0; j < 2; j++)
#pragma unroll
                for (int pl = 0; pl < NP; pl++) cur[pl][j] = nxt[pl][j];
        }
    } else if (warp == 2) {
        // ---- MMA issue (one thread) ---------------------------------------------
        if (lane == 0) {
            // a narrow tile multiplies only its columns, rounded up to the
            // MMA's N granularity of 16 (M = 128: N = 16..256, N % 16 == 0)
            constexpr uint32_t idesc = f16_idesc(TC_BM, TC_BN);
            bool ok = true;
            for (int q = 0; q < npairs && ok; q++) {
                const int sa = q % C::NA, sb = q % C::NB;
                if (!tc_wait(&a_full[sa], (q / C::NA) & 1, abort_flag) ||
                    !tc_wait(&b_full[sb], (q / C::NB) & 1, abort_flag)) {
                    ok = false;
                    break;
                }
                const int ps = q % TC_PSLOTS;
                if (!tc_wait(&t_empty[ps], ((q / TC_PSLOTS) & 1) ^ 1, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t a_addr = sbase + L::OFF_A + sa * A_STAGE;
                const uint32_t b_addr = sbase + L::OFF_B + sb * B_STAGE;
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    const uint32_t d = tmem + (uint32_t)((2 * ps + j) * TC_BN);
                    const uint32_t aj = a_addr + 64u * j, bj = b_addr + 64u * j;
                    tc_mma_f16(d, sw128_desc(aj), sw128_desc(bj), idesc, 0u);            // k 0-15
                    tc_mma_f16(d, sw128_desc(aj + 32), sw128_desc(bj + 32), idesc, 1u);  // k 16-31
                }
                tc_commit(smem_u32(&pair_done[q % TC_ND]));
            }
            // all issued MMAs complete before TMEM can be released
            tc_commit(smem_u32(mma_done));
            mbar_wait_bounded(mma_done, 0);
        }
    } else if (warp >= 4 && warp < 8) {
        // ---- converters: one weight row per thread, one block pair at a time ----
        const int row = tid - 128;
        for (int c = 0; c < nchunks; c++) {
            const int s = c % C::NR;
            if (!tc_wait_warp(&raw_full[s], (c / C::NR) & 1, abort_flag, lane)) break;
            const uint8_t *rrow = gbase + L::OFF_RAW + s * L::RAW_STAGE + row * C::RAWB;
            uint32_t hdr[4] = {0u, 0u, 0u, 0u};
            if constexpr (WT == WT_Q4_K) {
                const uint4 hv = *reinterpret_cast<const uint4 *>(rrow);
                hdr[0] = hv.x, hdr[1] = hv.y, hdr[2] = hv.z, hdr[3] = hv.w;
            }
            bool ok = true;
#pragma unroll
            for (int pp = 0; pp < CHUNK_PAIRS; pp++) {
                const int q = CHUNK_PAIRS * c + pp;
                const int sa = q % C::NA, ss = q % TC_NS;
                uint32_t w[PairWords<WT>::N];
                load_pair_words<WT>(rrow, pp, w);
                if (pp == CHUNK_PAIRS - 1) mbar_arrive(&raw_empty[s]);  // the chunk is in registers
                if ((q >= C::NA &&
                     !tc_wait_warp(&pair_done[(q - C::NA) % TC_ND], done_parity(q - C::NA), abort_flag, lane)) ||
                    !tc_wait_warp(&s_empty[ss], ((q / TC_NS) & 1) ^ 1, abort_flag, lane)) {
                    ok = false;
                    break;
                }
                // the stage was last read by the tensor core (async proxy):
                // order those reads before this thread's generic stores
                fence_proxy_async_smem();
                uint32_t v0[16], v1[16];
                float sc0, sc1, mn0, mn1;
                convert_pair<WT>(w, hdr, pp, v0, v1, sc0, sc1, mn0, mn1);
                const uint32_t a_addr = sbase + L::OFF_A + sa * A_STAGE;
                store_a_block(a_addr, row, 0, v0);
                store_a_block(a_addr, row, 1, v1);
                float *e = ring + ss * L::SC_PAIR;
                e[0 * 128 + row] = sc0;
                e[1 * 128 + row] = sc1;
                if constexpr (C::SCN == 4) {
                    e[4 * 128 + row] = mn0;
                    e[5 * 128 + row] = mn1;
                }
                fence_proxy_async_smem();
                mbar_arrive(&a_full[sa]);
                mbar_arrive(&s_full[ss]);
            }
            if (!ok) break;
        }
    } else if (warp >= 8) {
        // ---- epilogue: warp w reads TMEM lanes 32*(w%4).., columns 32*qc.. ------
        const int sub = warp & 3, qc = (warp - 8) >> 2;  // lane quarter, column quarter
        const int row = 32 * sub + lane;
        const bool live = 32 * qc < ncols;
        uint64_t acc2[16];  // columns (2i, 2i+1) of the warp's 32, as f32x2
#pragma unroll
        for (int i = 0; i < 16; i++) acc2[i] = 0;
        bool ok = live;
        for (int q = 0; q < npairs && ok; q++) {
            const int ss = q % TC_NS;
            if (!tc_wait_warp(&s_full[ss], (q / TC_NS) & 1, abort_flag, lane)) {
                ok = false;
                break;
            }
            const float *e = ring + ss * L::SC_PAIR;
            const int ps = q % TC_PSLOTS;
            if (!tc_wait_warp(&pair_done[q % TC_ND], done_parity(q), abort_flag, lane)) {
                ok = false;
                break;
            }
            tc_fence_after();
            // 4 chunks of 16 columns (2 blocks x 2); the load of chunk k+1 is in
            // flight while chunk k is scaled and accumulated
            const uint32_t tbase = tmem + ((uint32_t)(32 * sub) << 16) + (uint32_t)(2 * ps * TC_BN + 32 * qc);
            uint32_t ra[16], rb[16];
            tc_ld16(tbase, ra);
            tc_wait_ld();
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const int j = k >> 1, cc = k & 1;
                if (k + 1 < 4) {
                    const int jn = (k + 1) >> 1, cn = (k + 1) & 1;
                    if (k & 1)
                        tc_ld16(tbase + (uint32_t)(jn * TC_BN + 16 * cn), ra);
                    else
                        tc_ld16(tbase + (uint32_t)(jn * TC_BN + 16 * cn), rb);
                }
                const uint32_t(&r)[16] = (k & 1) ? rb : ra;
                const float sw = e[(0 * 2 + j) * 128 + row];
                const uint64_t sw2 = f2_pack(sw, sw);
                const float mw = C::SCN == 4 ? -e[(2 * 2 + j) * 128 + row] : 0.0f;
                const uint64_t mw2 = f2_pack(mw, mw);
                const float4 *dxv = reinterpret_cast<const float4 *>(e + (1 * 2 + j) * 128 + 32 * qc + 16 * cc);
                const float4 *xsv = reinterpret_cast<const float4 *>(e + (3 * 2 + j) * 128 + 32 * qc + 16 * cc);
#pragma unroll
                for (int i4 = 0; i4 < 4; i4++) {
                    const float4 dq = dxv[i4];
                    const uint64_t s01 = f2_mul(sw2, f2_pack(dq.x, dq.y));
                    const uint64_t s23 = f2_mul(sw2, f2_pack(dq.z, dq.w));
                    uint64_t &a01 = acc2[8 * cc + 2 * i4];
                    uint64_t &a23 = acc2[8 * cc + 2 * i4 + 1];
                    a01 = f2_fma(f2_pack_bits(r[4 * i4], r[4 * i4 + 1]), s01, a01);
                    a23 = f2_fma(f2_pack_bits(r[4 * i4 + 2], r[4 * i4 + 3]), s23, a23);
                    if constexpr (C::SCN == 4) {
                        const float4 xq = xsv[i4];
                        a01 = f2_fma(mw2, f2_pack(xq.x, xq.y), a01);
                        a23 = f2_fma(mw2, f2_pack(xq.z, xq.w), a23);
                    }
                }
                if (k + 1 < 4) tc_wait_ld();
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&t_empty[ps]);
                mbar_arrive(&s_empty[ss]);
            }
        }
        // The tile leaves through shared memory: staged as [column][128 rows]
        // in the A stages (free once every pair's MMAs have completed), then
        // each column's rows go out as one 512-byte store per warp (per-lane
        // scalar stores to 32 output rows were as slow as the main loop in
        // the split-f16 kernel).
        float *stage = reinterpret_cast<float *>(gbase + L::OFF_A);
        static_assert(C::NA * A_STAGE >= TC_BN * TC_BM * 4, "the output tile is staged in the A stages");
        if (ok) {
            float acc[32];
#pragma unroll
            for (int i = 0; i < 16; i++) f2_unpack(acc2[i], acc[2 * i], acc[2 * i + 1]);
#pragma unroll
            for (int i = 0; i < 32; i++) stage[(32 * qc + i) * TC_BM + row] = acc[i];
        }
        asm volatile("bar.sync 1, 512;" ::: "memory");  // the 16 epilogue warps
        if (!*abort_flag) {
            const int rows_valid = min(TC_BM, p.M - m0);
            const int r0 = 4 * lane;
            const int pb = PEER ? (int)((*p.peer.epoch + 1u) & 1u) : 0;
            for (int c = warp - 8; c < ncols; c += TC_EPI_WARPS) {
                const int r = xrow0 + c;
                float4 v = *reinterpret_cast<const float4 *>(stage + c * TC_BM + r0);
                uint8_t *dst;
                int owner = -1;
                bool plain = false;
                if (tw.tsplit >= 0) {
                    dst = reinterpret_cast<uint8_t *>(p.tail_partial +
                                                      (((uint64_t)tw.tsplit * tw.tail_n + tw.ttile) * TC_BN + c) * TC_BM);
                } else if (p.partial) {
                    dst = reinterpret_cast<uint8_t *>(p.partial + ((uint64_t)blockIdx.z * p.N + r) * p.M + m0);
                } else {
                    uint64_t off;
                    if (p.grouped) {
                        const int slot = p.g.rows[r];
                        int tok = slot / p.g.n_selected;
                        if (PEER && p.peer.owner_tokens > 0) {
                            owner = tok / p.peer.owner_tokens;
                            tok -= owner * p.peer.owner_tokens;
                        }
                        off = (uint64_t)(slot % p.g.n_selected) * p.g.dst_nb1 + (uint64_t)tok * p.g.dst_nb2;
                    } else {
                        off = (uint64_t)r * p.y_nb1;
                    }
                    off += (uint64_t)m0 * 4;
                    dst = PEER ? reinterpret_cast<uint8_t *>(off) : p.y + off;
                    plain = !PEER;
                }
                if (plain && (p.epi.bias || p.epi.silu)) {  // fused bias / SiLU on y
                    if (r0 < rows_valid) v.x = apply_act(v.x, p.epi, m0 + r0);
                    if (r0 + 1 < rows_valid) v.y = apply_act(v.y, p.epi, m0 + r0 + 1);
                    if (r0 + 2 < rows_valid) v.z = apply_act(v.z, p.epi, m0 + r0 + 2);
                    if (r0 + 3 < rows_valid) v.w = apply_act(v.w, p.epi, m0 + r0 + 3);
                }
                auto put = [&](uint8_t *base) {
                    float *o = reinterpret_cast<float *>(base) + r0;
                    if (r0 + 4 <= rows_valid && (reinterpret_cast<uintptr_t>(base) & 15) == 0) {
                        *reinterpret_cast<float4 *>(o) = v;
                    } else {
                        if (r0 < rows_valid) o[0] = v.x;
                        if (r0 + 1 < rows_valid) o[1] = v.y;
                        if (r0 + 2 < rows_valid) o[2] = v.z;
                        if (r0 + 3 < rows_valid) o[3] = v.w;
                    }
                };
                if (PEER && tw.tsplit < 0 && !p.partial) {  // NVLink stores into the owner's buffer, or every rank's
                    const uint64_t off = reinterpret_cast<uint64_t>(dst);
                    if (owner >= 0)
                        put(p.peer.y[pb][owner] + off);
                    else
                        for (int pr = 0; pr < p.peer.n; pr++) put(p.peer.y[pb][pr] + off);
                } else {
                    put(dst);
                }
            }
        }
    }

    // the epilogue threads' peer stores, before the CTA counts itself done
    if (PEER && warp >= 8) __threadfence_system();
    tc_fence_before();
    __syncthreads();
    if (*abort_flag && tid == 0) report_status(p.status, STATUS_TIMEOUT);
    if (PEER && tid == 0) peer_cta_done(p.peer);
    if (warp == 2) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TC_TMEM_COLS)
                     : "memory");
    }
}

// ---- split-f16 dequantizing GEMM (Q8_0, Q4_0) ---------------------------------
// Every dequantized operand value is an f16 block scale times a small
// integer: weights d*q (q in [-128, 127] for Q8_0, [-8, 7] for Q4_0), the
// Q8_0-rounded activations dx*qx (qx in [-127, 127]). Such a product has at
// most 11 + 8 significant bits, so it is exactly hi + lo with hi = rn16(d*q)
// and lo = d*q - hi (both f16; the f16 fma computes the remainder exactly).
// The tensor core then accumulates
//     D += Ahi*Bhi + Ahi*Blo + Alo*Bhi       (Alo*Blo < 2^-22 of each product)
// in f32 over the tile's whole K range: three MMAs per K step and no
// per-block epilogue; the accumulator is read once, at the end of the tile.
// Range: activation row t is scaled by a power of two 2^-e_t (exact) that
// puts its largest value below 2^15, and the epilogue multiplies by 2^e_t.
// Weights are used unscaled; a block scale whose products leave the f16
// range (Q8_0 |d| > 511.75, Q4_0 |d| > 8188) raises STATUS_RANGE.
//
// Operands: the weight tile (A) lives in tensor memory, written there by
// the converters (tcgen05.st, one TMEM lane per weight row), so the MMAs read
// only the activations from shared memory: three 128 x 128 x 16 MMAs with
// both operands in shared memory would need 96 KB of operand reads per block
// pair, as much shared-memory bandwidth as they have time for.
// Tiles are 128 weight rows x 192 activation rows: each converted weight
// tile feeds up to 192 columns, the MMAs (N up to 192) stay ahead of their
// issue, three activation stages fit beside the raw weight ring, and a
// mul_mat_id expert group of up to 192 routed rows is one tile.
// TMEM columns: [0, 192) the f32 accumulator ([0, 256) stacked); then T3Cfg::NA slots of 64
// columns, one block pair each (hi plane: 32 columns of two f16, lo plane:
// the next 32).
// An ungrouped product of at most 128 columns (one tile) stacks the
// activation planes (the STACK instantiation): the stage holds the hi rows, then the lo rows right
// after them (W = 64 * ceil(ncols / 64) rows each), and a K step is two
// MMAs instead of three: Ahi x [Bhi; Blo]
// (N = 2W, columns [0, W) += Ahi.Bhi and [W, 2W) += Ahi.Blo) and Alo x Bhi
// (N = W, into [0, W)); the epilogue adds the two halves. An MMA's cost has
// a floor well above its N / 2 cycles at small N, so fewer, wider MMAs win.
// Roles (512 threads):
//   warp 0      TMA: raw weight chunks (8 blocks x 128 rows), as gemm_tc_kernel.
//   warp 1      TMA: activation stages (192 rows x 64 f16, the hi and lo
//               planes) into a ring of T3Cfg::NBP block pairs.
//   warp 2      TMEM (512 columns) and the MMAs (one thread, one commit per
//               block pair, which frees its A slot and its B stage).
//   warp 3      gate: waits for a pair's A slot and B stage, then meets the
//               MMA warp at named barrier T3_GATE_BAR with its verdict, so
//               the MMA warp never polls a shared-memory barrier (those
//               polls are slow while the tensor core streams operands from
//               shared memory; a named barrier does not touch it).
//   warps 4-7   converters: one weight row (= TMEM lane) each; hi and lo of
//               a pair into an A slot.
//   warps 8-15  epilogue: lane quarter warp % 4, 96 columns each.
constexpr int T3_THREADS = 512;
constexpr int T3_GATE_BAR = 2;  // named barrier of warps 2 and 3 (0: __syncthreads, 1: epilogue)
constexpr int T3_BN = 192;
constexpr int T3_TMEM_COLS = 512;
constexpr int T3_ACC_COLS = 256;  // accumulator region; the A slots follow
constexpr int T3_HALF = T3_BN * 128;  // one plane of a block pair: 192 rows x 64 f16
constexpr int T3_XB = 64;              // activation rows per TMA box (T3_BN % T3_XB == 0, 8-row swizzle groups)
static_assert(T3_BN % T3_XB == 0 && T3_XB % 8 == 0, "activation boxes");

template <int WT>
struct T3Cfg;
template <>
struct T3Cfg<WT_Q8_0> {
    static constexpr int NR = 2, NA = 4, NBP = 3;
    static constexpr float kMaxScale = 65504.0f / 128.0f;
};
template <>
struct T3Cfg<WT_Q4_0> {
    static constexpr int NR = 4, NA = 4, NBP = 3;
    static constexpr float kMaxScale = 65504.0f / 8.0f;
};
// Q4_K: w = d*(sc*q) - dmin*m. sc*q <= 63*15 = 945 is an exact f16 integer, so
// d*(sc*q) splits into hi + lo exactly as the other types do; the min term is
// carried as extra contraction positions (below). Limits: d*945 and dmin*63
// within the f16 range.
template <>
struct T3Cfg<WT_Q4_K> {
    static constexpr int NR = 4, NA = 4, NBP = 3;
    static constexpr float kMaxScale = 65504.0f / 945.0f;
    static constexpr float kMaxMin = 65504.0f / 63.0f;
};

template <int WT>
struct T3Layout {
    using C = T3Cfg<WT>;
    static_assert(T3_BN <= T3_ACC_COLS && T3_ACC_COLS + 64 * C::NA <= T3_TMEM_COLS, "TMEM: accumulator + A slots");
    static constexpr int RAW_STAGE = TC_BM * TcCfg<WT>::RAWB;
    static constexpr int B_STAGE3 = 2 * T3_HALF;  // [hi plane][lo plane]
    static constexpr int OFF_B = 0;
    static constexpr int OFF_RAW = OFF_B + C::NBP * B_STAGE3;
    static constexpr int OFF_BAR = OFF_RAW + ((C::NR * RAW_STAGE + 1023) / 1024) * 1024;
    static constexpr int N_BARS = 2 * C::NR + C::NA + C::NBP + TC_ND + 1;
    // epilogue column table: destination (8 bytes), scale, owner rank
    static constexpr int OFF_COLS = OFF_BAR + ((N_BARS * 8 + 15) / 16) * 16;
    static constexpr int OFF_MISC = OFF_COLS + T3_BN * 16;
    static constexpr int BYTES = OFF_MISC + 16 + 1024;  // + alignment slack
    static_assert(C::NBP * B_STAGE3 >= T3_BN * TC_BM * 4, "the output tile is staged in the activation ring");
};

// The tile's output column c (row 0 of the tile): where it goes, its
// activation row scale, and (peer mode) the rank that receives it (-1: all).
struct T3Col {
    uint64_t dst;  // byte address (peer mode: byte offset in a rank's buffer)
    float scale;
    int owner;
};

// One block's 16 words of exact f16 integers (element order) times the
// block scale d, split into the hi and lo planes (16 words each).
__device__ __forceinline__ void split_block(const uint32_t (&v)[16], __half2 d2, uint32_t *hi, uint32_t *lo) {
#pragma unroll
    for (int i = 0; i < 16; i++) {
        const __half2 h = __hmul2(bits_h2(v[i]), d2);
        hi[i] = h2_bits(h);
        lo[i] = h2_bits(__hfma2(bits_h2(v[i]), d2, __hneg2(h)));
    }
}

template <int WT, bool PEER, bool STACK>
__global__ void __launch_bounds__(T3_THREADS, 1)
    gemm_tc3_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                    const TcParams p) {
    using C = T3Cfg<WT>;
    using L = T3Layout<WT>;
    using RC = TcCfg<WT>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
    uint8_t *gbase = smem_raw + (sbase - smem_u32(smem_raw));

    const TileWork tw = decode_tile(p, T3_BN);
    if (tw.unused) {  // unused tile (uniform, before any set-up)
        if (PEER && threadIdx.x == 0) peer_cta_done(p.peer);
        return;
    }
    const int m0 = tw.m0, xrow0 = tw.xrow0, ncols = tw.ncols, expert = tw.expert;
    const int chunk0 = tw.chunk0, nchunks = tw.nchunks;
    // Contraction steps ("pairs", 64 positions each). Q4_K: every two
    // super-blocks (8 pairs) are followed by one extra pair whose first 16
    // positions hold the 16 sub-blocks' -dmin*m against the activation block
    // sums (the rest of it is not multiplied); the activation planes are laid
    // out the same way (576 positions per 512 elements). Tiles and splits
    // cover whole super-block pairs, so chunk0 and nchunks are even.
    const int pair0 = WT == WT_Q4_K ? chunk0 / 2 * 9 : tw.pair0;
    const int npairs = WT == WT_Q4_K ? nchunks / 2 * 9 : tw.npairs;
    // STACK (an ungrouped product of at most 128 columns, one tile): the
    // activation planes are stacked, W rows each. Its rounding differs from
    // the three-MMA form's, and every column of the product is treated
    // alike, so permuting the columns permutes the output bits.
    static_assert(T3_XB == 64, "stacked planes use 64-row boxes");
    const int stack_w = STACK ? T3_XB * ((ncols + T3_XB - 1) / T3_XB) : 0;
    constexpr int acol0 = STACK ? T3_ACC_COLS : T3_BN;  // TMEM column of the first A slot

    uint64_t *bars = reinterpret_cast<uint64_t *>(gbase + L::OFF_BAR);
    uint64_t *raw_full = bars;
    uint64_t *raw_empty = raw_full + C::NR;
    uint64_t *a_full = raw_empty + C::NR;
    uint64_t *b_full = a_full + C::NA;
    uint64_t *pair_done = b_full + C::NBP;
    uint64_t *mma_done = pair_done + TC_ND;
    auto done_parity = [](int q) { return (uint32_t)((q / TC_ND) & 1); };
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(gbase + L::OFF_MISC);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(gbase + L::OFF_MISC + 4);
    int *range_flag = reinterpret_cast<int *>(gbase + L::OFF_MISC + 8);
    T3Col *cols = reinterpret_cast<T3Col *>(gbase + L::OFF_COLS);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    if (tid == 0) {
        for (int i = 0; i < C::NR; i++) {
            mbar_init(&raw_full[i], 1);
            mbar_init(&raw_empty[i], WT == WT_Q4_K ? 256 : 128);  // Q4_K: both converter groups
        }
        for (int i = 0; i < C::NA; i++) mbar_init(&a_full[i], 128);
        for (int i = 0; i < C::NBP; i++) {
            mbar_init(&b_full[i], 1);
        }
        for (int i = 0; i < TC_ND; i++) mbar_init(&pair_done[i], 1);
        mbar_init(mma_done, 1);
        *abort_flag = 0;
        *range_flag = 0;
        fence_barrier_init();
    }
    if (warp == 2) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(T3_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // Q4_K converters: group 0 is warps 4-7, group 1 warps 8-11 (which then
    // run the epilogue); warp w writes TMEM lanes 32*(w % 4) .. +31.
    auto convert_q4k = [&](auto grp_c) {
        constexpr int grp = decltype(grp_c)::value;
        if constexpr (WT == WT_Q4_K) {
            // Q4_K: a chunk is one super-block (4 pairs); after every second
            // one, the min-term pair of both (see the pair numbering above).
            // Group grp converts pairs 2grp and 2grp+1 of every super-block;
            // group 1 also the min-term pairs.
            const int row = 32 * (warp & 3) + lane;
            bool range_ok = true;
            float mins[8];  // -dmin*m of the previous (even) super-block, exact in f32
            for (int c = 0; c < nchunks; c++) {
                const int s = c % C::NR;
                if (!tc_wait_warp(&raw_full[s], (c / C::NR) & 1, abort_flag, lane)) break;
                const uint8_t *rrow = gbase + L::OFF_RAW + s * L::RAW_STAGE + row * RC::RAWB;
                const uint4 hv = *reinterpret_cast<const uint4 *>(rrow);
                const uint32_t hdr[4] = {hv.x, hv.y, hv.z, hv.w};
                uint32_t w[2][8];
#pragma unroll
                for (int j = 0; j < 2; j++) load_pair_words<WT>(rrow, 2 * grp + j, w[j]);
                mbar_arrive(&raw_empty[s]);  // the super-block is in registers
                const float d = f16_bits_to_f32((uint16_t)(hdr[0] & 0xFFFFu));
                const float dmin = f16_bits_to_f32((uint16_t)(hdr[0] >> 16));
                range_ok = range_ok && fabsf(d) <= C::kMaxScale && fabsf(dmin) <= C::kMaxMin;
                const __half2 d2 = __half2half2(__ushort_as_half((uint16_t)(hdr[0] & 0xFFFFu)));
                bool ok = true;
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    const int pp = 2 * grp + j;
                    const int q = (c >> 1) * 9 + (c & 1) * CHUNK_PAIRS + pp;
                    const int sa = q % C::NA;
                    int sc0, mn0, sc1, mn1;
                    q4k_scale_min(hdr, 2 * pp, sc0, mn0);
                    q4k_scale_min(hdr, 2 * pp + 1, sc1, mn1);
                    const __half2 s0 = __float2half2_rn((float)sc0), s1 = __float2half2_rn((float)sc1);
                    uint32_t v0[16], v1[16];
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        uint32_t lo[2], hi[2];
                        nib_word_to_f16<0>(w[j][i], lo, hi);
                        // sc * q: exact f16 integers (<= 945)
                        v0[2 * i] = h2_bits(__hmul2(bits_h2(lo[0]), s0));
                        v0[2 * i + 1] = h2_bits(__hmul2(bits_h2(lo[1]), s0));
                        v1[2 * i] = h2_bits(__hmul2(bits_h2(hi[0]), s1));
                        v1[2 * i + 1] = h2_bits(__hmul2(bits_h2(hi[1]), s1));
                    }
                    uint32_t h[32], l[32];
                    split_block(v0, d2, h, l);
                    split_block(v1, d2, h + 16, l + 16);
                    if (q >= C::NA &&
                        !tc_wait_warp(&pair_done[(q - C::NA) % TC_ND], done_parity(q - C::NA), abort_flag, lane)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t ta = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + (uint32_t)(acol0 + 64 * sa);
                    tc_st32(ta, h);
                    tc_st32(ta + 32u, l);
                    tc_wait_st();
                    tc_fence_before();
                    mbar_arrive(&a_full[sa]);
                }
                if (!ok) break;
                if constexpr (grp == 1) {
                    float cur[8];
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        int scj, mnj;
                        q4k_scale_min(hdr, j, scj, mnj);
                        cur[j] = -(dmin * (float)mnj);  // exact: 11 + 6 significant bits
                    }
                    if ((c & 1) == 0) {
#pragma unroll
                        for (int j = 0; j < 8; j++) mins[j] = cur[j];
                        continue;
                    }
                    // the min-term pair: 16 values (sub-blocks of super-blocks c-1, c)
                    const int q = (c >> 1) * 9 + 8;
                    const int sa = q % C::NA;
                    uint32_t h8[8], l8[8];
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        const float a = i < 4 ? mins[2 * i] : cur[2 * i - 8];
                        const float b = i < 4 ? mins[2 * i + 1] : cur[2 * i - 7];
                        const __half ha = __float2half_rn(a), hb = __float2half_rn(b);
                        const __half la = __float2half_rn(a - __half2float(ha)), lb = __float2half_rn(b - __half2float(hb));
                        h8[i] = (uint32_t)__half_as_ushort(ha) | ((uint32_t)__half_as_ushort(hb) << 16);
                        l8[i] = (uint32_t)__half_as_ushort(la) | ((uint32_t)__half_as_ushort(lb) << 16);
                    }
                    if (q >= C::NA &&
                        !tc_wait_warp(&pair_done[(q - C::NA) % TC_ND], done_parity(q - C::NA), abort_flag, lane))
                        break;
                    tc_fence_after();
                    const uint32_t ta = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + (uint32_t)(acol0 + 64 * sa);
                    tc_st8(ta, h8);
                    tc_st8(ta + 32u, l8);
                    tc_wait_st();
                    tc_fence_before();
                    mbar_arrive(&a_full[sa]);
                }
            }
            if (!range_ok) *range_flag = 1;
        }
    };

    if (warp == 0) {
        // ---- raw weight chunks ------------------------------------------------
        if (lane == 0) {
            int armed[C::NR];
            for (int i = 0; i < C::NR; i++) armed[i] = -1;
            for (int c = 0; c < nchunks; c++) {
                const int s = c % C::NR;
                if (!tc_wait(&raw_empty[s], ((c / C::NR) & 1) ^ 1, abort_flag, 64)) break;
                mbar_arrive_expect_tx(&raw_full[s], L::RAW_STAGE);
                const int gc = chunk0 + c;
                const int x0 = WT == WT_Q8_0 ? gc * (RC::RAWB / 2) : gc * RC::RAWB;
                tma_load_3d(sbase + L::OFF_RAW + s * L::RAW_STAGE, &tm_w, x0, m0, expert, smem_u32(&raw_full[s]));
                armed[s] = (c / C::NR) & 1;
            }
            if (*abort_flag)  // let the copies in flight land before the CTA exits
                for (int i = 0; i < C::NR; i++)
                    if (armed[i] >= 0) mbar_wait_bounded(&raw_full[i], (uint32_t)armed[i]);
        }
    } else if (warp == 1) {
        // ---- activation stages: both planes of a pair on one barrier ------------------
        // (boxes of T3_XB rows, only as many as the tile's live columns need:
        // a narrow tile's stages are written with fewer shared-memory bytes)
        if (lane == 0) {
            int armed[C::NBP];
            for (int i = 0; i < C::NBP; i++) armed[i] = -1;
            const int nbox = (ncols + T3_XB - 1) / T3_XB;
            for (int q = 0; q < npairs; q++) {
                const int s = q % C::NBP;
                if (q >= C::NBP && !tc_wait(&pair_done[(q - C::NBP) % TC_ND], done_parity(q - C::NBP), abort_flag, 16))
                    break;
                mbar_arrive_expect_tx(&b_full[s], (uint32_t)(2 * nbox * T3_XB * 128));
                const uint32_t dst = sbase + L::OFF_B + s * L::B_STAGE3;
                for (int b = 0; b < nbox; b++) {
                    const uint32_t o = (uint32_t)(b * T3_XB * 128);
                    tma_load_3d(dst + o, &tm_x, (pair0 + q) * 64, xrow0 + b * T3_XB, 0, smem_u32(&b_full[s]));
                    tma_load_3d(dst + (STACK ? (uint32_t)stack_w * 128u : (uint32_t)T3_HALF) + o, &tm_x,
                                (pair0 + q) * 64, xrow0 + b * T3_XB, 1, smem_u32(&b_full[s]));
                }
                armed[s] = (q / C::NBP) & 1;
            }
            if (*abort_flag)
                for (int i = 0; i < C::NBP; i++)
                    if (armed[i] >= 0) mbar_wait_bounded(&b_full[i], (uint32_t)armed[i]);
        }
    } else if (warp == 3) {
        // ---- gate: A slot + B stage of pair q, then the rendezvous --------------
        // Both warps take exactly one barrier step per pair until the OR of
        // their votes is set (this warp's bounded waits gave up), and leave
        // the loop at the same pair: the waits are bounded, so the MMA warp
        // is never left alone at the barrier.
        for (int q = 0; q < npairs; q++) {
            int ok = 0;
            if (lane == 0)
                ok = tc_wait(&a_full[q % C::NA], (q / C::NA) & 1, abort_flag) &&
                     tc_wait(&b_full[q % C::NBP], (q / C::NBP) & 1, abort_flag);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (named_bar_red_or(T3_GATE_BAR, 64, !ok)) break;
        }
    } else if (warp == 2) {
        // ---- MMA issue: the whole warp waits, one thread issues ------------------
        {
            // a narrow tile multiplies only its columns, rounded up to the
            // MMA's N granularity of 16 (M = 128: N = 16..256, N % 16 == 0)
            const int nmma = min(T3_BN, (ncols + 15) & ~15);
            const uint32_t idesc = f16_idesc(TC_BM, nmma);
            const uint32_t idesc_w = f16_idesc(TC_BM, STACK ? 2 * stack_w : 16), idesc_n = f16_idesc(TC_BM, STACK ? stack_w : 16);
            for (int q = 0; q < npairs; q++) {
                const int sa = q % C::NA, sb = q % C::NBP;
                // the gate's verdict for pair q (uniform over the warp)
                if (named_bar_red_or(T3_GATE_BAR, 64, false)) break;
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t a_hi = tmem + (uint32_t)(acol0 + 64 * sa), a_lo = a_hi + 32u;
                    const uint32_t b_hi = sbase + L::OFF_B + sb * L::B_STAGE3, b_lo = b_hi + T3_HALF;
                    // a Q4_K min-term pair uses its first K step only
                    const int nk = (WT == WT_Q4_K && q % 9 == 8) ? 1 : 4;
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        if (k >= nk) break;
                        // K step of 16: 8 TMEM columns of A; 32 bytes in the swizzled B rows
                        const uint32_t ka = 8u * k, kb = 64u * (k >> 1) + 32u * (k & 1);
                        if constexpr (STACK) {  // [Bhi; Blo] in one operand of 2W rows
                            tc_mma_f16_ts(tmem, a_hi + ka, sw128_desc(b_hi + kb), idesc_w, (q | k) ? 1u : 0u);
                            tc_mma_f16_ts(tmem, a_lo + ka, sw128_desc(b_hi + kb), idesc_n, 1u);
                        } else {
                            tc_mma_f16_ts(tmem, a_hi + ka, sw128_desc(b_hi + kb), idesc, (q | k) ? 1u : 0u);
                            tc_mma_f16_ts(tmem, a_hi + ka, sw128_desc(b_lo + kb), idesc, 1u);
                            tc_mma_f16_ts(tmem, a_lo + ka, sw128_desc(b_hi + kb), idesc, 1u);
                        }
                    }
                    tc_commit(smem_u32(&pair_done[q % TC_ND]));
                }
                __syncwarp();
            }
            // the accumulator is complete when every issued MMA has finished
            if (lane == 0) tc_commit(smem_u32(mma_done));
        }
    } else if (warp >= 4 && warp < 8) {
        // ---- converters: one weight row per thread, one block pair at a time ----
        if constexpr (WT == WT_Q4_K) {
            convert_q4k(std::integral_constant<int, 0>{});
        } else {
        const int row = tid - 128;
        bool range_ok = true;
        for (int c = 0; c < nchunks; c++) {
            const int s = c % C::NR;
            if (!tc_wait_warp(&raw_full[s], (c / C::NR) & 1, abort_flag, lane)) break;
            const uint8_t *rrow = gbase + L::OFF_RAW + s * L::RAW_STAGE + row * RC::RAWB;
            bool ok = true;
#pragma unroll
            for (int pp = 0; pp < CHUNK_PAIRS; pp++) {
                const int q = CHUNK_PAIRS * c + pp;
                const int sa = q % C::NA;
                uint32_t w[PairWords<WT>::N];
                load_pair_words_v<WT>(rrow, pp, w);
                if (pp == CHUNK_PAIRS - 1) mbar_arrive(&raw_empty[s]);  // the chunk is in registers
                uint32_t v0[16], v1[16];
                float sc0, sc1, mn0, mn1;
                convert_pair<WT>(w, nullptr, pp, v0, v1, sc0, sc1, mn0, mn1);
                range_ok = range_ok && fabsf(sc0) <= C::kMaxScale && fabsf(sc1) <= C::kMaxScale;
                uint32_t h[32], l[32];  // the pair's 64 elements, hi and lo
                split_block(v0, __float2half2_rn(sc0), h, l);
                split_block(v1, __float2half2_rn(sc1), h + 16, l + 16);
                // the slot was last read by the MMAs of pair q - NA
                if (q >= C::NA &&
                    !tc_wait_warp(&pair_done[(q - C::NA) % TC_ND], done_parity(q - C::NA), abort_flag, lane)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t ta = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + (uint32_t)(acol0 + 64 * sa);
                tc_st32(ta, h);
                tc_st32(ta + 32u, l);
                tc_wait_st();
                tc_fence_before();
                mbar_arrive(&a_full[sa]);
            }
            if (!ok) break;
        }
        if (!range_ok) *range_flag = 1;
        }
    } else if (warp >= 8) {
        if constexpr (WT == WT_Q4_K) {
            if (warp < 12) convert_q4k(std::integral_constant<int, 1>{});
        }
        // ---- epilogue ------------------------------------------------------------
        // (1) while the main loop runs: the column table (destinations of the
        //     tile's columns, their activation row scales);
        // (2) after the last MMA: TMEM -> the output tile staged in shared
        //     memory as [column][128 rows] (the activation ring is free);
        // (3) each column's 128 rows leave as one 512-byte store per warp.
        const int et = tid - 256;  // 0..255
        const int sub = warp & 3, half = (warp - 8) >> 2;
        const int row = 32 * sub + lane;
        for (int c = et; c < ncols; c += 256) {
            const int r = xrow0 + c;
            T3Col d;
            d.scale = p.xscale[r];
            d.owner = -1;
            if (tw.tsplit >= 0) {
                d.dst = reinterpret_cast<uint64_t>(p.tail_partial +
                                                   (((uint64_t)tw.tsplit * tw.tail_n + tw.ttile) * T3_BN + c) * TC_BM);
            } else if (p.partial) {
                d.dst = reinterpret_cast<uint64_t>(p.partial + ((uint64_t)blockIdx.z * p.N + r) * p.M + m0);
            } else {
                uint64_t off;
                if (p.grouped) {
                    const int slot = p.g.rows[r];
                    int tok = slot / p.g.n_selected;
                    if (PEER && p.peer.owner_tokens > 0) {
                        d.owner = tok / p.peer.owner_tokens;
                        tok -= d.owner * p.peer.owner_tokens;
                    }
                    off = (uint64_t)(slot % p.g.n_selected) * p.g.dst_nb1 + (uint64_t)tok * p.g.dst_nb2;
                } else {
                    off = (uint64_t)r * p.y_nb1;
                }
                off += (uint64_t)m0 * 4;
                d.dst = PEER ? off : reinterpret_cast<uint64_t>(p.y) + off;
            }
            cols[c] = d;
        }
        float *stage = reinterpret_cast<float *>(gbase + L::OFF_B);
        const bool live = tc_wait_warp(mma_done, 0, abort_flag, lane, 256) && !*abort_flag;
        if (live && 96 * half < ncols) {
            tc_fence_after();
            fence_proxy_async_smem();  // the ring was last written by TMA and read by the tensor core
#pragma unroll 1
            for (int cc = 0; cc < 3; cc++) {
                const int qc = 3 * half + cc;
                if (32 * qc >= ncols) break;
                uint32_t r[32];
                tc_ld32(tmem + ((uint32_t)(32 * sub) << 16) + (uint32_t)(32 * qc), r);
                tc_wait_ld();
                if constexpr (STACK) {  // + the Ahi.Blo half
                    uint32_t r2[32];
                    tc_ld32(tmem + ((uint32_t)(32 * sub) << 16) + (uint32_t)(stack_w + 32 * qc), r2);
                    tc_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; i++) r[i] = __float_as_uint(__uint_as_float(r[i]) + __uint_as_float(r2[i]));
                }
#pragma unroll
                for (int i = 0; i < 32; i++)
                    stage[(32 * qc + i) * TC_BM + row] = npairs > 0 ? __uint_as_float(r[i]) : 0.0f;
            }
        }
        asm volatile("bar.sync 1, 256;" ::: "memory");  // the 8 epilogue warps
        if (live) {
            const int rows_valid = min(TC_BM, p.M - m0);
            const int r0 = 4 * lane;  // this lane's 4 rows
            const int ep = (warp - 8);
            const int pb = PEER ? (int)((*p.peer.epoch + 1u) & 1u) : 0;  // this step's peer buffer
            for (int c = ep; c < ncols; c += 8) {
                const T3Col d = cols[c];
                float4 v = *reinterpret_cast<const float4 *>(stage + c * TC_BM + r0);
                v.x *= d.scale, v.y *= d.scale, v.z *= d.scale, v.w *= d.scale;
                if (!PEER && tw.tsplit < 0 && !p.partial && (p.epi.bias || p.epi.silu)) {  // fused bias / SiLU on y
                    if (r0 < rows_valid) v.x = apply_act(v.x, p.epi, m0 + r0);
                    if (r0 + 1 < rows_valid) v.y = apply_act(v.y, p.epi, m0 + r0 + 1);
                    if (r0 + 2 < rows_valid) v.z = apply_act(v.z, p.epi, m0 + r0 + 2);
                    if (r0 + 3 < rows_valid) v.w = apply_act(v.w, p.epi, m0 + r0 + 3);
                }
                auto put = [&](uint8_t *base) {
                    float *o = reinterpret_cast<float *>(base) + r0;
                    if (r0 + 4 <= rows_valid && (reinterpret_cast<uintptr_t>(base) & 15) == 0) {
                        *reinterpret_cast<float4 *>(o) = v;
                    } else {
                        if (r0 < rows_valid) o[0] = v.x;
                        if (r0 + 1 < rows_valid) o[1] = v.y;
                        if (r0 + 2 < rows_valid) o[2] = v.z;
                        if (r0 + 3 < rows_valid) o[3] = v.w;
                    }
                };
                if constexpr (PEER) {
                    if (tw.tsplit >= 0 || p.partial) {
                        put(reinterpret_cast<uint8_t *>(d.dst));
                    } else {  // NVLink stores into the owner's buffer, or every rank's
                        if (d.owner >= 0)
                            put(p.peer.y[pb][d.owner] + d.dst);
                        else
                            for (int pr = 0; pr < p.peer.n; pr++) put(p.peer.y[pb][pr] + d.dst);
                    }
                } else {
                    put(reinterpret_cast<uint8_t *>(d.dst));
                }
            }
        }
    }

    // the epilogue threads' peer stores, before the CTA counts itself done
    if (PEER && warp >= 8) __threadfence_system();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
        if (*abort_flag) report_status(p.status, STATUS_TIMEOUT);
        if (*range_flag) report_status(p.status, STATUS_RANGE);
    }
    if (PEER && tid == 0) peer_cta_done(p.peer);
    if (warp == 2) {
        // every issued MMA has completed before the columns are released
        if (lane == 0) mbar_wait_bounded(mma_done, 0);
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(T3_TMEM_COLS)
                     : "memory");
    }
}

// ---- activations: Q8_0 quantize into f16 operands -----------------------------
// One CTA per activation row r (with `routed`, the activation of routed slot
// r: token g.rows[r] / n_selected, for r < sum(counts)).
// hilo == false (the per-block kernel): q16[r][k] = qx as an f16 integer,
// dxT[b][r] = dx (the f16 block scale as f32), xsdT[b][r] = dx * sum(qx).
// hilo == true (the split-f16 kernel): the row's scale exponent e is chosen
// from its largest block scale D (D * 128 < 2^(e + 15)), then
// v = dx*qx * 2^-e (exact) is written as hi = rn16(v) to plane 0
// (q16[r][k]) and lo = v - hi to plane 1 (q16[rows + r][k]); xscale[r] = 2^e.
// With `chunks` > 1 (few rows: a cluster of `chunks` CTAs per row) each CTA
// takes a contiguous run of the row's blocks and the CTAs of the cluster
// exchange their maxima through distributed shared memory.
constexpr int QF_THREADS = 256;

__device__ __forceinline__ float ld_cluster_f32(const float *p, uint32_t rank) {
    uint32_t ra;
    float v;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(smem_u32(p)), "r"(rank));
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(ra) : "memory");
    return v;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__global__ void __launch_bounds__(QF_THREADS) quantize_q8_f16_kernel(const uint8_t *__restrict__ x, uint64_t x_nb1,
                                                                    int K, int rows, __half *__restrict__ q16,
                                                                    float *__restrict__ dxT, float *__restrict__ xsdT,
                                                                    float *__restrict__ xscale, bool hilo, bool ext,
                                                                    bool routed, GroupMap g, int chunks) {
    const int r = (int)blockIdx.x / chunks, part = (int)blockIdx.x % chunks, tid = threadIdx.x;
    int src = r;
    if (routed) {
        if (g.n_groups == 0 || r >= g.offsets[g.n_groups - 1] + g.counts[g.n_groups - 1]) return;
        src = g.rows[r] / g.n_selected;
    }
    const float *xr = reinterpret_cast<const float *>(x + (uint64_t)src * x_nb1);
    const int nblk = K / QK;
    // this CTA's blocks [b_lo, b_hi) of the row
    // (32-bit: part < 8 and nblk < 2^26)
    const int b_lo = chunks == 1 ? 0 : part * nblk / chunks, b_hi = chunks == 1 ? nblk : (part + 1) * nblk / chunks;
    // ext (Q4_K): 576 positions per 512 elements, the 64 after each 512
    // starting with the 16 blocks' sums (the min-term pair of the GEMM)
    const int KE = ext ? K / 512 * 576 : K;
    __half *orow = q16 + (uint64_t)r * KE;
    __half *orow_lo = q16 + ((uint64_t)rows + r) * KE;
    float down = 1.0f;  // 2^-e
    if (hilo) {
        __shared__ float wmax[QF_THREADS / 32];
        float amax = 0.0f;
        for (int k = b_lo * QK + 4 * tid; k < b_hi * QK; k += 4 * QF_THREADS) {
            const float4 v = *reinterpret_cast<const float4 *>(xr + k);
            amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        if ((tid & 31) == 0) wmax[tid >> 5] = amax;
        __syncthreads();
        amax = wmax[0];
#pragma unroll
        for (int w = 1; w < QF_THREADS / 32; w++) amax = fmaxf(amax, wmax[w]);
        if (chunks > 1) {  // the row's maximum over the cluster's CTAs
            __shared__ float part_max;
            if (tid == 0) part_max = amax;
            cluster_sync_all();
            for (int j = 0; j < chunks; j++) amax = fmaxf(amax, ld_cluster_f32(&part_max, (uint32_t)j));
            cluster_sync_all();  // every CTA has read before any leaves
        }
        // the largest block scale: the quantizer's d of the row maximum
        // (division and f16 rounding are monotonic)
        const float dmax = __half2float(__float2half_rn(__fdiv_rn(amax, 127.0f)));
        const float bound = dmax * (ext ? 4096.0f : 128.0f);  // ext: block sums up to 32 * 127 * d
        int e = 0;
        if (bound > 0.0f && isfinite(bound)) {
            int ex;
            frexpf(bound, &ex);  // bound < 2^ex
            e = ex - 15;
        }
        down = ldexpf(1.0f, -e);
        if (tid == 0 && part == 0) xscale[r] = ldexpf(1.0f, e);
    }
    // 8 lanes per block, 4 elements per lane; every lane of the warp calls the
    // quantize routine (uniform trip count)
    for (int base = b_lo; base < b_hi; base += QF_THREADS / 8) {
        const int b = base + (tid >> 3);
        const int k = b * QK + (tid & 7) * 4;
        const bool valid = b < b_hi;
        const float4 v = valid ? *reinterpret_cast<const float4 *>(xr + k) : make_float4(0.f, 0.f, 0.f, 0.f);
        uint16_t dbits;
        int qsum;
        const uint32_t q = quantize_q8_0_quad(v, dbits, qsum);
        if (!valid) continue;
        const float d = f16_bits_to_f32(dbits);
        const int kp = ext ? k + (k >> 9) * 64 : k;  // position in the operand row
        __half hq[4];
        if (hilo && ext && (tid & 7) == 0) {  // the block sum, as hi + lo (24 significant bits: lo rounds)
            const float xs = (d * (float)qsum) * down;
            const __half h = __float2half_rn(xs);
            const int pe = (b >> 4) * 576 + 512 + (b & 15);
            orow[pe] = h;
            orow_lo[pe] = __float2half_rn(xs - __half2float(h));
        }
        if (hilo) {
            __half lq[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float val = (d * (float)(int8_t)((q >> (8 * i)) & 0xFFu)) * down;  // exact
                hq[i] = __float2half_rn(val);
                lq[i] = __float2half_rn(val - __half2float(hq[i]));
            }
            *reinterpret_cast<uint2 *>(orow_lo + kp) = *reinterpret_cast<const uint2 *>(lq);
        } else {
#pragma unroll
            for (int i = 0; i < 4; i++) hq[i] = __int2half_rn((int)(int8_t)((q >> (8 * i)) & 0xFFu));
            if ((tid & 7) == 0) {
                dxT[(uint64_t)b * rows + r] = d;
                xsdT[(uint64_t)b * rows + r] = d * (float)qsum;
            }
        }
        *reinterpret_cast<uint2 *>(orow + kp) = *reinterpret_cast<const uint2 *>(hq);
    }
}

// y[n][m] = sum over z in order of partial[z][n][m] (deterministic), then
// the fused epilogue.
__global__ void tc_split_reduce_kernel(const float *__restrict__ partial, int splits, int M, int N, uint8_t *y,
                                       uint64_t y_nb1, const EpiAct epi) {
    const int64_t total = (int64_t)M * N;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        float acc = partial[i];
        for (int z = 1; z < splits; z++) acc += partial[(int64_t)z * total + i];
        const int n = (int)(i / M), m = (int)(i % M);
        reinterpret_cast<float *>(y + (uint64_t)n * y_nb1)[m] = apply_act(acc, epi, m);
    }
}

// Tail tiles: y = sum over s in order of the S partial tiles (deterministic),
// then the fused epilogue.
__global__ void tc_tail_reduce_kernel(const float *__restrict__ partial, int S, int n_tail, int tiles_n, int m0_tile,
                                      int M, int N, int bn, int bw, uint8_t *y, uint64_t y_nb1, const EpiAct epi) {
    const int64_t per = (int64_t)n_tail * bn * TC_BM;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < per; i += (int64_t)gridDim.x * blockDim.x) {
        const int tt = (int)(i / (bn * TC_BM)), rem = (int)(i % (bn * TC_BM));
        const int c = rem / TC_BM, rr = rem % TC_BM;
        const int m = (m0_tile + tt / tiles_n) * TC_BM + rr, n = (tt % tiles_n) * bw + c;
        if (c >= bw || m >= M || n >= N) continue;
        float acc = partial[i];
        for (int sp = 1; sp < S; sp++) acc += partial[(int64_t)sp * per + i];
        reinterpret_cast<float *>(y + (uint64_t)n * y_nb1)[m] = apply_act(acc, epi, m);
    }
}

// Grouped tail (mul_mat_id): each split tile's columns are summed over the
// splits in order (deterministic) and stored through the group map; the
// plan is recomputed from the routed column tile count (none: no work).
__global__ void tc_gtail_reduce_kernel(const TcParams p, int bn) {
    const int T = p.g.tile_start[p.g.n_groups];
    const int tiles_m = (p.M + TC_BM - 1) / TC_BM;
    TailPlan tp{};
    if (!tail_plan(tiles_m, T, p.K / QKK, p.gtail_sms, p.gtail_even, &tp)) return;
    const int n_tail = tp.rows * T;
    const int64_t per = (int64_t)n_tail * bn * TC_BM;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < per; i += (int64_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / (bn * TC_BM)), rem = (int)(i % (bn * TC_BM));
        const int c = rem / TC_BM, row = rem % TC_BM;
        const int m = (tiles_m - tp.rows + t / T) * TC_BM + row, tt = t % T;
        if (m >= p.M) continue;
        int e = 0;
        while (p.g.tile_start[e + 1] <= tt) e++;
        const int jt = tt - p.g.tile_start[e];
        if (c >= min(bn, p.g.counts[e] - jt * bn)) continue;
        float acc = p.tail_partial[((int64_t)t * bn + c) * TC_BM + row];
        for (int sp = 1; sp < tp.splits; sp++) acc += p.tail_partial[(((int64_t)sp * n_tail + t) * bn + c) * TC_BM + row];
        const int slot = p.g.rows[p.g.offsets[e] + jt * bn + c];
        const uint64_t off = (uint64_t)(slot % p.g.n_selected) * p.g.dst_nb1 +
                             (uint64_t)(slot / p.g.n_selected) * p.g.dst_nb2 + (uint64_t)m * 4;
        *reinterpret_cast<float *>(p.y + off) = apply_act(acc, p.epi, m);
    }
}

// ---- host side ---------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static std::once_flag once;
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    std::call_once(once, [] {
        void *q = nullptr;
        cudaDriverEntryPointQueryResult res;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &q, cudaEnableDefault, &res) == cudaSuccess &&
            res == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(q);
    });
    return fn;
}

// Tiled tensor map of rank 2 (dim2 == 0) or 3; strides in bytes.
int encode_map(CUtensorMap *map, CUtensorMapDataType dt, const void *base, uint64_t dim0, uint64_t dim1,
               uint64_t dim2, uint64_t stride1, uint64_t stride2, uint32_t box0, uint32_t box1,
               CUtensorMapSwizzle swz) {
    auto fn = encode_fn();
    if (!fn) return fb::set_error(FB_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    const cuuint32_t rank = dim2 ? 3 : 2;
    const cuuint64_t dims[3] = {dim0, dim1, dim2 ? dim2 : 1};
    const cuuint64_t strides[2] = {stride1, stride2};
    const cuuint32_t box[3] = {box0, box1, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, dt, rank, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fb::set_error(FB_ERR_CUDA, "tensor map encode failed (%d)", (int)r);
    return FB_OK;
}

// The split-f16 kernel runs Q8_0 and Q4_0, and Q4_K when K is a multiple of
// 512 (every min-term pair covers two whole super-blocks).
bool split_kernel(int32_t wtype, int64_t K) { return wtype != WT_Q4_K || K % 512 == 0; }
// Length of an activation operand row: K, or for the split-f16 Q4_K 576
// positions per 512 elements.
int64_t operand_k(int32_t wtype, int64_t K) { return wtype == WT_Q4_K && K % 512 == 0 ? K / 512 * 576 : K; }
// Q4_K K ranges (splits) cover whole super-block pairs.
int chunk_round(int32_t wtype, int chunks) { return wtype == WT_Q4_K ? (chunks + 1) / 2 * 2 : chunks; }

template <int WT, bool SPLIT>
constexpr int smem_bytes_of() {
    if constexpr (SPLIT)
        return T3Layout<WT>::BYTES;
    else
        return TcLayout<WT>::BYTES;
}

// rows: activation rows in the operand buffer; n_planes / w_nb2: weight
// planes (experts) of the grouped mode (1 / unused otherwise). SPLIT: the
// split-f16 kernel (Q8_0, Q4_0, Q4_K with K % 512 == 0), else the per-block
// kernel (Q4_K).
template <int WT, bool SPLIT>
int launch_tc_typed(const void *w, uint64_t w_nb1, uint64_t w_nb2, int64_t n_planes, const XQ16 &xa, int64_t K,
                    int64_t M, int64_t rows, void *y, uint64_t y_nb1, const GroupMap *groups, int32_t *status,
                    int splits, cudaStream_t s, const PeerOut *peer, const EpiAct &epi) {
    using C = TcCfg<WT>;
    using L = TcLayout<WT>;
    static_assert(L::BYTES <= 232448, "gemm_tc shared memory");
    // the split-f16 kernel over the hi / lo activation planes (Q4_K: the
    // extended rows with the block sums), or the per-block kernel over exact
    // f16 integers
    constexpr bool kSplit = SPLIT;
    constexpr int BN = kSplit ? T3_BN : TC_BN;
    constexpr int kBytes = smem_bytes_of<WT, SPLIT>();
    const int64_t KE = operand_k(WT, K);
    static_assert(kBytes <= 232448, "gemm_tc3 shared memory");
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
    // activations: [rows][K] f16 (Q4_K), or planes [2][rows][K] (hi, lo)
    rc = encode_map(&tx, CU_TENSOR_MAP_DATA_TYPE_UINT16, xa.q16, (uint64_t)KE, (uint64_t)rows, kSplit ? 2 : 0,
                    (uint64_t)KE * 2, kSplit ? (uint64_t)rows * (uint64_t)KE * 2 : 0, 64, kSplit ? T3_XB : BN,
                    CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    // the peer-store variant is a separate instantiation, so the plain kernel
    // carries none of its registers; so is the stacked one (an ungrouped
    // product of at most 128 columns)
    const bool stack = kSplit && !groups && !peer && rows <= 128;
    using KernFn = void (*)(const CUtensorMap, const CUtensorMap, const TcParams);
    KernFn kern;
    if constexpr (kSplit)
        kern = peer ? gemm_tc3_kernel<WT, true, false>  // peer stores: grouped only
                    : (stack ? gemm_tc3_kernel<WT, false, true> : gemm_tc3_kernel<WT, false, false>);
    else
        kern = peer ? gemm_tc_kernel<WT, true> : gemm_tc_kernel<WT, false>;
    static DeviceFlags configured[4];
    rc = raise_smem_limit((const void *)kern, kBytes, configured[(peer ? 2 : 0) + (stack ? 1 : 0)], "gemm_tc");
    if (rc) return rc;
    TcParams p{};
    p.M = (int)M;
    p.N = (int)rows;
    p.K = (int)K;
    // Ungrouped split-f16 tiles share the columns evenly (rounded to the
    // MMA's N step of 16): an MMA costs a floor of cycles well above N / 2 at
    // small N, so 176 + 176 + 160 columns beat 192 + 192 + 128.
    p.bw = BN;
    if (kSplit && !groups && rows > 0) {
        const int64_t nt = (rows + BN - 1) / BN;
        p.bw = (int)std::min<int64_t>(BN, ((rows + nt - 1) / nt + 15) / 16 * 16);
        if ((rows + p.bw - 1) / p.bw != nt) p.bw = BN;  // the same tile count as the planners assume
    }
    p.y = static_cast<uint8_t *>(y);
    p.y_nb1 = y_nb1;
    p.dxT = xa.dxT;
    p.xsdT = xa.xsdT;
    p.xscale = xa.xscale;
    p.status = status;
    p.grouped = groups != nullptr;
    if (groups) p.g = *groups;
    if (peer) p.peer = *peer;
    p.epi = epi;
    const int total_pairs = (int)(K / (2 * QK));
    if (splits > 1) {
        const int per_chunks = chunk_round(WT, (int)((K / QKK + splits - 1) / splits));
        p.split_pairs = per_chunks * CHUNK_PAIRS;
        splits = (total_pairs + p.split_pairs - 1) / p.split_pairs;
        p.partial = xa.partial;
    }
    const unsigned tiles_n = groups ? (unsigned)groups->max_tiles : (unsigned)((rows + BN - 1) / BN);
    if (tiles_n == 0 || M == 0) return FB_OK;
    if (tiles_n > 65535) return fb::set_error(FB_ERR_UNSUPPORTED, "gemm_tc: too many column tiles");
    dim3 grid((unsigned)((M + TC_BM - 1) / TC_BM), tiles_n, (unsigned)std::max(splits, 1));
    p.tail_full = -1;
    TailPlan tp{};
    if (!groups && splits <= 1 && gemm_tc_tail(WT, K, M, rows, &tp)) {
        const int tiles_m = (int)((M + TC_BM - 1) / TC_BM);
        p.tail_tiles_n = (int)tiles_n;
        p.tail_m0 = tiles_m - tp.rows;
        p.tail_full = p.tail_m0 * (int)tiles_n;
        p.tail_S = tp.splits;
        p.tail_n = tp.rows * (int)tiles_n;
        p.tail_split_pairs = tp.split_pairs;
        p.tail_partial = xa.partial;
        grid = dim3((unsigned)(p.tail_full + p.tail_n * p.tail_S), 1, 1);
    } else if (groups && !peer && splits <= 1 && ((M + TC_BM - 1) / TC_BM) * (int64_t)tiles_n > sm_count()) {
        // mul_mat_id whose largest tile count overflows one wave: the tail
        // split is planned in the kernel from the routed column tile count;
        // the grid covers the largest count plus one wave of split work
        // items (tail_plan: at most one per SM)
        p.gtail_sms = sm_count();
        p.gtail_even = WT == WT_Q4_K;
        p.tail_partial = xa.partial;
        grid = dim3((unsigned)(((M + TC_BM - 1) / TC_BM) * (int64_t)tiles_n + p.gtail_sms), 1, 1);
    }
    kern<<<grid, kSplit ? T3_THREADS : TC_THREADS, kBytes, s>>>(tw, tx, p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fb::set_error(FB_ERR_CUDA, "gemm_tc launch: %s", cudaGetErrorString(e));
    if (p.tail_full >= 0) {
        const int64_t total = (int64_t)p.tail_n * BN * TC_BM;
        const int blocks = (int)std::min<int64_t>((total + 255) / 256, 4 * sm_count());
        tc_tail_reduce_kernel<<<blocks, 256, 0, s>>>(p.tail_partial, p.tail_S, p.tail_n, p.tail_tiles_n, p.tail_m0,
                                                     (int)M, (int)rows, BN, p.bw, static_cast<uint8_t *>(y), y_nb1, epi);
        e = cudaGetLastError();
        if (e != cudaSuccess) return fb::set_error(FB_ERR_CUDA, "gemm_tc tail reduce launch: %s", cudaGetErrorString(e));
    }
    if (p.gtail_sms > 0) {
        const int64_t total = (int64_t)p.gtail_sms * BN * TC_BM;  // the largest tail
        const int blocks = (int)std::min<int64_t>((total + 255) / 256, 4 * sm_count());
        tc_gtail_reduce_kernel<<<blocks, 256, 0, s>>>(p, BN);
        e = cudaGetLastError();
        if (e != cudaSuccess) return fb::set_error(FB_ERR_CUDA, "gemm_tc tail reduce launch: %s", cudaGetErrorString(e));
    }
    if (p.partial) {
        const int64_t total = M * rows;
        const int blocks = (int)std::min<int64_t>((total + 255) / 256, 4 * sm_count());
        tc_split_reduce_kernel<<<blocks, 256, 0, s>>>(p.partial, splits, (int)M, (int)rows, static_cast<uint8_t *>(y),
                                                      y_nb1, epi);
        e = cudaGetLastError();
        if (e != cudaSuccess) return fb::set_error(FB_ERR_CUDA, "gemm_tc split reduce launch: %s", cudaGetErrorString(e));
    }
    return FB_OK;
}

uint64_t pad256(uint64_t v) { return (v + 255) & ~uint64_t(255); }

}  // namespace

int encode_tensor_map_2d(CUtensorMap *map, CUtensorMapDataType dt, const void *base, uint64_t dim0, uint64_t dim1,
                         uint64_t stride1, uint32_t box0, uint32_t box1) {
    return encode_map(map, dt, base, dim0, dim1, 0, stride1, 0, box0, box1, CU_TENSOR_MAP_SWIZZLE_NONE);
}

int encode_tensor_map_2d_sw128(CUtensorMap *map, CUtensorMapDataType dt, const void *base, uint64_t dim0,
                               uint64_t dim1, uint64_t stride1, uint32_t box0, uint32_t box1) {
    return encode_map(map, dt, base, dim0, dim1, 0, stride1, 0, box0, box1, CU_TENSOR_MAP_SWIZZLE_128B);
}

bool gemm_tc_supported(int32_t wtype, int64_t K, int64_t M, int64_t N, const void *w, uint64_t w_nb1) {
    if (wtype != WT_Q8_0 && wtype != WT_Q4_0 && wtype != WT_Q4_K) return false;
    if (K <= 0 || K % QKK || K > (1 << 24) || M <= 0 || N <= 0 || M > INT32_MAX || N > INT32_MAX / 64) return false;
    if (((reinterpret_cast<uintptr_t>(w) | w_nb1) & 15) != 0) return false;
    return (N + gemm_tc_block_n(wtype, K) - 1) / gemm_tc_block_n(wtype, K) <= 65535;
}

int gemm_tc_block_n(int32_t wtype, int64_t K) { return split_kernel(wtype, K) ? T3_BN : TC_BN; }

// Split-K when the tile grid leaves most SMs idle (ungrouped only): one CTA
// per SM in a single wave, every split at least two weight chunks.
int gemm_tc_splits(int32_t wtype, int64_t K, int64_t M, int64_t N) {
    const int64_t bn = gemm_tc_block_n(wtype, K);
    const int64_t tiles = ((M + TC_BM - 1) / TC_BM) * ((N + bn - 1) / bn);
    const int64_t nchunks = K / QKK, sms = sm_count();
    if (tiles * 2 > sms || nchunks < 4) return 1;
    const int64_t splits = std::min<int64_t>({sms / tiles, nchunks / 2, 16});
    if (splits < 2) return 1;
    const int64_t per = chunk_round(wtype, (int)((nchunks + splits - 1) / splits));
    return (int)((nchunks + per - 1) / per);
}

// Tail split of an ungrouped GEMM (tail_plan).
bool gemm_tc_tail(int32_t wtype, int64_t K, int64_t M, int64_t N, TailPlan *tp) {
    const int64_t bn = gemm_tc_block_n(wtype, K);
    TailPlan t{};
    const bool on = tail_plan((M + TC_BM - 1) / TC_BM, (N + bn - 1) / bn, K / QKK, sm_count(), wtype == WT_Q4_K, &t);
    if (on && tp) *tp = t;
    return on;
}

// Split-f16 (Q8_0, Q4_0, Q4_K with K % 512 == 0): the hi and lo planes and
// the row scales. Per-block (other Q4_K): the f16 integers and the two
// block-scale arrays.
uint64_t xq16_bytes(int32_t wtype, int64_t K, int64_t rows, int64_t M, bool grouped) {
    const uint64_t nblk = (uint64_t)K / QK, KE = (uint64_t)operand_k(wtype, K);
    uint64_t b = !split_kernel(wtype, K)
                     ? pad256((uint64_t)rows * (uint64_t)K * 2) + 2 * pad256(nblk * (uint64_t)rows * 4)
                     : pad256(2 * (uint64_t)rows * KE * 2) + pad256((uint64_t)rows * 4);
    if (grouped) {  // the tail split's partial tiles: at most one per SM
        b += pad256((uint64_t)sm_count() * gemm_tc_block_n(wtype, K) * TC_BM * 4);
    } else {
        const int sp = gemm_tc_splits(wtype, K, M, rows);
        TailPlan tp{};
        if (sp > 1)
            b += pad256((uint64_t)sp * (uint64_t)M * (uint64_t)rows * 4);
        else if (gemm_tc_tail(wtype, K, M, rows, &tp)) {
            const int64_t bn = gemm_tc_block_n(wtype, K);
            b += pad256((uint64_t)tp.splits * tp.rows * ((rows + bn - 1) / bn) * bn * TC_BM * 4);
        }
    }
    return b;
}

XQ16 xq16_carve(int32_t wtype, void *base, int64_t K, int64_t rows) {
    const uint64_t nblk = (uint64_t)K / QK;
    uint8_t *p = static_cast<uint8_t *>(base);
    XQ16 r{};
    r.q16 = p;
    if (!split_kernel(wtype, K)) {
        p += pad256((uint64_t)rows * (uint64_t)K * 2);
        r.dxT = reinterpret_cast<float *>(p);
        p += pad256(nblk * (uint64_t)rows * 4);
        r.xsdT = reinterpret_cast<float *>(p);
        p += pad256(nblk * (uint64_t)rows * 4);
    } else {
        p += pad256(2 * (uint64_t)rows * (uint64_t)operand_k(wtype, K) * 2);
        r.xscale = reinterpret_cast<float *>(p);
        p += pad256((uint64_t)rows * 4);
    }
    r.partial = reinterpret_cast<float *>(p);
    return r;
}

int launch_quantize_q8_f16(const void *x, uint64_t x_nb1, int64_t K, int64_t N, const XQ16 &out,
                           const GroupMap *routed, cudaStream_t s, int32_t wtype) {
    const int64_t rows = routed ? N * routed->n_selected : N;
    if (rows == 0) return FB_OK;
    if (K % QK || K <= 0 || K > INT32_MAX / 4 || rows > INT32_MAX)
        return fb::set_error(FB_ERR_UNSUPPORTED, "quantize_q8_f16: unsupported shape");
    if ((reinterpret_cast<uintptr_t>(x) | x_nb1) & 15)
        return fb::set_error(FB_ERR_INVALID, "quantize_q8_f16: activations must be 16-byte aligned");
    GroupMap g{};
    if (routed) g = *routed;
    const bool hilo = split_kernel(wtype, K), ext = wtype == WT_Q4_K && hilo;
    // Few long rows (K >= 8192): a cluster of CTAs per row, up to two waves
    // of CTAs, at least 32 blocks per CTA, a power of two up to 8. (Rows of
    // 4096 were measured faster as one CTA each: the cluster barriers cost
    // more than the split saves.)
    int chunks = 1;
    if (hilo && K / QK >= 256)
        while (chunks < 8 && rows * chunks < 2 * (int64_t)sm_count() && K / QK >= 64 * chunks) chunks *= 2;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)(rows * chunks));
    cfg.blockDim = dim3(QF_THREADS);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)chunks;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaSuccess;
    if (chunks == 1)
        quantize_q8_f16_kernel<<<(unsigned)rows, QF_THREADS, 0, s>>>(static_cast<const uint8_t *>(x), x_nb1, (int)K,
                                                                      (int)rows, static_cast<__half *>(out.q16), out.dxT,
                                                                      out.xsdT, out.xscale, hilo, ext, routed != nullptr,
                                                                      g, 1);
    else
        e = cudaLaunchKernelEx(&cfg, quantize_q8_f16_kernel, static_cast<const uint8_t *>(x), x_nb1, (int)K, (int)rows,
                               static_cast<__half *>(out.q16), out.dxT, out.xsdT, out.xscale, hilo, ext,
                               routed != nullptr, g, chunks);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return fb::set_error(FB_ERR_CUDA, "quantize_q8_f16 launch: %s", cudaGetErrorString(e));
    return FB_OK;
}

int launch_gemm_tc(int32_t wtype, const void *w, uint64_t w_nb1, const XQ16 &xa, int64_t K, int64_t M, int64_t N,
                   void *y, uint64_t y_nb1, const GroupMap *groups, int32_t *status, cudaStream_t s,
                   const PeerOut *peer, const EpiAct *epi) {
    if (epi_active(epi) && groups) return fb::set_error(FB_ERR_INVALID, "gemm_tc: fused epilogue needs the ungrouped mode");
    const EpiAct ep = epi ? *epi : EpiAct{nullptr, 0};
    if (peer && (!groups || peer->n < 1 || peer->n > kMaxPeers || !peer->count || !peer->epoch))
        return fb::set_error(FB_ERR_INVALID, "gemm_tc: peer outputs need the grouped mode and a full peer set");
    const int64_t rows = groups ? N * groups->n_selected : N;
    if (!gemm_tc_supported(wtype, K, M, rows, w, w_nb1))
        return fb::set_error(FB_ERR_UNSUPPORTED, "gemm_tc: unsupported shape or alignment");
    const uint64_t w_nb2 = groups ? groups->w_group_stride : 0;
    const int64_t planes = groups ? groups->n_groups : 1;
    if (groups && (groups->n_groups < 1 || (w_nb2 & 15) || ((groups->dst_nb1 | groups->dst_nb2) & 3)))
        return fb::set_error(FB_ERR_INVALID, "gemm_tc: grouped strides");
    if ((reinterpret_cast<uintptr_t>(y) | y_nb1) & 3) return fb::set_error(FB_ERR_INVALID, "gemm_tc: output alignment");
    const int splits = groups ? 1 : gemm_tc_splits(wtype, K, M, rows);
    switch (wtype) {
    case WT_Q8_0:
        return launch_tc_typed<WT_Q8_0, true>(w, w_nb1, w_nb2, planes, xa, K, M, rows, y, y_nb1, groups, status,
                                              splits, s, peer, ep);
    case WT_Q4_0:
        return launch_tc_typed<WT_Q4_0, true>(w, w_nb1, w_nb2, planes, xa, K, M, rows, y, y_nb1, groups, status,
                                              splits, s, peer, ep);
    default:
        if (split_kernel(wtype, K))
            return launch_tc_typed<WT_Q4_K, true>(w, w_nb1, w_nb2, planes, xa, K, M, rows, y, y_nb1, groups, status,
                                                  splits, s, peer, ep);
        return launch_tc_typed<WT_Q4_K, false>(w, w_nb1, w_nb2, planes, xa, K, M, rows, y, y_nb1, groups, status,
                                               splits, s, peer, ep);
    }
}

}  // namespace fbk
