// Device helpers shared by the sm_100a kernels: ggml block formats, byte-level
// loads from 2-byte-aligned block fields, mbarrier / bulk-copy (TMA) PTX with
// bounded waits, and the quantize_row_q8_0 warp routine.
#pragma once

#include <cuda_fp16.h>
#include <cstdint>

namespace fbk {

// ggml block sizes (feml-core/src/dtype.rs:60,64,68).
constexpr int QK = 32;            // Q8_0 / Q4_0 block, Q4_K sub-block
constexpr int QKK = 256;          // Q4_K super-block
constexpr int Q8_0_BYTES = 34;    // f16 d + 32 x i8
constexpr int Q4_0_BYTES = 18;    // f16 d + 16 x (2 nibbles)
constexpr int Q4_K_BYTES = 144;   // f16 d, f16 dmin, 12 B scales, 128 B nibbles
constexpr int Q5_K_BYTES = 176;   // f16 d, f16 dmin, 12 B scales, 32 B fifth bits, 128 B nibbles
constexpr int Q6_K_BYTES = 210;   // 128 B low nibbles, 64 B top 2 bits, 16 x i8 scales, f16 d

// dtype discriminants used by the kernels (feml-core/src/dtype.rs:14-35).
constexpr int WT_F32 = 5, WT_Q4_0 = 7, WT_Q8_0 = 11, WT_Q4_K = 15, WT_Q5_K = 16, WT_Q6_K = 17;

// status bits written by kernels into the backend's device status word.
constexpr int STATUS_TIMEOUT = 1 << 0;    // a bounded wait gave up
constexpr int STATUS_BAD_ID = 1 << 1;     // mul_mat_id id outside [0, n_experts)
constexpr int STATUS_BAD_ARGS = 1 << 2;   // launch arguments failed a device-side check
constexpr int STATUS_RANGE = 1 << 3;      // a dequantized weight left the f16 range of the split-f16 GEMM

// Bound on mbarrier polls before a wait is declared failed (each try_wait
// suspends for a hardware-defined slice, so this is seconds, not forever).
constexpr uint32_t kWaitLimit = 1u << 24;

__device__ __forceinline__ float f16_bits_to_f32(uint16_t h) { return __half2float(__ushort_as_half(h)); }

__device__ __forceinline__ uint16_t ld_u16(const uint8_t *p) { return *reinterpret_cast<const uint16_t *>(p); }

// Load `N` little-endian 32-bit words starting at a 2-byte-aligned address
// (ggml block fields after the f16 scale are only 2-byte aligned).
template <int N>
__device__ __forceinline__ void ld_words_a2(const uint8_t *p, uint32_t (&out)[N]) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t *base = reinterpret_cast<const uint32_t *>(a & ~uintptr_t(3));
    const uint32_t sh = (uint32_t)(a & 3) * 8u;
    uint32_t w[N + 1];
#pragma unroll
    for (int i = 0; i <= N; i++) w[i] = base[i];
#pragma unroll
    for (int i = 0; i < N; i++) out[i] = __funnelshift_r(w[i], w[i + 1], sh);
}

// 6-bit (scale, min) pair j of a Q4_K super-block from its 12 packed bytes
// (public ggml get_scale_min_k4 layout).
__device__ __forceinline__ void q4k_scale_min(int j, const uint8_t *q, int &sc, int &m) {
    if (j < 4) {
        sc = q[j] & 63;
        m = q[j + 4] & 63;
    } else {
        sc = (q[j + 4] & 0x0f) | ((q[j - 4] >> 6) << 4);
        m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// quantize_row_q8_0 for one 32-element block spread over 8 consecutive lanes
// (group aligned to 8) holding 4 elements each:
//   d = amax / 127 (IEEE division), id = 1/d (IEEE reciprocal, 0 when d == 0),
//   q = roundf(x * id) (half away from zero).
// Returns the lane's 4 values packed little-endian; the f16 bits of d and the
// block's integer sum come back through the refs. All 32 lanes must call it.
__device__ __forceinline__ uint32_t quantize_q8_0_quad(float4 v, uint16_t &d_bits, int &qsum) {
    float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __frcp_rn(d) : 0.0f;
    const int q0 = (int)roundf(__fmul_rn(v.x, id));
    const int q1 = (int)roundf(__fmul_rn(v.y, id));
    const int q2 = (int)roundf(__fmul_rn(v.z, id));
    const int q3 = (int)roundf(__fmul_rn(v.w, id));
    int s = q0 + q1 + q2 + q3;
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    d_bits = __half_as_ushort(__float2half_rn(d));
    qsum = s;
    return (uint32_t)(q0 & 0xff) | ((uint32_t)(q1 & 0xff) << 8) | ((uint32_t)(q2 & 0xff) << 16) |
           ((uint32_t)(q3 & 0xff) << 24);
}

// ---------------------------------------------------------------------------
// mbarrier + bulk async copy (TMA, non-tensor form). All waits are bounded.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for phase `parity` of `bar` to complete; false if the bound ran out.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity) {
    for (uint32_t i = 0; i < kWaitLimit; i++)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}

// Global -> shared bulk copy completing on `bar` (dst, src 16-B aligned,
// bytes a multiple of 16). The L2 policy marks streamed weights evict-first.
__device__ __forceinline__ void bulk_g2s(void *smem_dst, const void *gmem_src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void bulk_g2s_evict_first(void *smem_dst, const void *gmem_src, uint32_t bytes,
                                                     uint64_t *bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
        "%4;" ::"r"(smem_u32(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// TMA prefetch of a global range into L2 (16-byte aligned, multiple of 16).
__device__ __forceinline__ void bulk_prefetch_l2(const void *gmem_src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(gmem_src), "r"(bytes) : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Programmatic dependent launch: wait for the preceding grid's results.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Thread-block clusters: rank, size, barrier, distributed shared memory.
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_size() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
// Address of the same shared-memory location in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t dsmem_map(const void *local, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(local)), "r"(rank));
    return r;
}
__device__ __forceinline__ int4 dsmem_ld16(uint32_t addr) {
    int4 v;
    asm volatile("ld.shared::cluster.v4.s32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(addr)
                 : "memory");
    return v;
}
__device__ __forceinline__ uint32_t dsmem_ld4(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
    return v;
}

__device__ __forceinline__ void report_status(int *status, int bits) {
    if (status) atomicOr(status, bits);
}

}  // namespace fbk
