// 2D TMA tensor maps shared by the kernels that move tiles with
// cp.async.bulk.tensor (the tcgen05 GEMM and the K-split decode GEMV).
#pragma once
#include <cuda.h>

#include <cstdint>

namespace fbk {

// 2D tiled tensor map, no swizzle; dim0 is contiguous, stride1 in bytes.
int encode_tensor_map_2d(CUtensorMap *map, CUtensorMapDataType dt, const void *base, uint64_t dim0, uint64_t dim1,
                         uint64_t stride1, uint32_t box0, uint32_t box1);
// The same with the 128-byte swizzle: box0 * element size must be 128 bytes;
// in shared memory (box start 1024-byte aligned) row y's 16-byte unit u lands
// at y * 128 + ((u ^ (y % 8)) * 16).
int encode_tensor_map_2d_sw128(CUtensorMap *map, CUtensorMapDataType dt, const void *base, uint64_t dim0,
                               uint64_t dim1, uint64_t stride1, uint32_t box0, uint32_t box1);

#ifdef __CUDACC__
// One 2D box into shared memory, completing on `bar` (no multicast). The
// innermost coordinate times the element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int c0, int c1, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar)
        : "memory");
}
#endif

}  // namespace fbk
