// mul_mat_id front end: routing tables for the grouped GEMMs.
//
// Slot i = s + t*n_selected (ggml ids [n_selected, N]) selects expert
// ids[s, t]. With expert sharding, expert e belongs to shard e % n_shards
// and is local expert e / n_shards there; slots of other shards are skipped
// (their owner computes them), ids outside [0, E) are invalid. The tables
// list, per local expert, its slots in ascending order:
//   counts[e], offsets[e] (exclusive prefix), rows[offsets[e] + r],
//   tile_start[e] = sum_{e' < e} ceil(counts[e'] / block_n)   (e = 0..E)
// One CTA builds them: slots are processed in 1024-slot chunks; within a
// chunk each warp ranks its lanes per expert with __match_any_sync and a
// per-(warp, expert) prefix places them, so the order is the stable
// ascending slot order (bit-identical to a sequential scan).
#include <cuda_runtime.h>

#include "../host_common.h"
#include "common.cuh"
#include "kernels.h"

namespace fbk {

namespace {

constexpr int kRouteThreads = 1024;
constexpr int kRouteWarps = kRouteThreads / 32;
constexpr int kMaxExperts = 256;

__global__ void __launch_bounds__(kRouteThreads) moe_route_kernel(const int32_t *__restrict__ ids, uint64_t ids_stride,
                                                                   int n_sel, int N, int E, int shard, int n_shards,
                                                                   int n_local, int32_t *counts,
                                                                   int32_t *offsets, int32_t *rows,
                                                                   int32_t *tile_start, int block_n, int32_t *status,
                                                                   uint8_t *dst, uint64_t dst_nb1, uint64_t dst_nb2,
                                                                   int M, uint8_t *dst_alt, const uint32_t *epoch,
                                                                   int owner_tokens) {
    __shared__ int cnt[kMaxExperts];
    __shared__ int base[kMaxExperts];
    __shared__ int off[kMaxExperts];
    __shared__ int wcnt[kRouteWarps][kMaxExperts];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n_slots = n_sel * N;
    // local expert of a slot: -1 = another shard's, -2 = invalid id
    auto local_of = [&](int e) -> int {
        if (e < 0 || e >= E) return -2;
        return (e % n_shards) == shard ? e / n_shards : -1;
    };
    for (int e = tid; e < n_local; e += kRouteThreads) {
        cnt[e] = 0;
        base[e] = 0;
    }
    __syncthreads();
    int bad = 0;
    for (int i = tid; i < n_slots; i += kRouteThreads) {
        const int le = local_of(ids[(uint64_t)(i / n_sel) * ids_stride + (i % n_sel)]);
        if (le >= 0)
            atomicAdd(&cnt[le], 1);
        else if (le == -2)
            bad = 1;
    }
    const int any_bad = __syncthreads_or(bad);
    if (any_bad && tid == 0) report_status(status, STATUS_BAD_ID);
    if (epoch && ((*epoch + 1u) & 1u)) dst = dst_alt;  // this step's buffer of a fused multi-GPU step
    if (any_bad && dst) {  // slots with an invalid id produce zeros
        for (int i = 0; i < n_slots; i++) {
            const int t = i / n_sel, s = i % n_sel;
            const int e = ids[(uint64_t)t * ids_stride + s];
            if (local_of(e) != -2) continue;
            int lt = t;  // token index in dst
            if (owner_tokens > 0) {
                if (t / owner_tokens != shard) continue;  // another rank's token: its owner zeroes it
                lt = t % owner_tokens;
            }
            float *col = reinterpret_cast<float *>(dst + (uint64_t)s * dst_nb1 + (uint64_t)lt * dst_nb2);
            for (int m = tid; m < M; m += kRouteThreads) col[m] = 0.0f;
        }
    }
    if (tid == 0) {
        int run = 0, tiles = 0;
        for (int e = 0; e < n_local; e++) {
            off[e] = run;
            counts[e] = cnt[e];
            offsets[e] = run;
            if (tile_start) tile_start[e] = tiles;
            run += cnt[e];
            tiles += (cnt[e] + block_n - 1) / block_n;
        }
        if (tile_start) tile_start[n_local] = tiles;
    }
    __syncthreads();
    for (int c0 = 0; c0 < n_slots; c0 += kRouteThreads) {
        for (int i = tid; i < kRouteWarps * n_local; i += kRouteThreads) wcnt[i / n_local][i % n_local] = 0;
        __syncthreads();
        const int i = c0 + tid;
        int e = -1;
        if (i < n_slots) {
            e = local_of(ids[(uint64_t)(i / n_sel) * ids_stride + (i % n_sel)]);
            if (e < 0) e = -1;
        }
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        const int rank = __popc(peers & ((1u << lane) - 1u));
        if (e >= 0 && rank == 0) wcnt[warp][e] = __popc(peers);
        __syncthreads();
        // exclusive prefix over warps, per expert; advance the expert base
        for (int x = tid; x < n_local; x += kRouteThreads) {
            int run = base[x];
            for (int w = 0; w < kRouteWarps; w++) {
                const int v = wcnt[w][x];
                wcnt[w][x] = run;
                run += v;
            }
            base[x] = run;
        }
        __syncthreads();
        if (e >= 0) rows[off[e] + wcnt[warp][e] + rank] = i;
        __syncthreads();
    }
}

}  // namespace

int launch_moe_route(const int32_t *ids, uint64_t ids_nb1, int64_t n_selected, int64_t N, int64_t n_experts,
                     int64_t shard, int64_t n_shards, int32_t *counts, int32_t *offsets, int32_t *rows,
                     int32_t *tile_start, int32_t block_n, int32_t *status, void *dst, uint64_t dst_nb1,
                     uint64_t dst_nb2, int64_t M, cudaStream_t s, void *dst_alt, const uint32_t *epoch,
                     int64_t owner_tokens) {
    if (n_experts < 1 || n_experts > kMaxExperts)
        return fb::set_error(FB_ERR_UNSUPPORTED, "mul_mat_id: n_experts %ld not in [1, %d]", (long)n_experts, kMaxExperts);
    if (n_shards < 1 || shard < 0 || shard >= n_shards)
        return fb::set_error(FB_ERR_INVALID, "mul_mat_id: shard %ld of %ld", (long)shard, (long)n_shards);
    const int64_t n_local = local_experts(n_experts, shard, n_shards);
    if (n_selected < 1 || N < 0 || n_selected * N > INT32_MAX / 2)
        return fb::set_error(FB_ERR_INVALID, "mul_mat_id: bad slot count");
    if (ids_nb1 % 4 || (reinterpret_cast<uintptr_t>(ids) & 3))
        return fb::set_error(FB_ERR_INVALID, "mul_mat_id: ids must be 4-byte aligned");
    if (owner_tokens < 0 || owner_tokens > INT32_MAX || (owner_tokens > 0 && owner_tokens * n_shards < N))
        return fb::set_error(FB_ERR_INVALID, "mul_mat_id: %ld tokens per owner for %ld tokens on %ld shards",
                             (long)owner_tokens, (long)N, (long)n_shards);
    moe_route_kernel<<<1, kRouteThreads, 0, s>>>(ids, ids_nb1 / 4, (int)n_selected, (int)N, (int)n_experts, (int)shard,
                                                 (int)n_shards, (int)n_local, counts,
                                                 offsets, rows, tile_start, block_n, status,
                                                 static_cast<uint8_t *>(dst), dst_nb1, dst_nb2, (int)M,
                                                 static_cast<uint8_t *>(dst_alt), epoch, (int)owner_tokens);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fb::set_error(FB_ERR_CUDA, "moe_route launch: %s", cudaGetErrorString(e));
    return FB_OK;
}

}  // namespace fbk
