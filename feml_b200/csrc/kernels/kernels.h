// Host-side launch interface of the sm_100a kernels (one .cu per family).
// Every launcher validates its arguments, enqueues on `stream` and returns an
// FB_* status (recording the message through fb::set_error on failure).
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>

#include "../host_common.h"

namespace fbk {

// Per-device "done" flags of a launcher's one-time kernel attribute setup.
using DeviceFlags = std::atomic<bool>[64];

// Raise `func`'s dynamic shared-memory limit to `bytes` the first time it is
// launched on the current device. The flag is atomic, so host threads that
// launch concurrently do not race on it; two threads that both see it unset
// both set the attribute, which is idempotent.
inline int raise_smem_limit(const void *func, int bytes, DeviceFlags &done, const char *what) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) dev = -1;
    const bool tracked = dev >= 0 && dev < 64;
    if (tracked && done[dev].load(std::memory_order_acquire)) return FB_OK;
    const cudaError_t e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return fb::set_error(FB_ERR_CUDA, "%s: smem attribute: %s", what, cudaGetErrorString(e));
    if (tracked) done[dev].store(true, std::memory_order_release);
    return FB_OK;
}

// Fused output epilogue of a mul_mat (a plan's mul_mat -> add(bias) -> silu
// chain computed by the mul_mat's kernel): out[n][m] = act(y[n][m] + bias[m]).
// The standalone add and silu kernels use the same expressions, so a fused
// chain gives the bits of the node-by-node one.
struct EpiAct {
    const float *bias;  // M floats, or nullptr
    int silu;           // apply SiLU, x / (1 + exp(-x)), after the bias
};
inline bool epi_active(const EpiAct *e) { return e && (e->bias || e->silu); }
#ifdef __CUDACC__
__device__ __forceinline__ float silu_f32(float v) { return __fdiv_rn(v, __fadd_rn(1.0f, expf(-v))); }
__device__ __forceinline__ float apply_act(float v, const EpiAct &e, int m) {
    if (e.bias) v = __fadd_rn(v, e.bias[m]);
    if (e.silu) v = silu_f32(v);
    return v;
}
#endif

// Planar Q8_0 activations: the device-internal form the quantized kernels
// read. Column n of an activation matrix [K, N] becomes qs[n*K .. n*K+K)
// (int8), d[n*(K/32) + b] (the f16-rounded block scale as f32) and
// sum[n*(K/32) + b] (sum of the block's 32 integers).
struct Q8Planar {
    int8_t *qs;
    float *d;
    int32_t *sum;
};

// Bytes of a planar Q8_0 buffer for [K, N] activations (each part padded to
// 256 bytes).
uint64_t q8_planar_bytes(int64_t K, int64_t N);
Q8Planar q8_planar_carve(void *base, int64_t K, int64_t N);

// quantize.cu
int launch_quantize_rows(int32_t dtype, const void *x, uint64_t x_row_stride, void *y, int64_t rows, int64_t k,
                         cudaStream_t s);
// quantize_row_q8_0 into planar form; columns of x at x + n*x_nb1.
int launch_quantize_q8_planar(const void *x, uint64_t x_nb1, int64_t K, int64_t N, Q8Planar out, cudaStream_t s);

// gemv.cu: dequant-fused GEMV for small N (1..8). When `xq` is non-null the
// activations were quantized by a preceding kernel (read after a
// programmatic-dependent-launch wait); otherwise each CTA quantizes them
// itself (fused path, no workspace).
bool gemv_supported(int32_t wtype, int64_t K, int64_t N);
bool gemv_fused_ok(int64_t K, int64_t N);
int gemv_max_cols();  // largest N the GEMV takes
// Peer outputs of a row-sharded GEMV: y[b][r] is output buffer b (0/1,
// alternating by step) of rank r at this rank's first row (device pointers
// valid here: own memory or an IPC mapping of a peer's), flag[r] rank r's
// step flag, count a zeroed device counter of this rank, epoch this rank's
// count of completed steps (buffer = (epoch + 1) & 1). The last warp of the
// grid raises every flag by one.
// owner_tokens > 0 (grouped GEMM only): outputs are not replicated; token t
// belongs to rank t / owner_tokens, whose buffers hold its owner_tokens
// tokens, and a slot of token t is stored only there, at local token
// t % owner_tokens.
constexpr int kMaxPeers = 8;
struct PeerOut {
    uint8_t *y[2][kMaxPeers];
    uint32_t *flag[kMaxPeers];
    uint32_t *count;
    const uint32_t *epoch;
    int n;
    int owner_tokens;
};
// With `norm_eps` (in-kernel quantization only: xq and peer null) every
// activation column is rms-normalized with that eps before it is quantized.
// With `epi` the outputs go through the fused bias / SiLU epilogue.
int launch_gemv(int32_t wtype, const void *w, uint64_t w_nb1, const void *x, uint64_t x_nb1, void *y,
                uint64_t y_nb1, int64_t K, int64_t M, int64_t N, const Q8Planar *xq, int32_t *status,
                cudaStream_t s, bool pdl, const PeerOut *peer = nullptr, const float *norm_eps = nullptr,
                const EpiAct *epi = nullptr);
// Wait until this rank's flag reaches (epoch + 1) * n_ranks, then advance
// the epoch (bounded by timeout_us; STATUS_TIMEOUT on expiry).
constexpr uint64_t kPeerWaitTimeoutUs = 1000000;  // default bound: one second
int launch_peer_wait(const uint32_t *flag, uint32_t *epoch, int32_t n_ranks, int32_t *status, cudaStream_t s,
                     uint64_t timeout_us = kPeerWaitTimeoutUs);

// norm.cu: rms_norm along ne0 (y may alias x); ne[4], strides in bytes.
int launch_rms_norm(const void *x, const uint64_t *xnb, void *y, const uint64_t *ynb, const int64_t *ne, float eps,
                    cudaStream_t s);

// gemm_f32.cu: F32 mul_mat on SIMT FP32 (any N), bit-exact with the
// reference's sequential order. `status` receives STATUS_TIMEOUT if a bounded
// pipeline wait gives up.
int launch_gemm_f32(const void *w, uint64_t w_nb1, const void *x, uint64_t x_nb1, void *y, uint64_t y_nb1,
                    int64_t K, int64_t M, int64_t N, int32_t *status, cudaStream_t s);

// gemm_q.cu: quantized mul_mat for large N on Q8Planar activations. The
// optional gather maps (MoE) select activation columns and output columns.
struct GroupMap {
    const int32_t *counts;   // [n_groups] columns per group (device)
    const int32_t *offsets;  // [n_groups] exclusive prefix (device)
    const int32_t *rows;     // [n_slots] slot ids in group order (device)
    const int32_t *tile_start;  // [n_groups + 1] prefix of ceil(count/BN) (device)
    int32_t n_groups;
    int32_t n_selected;
    uint64_t w_group_stride;   // bytes between experts' weights
    uint64_t dst_nb1, dst_nb2; // dst column (s, t) at dst + s*nb1 + t*nb2
    int32_t max_tiles;         // upper bound of total column tiles
};
int launch_gemm_f32_grouped(const void *w, uint64_t w_nb1, const void *x, uint64_t x_nb1, int64_t K, int64_t M,
                            void *dst, const GroupMap &g, cudaStream_t s);
int gemm_f32_block_n();
bool gemm_q_supported(int32_t wtype, int64_t K, const void *w, uint64_t w_nb1);
// split_ws (ungrouped only): gemm_q_split_bytes(K, M, N) bytes for the
// split-K partial tiles; null runs without split-K.
int launch_gemm_q(int32_t wtype, const void *w, uint64_t w_nb1, const Q8Planar &xq, int64_t K, int64_t M, int64_t N,
                  void *y, uint64_t y_nb1, const GroupMap *groups, cudaStream_t s, void *split_ws = nullptr);
int gemm_q_block_n();
int gemm_q_splits(int64_t K, int64_t M, int64_t N);
uint64_t gemm_q_split_bytes(int64_t K, int64_t M, int64_t N);

// gemm_tc.cu: tcgen05/TMEM GEMM for Q8_0 / Q4_0 / Q4_K weights (K % 256 == 0,
// 16-byte aligned rows). Activations come quantized to Q8_0 as XQ16. For the
// split-f16 kernel (Q8_0, Q4_0, and Q4_K with K % 512 == 0): q16 holds two
// planes [2][rows][KE] of f16, hi and lo of the dequantized activation times
// 2^-e_row (Q4_K: KE = 576 per 512 elements, the block sums after each 512),
// and xscale [rows] = 2^e_row. For the per-block kernel (other Q4_K): q16
// [rows][K] exact f16 integers, dxT / xsdT [K/32][rows] (block scale and
// scale * integer sum). Both leave room for split-K partial tiles.
struct XQ16 {
    void *q16;
    float *dxT;
    float *xsdT;
    float *xscale;
    float *partial;
};
// Bytes of an XQ16 buffer for `rows` activation rows (plus the split-K
// partials of an ungrouped M x rows GEMM).
uint64_t xq16_bytes(int32_t wtype, int64_t K, int64_t rows, int64_t M, bool grouped);
XQ16 xq16_carve(int32_t wtype, void *base, int64_t K, int64_t rows);
bool gemm_tc_supported(int32_t wtype, int64_t K, int64_t M, int64_t N, const void *w, uint64_t w_nb1);
int gemm_tc_splits(int32_t wtype, int64_t K, int64_t M, int64_t N);
// Tail split of a multi-wave ungrouped GEMM: the last `rows` m-tile rows
// split `splits` ways in K (split_pairs block pairs each) and summed by a
// reduction kernel; false when the grid gains nothing from it.
struct TailPlan {
    int rows, splits, split_pairs;
};
bool gemm_tc_tail(int32_t wtype, int64_t K, int64_t M, int64_t N, TailPlan *tp);
// With `routed` (mul_mat_id), the N * n_selected operand rows are the routed
// slots in expert order (row r from token routed->rows[r] / n_selected).
// `wtype` is the weight type of the GEMM that reads the result (it picks
// the operand form above).
int launch_quantize_q8_f16(const void *x, uint64_t x_nb1, int64_t K, int64_t N, const XQ16 &out,
                           const GroupMap *routed, cudaStream_t s, int32_t wtype);
// With `groups` (mul_mat_id): expert planes w + e*groups->w_group_stride,
// activation rows = routed slots (N tokens x n_selected), outputs through
// the group map. Column tiles of groups->tile_start use gemm_tc_block_n(wtype, K).
// With `peer` (grouped mode only): each output value is stored into every
// rank's buffer of this step instead of y (see PeerOut), then every rank's
// flag is raised once by the grid's last CTA.
// With `epi` (ungrouped only) the outputs go through the fused bias / SiLU
// epilogue.
int launch_gemm_tc(int32_t wtype, const void *w, uint64_t w_nb1, const XQ16 &xa, int64_t K, int64_t M, int64_t N,
                   void *y, uint64_t y_nb1, const GroupMap *groups, int32_t *status, cudaStream_t s,
                   const PeerOut *peer = nullptr, const EpiAct *epi = nullptr);
// Column-tile width of the kernel that runs `wtype` at this K (192 split-f16,
// 128 per-block).
int gemm_tc_block_n(int32_t wtype, int64_t K);

// Per-block int32 sums (bit-exactness probe); xq in ggml Q8_0 layout.
int launch_block_dots(int32_t wtype, const void *w, uint64_t w_nb1, const void *xq, int64_t K, int64_t M, int64_t N,
                      int32_t *out, cudaStream_t s);

// moe.cu: routing tables + column-tile prefix for gemm_q's grouped mode.
// When dst is non-null, output columns of slots with an invalid id are
// zeroed (and STATUS_BAD_ID is raised).
// Expert sharding: expert e belongs to shard e % n_shards as local expert
// e / n_shards; other shards' slots are skipped (no write). With `epoch`
// (fused multi-GPU steps) the zeroed buffer is dst_alt when (*epoch + 1) is
// odd, dst otherwise.
inline int64_t local_experts(int64_t n_experts, int64_t shard, int64_t n_shards) {
    return n_experts > shard ? (n_experts - shard + n_shards - 1) / n_shards : 0;
}
// With owner_tokens > 0 dst holds only this shard's tokens [shard *
// owner_tokens, +owner_tokens) (token t at local index t % owner_tokens),
// and only their invalid slots are zeroed.
int launch_moe_route(const int32_t *ids, uint64_t ids_nb1, int64_t n_selected, int64_t N, int64_t n_experts,
                     int64_t shard, int64_t n_shards, int32_t *counts, int32_t *offsets, int32_t *rows,
                     int32_t *tile_start, int32_t block_n, int32_t *status, void *dst, uint64_t dst_nb1,
                     uint64_t dst_nb2, int64_t M, cudaStream_t s, void *dst_alt = nullptr,
                     const uint32_t *epoch = nullptr, int64_t owner_tokens = 0);

// elementwise.cu: the reference's broadcasting add (feml-cpu/src/ops/
// elementwise.rs), SiLU, and the bias / SiLU epilogue applied in place to a
// finished mul_mat output y [N][M] (row n at y + n*y_nb1). ne[4] and byte
// strides nb[4] as in feml-core layouts; c may alias a or b exactly.
int launch_add_f32(const void *a, const int64_t *ane, const uint64_t *anb, const void *b, const int64_t *bne,
                   const uint64_t *bnb, void *c, const int64_t *cne, const uint64_t *cnb, cudaStream_t s);
int launch_silu_f32(const void *x, const uint64_t *xnb, void *y, const uint64_t *ynb, const int64_t *ne,
                    cudaStream_t s);
int launch_bias_act(void *y, uint64_t y_nb1, int64_t M, int64_t N, const EpiAct &epi, cudaStream_t s);

int sm_count();

}  // namespace fbk
