// On-device quantizers: quantize_row_q8_0 (activations, ggml or planar form)
// and the weight quantizers Q8_0 / Q4_0 / Q4_K. One warp per block; every
// arithmetic step is a correctly rounded IEEE operation written with explicit
// _rn intrinsics, so the bytes equal the CPU restatement's bit for bit.
#include <cuda_runtime.h>

#include <algorithm>

#include "../host_common.h"
#include "common.cuh"
#include "kernels.h"

namespace fbk {

namespace {

constexpr int kWarps = 8;

// Q8_0 in ggml layout: the same 8-lanes-per-block routine as the planar and
// in-GEMV activation quantizers (one implementation of quantize_row_q8_0).
__global__ void __launch_bounds__(256) quantize_q8_0_kernel(const uint8_t *__restrict__ x, uint64_t x_stride,
                                                            uint8_t *__restrict__ y, int64_t rows, int64_t k) {
    const int64_t qpr = k / 4;
    const int64_t nq = rows * qpr;  // a multiple of 8
    for (int64_t base = (int64_t)blockIdx.x * 256; base < nq; base += (int64_t)gridDim.x * 256) {
        const int64_t q = base + threadIdx.x;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        int64_t r = 0, e = 0;
        if (q < nq) {
            r = q / qpr;
            e = (q % qpr) * 4;
            const float *xr = reinterpret_cast<const float *>(x + r * x_stride);
            v = make_float4(xr[e], xr[e + 1], xr[e + 2], xr[e + 3]);
        }
        uint16_t dbits;
        int qsum;
        const uint32_t packed = quantize_q8_0_quad(v, dbits, qsum);
        if (q < nq) {
            uint8_t *yb = y + (r * (k / QK) + e / QK) * Q8_0_BYTES;
            const int o = (int)(e % QK);
            // 2-byte-aligned destination: two 16-bit stores
            *reinterpret_cast<uint16_t *>(yb + 2 + o) = (uint16_t)(packed & 0xffffu);
            *reinterpret_cast<uint16_t *>(yb + 4 + o) = (uint16_t)(packed >> 16);
            if ((threadIdx.x & 7u) == 0) *reinterpret_cast<uint16_t *>(yb) = dbits;
        }
    }
}

// Planar activations: one float4 quad per thread per pass, 8 lanes per block,
// so every thread has its load in flight at once.
__global__ void __launch_bounds__(256) quantize_q8_planar_kernel(const uint8_t *__restrict__ x, uint64_t x_nb1,
                                                                 int64_t K, int64_t N, Q8Planar out) {
    const int64_t nblk = K / QK;
    const int64_t qpr = K / 4;       // quads per column
    const int64_t nq = N * qpr;      // a multiple of 8: groups never straddle the end
    for (int64_t base = (int64_t)blockIdx.x * 256; base < nq; base += (int64_t)gridDim.x * 256) {
        const int64_t q = base + threadIdx.x;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        int64_t n = 0, e = 0;
        if (q < nq) {
            n = q / qpr;
            e = (q % qpr) * 4;
            const float *xr = reinterpret_cast<const float *>(x + n * x_nb1);
            v = make_float4(xr[e], xr[e + 1], xr[e + 2], xr[e + 3]);
        }
        uint16_t dbits;
        int qsum;
        const uint32_t packed = quantize_q8_0_quad(v, dbits, qsum);  // all lanes take part
        if (q < nq) {
            *reinterpret_cast<uint32_t *>(out.qs + n * K + e) = packed;
            if ((threadIdx.x & 7u) == 0) {
                out.d[n * nblk + e / QK] = f16_bits_to_f32(dbits);
                out.sum[n * nblk + e / QK] = qsum;
            }
        }
    }
    // Let a dependent (programmatic) launch start its prologue.
    grid_launch_dependents();
}

// Q4_0: d = max / -8 with max the first element of largest magnitude;
// nibble = min(15, trunc(x * (1/d) + 8.5)).
__global__ void __launch_bounds__(kWarps * 32) quantize_q4_0_kernel(const uint8_t *__restrict__ x, uint64_t x_stride,
                                                                     uint8_t *__restrict__ y, int64_t rows,
                                                                     int64_t nblk) {
    const int lane = threadIdx.x & 31;
    const int64_t total = rows * nblk;
    for (int64_t i = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5); i < total; i += (int64_t)gridDim.x * kWarps) {
        const int64_t r = i / nblk, b = i % nblk;
        const float v = reinterpret_cast<const float *>(x + r * x_stride)[b * QK + lane];
        // first index of the largest |v| (ties -> lowest index, like a forward scan with '<')
        float a = fabsf(v);
        int idx = lane;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float oa = __shfl_xor_sync(0xffffffffu, a, o);
            const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
            if (oa > a || (oa == a && oi < idx)) { a = oa; idx = oi; }
        }
        float mx = __shfl_sync(0xffffffffu, v, idx);
        if (a == 0.0f) mx = 0.0f;  // the scan never updates `max` when every |v| is 0
        const float d = __fdiv_rn(mx, -8.0f);
        const float id = d != 0.0f ? __frcp_rn(d) : 0.0f;
        const float xv = __fadd_rn(__fmul_rn(v, id), 8.5f);
        int q = (int)(int8_t)(int)xv;  // truncation toward zero, as the (int8_t) cast
        q = q > 15 ? 15 : q;
        const int qhi = __shfl_down_sync(0xffffffffu, q, 16);
        uint8_t *yb = y + (r * nblk + b) * Q4_0_BYTES;
        if (lane < 16) yb[2 + lane] = (uint8_t)(q | (qhi << 4));
        if (lane == 0) *reinterpret_cast<uint16_t *>(yb) = __half_as_ushort(__float2half_rn(d));
    }
}

// Q4_K (this library's deterministic single-pass scheme): one warp per
// 256-element super-block; lane l owns element l of each of the 8 sub-blocks.
__global__ void __launch_bounds__(kWarps * 32) quantize_q4_k_kernel(const uint8_t *__restrict__ x, uint64_t x_stride,
                                                                     uint8_t *__restrict__ y, int64_t rows,
                                                                     int64_t nsb) {
    const int lane = threadIdx.x & 31;
    const int64_t total = rows * nsb;
    for (int64_t i = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5); i < total; i += (int64_t)gridDim.x * kWarps) {
        const int64_t r = i / nsb, s = i % nsb;
        const float *xs = reinterpret_cast<const float *>(x + r * x_stride) + s * QKK;
        float v[8], scale[8], minv[8];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            v[j] = xs[32 * j + lane];
            float lo = v[j], hi = v[j];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float olo = __shfl_xor_sync(0xffffffffu, lo, o);
                const float ohi = __shfl_xor_sync(0xffffffffu, hi, o);
                lo = olo < lo ? olo : lo;
                hi = ohi > hi ? ohi : hi;
            }
            // a forward scan from +0.0 with strict compares keeps +0.0 unless a
            // strictly negative (positive) element exists
            lo = lo < 0.0f ? lo : 0.0f;
            hi = hi > 0.0f ? hi : 0.0f;
            scale[j] = __fdiv_rn(__fsub_rn(hi, lo), 15.0f);
            minv[j] = -lo;
        }
        float max_scale = 0.0f, max_min = 0.0f;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            max_scale = scale[j] > max_scale ? scale[j] : max_scale;
            max_min = minv[j] > max_min ? minv[j] : max_min;
        }
        const uint16_t dh = __half_as_ushort(__float2half_rn(__fdiv_rn(max_scale, 63.0f)));
        const uint16_t mh = __half_as_ushort(__float2half_rn(__fdiv_rn(max_min, 63.0f)));
        const float df = f16_bits_to_f32(dh), mf = f16_bits_to_f32(mh);
        int sc[8], mm[8], q[8];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            int a = df > 0.0f ? (int)roundf(__fdiv_rn(scale[j], df)) : 0;
            int m = mf > 0.0f ? (int)roundf(__fdiv_rn(minv[j], mf)) : 0;
            sc[j] = a > 63 ? 63 : a;
            mm[j] = m > 63 ? 63 : m;
            const float ds = __fmul_rn(df, (float)sc[j]);
            const float dm = __fmul_rn(mf, (float)mm[j]);
            int t = 0;
            if (ds > 0.0f) {
                t = (int)roundf(__fdiv_rn(__fadd_rn(v[j], dm), ds));
                t = t < 0 ? 0 : (t > 15 ? 15 : t);
            }
            q[j] = t;
        }
        uint8_t *yb = y + (r * nsb + s) * Q4_K_BYTES;
#pragma unroll
        for (int g = 0; g < 4; g++) yb[16 + 32 * g + lane] = (uint8_t)(q[2 * g] | (q[2 * g + 1] << 4));
        if (lane == 0) {
            *reinterpret_cast<uint16_t *>(yb) = dh;
            *reinterpret_cast<uint16_t *>(yb + 2) = mh;
            uint8_t scales[12];
#pragma unroll
            for (int j = 0; j < 12; j++) scales[j] = 0;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                if (j < 4) {
                    scales[j] = (uint8_t)sc[j];
                    scales[j + 4] = (uint8_t)mm[j];
                } else {
                    scales[j + 4] = (uint8_t)((sc[j] & 0x0f) | ((mm[j] & 0x0f) << 4));
                    scales[j - 4] |= (uint8_t)((sc[j] >> 4) << 6);
                    scales[j] |= (uint8_t)((mm[j] >> 4) << 6);
                }
            }
#pragma unroll
            for (int j = 0; j < 12; j++) yb[4 + j] = scales[j];
        }
    }
}

__global__ void copy_rows_kernel(const uint8_t *__restrict__ x, uint64_t x_stride, uint8_t *__restrict__ y,
                                 int64_t rows, int64_t row_bytes) {
    const int64_t total = rows * row_bytes;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / row_bytes, c = i % row_bytes;
        y[i] = x[r * x_stride + c];
    }
}

int grid_for(int64_t work_items) {
    int64_t g = (work_items + kWarps - 1) / kWarps;
    const int64_t cap = (int64_t)sm_count() * 16;
    if (g > cap) g = cap;
    return (int)(g < 1 ? 1 : g);
}

}  // namespace

uint64_t q8_planar_bytes(int64_t K, int64_t N) {
    auto pad = [](uint64_t v) { return (v + 255) / 256 * 256; };
    const uint64_t nblk = (uint64_t)(K / QK);
    return pad((uint64_t)K * N) + pad(nblk * N * 4) + pad(nblk * N * 4);
}

Q8Planar q8_planar_carve(void *base, int64_t K, int64_t N) {
    auto pad = [](uint64_t v) { return (v + 255) / 256 * 256; };
    const uint64_t nblk = (uint64_t)(K / QK);
    uint8_t *p = static_cast<uint8_t *>(base);
    Q8Planar q;
    q.qs = reinterpret_cast<int8_t *>(p);
    p += pad((uint64_t)K * N);
    q.d = reinterpret_cast<float *>(p);
    p += pad(nblk * N * 4);
    q.sum = reinterpret_cast<int32_t *>(p);
    return q;
}

int launch_quantize_rows(int32_t dtype, const void *x, uint64_t x_row_stride, void *y, int64_t rows, int64_t k,
                         cudaStream_t s) {
    if (rows < 0 || k < 0) return fb::set_error(FB_ERR_INVALID, "quantize: negative size");
    if (rows == 0 || k == 0) return FB_OK;
    if (!x || !y) return fb::set_error(FB_ERR_INVALID, "quantize: null pointer");
    if ((reinterpret_cast<uintptr_t>(x) & 3) || (x_row_stride & 3))
        return fb::set_error(FB_ERR_INVALID, "quantize: f32 source must be 4-byte aligned");
    const auto *xb = static_cast<const uint8_t *>(x);
    auto *yb = static_cast<uint8_t *>(y);
    switch (dtype) {
    case WT_Q8_0:
    case WT_Q4_0: {
        if (k % QK) return fb::set_error(FB_ERR_SHAPE, "quantize: k %ld is not a multiple of 32", (long)k);
        if (reinterpret_cast<uintptr_t>(y) & 1) return fb::set_error(FB_ERR_INVALID, "quantize: y must be 2-byte aligned");
        const int64_t nblk = k / QK;
        if (dtype == WT_Q8_0) {
            const int grid = (int)std::min<int64_t>((rows * k / 4 + 255) / 256, (int64_t)sm_count() * 16);
            quantize_q8_0_kernel<<<grid, 256, 0, s>>>(xb, x_row_stride, yb, rows, k);
        } else
            quantize_q4_0_kernel<<<grid_for(rows * nblk), kWarps * 32, 0, s>>>(xb, x_row_stride, yb, rows, nblk);
        break;
    }
    case WT_Q4_K: {
        if (k % QKK) return fb::set_error(FB_ERR_SHAPE, "quantize: k %ld is not a multiple of 256", (long)k);
        if (reinterpret_cast<uintptr_t>(y) & 1) return fb::set_error(FB_ERR_INVALID, "quantize: y must be 2-byte aligned");
        const int64_t nsb = k / QKK;
        quantize_q4_k_kernel<<<grid_for(rows * nsb), kWarps * 32, 0, s>>>(xb, x_row_stride, yb, rows, nsb);
        break;
    }
    case WT_F32: {
        const int64_t rb = 4 * k;
        copy_rows_kernel<<<grid_for(rows * rb / 256 + 1), 256, 0, s>>>(xb, x_row_stride, yb, rows, rb);
        break;
    }
    default:
        return fb::set_error(FB_ERR_UNSUPPORTED, "quantize: dtype %d not supported", dtype);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fb::set_error(FB_ERR_CUDA, "quantize launch: %s", cudaGetErrorString(e));
    return FB_OK;
}

int launch_quantize_q8_planar(const void *x, uint64_t x_nb1, int64_t K, int64_t N, Q8Planar out, cudaStream_t s) {
    if (K % QK) return fb::set_error(FB_ERR_SHAPE, "quantize_q8_0: K %ld is not a multiple of 32", (long)K);
    if (N == 0 || K == 0) return FB_OK;
    if ((reinterpret_cast<uintptr_t>(x) & 3) || (x_nb1 & 3))
        return fb::set_error(FB_ERR_INVALID, "quantize_q8_0: activations must be 4-byte aligned");
    const int64_t nq = N * K / 4;
    const int grid = (int)std::min<int64_t>((nq + 255) / 256, (int64_t)sm_count() * 16);
    quantize_q8_planar_kernel<<<grid, 256, 0, s>>>(static_cast<const uint8_t *>(x), x_nb1, K, N, out);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fb::set_error(FB_ERR_CUDA, "quantize_q8_0 launch: %s", cudaGetErrorString(e));
    return FB_OK;
}

}  // namespace fbk
