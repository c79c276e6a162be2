// RMS normalization (Op::RmsNorm { eps }, feml-core/src/op.rs:26; built by
// GraphBuilder::rms_norm, graph.rs:140-142; the reference has no kernel):
//   y[k] = x[k] * (1 / sqrt(sum_k x[k]^2 / ne0 + eps))   along ne0, per row.
// One CTA per row: each thread accumulates its strided elements, the warp
// sums meet in shared memory and are added in warp order (deterministic), then
// the row is scaled. In-place (y == x) is safe: every write comes after the
// row's sum is complete. The decode GEMV applies the same normalization to
// its activations itself when a plan feeds rms_norm straight into mul_mat
// (gemv.cu), so this kernel runs only where the normalized tensor is needed.
#include <cuda_runtime.h>

#include "../host_common.h"
#include "common.cuh"
#include "kernels.h"

namespace fbk {

namespace {

constexpr int kNormThreads = 256;

struct NormParams {
    const uint8_t *x;
    uint8_t *y;
    int64_t ne0, ne1, ne2;
    uint64_t xnb1, xnb2, xnb3, ynb1, ynb2, ynb3;
    float eps;
};

__global__ void __launch_bounds__(kNormThreads) rms_norm_kernel(const NormParams p) {
    __shared__ float s_part[kNormThreads / 32];
    __shared__ float s_scale;
    const int64_t r = blockIdx.x;
    const int64_t i1 = r % p.ne1, i2 = (r / p.ne1) % p.ne2, i3 = r / (p.ne1 * p.ne2);
    const float *x = reinterpret_cast<const float *>(p.x + i1 * p.xnb1 + i2 * p.xnb2 + i3 * p.xnb3);
    float *y = reinterpret_cast<float *>(p.y + i1 * p.ynb1 + i2 * p.ynb2 + i3 * p.ynb3);
    float ss = 0.0f;
    for (int64_t k = threadIdx.x; k < p.ne0; k += kNormThreads) {
        const float v = x[k];
        ss = fmaf(v, v, ss);
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.0f;
#pragma unroll
        for (int w = 0; w < kNormThreads / 32; w++) t += s_part[w];
        s_scale = 1.0f / sqrtf(t / (float)p.ne0 + p.eps);
    }
    __syncthreads();
    const float sc = s_scale;
    for (int64_t k = threadIdx.x; k < p.ne0; k += kNormThreads) y[k] = x[k] * sc;
}

}  // namespace

int launch_rms_norm(const void *x, const uint64_t *xnb, void *y, const uint64_t *ynb, const int64_t *ne, float eps,
                    cudaStream_t s) {
    if (!x || !y || !xnb || !ynb || !ne) return fb::set_error(FB_ERR_INVALID, "rms_norm: null argument");
    if (xnb[0] != 4 || ynb[0] != 4) return fb::set_error(FB_ERR_UNSUPPORTED, "rms_norm: rows must be contiguous f32");
    if (((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 3) != 0)
        return fb::set_error(FB_ERR_INVALID, "rms_norm: operands must be 4-byte aligned");
    for (int d = 0; d < 4; d++)
        if (ne[d] < 0) return fb::set_error(FB_ERR_SHAPE, "rms_norm: negative dimension");
    const int64_t rows = ne[1] * ne[2] * ne[3];
    if (rows == 0 || ne[0] == 0) return FB_OK;
    if (rows > INT32_MAX) return fb::set_error(FB_ERR_UNSUPPORTED, "rms_norm: too many rows");
    NormParams p;
    p.x = static_cast<const uint8_t *>(x);
    p.y = static_cast<uint8_t *>(y);
    p.ne0 = ne[0];
    p.ne1 = ne[1];
    p.ne2 = ne[2];
    p.xnb1 = xnb[1];
    p.xnb2 = xnb[2];
    p.xnb3 = xnb[3];
    p.ynb1 = ynb[1];
    p.ynb2 = ynb[2];
    p.ynb3 = ynb[3];
    p.eps = eps;
    rms_norm_kernel<<<(unsigned)rows, kNormThreads, 0, s>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fb::set_error(FB_ERR_CUDA, "rms_norm launch: %s", cudaGetErrorString(e));
    return FB_OK;
}

}  // namespace fbk
