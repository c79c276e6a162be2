// Elementwise f32 ops of the plans that feed and follow mul_mat: the
// reference's broadcasting add (feml-cpu/src/ops/elementwise.rs:30-96: a
// source dimension of size 1 broadcasts; c may alias a or b exactly), SiLU
// (feml-core/src/op.rs:32, x / (1 + exp(-x)); the reference has no kernel for
// it), and the bias / SiLU epilogue applied in place to a finished mul_mat
// output when the producing kernel has no fused epilogue. Each element is
// read before it is written by the same thread, so exact aliasing is safe.
// The arithmetic is apply_act's (kernels.h), so a chain computed here gives
// the same bits as the epilogue fused into a mul_mat kernel.
#include <cuda_runtime.h>

#include <algorithm>

#include "../host_common.h"
#include "common.cuh"
#include "kernels.h"

namespace fbk {

namespace {

constexpr int kEwThreads = 256;

struct Dims4 {
    int64_t ne[4];
    uint64_t anb[4], bnb[4], cnb[4];
    int64_t ane[4], bne[4];
};

__global__ void add_f32_kernel(const uint8_t *__restrict__ a, const uint8_t *__restrict__ b, uint8_t *c,
                               const Dims4 d, int64_t total) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        int64_t r = i;
        uint64_t oa = 0, ob = 0, oc = 0;
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int64_t ik = r % d.ne[k];
            r /= d.ne[k];
            oa += (uint64_t)(d.ane[k] == 1 ? 0 : ik) * d.anb[k];
            ob += (uint64_t)(d.bne[k] == 1 ? 0 : ik) * d.bnb[k];
            oc += (uint64_t)ik * d.cnb[k];
        }
        const float x = *reinterpret_cast<const float *>(a + oa);
        const float y = *reinterpret_cast<const float *>(b + ob);
        *reinterpret_cast<float *>(c + oc) = __fadd_rn(x, y);
    }
}

__global__ void silu_f32_kernel(const uint8_t *x, uint8_t *y, const Dims4 d, int64_t total) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        int64_t r = i;
        uint64_t ox = 0, oy = 0;
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int64_t ik = r % d.ne[k];
            r /= d.ne[k];
            ox += (uint64_t)ik * d.anb[k];
            oy += (uint64_t)ik * d.cnb[k];
        }
        *reinterpret_cast<float *>(y + oy) = silu_f32(*reinterpret_cast<const float *>(x + ox));
    }
}

__global__ void bias_act_kernel(uint8_t *y, uint64_t y_nb1, int M, int64_t total, const EpiAct e) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int m = (int)(i % M);
        float *p = reinterpret_cast<float *>(y + (uint64_t)(i / M) * y_nb1) + m;
        *p = apply_act(*p, e, m);
    }
}

unsigned grid_for(int64_t total) {
    return (unsigned)std::max<int64_t>(1, std::min<int64_t>((total + kEwThreads - 1) / kEwThreads, 8 * sm_count()));
}

bool aligned4(const void *p, const uint64_t *nb) {
    uint64_t v = reinterpret_cast<uintptr_t>(p);
    for (int k = 0; k < 4; k++) v |= nb[k];
    return (v & 3) == 0;
}

}  // namespace

int launch_add_f32(const void *a, const int64_t *ane, const uint64_t *anb, const void *b, const int64_t *bne,
                   const uint64_t *bnb, void *c, const int64_t *cne, const uint64_t *cnb, cudaStream_t s) {
    Dims4 d{};
    int64_t total = 1;
    for (int k = 0; k < 4; k++) {
        if (cne[k] < 0 || ane[k] < 1 || bne[k] < 1) return fb::set_error(FB_ERR_SHAPE, "shape error: add: bad shape");
        if ((ane[k] != 1 && ane[k] != cne[k]) || (bne[k] != 1 && bne[k] != cne[k]))
            return fb::set_error(FB_ERR_SHAPE, "shape error: add: dim %d: %ld and %ld do not broadcast to %ld", k,
                                 (long)ane[k], (long)bne[k], (long)cne[k]);
        d.ne[k] = cne[k];
        d.ane[k] = ane[k];
        d.bne[k] = bne[k];
        d.anb[k] = anb[k];
        d.bnb[k] = bnb[k];
        d.cnb[k] = cnb[k];
        total *= cne[k];
    }
    if (total == 0) return FB_OK;
    if (!aligned4(a, anb) || !aligned4(b, bnb) || !aligned4(c, cnb))
        return fb::set_error(FB_ERR_INVALID, "add: f32 operands must be 4-byte aligned");
    add_f32_kernel<<<grid_for(total), kEwThreads, 0, s>>>(static_cast<const uint8_t *>(a),
                                                            static_cast<const uint8_t *>(b),
                                                            static_cast<uint8_t *>(c), d, total);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? FB_OK : fb::set_error(FB_ERR_CUDA, "add launch: %s", cudaGetErrorString(e));
}

int launch_silu_f32(const void *x, const uint64_t *xnb, void *y, const uint64_t *ynb, const int64_t *ne,
                    cudaStream_t s) {
    Dims4 d{};
    int64_t total = 1;
    for (int k = 0; k < 4; k++) {
        if (ne[k] < 0) return fb::set_error(FB_ERR_SHAPE, "shape error: silu: bad shape");
        d.ne[k] = ne[k];
        d.anb[k] = xnb[k];
        d.cnb[k] = ynb[k];
        total *= ne[k];
    }
    if (total == 0) return FB_OK;
    if (!aligned4(x, xnb) || !aligned4(y, ynb)) return fb::set_error(FB_ERR_INVALID, "silu: f32 operands must be 4-byte aligned");
    silu_f32_kernel<<<grid_for(total), kEwThreads, 0, s>>>(static_cast<const uint8_t *>(x), static_cast<uint8_t *>(y),
                                                             d, total);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? FB_OK : fb::set_error(FB_ERR_CUDA, "silu launch: %s", cudaGetErrorString(e));
}

int launch_bias_act(void *y, uint64_t y_nb1, int64_t M, int64_t N, const EpiAct &epi, cudaStream_t s) {
    if (!epi_active(&epi) || M == 0 || N == 0) return FB_OK;
    if (M > INT32_MAX || ((reinterpret_cast<uintptr_t>(y) | y_nb1) & 3))
        return fb::set_error(FB_ERR_INVALID, "bias/silu epilogue: bad output");
    const int64_t total = M * N;
    bias_act_kernel<<<grid_for(total), kEwThreads, 0, s>>>(static_cast<uint8_t *>(y), y_nb1, (int)M, total, epi);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? FB_OK : fb::set_error(FB_ERR_CUDA, "bias/silu launch: %s", cudaGetErrorString(e));
}

}  // namespace fbk
