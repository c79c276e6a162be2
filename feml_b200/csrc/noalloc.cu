// mul_mat with a fixed, library-owned scratch area instead of a workspace
// from the caller.
//
// feml_b200_mul_mat takes its activation scratch (the Q8_0-quantized
// activations of the multi-column GEMV and the tiled GEMM) from the caller.
// Some callers cannot provide one: a host whose device memory is laid out
// once, up front, by a planner (every byte of a GraphPlan is placed ahead of
// time and an operator may not ask for more), or a caller on a stream that
// must not stall, since cudaFree synchronizes the whole device and
// cudaMalloc may. feml_b200_mul_mat_noalloc serves them: its scratch is the
// file-scope device array below, so the call allocates no memory of any
// kind; it runs the same kernels as feml_b200_mul_mat.
//
// Rules of the shared array:
//   * one array per device (the module's __device__ variable); its address is
//     looked up with cudaGetSymbolAddress on the first call made on each
//     device, with that device current. That first call also loads the
//     module on the device if nothing else has, so make it before any stream
//     capture.
//   * every call on a device uses the same bytes. Calls whose kernels may run
//     at the same time (different streams with no ordering between them,
//     host threads on different streams) race on them and give wrong results;
//     calls on one stream are ordered and safe.
//   * nothing in it needs to start at zero: each call writes the quantized
//     activations it reads before reading them.
//   * shapes whose scratch exceeds kStaticScratchBytes are rejected with
//     FB_ERR_UNSUPPORTED before any work is queued; arguments are checked
//     first, as feml_b200_mul_mat checks them (negative dimensions give
//     FB_ERR_INVALID, an empty output returns FB_OK, an unsupported weight
//     dtype gives FB_ERR_UNSUPPORTED).
//   * when the 16 MiB are taken: this file is its own device module (the
//     library is built without relocatable device code). Under lazy module
//     loading (CUDA_MODULE_LOADING=LAZY, the default of CUDA 12) the module,
//     and with it the array, is loaded into a device's context by the first
//     call on that device; under CUDA_MODULE_LOADING=EAGER every context the
//     process creates on any device reserves the 16 MiB at creation, whether
//     or not it ever calls this entry point.
#include <cuda_runtime.h>

#include <mutex>

#include "host_common.h"

namespace {

constexpr unsigned long long kStaticScratchBytes = 16ull << 20;  // 16 MiB
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_mul_mat_scratch[kStaticScratchBytes];

std::mutex g_mu;
void *g_scratch_addr[kMaxDevices];

int static_scratch(void **out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fb::set_error(FB_ERR_CUDA, "mul_mat_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices)
        return fb::set_error(FB_ERR_DEVICE, "mul_mat_noalloc: device %d beyond the %d supported", dev, kMaxDevices);
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scratch_addr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_mul_mat_scratch);
        if (e != cudaSuccess || !p)
            return fb::set_error(FB_ERR_CUDA, "mul_mat_noalloc: cudaGetSymbolAddress on device %d: %s", dev,
                                 cudaGetErrorString(e));
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return FB_OK;
}

}  // namespace

extern "C" {

uint64_t feml_b200_mul_mat_noalloc_limit(void) { return kStaticScratchBytes; }

int feml_b200_mul_mat_noalloc(int32_t wtype, const void *w, uint64_t w_nb1, const void *x, uint64_t x_nb1, void *dst,
                              uint64_t dst_nb1, int64_t K, int64_t M, int64_t N, void *stream) {
    if (K < 0 || M < 0 || N < 0) return fb::set_error(FB_ERR_INVALID, "mul_mat_noalloc: negative dimension");
    if (M == 0 || N == 0) return FB_OK;
    const int32_t dts[2] = {wtype, FB_F32};
    if (!feml_b200_supports_op(nullptr, FB_OP_MUL_MAT, dts, 2))
        return fb::set_error(FB_ERR_UNSUPPORTED, "mul_mat_noalloc: weight dtype %d not supported", wtype);
    uint64_t need = 0;
    int rc = feml_b200_mul_mat_workspace(wtype, K, M, N, &need);
    if (rc) return rc;
    if (need > kStaticScratchBytes)
        return fb::set_error(FB_ERR_UNSUPPORTED,
                             "mul_mat_noalloc: this shape needs %llu bytes of scratch, the static scratch holds %llu "
                             "(use feml_b200_mul_mat with a workspace)",
                             (unsigned long long)need, kStaticScratchBytes);
    void *ws = nullptr;
    if (need > 0) {
        rc = static_scratch(&ws);
        if (rc) return rc;
    }
    return feml_b200_mul_mat(wtype, w, w_nb1, x, x_nb1, dst, dst_nb1, K, M, N, ws, need > 0 ? kStaticScratchBytes : 0,
                             stream);
}

}  // extern "C"
