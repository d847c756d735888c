// Allocation-free normalised matrix-vector product.
//
// Some hosts cannot call cudaMalloc at the point where they need this product: code running while
// another component owns the device memory budget (a fixed pool carved out at start-up), or an
// embedding runtime that forbids allocation on its inference thread. This entry point allocates
// nothing. The caller passes device pointers for every input and output; the one intermediate (the
// RMS-normalised input rows, which the regular path keeps in a per-stage buffer) lives in a fixed
// device array in this file.
//
// The array is a file-scope __device__ variable, so every GPU that loads this library holds
// XJC_NOALLOC_MAX_FLOATS floats (256 KiB) of it until the process exits. All calls on a device share
// it and it keeps the last call's contents; each call overwrites every element it reads, so nothing
// needs to start at zero. Calls whose work overlaps on the GPU (other threads, other streams) race on
// the array: serialise them.
//
// In host code the array's name is not a device address. The first call on a device, with that device
// current, looks its address up with cudaGetSymbolAddress and caches it for that device; make that
// first call before any stream capture.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>

#include "../../include/xj_cuda.h"
#include "kernels.cuh"

using namespace xjk;

namespace {

static __device__ __align__(256) float g_noalloc_scratch[XJC_NOALLOC_MAX_FLOATS];

// Device address of g_noalloc_scratch per device, looked up once per device by the first call made
// with that device current. Atomic, so calls from several host threads may race on the first lookup
// harmlessly (each stores the same address). A cudaDeviceReset, or any other end of the device's
// primary context, invalidates the cached address: call xj_cuda_norm_gemv_noalloc only within one
// context lifetime per device.
constexpr int MAXDEV = 64;
std::atomic<float *> g_scratch_addr[MAXDEV];

void seterr(char *err, size_t errlen, const char *fmt, ...) {
    if (!err || !errlen) return;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(err, errlen, fmt, ap);
    va_end(ap);
}

uint64_t row_bytes(int type, int64_t n) {
    switch (type) {
    case XJ_F32: return (uint64_t)n * 4;
    case XJ_F16: case XJ_BF16: return (uint64_t)n * 2;
    case XJ_Q8_0: return (uint64_t)(n / 32) * 34;
    case XJ_Q4_K: return (uint64_t)(n / 256) * 144;
    case XJ_Q5_K: return (uint64_t)(n / 256) * 176;
    case XJ_Q6_K: return (uint64_t)(n / 256) * 210;
    default: return 0;
    }
}

}  // namespace

extern "C" int xj_cuda_norm_gemv_noalloc(int type, const void *w_dev, int k, int n, const float *x_dev,
                                         const float *norm_w_dev, float eps, int T, float *y_dev, char *err,
                                         size_t errlen) {
    const uint64_t rb = row_bytes(type, k);
    if (!rb || k <= 0 || k % 8 || (type != XJ_F32 && type != XJ_F16 && type != XJ_BF16 && k % 32) ||
        ((type == XJ_Q4_K || type == XJ_Q5_K || type == XJ_Q6_K) && k % 256)) {
        seterr(err, errlen, "unsupported type %d or row length %d", type, k);
        return -1;
    }
    if (n <= 0 || T < 1 || T > MAXT) { seterr(err, errlen, "need n >= 1 and 1 <= T <= %d", MAXT); return -1; }
    if ((long long)T * k > XJC_NOALLOC_MAX_FLOATS) {
        seterr(err, errlen, "T*k = %lld exceeds the fixed scratch of %d floats", (long long)T * k, XJC_NOALLOC_MAX_FLOATS);
        return -1;
    }
    if (!w_dev || !x_dev || !norm_w_dev || !y_dev) { seterr(err, errlen, "null device pointer"); return -1; }
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= MAXDEV) { seterr(err, errlen, "no usable current device"); return -1; }
    float *hn = g_scratch_addr[dev].load(std::memory_order_acquire);
    if (!hn) {
        e = cudaGetSymbolAddress((void **)&hn, g_noalloc_scratch);
        if (e != cudaSuccess || !hn) {
            seterr(err, errlen, "cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
            return -1;
        }
        g_scratch_addr[dev].store(hn, std::memory_order_release);
    }
    // rows of the normalised input (core/xj_cpu.c:56-61), then the product (core/xj_cpu.c:36-54)
    k_rmsnorm<<<T, 256>>>(x_dev, (long long)k, norm_w_dev, hn, (long long)k, k, eps);
    GemvArgs a{};
    a.job[0].w = DevMat{(const uint8_t *)w_dev, type, k, n, (long long)rb};
    a.job[0].y = y_dev;
    a.job[0].ldy = n;
    a.job[0].accumulate = 0;
    a.njob = 1;
    a.row_start[0] = 0;
    a.row_start[1] = n;
    a.x = hn;
    a.ldx = k;
    a.T = T;
    k_gemv_generic<<<(n + 7) / 8, 256>>>(a);
    e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaStreamSynchronize(0);
    if (e != cudaSuccess) { seterr(err, errlen, "CUDA error: %s", cudaGetErrorString(e)); return -1; }
    return 0;
}
