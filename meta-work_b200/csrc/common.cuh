// Shared device helpers for the xj CUDA backend (sm_100a).
#pragma once
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cstdint>

#include "../../include/xj_abi.h"

#define XJ_DEV __device__ __forceinline__

// A weight matrix resident in HBM: N rows of K elements. Row-major GGUF block layout (row r at
// p + r*ld) and/or the tensor-core tiled layout (tq/th/ts/td, see gemv_mma.cuh); either may be absent.
struct DevMat {
    const uint8_t *p;
    int type;        // enum xj_type
    int K, N;
    long long ld;    // bytes between rows (row-major layout)
    const uint8_t *tq = nullptr, *th = nullptr, *ts = nullptr, *td = nullptr;
};

XJ_DEV float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

XJ_DEV double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

XJ_DEV float warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide double sum; `red` must hold blockDim.x/32 doubles. All threads get the result.
XJ_DEV double block_sum_d(double v, double *red) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_sum_d(v);
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    double t = 0;
    for (int i = 0; i < nw; i++) t += red[i];
    return t;
}

XJ_DEV float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
XJ_DEV float bf2f(uint16_t h) { return __uint_as_float((uint32_t)h << 16); }
XJ_DEV uint16_t ld_u16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

// The math of the reference CPU path uses these exact forms (core/xj_cpu.c:63-65).
XJ_DEV float silu_f(float x) { return x / (1.0f + expf(-x)); }
XJ_DEV float sigm_f(float x) { return 1.0f / (1.0f + expf(-x)); }
XJ_DEV float softplus_f(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

// 6-bit (scale, min) of sub-block j of a K-quant super-block (layout of core/xj_quant.h:49-52).
XJ_DEV void k4_scale_min(int j, const uint8_t *q, int &d, int &m) {
    if (j < 4) { d = q[j] & 63; m = q[j + 4] & 63; }
    else { d = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4); m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4); }
}

// Dequantise 8 consecutive elements [e0, e0+8) (e0 % 8 == 0) of one row. The arithmetic per element
// is the reference's (core/xj_quant.h:55-122) with each product and difference rounded separately
// (no fused multiply-add, as the reference build evaluates it), so results are bit-identical.
XJ_DEV void dequant8(int type, const uint8_t *row, int e0, float *y) {
    switch (type) {
    case XJ_F32: {
        const float4 *p = reinterpret_cast<const float4 *>(row + 4 * (size_t)e0);
        float4 a = p[0], b = p[1];
        y[0] = a.x; y[1] = a.y; y[2] = a.z; y[3] = a.w; y[4] = b.x; y[5] = b.y; y[6] = b.z; y[7] = b.w;
        return;
    }
    case XJ_F16: case XJ_BF16: {
        uint4 v = *reinterpret_cast<const uint4 *>(row + 2 * (size_t)e0);
        uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            uint16_t lo = (uint16_t)(w[i] & 0xffff), hi = (uint16_t)(w[i] >> 16);
            y[2 * i] = type == XJ_F16 ? h2f(lo) : bf2f(lo);
            y[2 * i + 1] = type == XJ_F16 ? h2f(hi) : bf2f(hi);
        }
        return;
    }
    case XJ_Q8_0: {
        const uint8_t *b = row + (size_t)(e0 / 32) * 34;
        const float d = h2f(ld_u16(b));
        const int8_t *q = reinterpret_cast<const int8_t *>(b + 2 + (e0 % 32));
#pragma unroll
        for (int l = 0; l < 8; l++) y[l] = __fmul_rn(d, (float)q[l]);
        return;
    }
    case XJ_Q4_K: case XJ_Q5_K: {
        const int bb = type == XJ_Q4_K ? 144 : 176;
        const uint8_t *b = row + (size_t)(e0 / 256) * bb;
        const int w = e0 % 256, j = w / 32, l0 = w % 32;
        const float d = h2f(ld_u16(b)), dmin = h2f(ld_u16(b + 2));
        int s, m;
        k4_scale_min(j, b + 4, s, m);
        const float d1 = __fmul_rn(d, (float)s), m1 = __fmul_rn(dmin, (float)m);
        if (type == XJ_Q4_K) {
            uint2 v = *reinterpret_cast<const uint2 *>(b + 16 + 32 * (j / 2) + l0);
            const uint8_t *q = reinterpret_cast<const uint8_t *>(&v);
#pragma unroll
            for (int l = 0; l < 8; l++) {
                int qv = (j & 1) ? (q[l] >> 4) : (q[l] & 0xF);
                y[l] = __fsub_rn(__fmul_rn(d1, (float)qv), m1);
            }
        } else {
            uint2 vh = *reinterpret_cast<const uint2 *>(b + 16 + l0);
            uint2 vl = *reinterpret_cast<const uint2 *>(b + 48 + 32 * (j / 2) + l0);
            const uint8_t *qh = reinterpret_cast<const uint8_t *>(&vh);
            const uint8_t *ql = reinterpret_cast<const uint8_t *>(&vl);
#pragma unroll
            for (int l = 0; l < 8; l++) {
                int qv = ((j & 1) ? (ql[l] >> 4) : (ql[l] & 0xF)) + ((qh[l] >> j) & 1 ? 16 : 0);
                y[l] = __fsub_rn(__fmul_rn(d1, (float)qv), m1);
            }
        }
        return;
    }
    case XJ_Q6_K: {
        const uint8_t *b = row + (size_t)(e0 / 256) * 210;
        const int w = e0 % 256, h = w / 128, r = w % 128, part = r / 32, l0 = r % 32;
        const float d = h2f(ld_u16(b + 208));
        const uint8_t *ql = b + 64 * h + (part & 1) * 32 + l0;
        const uint8_t *qh = b + 128 + 32 * h + l0;
        const int8_t *sc = reinterpret_cast<const int8_t *>(b + 192 + 8 * h);
        const int shl = (part >> 1) * 4, shh = 2 * part;
        const float ds = __fmul_rn(d, (float)sc[l0 / 16 + 2 * part]);
#pragma unroll
        for (int l = 0; l < 8; l++) {
            int qv = (((ql[l] >> shl) & 0xF) | (((qh[l] >> shh) & 3) << 4)) - 32;
            y[l] = __fmul_rn(ds, (float)qv);
        }
        return;
    }
    default:
#pragma unroll
        for (int l = 0; l < 8; l++) y[l] = 0.0f;
    }
}
