// Tensor-core decode GEMV for Q4_K / Q6_K / Q8_0 weights: y[t][r] (+)= W[r] . f(x[t]), T <= 4 tokens.
//
// The arithmetic is the reference matmul (core/xj_cpu.c:36-54: dequantise, fp32 dot product) reorganised
// so the tensor cores do the multiply-adds without losing fp32 accuracy:
//
//   * weights enter the MMA as their exact small integer codes (Q4_K q in 0..15, Q6_K q-32 as
//     lo + 16*hi - 32, Q8_0 q in -127..127), which fp16 represents exactly;
//   * each activation is split into two fp16 values x = hi + lo (after an exact power-of-two range
//     scaling), so the pair carries ~22 mantissa bits; the two halves are separate MMA columns;
//   * the per-block scales (d*sc, dmin*m, d) multiply the fp32 MMA partial sums of each 16- or 32-wide
//     block, and the Q4_K "- dmin*m" term is applied once per block via the block sums of x.
//
// mma.sync.m16n8k16 (f16 inputs, f32 accumulate): A = 16 weight rows x 16 codes, B = 16 codes x 8
// columns where column n = 2*token + split. The weights are re-laid-out at upload ("tiled" layout, same
// byte count, bit-exact re-encoding of the GGUF blocks): for every 16-row tile the payload of each warp
// k-step is stored in the exact register order of the A fragment, and every (tile, unit) is contiguous.
//
// Streaming: at most one CTA per SM; each CTA owns a contiguous range of tiles and streams their
// weights through a ring of shared-memory stages filled by bulk asynchronous copies (cp.async.bulk with
// an mbarrier per stage; no multicast). The first stages are requested before griddepcontrol.wait, so
// under programmatic dependent launch a kernel's weight stream starts while its predecessor finishes;
// registers stay free, so the two kernels' CTAs fit on an SM together.
//
// Fused prologues f: RMSNorm (core/xj_cpu.c:56-61), SwiGLU silu(g)*u (:273). Fused epilogues:
// store, residual add (:268,275), causal conv + SiLU over the T tokens of each channel (:172-182, the
// GDN qkv rows), per-tile argmax partials of the LM head (core/xj_spec.c:12-16).
//
// Every token column is computed independently in a fixed order, so a token's result does not depend
// on how many other tokens share the launch (decode T=1 and speculative verify T>1 agree bit for bit).
#pragma once
#include <cmath>
#include <cstring>
#include <vector>

#include "kernels.cuh"

namespace xjk {

constexpr int MMA_MAXT = 4;
constexpr int MMA_WIDE_T = 16;    // tokens of a wide launch (k_gemv_wide: 4 n-tiles per decoded fragment)
constexpr int MMA_WARPS = 16;
constexpr int MMA_KMAX_PT = 12;   // prologue elements per thread: K <= 12 * 512

enum { PRO_NONE = 0, PRO_NORM = 1, PRO_SWIGLU = 2 };
enum { EPI_STORE = 0, EPI_ADD = 1, EPI_CONV = 2, EPI_ARGMAX = 3 };

// Tiled weight (see repack_tiled below).
struct Tiled {
    const uint8_t *q = nullptr;   // fragment-ordered codes (F16: the fp16 values)
    const uint8_t *h = nullptr;   // Q6_K high 2-bit planes, Q5_K high-bit plane
    const uint8_t *s = nullptr;   // per-row block headers (scales)
    const uint8_t *d = nullptr;   // Q6_K / Q8_0 fp16 d per row-block, F16 power-of-two row-block scales
    int type = 0, K = 0, N = 0;   // type: the tiled layout (Q4_K, Q5_K, Q6_K, Q8_0 or F16)
    int nu = 0;                   // units per row: K-quant super-blocks (K/256), Q8_0 / F16 blocks (K/32)
};

inline Tiled tiled_of(const DevMat &m) {
    Tiled t;
    t.q = m.tq; t.h = m.th; t.s = m.ts; t.d = m.td; t.K = m.K; t.N = m.N;
    t.type = m.type == XJ_BF16 ? XJ_F16 : m.type;   // BF16 is tiled as scaled fp16
    t.nu = t.type == XJ_Q8_0 || t.type == XJ_F16 ? m.K / 32 : m.K / 256;
    return t;
}
inline int tiled_type(int gguf_type) { return gguf_type == XJ_BF16 ? XJ_F16 : gguf_type; }

struct MmaJob {
    Tiled w;
    float *y;              // output rows (may be null for EPI_ARGMAX)
    long long ldy;
    int epi;
    // EPI_CONV: rows are conv channels; state [N][kc-1], weights [N][kc], checkpoints [T-1][N][kc-1]
    float *conv_state;
    const float *conv_w;
    float *conv_ck;
    int kc;
    long long conv_bstride;   // nonzero: token t is its own sequence, with its state at conv_state + t*conv_bstride
    // EPI_ARGMAX (T = 1): per-tile best value, runner-up value, best index
    float *pbest, *psecond;
    int *pidx;
};

struct MmaArgs {
    MmaJob job[4];
    int njob;
    int tile_start[5];     // prefix sums of 16-row tiles over jobs
    int tiles_per_cta;     // each CTA owns tiles [blockIdx.x * tiles_per_cta, ...)
    const float *x;        // input [T][K] (PRO_SWIGLU: gate values)
    const float *x2;       // PRO_SWIGLU: up values
    long long ldx;
    int T, K;
    int pro;
    const float *norm_w;   // PRO_NORM weights
    float eps;
    int *err;              // set to 1 when a wait for the weight stream gives up
};

// Bytes per unit in each tiled region, units per streamed chunk, ring depth.
template <int TYPE> struct Geo;
// A ring of ~54 KB per CTA keeps enough bytes in flight per SM for HBM bandwidth while leaving room
// for the next kernel's CTA on the same SM.
template <> struct Geo<XJ_Q4_K> { static constexpr int QB = 2048, HB = 0, SB = 256, DB = 0, CU = 8, STAGES = 3; };
template <> struct Geo<XJ_Q6_K> { static constexpr int QB = 2048, HB = 1024, SB = 256, DB = 32, CU = 8, STAGES = 2; };
template <> struct Geo<XJ_Q8_0> { static constexpr int QB = 512, HB = 0, SB = 0, DB = 32, CU = 32, STAGES = 3; };
// Q5_K: the low nibbles as Q4_K's, the high bits as a 1-bit plane, Q4_K's block headers
template <> struct Geo<XJ_Q5_K> { static constexpr int QB = 2048, HB = 512, SB = 256, DB = 0, CU = 8, STAGES = 2; };
// F16 and BF16 matrices as fp16 values in A-fragment order (16 rows x 32 elements per unit) with a
// power-of-two fp16 scale per row and 32-element block (1 for F16)
template <> struct Geo<XJ_F16> { static constexpr int QB = 1024, HB = 0, SB = 0, DB = 32, CU = 16, STAGES = 3; };
// K-quant units (256 elements per row, split over two warps) or 32-element units
template <int TYPE> constexpr bool kquant() { return TYPE == XJ_Q4_K || TYPE == XJ_Q5_K || TYPE == XJ_Q6_K; }
template <int TYPE> constexpr int unit_k() { return kquant<TYPE>() ? 256 : 32; }
template <int TYPE> constexpr int unit_bytes() { return Geo<TYPE>::QB + Geo<TYPE>::HB + Geo<TYPE>::SB + Geo<TYPE>::DB; }
template <int TYPE> constexpr int stage_bytes() { return Geo<TYPE>::CU * unit_bytes<TYPE>(); }

// ------------------------------------------------------------------ PTX helpers
XJ_DEV uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

XJ_DEV void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(bar)), "r"(count) : "memory");
}
XJ_DEV void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(smem_u32(bar)), "r"(bytes) : "memory");
}
XJ_DEV bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
                 : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}
// Bounded wait: gives up after a fixed number of polls (each poll may suspend the thread briefly),
// records the failure in *err and returns false instead of hanging.
XJ_DEV bool mbar_wait(uint64_t *bar, uint32_t parity, int *err) {
    for (int it = 0; it < (1 << 22); it++)
        if (mbar_try_wait(bar, parity)) return true;
    if (err) atomicExch(err, 1);
    return false;
}
XJ_DEV void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

XJ_DEV uint32_t lop3_and_or(uint32_t a, uint32_t mask, uint32_t magic) {
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(mask), "r"(magic));   // (a & b) | c
    return r;
}

XJ_DEV uint32_t hsub2(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("sub.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

XJ_DEV uint32_t hadd2(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("add.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

XJ_DEV uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}

XJ_DEV void mma16816(float *d, const uint32_t *a, uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Q4_K / Q6_K low nibbles of one k-step word -> exact fp16 codes in A-fragment order.
// Word bits: a0 at 0-3 / 16-19, a1 at 4-7 / 20-23, a2 at 8-11 / 24-27, a3 at 12-15 / 28-31.
XJ_DEV void nib_frag(uint32_t w, uint32_t *a) {
    const uint32_t w8 = w >> 8;
    a[0] = hsub2(lop3_and_or(w, 0x000F000Fu, 0x64006400u), 0x64006400u);    // 1024 + q - 1024
    a[1] = hsub2(lop3_and_or(w, 0x00F000F0u, 0x54005400u), 0x54005400u);    //   64 + q - 64
    a[2] = hsub2(lop3_and_or(w8, 0x000F000Fu, 0x64006400u), 0x64006400u);
    a[3] = hsub2(lop3_and_or(w8, 0x00F000F0u, 0x54005400u), 0x54005400u);
}

// Q6_K high 2-bit fields (bits 2r..2r+1 of each half of hw) -> 16*h - 32, exact in fp16.
XJ_DEV void hi_frag(uint32_t hw, uint32_t *a) {
    a[0] = hfma2(lop3_and_or(hw, 0x00030003u, 0x64006400u), 0x4C004C00u, 0xF402F402u);   // (1024+h)*16 - 16416
    a[1] = hfma2(lop3_and_or(hw, 0x000C000Cu, 0x5C005C00u), 0x4C004C00u, 0xEC08EC08u);   // ( 256+h)*16 -  4128
    a[2] = hfma2(lop3_and_or(hw, 0x00300030u, 0x54005400u), 0x4C004C00u, 0xE420E420u);   // (  64+h)*16 -  1056
    a[3] = hfma2(lop3_and_or(hw, 0x00C000C0u, 0x4C004C00u), 0x4C004C00u, 0xDC80DC80u);   // (  16+h)*16 -   288
}

// Q8_0 signed bytes [p0 p1 p2 p3] -> fp16 pairs (p0, p1) and (p2, p3), exact.
XJ_DEV void q8_frag(uint32_t w0, uint32_t w1, uint32_t *a) {
    const uint32_t u0 = w0 ^ 0x80808080u, u1 = w1 ^ 0x80808080u;                 // q + 128
    a[0] = hsub2(__byte_perm(u0, 0x64646464u, 0x4140), 0x64806480u);             // 1024 + 128 + q - 1152
    a[1] = hsub2(__byte_perm(u0, 0x64646464u, 0x4342), 0x64806480u);
    a[2] = hsub2(__byte_perm(u1, 0x64646464u, 0x4140), 0x64806480u);
    a[3] = hsub2(__byte_perm(u1, 0x64646464u, 0x4342), 0x64806480u);
}

XJ_DEV uint32_t word_of(const uint4 &v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }
XJ_DEV uint32_t byte_of(const uint4 &v, int i) { return (word_of(v, i >> 2) >> (8 * (i & 3))) & 0xffu; }

// Q4_K codes of one k-step word as fp16 (64 + q), exact; the constant 64 is removed through the
// block-sum term (d*sc*(D - 64*S) - dmin*m*S = d*sc*D - (64*d*sc + dmin*m)*S).
XJ_DEV void nib_frag64(uint32_t w, uint32_t *a) {
    a[0] = lop3_and_or(w << 4, 0x00F000F0u, 0x54005400u);
    a[1] = lop3_and_or(w, 0x00F000F0u, 0x54005400u);
    a[2] = lop3_and_or(w >> 4, 0x00F000F0u, 0x54005400u);
    a[3] = lop3_and_or(w >> 8, 0x00F000F0u, 0x54005400u);
}

// Q5_K codes of one k-step as fp16 (64 + q, q = low nibble + 16 * high bit), exact: the nibbles as
// nib_frag64, the high bit into mantissa bit 8 (weight 16 above 64). Word hw of the high-bit plane
// holds k-steps 4j .. 4j+3; k-step S = s & 3 keeps register r's bits at 4S + r (first half) and
// 16 + 4S + r (second half).
XJ_DEV void nib5_frag64(uint32_t w, uint32_t hw, int S, uint32_t *a) {   // S: a constant after unrolling
    nib_frag64(w, a);
#pragma unroll
    for (int r = 0; r < 4; r++) {
        const int sh = 8 - 4 * S - r;
        const uint32_t hb = sh >= 0 ? hw << sh : hw >> -sh;
        a[r] = lop3_and_or(hb, 0x01000100u, a[r]);
    }
}

// Position of column k (0..15) of a k-step in the staged activations: lane quad c finds columns
// 2c, 2c+1, 2c+8, 2c+9 (its two B-fragment registers) as 4 adjacent halves.
__host__ __device__ inline int bperm(int k) { return ((k & 7) >> 1) * 4 + (k >> 3) * 2 + (k & 1); }

// ------------------------------------------------------------------ one unit from a shared-memory stage
// Accumulate into (yg[n], yg8[n]) (rows g, g+8 of the tile, tokens 4n + c) unit ui of the staged chunk
// (global unit u of its tile) for up to 4*NT tokens: the A fragment is decoded once per k-step and
// multiplied with NT B fragments (8 columns each: tokens 4n..4n+3, hi and lo), so a token's result does
// not depend on NT or on the other tokens of the launch. K-quant units are shared by two warps: half hh
// takes k-steps 8hh..8hh+7. xb: this lane's B-fragment row of n-tile 0 (column g); the row of n-tile n
// is 8n columns further. xsum: 32-wide block sums [T][nblk] (Q4_K, Q5_K); scw: this warp's 128-float
// scale scratch.
template <int TYPE, int NT>
XJ_DEV void unit_compute_n(const uint8_t *stage, int ui, int u, int hh, int lane, int T, const __half *xb,
                           int xstride, const float *xsum, int nblk, float *scw, float (&yg)[NT], float (&yg8)[NT]) {
    using G = Geo<TYPE>;
    const int g = lane >> 2, c = lane & 3;
    const uint8_t *qs = stage + ui * G::QB;
    if constexpr (TYPE == XJ_Q4_K || TYPE == XJ_Q5_K) {
        const uint8_t *ss = stage + G::CU * (G::QB + G::HB) + ui * G::SB;
        const uint4 q0 = *reinterpret_cast<const uint4 *>(qs + ((2 * hh) * 32 + lane) * 16);
        const uint4 q1 = *reinterpret_cast<const uint4 *>(qs + ((2 * hh + 1) * 32 + lane) * 16);
        uint2 hq = make_uint2(0u, 0u);   // Q5_K: this half's two words of the lane's high-bit record
        if constexpr (TYPE == XJ_Q5_K) hq = *reinterpret_cast<const uint2 *>(stage + G::CU * G::QB + ui * G::HB + lane * 16 + hh * 8);
        {
            const int r = lane & 15;
            const uint4 hdr = *reinterpret_cast<const uint4 *>(ss + r * 16);
            const float d = h2f((uint16_t)(hdr.x & 0xffff)), dmin = h2f((uint16_t)(hdr.x >> 16));
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const int sbl = 2 * (lane >> 4) + e, sb = 4 * hh + sbl;
                int s_, m_;
                if (sb < 4) { s_ = byte_of(hdr, 4 + sb) & 63; m_ = byte_of(hdr, 8 + sb) & 63; }
                else {
                    s_ = (byte_of(hdr, 8 + sb) & 0xF) | ((byte_of(hdr, sb) >> 6) << 4);
                    m_ = (byte_of(hdr, 8 + sb) >> 4) | ((byte_of(hdr, 4 + sb) >> 6) << 4);
                }
                const float d1 = d * (float)s_, m1 = dmin * (float)m_;
                float *o = scw + ((sbl * 8 + (r & 7)) * 4 + (r >> 3) * 2);
                o[0] = d1;
                o[1] = 64.0f * d1 + m1;
            }
        }
        __syncwarp();
        const int kb = u * 256;
#pragma unroll
        for (int sbl = 0; sbl < 4; sbl++) {
            float d4[NT][4];
#pragma unroll
            for (int n = 0; n < NT; n++) { d4[n][0] = d4[n][1] = d4[n][2] = d4[n][3] = 0.0f; }
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const int s = 8 * hh + 2 * sbl + e;
                uint32_t af[4];
                const uint32_t wq = word_of(e + 2 * sbl < 4 ? q0 : q1, (2 * sbl + e) & 3);
                if constexpr (TYPE == XJ_Q5_K) nib5_frag64(wq, (2 * sbl + e) < 4 ? hq.x : hq.y, (2 * sbl + e) & 3, af);
                else nib_frag64(wq, af);
#pragma unroll
                for (int n = 0; n < NT; n++) {
                    uint2 bv = make_uint2(0u, 0u);
                    if (8 * n + g < 2 * T) bv = *reinterpret_cast<const uint2 *>(xb + (size_t)(8 * n) * xstride + kb + 16 * s);
                    mma16816(d4[n], af, bv.x, bv.y);
                }
            }
            const float4 sc4 = *reinterpret_cast<const float4 *>(scw + (sbl * 8 + g) * 4);
#pragma unroll
            for (int n = 0; n < NT; n++) {
                const int t = 4 * n + c;
                const float S = t < T ? xsum[t * nblk + (kb >> 5) + 4 * hh + sbl] : 0.0f;
                yg[n] = fmaf(sc4.x, d4[n][0] + d4[n][1], yg[n]);
                yg[n] = fmaf(-sc4.y, S, yg[n]);
                yg8[n] = fmaf(sc4.z, d4[n][2] + d4[n][3], yg8[n]);
                yg8[n] = fmaf(-sc4.w, S, yg8[n]);
            }
        }
        __syncwarp();
    } else if constexpr (TYPE == XJ_Q6_K) {
        const uint8_t *hs = stage + G::CU * G::QB + ui * G::HB;
        const uint8_t *ss = stage + G::CU * (G::QB + G::HB) + ui * G::SB;
        const uint8_t *ds = stage + G::CU * (G::QB + G::HB + G::SB) + ui * G::DB;
        const uint4 q0 = *reinterpret_cast<const uint4 *>(qs + ((2 * hh) * 32 + lane) * 16);
        const uint4 q1 = *reinterpret_cast<const uint4 *>(qs + ((2 * hh + 1) * 32 + lane) * 16);
        const uint4 hq = *reinterpret_cast<const uint4 *>(hs + (hh * 32 + lane) * 16);
        {
            const int r = lane & 15;
            const uint4 sc = *reinterpret_cast<const uint4 *>(ss + r * 16);
            const float d = h2f(*reinterpret_cast<const uint16_t *>(ds + r * 2));
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int sl = 4 * (lane >> 4) + e;
                scw[(sl * 8 + (r & 7)) * 2 + (r >> 3)] = d * (float)(int8_t)byte_of(sc, 8 * hh + sl);
            }
        }
        __syncwarp();
        const int kb = u * 256;
#pragma unroll
        for (int sl = 0; sl < 8; sl++) {
            const int s = 8 * hh + sl;
            uint32_t af[4], ah[4];
            nib_frag(word_of(sl < 4 ? q0 : q1, sl & 3), af);
            uint32_t hw = word_of(hq, sl >> 1);
            if (sl & 1) hw >>= 8;
            hi_frag(hw, ah);
            const float2 sc2 = *reinterpret_cast<const float2 *>(scw + (sl * 8 + g) * 2);
#pragma unroll
            for (int n = 0; n < NT; n++) {
                float d4[4] = {0.f, 0.f, 0.f, 0.f};
                uint2 bv = make_uint2(0u, 0u);
                if (8 * n + g < 2 * T) bv = *reinterpret_cast<const uint2 *>(xb + (size_t)(8 * n) * xstride + kb + 16 * s);
                mma16816(d4, af, bv.x, bv.y);
                mma16816(d4, ah, bv.x, bv.y);
                yg[n] = fmaf(sc2.x, d4[0] + d4[1], yg[n]);
                yg8[n] = fmaf(sc2.y, d4[2] + d4[3], yg8[n]);
            }
        }
        __syncwarp();
    } else if constexpr (TYPE == XJ_F16) {
        // the fp16 values are the A fragments; k-step e's 16 bytes of lane l at 512 e + 16 l
        const uint8_t *ds = stage + G::CU * G::QB + ui * G::DB;
        const uint4 q0 = *reinterpret_cast<const uint4 *>(qs + lane * 16);
        const uint4 q1 = *reinterpret_cast<const uint4 *>(qs + 512 + lane * 16);
        const float dv = lane < 16 ? h2f(*reinterpret_cast<const uint16_t *>(ds + lane * 2)) : 0.0f;
        const float dg = __shfl_sync(0xffffffffu, dv, g), dg8 = __shfl_sync(0xffffffffu, dv, g + 8);
        const int kb = u * 32;
        const uint32_t af[2][4] = {{q0.x, q0.y, q0.z, q0.w}, {q1.x, q1.y, q1.z, q1.w}};
#pragma unroll
        for (int n = 0; n < NT; n++) {
            float d4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int e = 0; e < 2; e++) {
                uint2 bv = make_uint2(0u, 0u);
                if (8 * n + g < 2 * T) bv = *reinterpret_cast<const uint2 *>(xb + (size_t)(8 * n) * xstride + kb + 16 * e);
                mma16816(d4, af[e], bv.x, bv.y);
            }
            yg[n] = fmaf(dg, d4[0] + d4[1], yg[n]);
            yg8[n] = fmaf(dg8, d4[2] + d4[3], yg8[n]);
        }
    } else {
        const uint8_t *ds = stage + G::CU * G::QB + ui * G::DB;
        const uint4 q = *reinterpret_cast<const uint4 *>(qs + lane * 16);
        const float dv = lane < 16 ? h2f(*reinterpret_cast<const uint16_t *>(ds + lane * 2)) : 0.0f;
        const float dg = __shfl_sync(0xffffffffu, dv, g), dg8 = __shfl_sync(0xffffffffu, dv, g + 8);
        const int kb = u * 32;
        uint32_t af[2][4];
#pragma unroll
        for (int e = 0; e < 2; e++) q8_frag(word_of(q, 2 * e), word_of(q, 2 * e + 1), af[e]);
#pragma unroll
        for (int n = 0; n < NT; n++) {
            float d4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int e = 0; e < 2; e++) {
                uint2 bv = make_uint2(0u, 0u);
                if (8 * n + g < 2 * T) bv = *reinterpret_cast<const uint2 *>(xb + (size_t)(8 * n) * xstride + kb + 16 * e);
                mma16816(d4, af[e], bv.x, bv.y);
            }
            yg[n] = fmaf(dg, d4[0] + d4[1], yg[n]);
            yg8[n] = fmaf(dg8, d4[2] + d4[3], yg8[n]);
        }
    }
}

// ------------------------------------------------------------------ shared-memory layout
struct MmaSmem {
    int T, K, xstride;        // halves per activation column (row of the staged B operand)
    size_t off_ring, off_xs, off_sum, off_sc, off_red, bytes;
    __host__ __device__ MmaSmem(int T_, int K_, int ring_bytes, int tmax = MMA_MAXT) : T(T_), K(K_) {
        xstride = K + 16;                                   // 16-half pad: conflict-free 8-byte B loads
        off_ring = 0;                                       // weight stages (16-byte aligned)
        off_xs = off_ring + (size_t)ring_bytes;
        off_sum = off_xs + (size_t)2 * T * xstride * 2;     // fp16 columns 2t (hi) and 2t+1 (lo)
        off_sum = (off_sum + 15) & ~(size_t)15;
        off_sc = off_sum + (size_t)T * (K / 32) * 4;        // fp32 sums of hi+lo per 32-wide block
        off_sc = (off_sc + 15) & ~(size_t)15;
        off_red = off_sc + (size_t)MMA_WARPS * 128 * 4;     // per-warp staged scales
        bytes = off_red + (size_t)MMA_WARPS * 16 * tmax * 4 + 64;
    }
};

// ------------------------------------------------------------------ kernel
template <int TYPE, int NT>
__global__ void __launch_bounds__(MMA_WARPS * 32, NT == 1 ? 2 : 1) k_gemv_mma(MmaArgs a) {
    using G = Geo<TYPE>;
    constexpr int SB = stage_bytes<TYPE>(), NS = G::STAGES, TMAX = 4 * NT;
    constexpr bool KQ = kquant<TYPE>();                  // K-quant units are split over two warps
    extern __shared__ __align__(128) uint8_t smem[];
    const MmaSmem L(a.T, a.K, SB * NS, TMAX);
    uint8_t *ring = smem + L.off_ring;
    __half *xs = reinterpret_cast<__half *>(smem + L.off_xs);
    float *xsum = reinterpret_cast<float *>(smem + L.off_sum);
    float *scs = reinterpret_cast<float *>(smem + L.off_sc);
    float *red = reinterpret_cast<float *>(smem + L.off_red);
    __shared__ __align__(8) uint64_t bars[NS];
    __shared__ float tok_scale[TMAX], tok_nsc[TMAX];
    __shared__ float pred[MMA_WARPS][2];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, c = lane & 3;
    const int T = a.T, K = a.K;
    const int total = a.tile_start[a.njob];
    const int ta = blockIdx.x * a.tiles_per_cta;
    const int tb = ta + a.tiles_per_cta < total ? ta + a.tiles_per_cta : total;
    const int nu = a.job[0].w.nu;                       // all jobs of a launch share K
    const int nch = (nu + G::CU - 1) / G::CU;           // chunks per tile
    const int nchunks = (tb - ta) * nch;

    // chunk i -> (job, tile within job, first unit, units)
    auto chunk_of = [&](int i, int &j, int &tile, int &u0, int &cu) {
        const int tg = ta + i / nch, ci = i % nch;
        j = 0;
        while (tg >= a.tile_start[j + 1]) j++;
        tile = tg - a.tile_start[j];
        u0 = ci * G::CU;
        cu = nu - u0 < G::CU ? nu - u0 : G::CU;
    };
    auto issue = [&](int i) {   // one thread: request chunk i into stage i % NS
        int j, tile, u0, cu;
        chunk_of(i, j, tile, u0, cu);
        const Tiled &W = a.job[j].w;
        uint8_t *st = ring + (size_t)(i % NS) * SB;
        uint64_t *bar = &bars[i % NS];
        const size_t tu0 = (size_t)tile * nu + u0;
        mbar_expect_tx(bar, (uint32_t)(cu * unit_bytes<TYPE>()));
        bulk_g2s(st, W.q + tu0 * G::QB, cu * G::QB, bar);
        if (G::HB) bulk_g2s(st + G::CU * G::QB, W.h + tu0 * G::HB, cu * G::HB, bar);
        if (G::SB) bulk_g2s(st + G::CU * (G::QB + G::HB), W.s + tu0 * G::SB, cu * G::SB, bar);
        if (G::DB) bulk_g2s(st + G::CU * (G::QB + G::HB + G::SB), W.d + tu0 * G::DB, cu * G::DB, bar);
    };

    // ---- 1. request the first stages of weights (independent of the producer kernel)
    if (tid == 0) {
        for (int s = 0; s < NS; s++) mbar_init(&bars[s], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (int i = 0; i < NS && i < nchunks; i++) issue(i);
    }
    griddep_launch();
    griddep_wait();

    // ---- 2. prologue: f(x) -> range scale -> fp16 hi/lo columns (+ Q4_K block sums); x read once
    constexpr int XPT = MMA_KMAX_PT;
    for (int t = 0; t < T; t++) {
        const float *xr = a.x + t * a.ldx;
        float v[XPT];
        float ss = 0.0f, am = 0.0f;
#pragma unroll
        for (int k = 0; k < XPT; k++) {
            const int i = tid + k * MMA_WARPS * 32;
            float val = 0.0f;
            if (i < K) {
                const float xv = xr[i];
                if (a.pro == PRO_NORM) { ss = fmaf(xv, xv, ss); val = xv * a.norm_w[i]; }
                else if (a.pro == PRO_SWIGLU) val = silu_f(xv) * a.x2[t * a.ldx + i];
                else val = xv;
                v[k] = a.pro == PRO_NORM ? xv : val;
            }
            am = fmaxf(am, fabsf(val));
        }
        ss = warp_sum(ss);
        am = warp_max(am);
        if (lane == 0) { pred[warp][0] = ss; pred[warp][1] = am; }
        __syncthreads();
        if (tid == 0) {
            double tss = 0;
            float tam = 0.0f;
            for (int w = 0; w < MMA_WARPS; w++) { tss += pred[w][0]; tam = fmaxf(tam, pred[w][1]); }
            float nsc = 1.0f;
            if (a.pro == PRO_NORM) nsc = 1.0f / sqrtf((float)(tss / K) + a.eps);
            // the largest |f(x)| lands in [2^14, 2^15): fp16 hi/lo stay finite with full relative precision
            const float m = tam * nsc;
            tok_nsc[t] = nsc;
            tok_scale[t] = ldexpf(1.0f, 14 - (m > 0.0f ? ilogbf(m) : 0));
        }
        __syncthreads();
        const float sc = tok_scale[t], nsc = tok_nsc[t];
        __half *col_hi = xs + (size_t)(2 * t) * L.xstride, *col_lo = xs + (size_t)(2 * t + 1) * L.xstride;
#pragma unroll
        for (int k = 0; k < XPT; k++) {
            const int i = tid + k * MMA_WARPS * 32;
            if (i < K) {
                // PRO_NORM: (x * nsc) * w as core/xj_cpu.c:60, then the exact power-of-two scale
                const float val = (a.pro == PRO_NORM ? (v[k] * nsc) * a.norm_w[i] : v[k]) * sc;
                const __half hi = __float2half_rn(val);
                const __half lo = __float2half_rn(val - __half2float(hi));
                const int pos = (i & ~15) + bperm(i & 15);
                col_hi[pos] = hi;
                col_lo[pos] = lo;
                if (TYPE == XJ_Q4_K || TYPE == XJ_Q5_K) {
                    // elements i..i+31 of a warp form one 32-wide block; sum what the MMA multiplies
                    const float bs = warp_sum(__half2float(hi) + __half2float(lo));
                    if (lane == 0) xsum[t * (K / 32) + (i >> 5)] = bs;
                }
            }
        }
    }
    __syncthreads();

    // ---- 3. stream the chunks: wait for the stage, compute, release, refill
    const __half *xb = xs + (size_t)g * L.xstride + 4 * c;
    float *scw = scs + warp * 128;
    float yg[NT], yg8[NT];
#pragma unroll
    for (int n = 0; n < NT; n++) { yg[n] = 0.0f; yg8[n] = 0.0f; }
    for (int i = 0; i < nchunks; i++) {
        int j, tile, u0, cu;
        chunk_of(i, j, tile, u0, cu);
        mbar_wait(&bars[i % NS], (uint32_t)((i / NS) & 1), a.err);
        const uint8_t *st = ring + (size_t)(i % NS) * SB;
        if (KQ) {
            const int ui = warp >> 1;
            if (ui < cu) unit_compute_n<TYPE, NT>(st, ui, u0 + ui, warp & 1, lane, T, xb, L.xstride, xsum, K / 32, scw, yg, yg8);
        } else {
#pragma unroll
            for (int k = 0; k < G::CU / MMA_WARPS; k++) {
                const int ui = warp + k * MMA_WARPS;
                if (ui < cu) unit_compute_n<TYPE, NT>(st, ui, u0 + ui, 0, lane, T, xb, L.xstride, xsum, K / 32, scw, yg, yg8);
            }
        }
        const bool tile_end = (i % nch) == nch - 1;
        if (tile_end) {
#pragma unroll
            for (int n = 0; n < NT; n++) {
                red[(warp * 16 + g) * TMAX + 4 * n + c] = yg[n];
                red[(warp * 16 + g + 8) * TMAX + 4 * n + c] = yg8[n];
                yg[n] = 0.0f; yg8[n] = 0.0f;
            }
        }
        __syncthreads();   // stage i % NS is free; red holds the tile's per-warp partials
        if (tid == 0 && i + NS < nchunks) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue(i + NS);
        }
        if (!tile_end) continue;
        // ---- 4. epilogue of the tile: fixed-order sum over warps
        const MmaJob &jb = a.job[j];
        if (jb.epi == EPI_CONV && jb.conv_bstride) {
            // batch of sequences: each token through its own sequence's conv state, no checkpoints
            if (tid < 16 && tile * 16 + tid < jb.w.N) {
                const int ch = tile * 16 + tid, kc = jb.kc;
                const float *wc = jb.conv_w + (size_t)ch * kc;
                for (int t = 0; t < T; t++) {
                    float *st = jb.conv_state + t * jb.conv_bstride + (size_t)ch * (kc - 1);
                    float cs[8];
                    for (int k = 0; k < kc - 1; k++) cs[k] = st[k];
                    float s = 0.0f;
#pragma unroll
                    for (int w = 0; w < MMA_WARPS; w++) s += red[(w * 16 + tid) * TMAX + t];
                    s /= tok_scale[t];
                    float acc = 0.0f;
                    for (int k = 0; k < kc - 1; k++) acc = fmaf(cs[k], wc[k], acc);
                    acc = fmaf(s, wc[kc - 1], acc);
                    for (int k = 0; k < kc - 2; k++) st[k] = cs[k + 1];
                    st[kc - 2] = s;
                    jb.y[t * jb.ldy + ch] = silu_f(acc);
                }
            }
        } else if (jb.epi == EPI_CONV) {
            // one thread per channel: the T tokens in order through the rolling conv state
            if (tid < 16 && tile * 16 + tid < jb.w.N) {
                const int ch = tile * 16 + tid, kc = jb.kc;
                float cs[8];
                for (int k = 0; k < kc - 1; k++) cs[k] = jb.conv_state[(size_t)ch * (kc - 1) + k];
                const float *wc = jb.conv_w + (size_t)ch * kc;
                for (int t = 0; t < T; t++) {
                    float s = 0.0f;
#pragma unroll
                    for (int w = 0; w < MMA_WARPS; w++) s += red[(w * 16 + tid) * TMAX + t];
                    s /= tok_scale[t];
                    float acc = 0.0f;
                    for (int k = 0; k < kc - 1; k++) acc = fmaf(cs[k], wc[k], acc);
                    acc = fmaf(s, wc[kc - 1], acc);
                    for (int k = 0; k < kc - 2; k++) cs[k] = cs[k + 1];
                    cs[kc - 2] = s;
                    jb.y[t * jb.ldy + ch] = silu_f(acc);
                    if (jb.conv_ck && t < T - 1)
                        for (int k = 0; k < kc - 1; k++) jb.conv_ck[((size_t)t * jb.w.N + ch) * (kc - 1) + k] = cs[k];
                }
                for (int k = 0; k < kc - 1; k++) jb.conv_state[(size_t)ch * (kc - 1) + k] = cs[k];
            }
        } else if (jb.epi == EPI_ARGMAX) {
            if (tid < 32) {
                const int row = tid & 15;
                float s = 0.0f;
#pragma unroll
                for (int w = 0; w < MMA_WARPS; w++) s += red[(w * 16 + row) * TMAX + 0];
                s /= tok_scale[0];
                const bool real = tile * 16 + row < jb.w.N;   // rows past N pad the last tile
                if (jb.y && tid < 16 && real) jb.y[(size_t)tile * 16 + row] = s;
                if (!real) s = -INFINITY;
                // best / runner-up / lowest index of the tile's 16 rows (lanes 16..31 mirror 0..15)
                float b = s, b2 = -INFINITY;
                int bi = tile * 16 + row;
#pragma unroll
                for (int o = 8; o; o >>= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, b, o), ov2 = __shfl_xor_sync(0xffffffffu, b2, o);
                    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                    if (ov > b || (ov == b && oi < bi)) { b2 = fmaxf(b, ov2); b = ov; bi = oi; }
                    else b2 = fmaxf(b2, ov);
                }
                if (tid == 0) { jb.pbest[tile] = b; jb.psecond[tile] = b2; jb.pidx[tile] = bi; }
            }
        } else if (tid < 16 * TMAX) {
            const int row = tid / TMAX, t = tid % TMAX;
            if (t < T && tile * 16 + row < jb.w.N) {
                float s = 0.0f;
#pragma unroll
                for (int w = 0; w < MMA_WARPS; w++) s += red[(w * 16 + row) * TMAX + t];
                s /= tok_scale[t];
                float *yp = jb.y + t * jb.ldy + (size_t)tile * 16 + row;
                *yp = jb.epi == EPI_ADD ? *yp + s : s;
            }
        }
        __syncthreads();   // red is reused by the next tile
    }
}

// ------------------------------------------------------------------ wide launches (5..16 tokens)
// Activations for a wide launch are prepared once per GEMV by k_prep_xt (one block per token, the same
// arithmetic as k_gemv_mma's prologue: identical hi/lo values, block sums and range scales) into a
// global buffer laid out as k_gemv_mma stages them: per token, columns hi and lo of xstride = K + 16
// halves (bperm order within each 16), then the 32-wide block sums, then the range scales.
struct WideX {
    __half *cols;        // [T][2][xstride]
    float *xsum;         // [T][sstride]: K/32 block sums, rows padded to 16 bytes (bulk-copy granularity)
    float *scale;        // [T]
    int sstride;
};
__host__ __device__ inline int wide_sstride(int K) { return (K / 32 + 3) & ~3; }
inline size_t wide_x_bytes(int T, int K) {
    return ((size_t)T * 2 * (K + 16) * 2 + 255) / 256 * 256 + ((size_t)T * wide_sstride(K) * 4 + 255) / 256 * 256 + 256;
}
__host__ __device__ inline WideX wide_x_of(void *buf, int T, int K) {
    WideX w;
    uint8_t *p = (uint8_t *)buf;
    w.cols = (__half *)p;
    p += ((size_t)T * 2 * (K + 16) * 2 + 255) / 256 * 256;
    w.xsum = (float *)p;
    w.sstride = wide_sstride(K);
    p += ((size_t)T * w.sstride * 4 + 255) / 256 * 256;
    w.scale = (float *)p;
    return w;
}

// Layout of a 64-token launch's activations (k_gemv_b64): K in chunks of B64_CK = 128; chunk c is one
// record: per token a row of B64_XROW bytes holding each element as the pair (hi, lo) of fp16 halves,
// each 16-element group as four 16-byte lane quads (quad c: elements 2c, 2c+1, 2c+8, 2c+9, the B
// fragments of two MMA k-steps), then the 32-wide block sums [4][64] (sub-block major); the T range
// scales follow the last record. One bulk copy moves a whole record into shared memory.
constexpr int B64_T = 64;           // tokens of one launch, at most
constexpr int B64_CK = 128;         // K per chunk: half a K-quant super-block, four Q8_0 blocks
constexpr int B64_XROW = B64_CK * 4 + 64;   // bytes per token row (the pad makes B-fragment loads conflict-free)
__host__ __device__ inline int b64_rec_bytes(int T) { return T * B64_XROW + 4 * B64_T * 4; }
inline size_t b64_x_bytes(int T, int K) { return (size_t)(K / B64_CK) * b64_rec_bytes(T) + (size_t)T * 4 + 256; }
// position (in halves) of element e (0..15) of a 16-element group in its 64-byte lane-quad layout
__host__ __device__ inline int b64_pos(int e) { return ((e & 7) >> 1) * 8 + ((e & 1) + 2 * (e >> 3)) * 2; }

// Layout of a tensor-core (tcgen05) launch's activations (k_gemm_tc, up to 64 tokens): K in chunks of
// 128; chunk c is one 36 KB record: two planes (hi, then lo), each [64 tokens][128 halves] in the
// core-matrix layout of a K-major MMA operand (8 x 8 blocks of 128 bytes, block (i, j) at byte
// (i * 16 + j) * 128), then per 64-wide half a block-sum plane [64 tokens][16 halves] (same layout):
// for the half's two 32-element blocks b, columns 3b, 3b+1, 3b+2 = (Sh, Sl, Sh) with Sh + Sl = 2^-6 *
// (the block's sum of hi + lo), columns 6..15 zero (the Q4_K minimum term as one MMA). The 64 range
// scales follow the last record.
constexpr int TC_T = 64, TC_CK = 128;
constexpr int TC_PLANE_X = TC_T * TC_CK * 2;
constexpr int TC_PLANE_S = TC_T * 16 * 2;            // one block-sum plane (2 KB)
constexpr int TC_REC = 2 * TC_PLANE_X + 2 * TC_PLANE_S;
inline size_t tc_x_bytes(int K) { return (size_t)(K / TC_CK) * TC_REC + TC_T * 4 + 256; }
// A forward of more than 64 tokens prepares all of them in one launch: token t goes to 64-token chunk
// t / 64, whose records start TC_XSTRIDE bytes after the previous chunk's (room for the longest row).
constexpr size_t TC_XSTRIDE = (((size_t)(MMA_KMAX_PT * MMA_WARPS * 32 / TC_CK) * TC_REC + TC_T * 4 + 256) + 1023) / 1024 * 1024;
__host__ __device__ inline uint32_t tc_xoff(int t, int k) {   // byte of (token t, element k) in a plane
    return (uint32_t)((((t >> 3) * (TC_CK >> 3) + (k >> 3)) << 7) + ((t & 7) << 4) + ((k & 7) << 1));
}
__host__ __device__ inline uint32_t tc_soff(int t, int k) {   // byte of (token t, column k < 16) in a block-sum plane
    return (uint32_t)((((t >> 3) * 2 + (k >> 3)) << 7) + ((t & 7) << 4) + ((k & 7) << 1));
}
enum { PREP_WIDE = 0, PREP_B64 = 1, PREP_TC = 2 };

// Grid T, MMA_WARPS*32 threads: f(x[t]) -> range scale -> hi/lo columns + block sums of token t, in the
// wide layout (PREP_WIDE), the 64-token chunk layout (PREP_B64) or the tensor-core operand layout
// (PREP_TC, no block sums; token t in 64-token chunk t / 64 at TC_XSTRIDE bytes per chunk); the values
// are the same.
template <int L>
static __global__ void __launch_bounds__(MMA_WARPS * 32) k_prep_xt(const float *x, const float *x2, long long ldx, int K, int pro,
                                                                   const float *norm_w, float eps, void *buf, int T) {
    griddep_wait();
    griddep_launch();   // successors may start their prologue; they wait for this grid before reading
    __shared__ float pred[MMA_WARPS][2];
    __shared__ float s_scale, s_nsc;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, t = blockIdx.x;
    const WideX W = wide_x_of(buf, T, K);
    uint8_t *tcb = (uint8_t *)buf + (size_t)(t / TC_T) * TC_XSTRIDE;   // PREP_TC: this token's chunk
    const int tt = t % TC_T;                                          // PREP_TC: its row in the chunk
    const int xstride = K + 16;
    constexpr int XPT = MMA_KMAX_PT;
    const float *xr = x + t * ldx;
    float v[XPT];
    float ss = 0.0f, am = 0.0f;
#pragma unroll
    for (int k = 0; k < XPT; k++) {
        const int i = tid + k * MMA_WARPS * 32;
        float val = 0.0f;
        if (i < K) {
            const float xv = xr[i];
            if (pro == PRO_NORM) { ss = fmaf(xv, xv, ss); val = xv * norm_w[i]; }
            else if (pro == PRO_SWIGLU) val = silu_f(xv) * x2[t * ldx + i];
            else val = xv;
            v[k] = pro == PRO_NORM ? xv : val;
        }
        am = fmaxf(am, fabsf(val));
    }
    ss = warp_sum(ss);
    am = warp_max(am);
    if (lane == 0) { pred[warp][0] = ss; pred[warp][1] = am; }
    __syncthreads();
    if (tid == 0) {
        double tss = 0;
        float tam = 0.0f;
        for (int w = 0; w < MMA_WARPS; w++) { tss += pred[w][0]; tam = fmaxf(tam, pred[w][1]); }
        float nsc = 1.0f;
        if (pro == PRO_NORM) nsc = 1.0f / sqrtf((float)(tss / K) + eps);
        const float m = tam * nsc;
        s_nsc = nsc;
        s_scale = ldexpf(1.0f, 14 - (m > 0.0f ? ilogbf(m) : 0));
        if (L == PREP_B64) reinterpret_cast<float *>((uint8_t *)buf + (size_t)(K / B64_CK) * b64_rec_bytes(T))[t] = s_scale;
        else if (L == PREP_TC) reinterpret_cast<float *>(tcb + (size_t)(K / TC_CK) * TC_REC)[tt] = s_scale;
        else W.scale[t] = s_scale;
    }
    __syncthreads();
    const float sc = s_scale, nsc = s_nsc;
    __half *col_hi = W.cols + (size_t)(2 * t) * xstride, *col_lo = W.cols + (size_t)(2 * t + 1) * xstride;
#pragma unroll
    for (int k = 0; k < XPT; k++) {
        const int i = tid + k * MMA_WARPS * 32;
        if (i < K) {
            const float val = (pro == PRO_NORM ? (v[k] * nsc) * norm_w[i] : v[k]) * sc;
            const __half hi = __float2half_rn(val);
            const __half lo = __float2half_rn(val - __half2float(hi));
            const float bs = warp_sum(__half2float(hi) + __half2float(lo));
            if (L == PREP_TC) {
                uint8_t *rec = tcb + (size_t)(i / TC_CK) * TC_REC;
                const int ci = i & (TC_CK - 1);
                const uint32_t o = tc_xoff(tt, ci);
                *reinterpret_cast<__half *>(rec + o) = hi;
                *reinterpret_cast<__half *>(rec + TC_PLANE_X + o) = lo;
                if (lane == 0) {   // this warp's 32 elements are one block: its scaled sum as (Sh, Sl, Sh)
                    uint8_t *sp = rec + 2 * TC_PLANE_X + (ci >> 6) * TC_PLANE_S;
                    const int b = (ci >> 5) & 1;
                    const float sv = bs * 0.015625f;
                    const __half sh = __float2half_rn(sv), sl = __float2half_rn(sv - __half2float(sh));
                    *reinterpret_cast<__half *>(sp + tc_soff(tt, 3 * b)) = sh;
                    *reinterpret_cast<__half *>(sp + tc_soff(tt, 3 * b + 1)) = sl;
                    *reinterpret_cast<__half *>(sp + tc_soff(tt, 3 * b + 2)) = sh;
                }
                continue;
            }
            if (L == PREP_B64) {
                const int ci = i & (B64_CK - 1);
                uint8_t *rec = (uint8_t *)buf + (size_t)(i / B64_CK) * b64_rec_bytes(T);
                __half *row = reinterpret_cast<__half *>(rec + (size_t)t * B64_XROW) + (ci & ~15) * 2 + b64_pos(ci & 15);
                *reinterpret_cast<__half2 *>(row) = __halves2half2(hi, lo);
                if (lane == 0) reinterpret_cast<float *>(rec + (size_t)T * B64_XROW)[(ci >> 5) * B64_T + t] = bs;
            } else {
                const int pos = (i & ~15) + bperm(i & 15);
                col_hi[pos] = hi;
                col_lo[pos] = lo;
                if (lane == 0) W.xsum[t * W.sstride + (i >> 5)] = bs;
            }
        }
    }
}

constexpr int WIDE_SLICE = 2048;          // largest K per staged activation slice (one chunk of units)
constexpr int WIDE_MAXTILES = 4;          // tiles a CTA may own when a tile spans several slices
struct WideSmem {
    size_t off_ring, off_xs, off_sum, off_sc, off_red, bytes;
    int xstride;
    __host__ __device__ WideSmem(int ring_bytes) {
        xstride = WIDE_SLICE + 16;
        off_ring = 0;
        off_xs = (size_t)ring_bytes;
        off_sum = off_xs + (size_t)2 * MMA_WIDE_T * xstride * 2;
        off_sc = off_sum + (size_t)MMA_WIDE_T * (WIDE_SLICE / 32) * 4;
        off_red = off_sc + (size_t)MMA_WARPS * 128 * 4;
        bytes = off_red + (size_t)MMA_WARPS * 16 * MMA_WIDE_T * 4 + 64;
    }
};

// 5..16 tokens: each CTA owns a contiguous range of tiles; the activations arrive one K-slice at a
// time (bulk copies of the prepared columns), the weights through the same chunk ring as k_gemv_mma in
// slice-major order; each tile's partial rows are carried across slices in registers, so a tile's
// arithmetic is k_gemv_mma's (same units in the same order per warp, same fixed-order epilogue).
template <int TYPE>
__global__ void __launch_bounds__(MMA_WARPS * 32, 1) k_gemv_wide(MmaArgs a, const void *xbuf) {
    using G = Geo<TYPE>;
    constexpr int SB = stage_bytes<TYPE>(), NS = G::STAGES, NT = MMA_WIDE_T / 4, TMAX = MMA_WIDE_T;
    constexpr bool KQ = kquant<TYPE>();
    constexpr int USL = G::CU;                                  // units per slice: one chunk
    constexpr int SLK = USL * unit_k<TYPE>();                   // K per slice
    static_assert(SLK <= WIDE_SLICE, "slice fits the staging area");
    extern __shared__ __align__(128) uint8_t smem[];
    const WideSmem L(SB * NS);
    uint8_t *ring = smem + L.off_ring;
    __half *xs = reinterpret_cast<__half *>(smem + L.off_xs);
    float *xsum = reinterpret_cast<float *>(smem + L.off_sum);
    float *scs = reinterpret_cast<float *>(smem + L.off_sc);
    float *red = reinterpret_cast<float *>(smem + L.off_red);
    __shared__ __align__(8) uint64_t bars[NS];
    __shared__ __align__(8) uint64_t xbar;
    __shared__ float tok_scale[TMAX];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, c = lane & 3;
    const int T = a.T, K = a.K;
    const WideX X = wide_x_of(const_cast<void *>(xbuf), T, K);
    const int total = a.tile_start[a.njob];
    const int ta = blockIdx.x * a.tiles_per_cta;
    const int tb = ta + a.tiles_per_cta < total ? ta + a.tiles_per_cta : total;
    const int ntl = tb - ta;
    const int nu = a.job[0].w.nu;
    const int nsl = (nu + USL - 1) / USL;                   // slices (chunks per tile)
    const int nchunks = ntl * nsl;
    // chunk i (slice-major: i = s * ntl + tile) -> (job, tile, first unit, units)
    auto chunk_of = [&](int i, int &j, int &tile, int &u0, int &cu) {
        const int s = i / ntl, tg = ta + i % ntl;
        j = 0;
        while (tg >= a.tile_start[j + 1]) j++;
        tile = tg - a.tile_start[j];
        u0 = s * USL;
        cu = nu - u0 < USL ? nu - u0 : USL;
    };
    auto issue = [&](int i) {
        int j, tile, u0, cu;
        chunk_of(i, j, tile, u0, cu);
        const Tiled &W = a.job[j].w;
        uint8_t *st = ring + (size_t)(i % NS) * SB;
        uint64_t *bar = &bars[i % NS];
        const size_t tu0 = (size_t)tile * nu + u0;
        mbar_expect_tx(bar, (uint32_t)(cu * unit_bytes<TYPE>()));
        bulk_g2s(st, W.q + tu0 * G::QB, cu * G::QB, bar);
        if (G::HB) bulk_g2s(st + G::CU * G::QB, W.h + tu0 * G::HB, cu * G::HB, bar);
        if (G::SB) bulk_g2s(st + G::CU * (G::QB + G::HB), W.s + tu0 * G::SB, cu * G::SB, bar);
        if (G::DB) bulk_g2s(st + G::CU * (G::QB + G::HB + G::SB), W.d + tu0 * G::DB, cu * G::DB, bar);
    };
    if (tid == 0) {
        for (int q = 0; q < NS; q++) mbar_init(&bars[q], 1);
        mbar_init(&xbar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (int i = 0; i < NS && i < nchunks; i++) issue(i);
    }
    griddep_launch();
    griddep_wait();
    if (tid < T) tok_scale[tid] = X.scale[tid];
    const __half *xb = xs + (size_t)g * L.xstride + 4 * c;
    float *scw = scs + warp * 128;
    float yg[WIDE_MAXTILES][NT], yg8[WIDE_MAXTILES][NT];
#pragma unroll
    for (int q = 0; q < WIDE_MAXTILES; q++)
#pragma unroll
        for (int n = 0; n < NT; n++) { yg[q][n] = 0.0f; yg8[q][n] = 0.0f; }
    for (int sl = 0; sl < nsl; sl++) {
        // ---- activation slice sl of every token (columns hi, lo; block sums)
        const int k0 = sl * SLK, kl = K - k0 < SLK ? K - k0 : SLK;
        __syncthreads();                                   // the previous slice is no longer read
        if (tid == 0) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            const int nb4 = ((kl / 32) + 3) & ~3;              // block sums copied, rounded up to 16 bytes
            mbar_expect_tx(&xbar, (uint32_t)(2 * T * kl * 2 + T * nb4 * 4));
            for (int col = 0; col < 2 * T; col++)
                bulk_g2s(xs + (size_t)col * L.xstride, X.cols + (size_t)col * (K + 16) + k0, kl * 2, &xbar);
            for (int t = 0; t < T; t++)
                bulk_g2s(xsum + t * (WIDE_SLICE / 32), X.xsum + (size_t)t * X.sstride + k0 / 32, nb4 * 4, &xbar);
        }
        mbar_wait(&xbar, (uint32_t)(sl & 1), a.err);
        for (int tl = 0; tl < ntl; tl++) {
            const int i = sl * ntl + tl;
            int j, tile, u0, cu;
            chunk_of(i, j, tile, u0, cu);
            mbar_wait(&bars[i % NS], (uint32_t)((i / NS) & 1), a.err);
            const uint8_t *st = ring + (size_t)(i % NS) * SB;
            float zg[NT], zg8[NT];
            const int q = nsl > 1 ? tl : 0;                 // carried accumulators when a tile spans slices
#pragma unroll
            for (int n = 0; n < NT; n++) { zg[n] = yg[q][n]; zg8[n] = yg8[q][n]; }
            if (KQ) {
                const int ui = warp >> 1;
                if (ui < cu) unit_compute_n<TYPE, NT>(st, ui, ui, warp & 1, lane, T, xb, L.xstride, xsum, WIDE_SLICE / 32, scw, zg, zg8);
            } else {
#pragma unroll
                for (int k = 0; k < G::CU / MMA_WARPS; k++) {
                    const int ui = warp + k * MMA_WARPS;
                    if (ui < cu) unit_compute_n<TYPE, NT>(st, ui, ui, 0, lane, T, xb, L.xstride, xsum, WIDE_SLICE / 32, scw, zg, zg8);
                }
            }
            __syncthreads();                               // the stage is free
            if (tid == 0 && i + NS < nchunks) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                issue(i + NS);
            }
            if (sl < nsl - 1) {
#pragma unroll
                for (int n = 0; n < NT; n++) { yg[q][n] = zg[n]; yg8[q][n] = zg8[n]; }
                continue;
            }
            // ---- last slice of the tile: fixed-order sum over warps, epilogue
#pragma unroll
            for (int n = 0; n < NT; n++) {
                red[(warp * 16 + g) * TMAX + 4 * n + c] = zg[n];
                red[(warp * 16 + g + 8) * TMAX + 4 * n + c] = zg8[n];
                yg[q][n] = 0.0f; yg8[q][n] = 0.0f;
            }
            __syncthreads();
            const MmaJob &jb = a.job[j];
            if (jb.epi == EPI_CONV && jb.conv_bstride) {
                if (tid < 16 && tile * 16 + tid < jb.w.N) {
                    const int ch = tile * 16 + tid, kc = jb.kc;
                    const float *wc = jb.conv_w + (size_t)ch * kc;
                    for (int t = 0; t < T; t++) {
                        float *stt = jb.conv_state + t * jb.conv_bstride + (size_t)ch * (kc - 1);
                        float cs[8];
                        for (int k = 0; k < kc - 1; k++) cs[k] = stt[k];
                        float sv = 0.0f;
#pragma unroll
                        for (int w = 0; w < MMA_WARPS; w++) sv += red[(w * 16 + tid) * TMAX + t];
                        sv /= tok_scale[t];
                        float acc = 0.0f;
                        for (int k = 0; k < kc - 1; k++) acc = fmaf(cs[k], wc[k], acc);
                        acc = fmaf(sv, wc[kc - 1], acc);
                        for (int k = 0; k < kc - 2; k++) stt[k] = cs[k + 1];
                        stt[kc - 2] = sv;
                        jb.y[t * jb.ldy + ch] = silu_f(acc);
                    }
                }
            } else if (jb.epi == EPI_CONV) {
                if (tid < 16 && tile * 16 + tid < jb.w.N) {
                    const int ch = tile * 16 + tid, kc = jb.kc;
                    float cs[8];
                    for (int k = 0; k < kc - 1; k++) cs[k] = jb.conv_state[(size_t)ch * (kc - 1) + k];
                    const float *wc = jb.conv_w + (size_t)ch * kc;
                    for (int t = 0; t < T; t++) {
                        float sv = 0.0f;
#pragma unroll
                        for (int w = 0; w < MMA_WARPS; w++) sv += red[(w * 16 + tid) * TMAX + t];
                        sv /= tok_scale[t];
                        float acc = 0.0f;
                        for (int k = 0; k < kc - 1; k++) acc = fmaf(cs[k], wc[k], acc);
                        acc = fmaf(sv, wc[kc - 1], acc);
                        for (int k = 0; k < kc - 2; k++) cs[k] = cs[k + 1];
                        cs[kc - 2] = sv;
                        jb.y[t * jb.ldy + ch] = silu_f(acc);
                        if (jb.conv_ck && t < T - 1)
                            for (int k = 0; k < kc - 1; k++) jb.conv_ck[((size_t)t * jb.w.N + ch) * (kc - 1) + k] = cs[k];
                    }
                    for (int k = 0; k < kc - 1; k++) jb.conv_state[(size_t)ch * (kc - 1) + k] = cs[k];
                }
            } else if (tid < 16 * TMAX) {
                const int row = tid / TMAX, t = tid % TMAX;
                if (t < T && tile * 16 + row < jb.w.N) {
                    float sv = 0.0f;
#pragma unroll
                    for (int w = 0; w < MMA_WARPS; w++) sv += red[(w * 16 + row) * TMAX + t];
                    sv /= tok_scale[t];
                    float *yp = jb.y + t * jb.ldy + (size_t)tile * 16 + row;
                    *yp = jb.epi == EPI_ADD ? *yp + sv : sv;
                }
            }
            __syncthreads();   // red is reused by the next tile
        }
    }
}


// ------------------------------------------------------------------ 64-token launches (batches of sequences)
// 17..64 independent tokens (one per sequence of a batch): the weights stream once per launch and every
// decoded A fragment feeds all 2T columns. A CTA of B64_WARPS warps owns a block of 16 row tiles (warp
// w: tiles w and w + 8, sharing each B fragment) and a range of K chunks; the chunk's activations (all
// tokens, one 128-wide K slice) and the 16 tiles' weights for it arrive together in one stage. When a
// block's K is split over several CTAs, those CTAs form one thread-block cluster: CTA r owns rows
// [r*256/ns, (r+1)*256/ns) of the block; every CTA stages its partial sums in its own shared memory and
// sends each owner its rows with one bulk copy into the owner's receive buffer (distributed shared
// memory, completion on the owner's mbarrier); CTA r then adds the ns partials in rank order and runs
// the epilogue, so the result is deterministic. Per block and split the
// arithmetic is unit_compute_n's (same fragments, same per-block scale terms); only the summation order
// over K differs from the 1..16-token kernels.
constexpr int B64_WARPS = 8;
constexpr int B64_TILES = 2 * B64_WARPS;          // row tiles per block
constexpr int B64_ROWS = 16 * B64_TILES;          // 256
constexpr int B64_RS = B64_T + 4;                 // partial-sum row stride (floats): rows stay 16-byte aligned
constexpr int B64_MAXSPLIT = 16;                  // CTAs per block: up to a (non-portable) 16-CTA cluster
constexpr int B64_RECV_ROWS = B64_ROWS + B64_MAXSPLIT;   // >= ns * ceil(256 / ns) for every ns <= B64_MAXSPLIT
template <int TYPE> struct B64Geo;                // weight bytes per tile and chunk, and their layout
template <> struct B64Geo<XJ_Q4_K> { static constexpr int Q = 1024, H = 0, S = 256, D = 0; };
template <> struct B64Geo<XJ_Q6_K> { static constexpr int Q = 1024, H = 512, S = 256, D = 32; };
template <> struct B64Geo<XJ_Q8_0> { static constexpr int Q = 2048, H = 0, S = 0, D = 128; };
template <int TYPE> constexpr int b64_wbytes() { return B64Geo<TYPE>::Q + B64Geo<TYPE>::H + B64Geo<TYPE>::S + B64Geo<TYPE>::D; }
constexpr int B64_ACT = B64_T * B64_XROW + 4 * B64_T * 4;       // largest activation record
template <int TYPE> constexpr int b64_stage() { return B64_ACT + B64_TILES * b64_wbytes<TYPE>(); }
constexpr int B64_STAGES = 2;
constexpr size_t B64_RECV = (size_t)B64_RECV_ROWS * B64_RS * 4;
template <int TYPE> constexpr size_t b64_smem() {
    return (size_t)B64_STAGES * b64_stage<TYPE>() + (size_t)B64_WARPS * 2 * 128 * 4 + B64_RECV;
}
static_assert(b64_smem<XJ_Q8_0>() <= 227 * 1024, "fits one SM");

struct B64Args {
    MmaJob job[4];
    int njob, T, K;
    int nsplit;            // CTAs per block (= cluster size), each a contiguous range of K chunks
    int blk_start[5];      // prefix sums of 256-row blocks over jobs
    const void *xbuf;      // activations in the 64-token chunk layout (k_prep_xt<PREP_B64>)
    int *err;
};

XJ_DEV uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
XJ_DEV void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
XJ_DEV void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
// Address of this CTA's shared variable p in the shared memory of cluster CTA `rank`.
XJ_DEV uint32_t peer_addr(const void *p, uint32_t rank) {
    uint32_t ra;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(smem_u32(p)), "r"(rank));
    return ra;
}
// Bulk copy of `bytes` (multiple of 16, both ends 16-byte aligned) from this CTA's shared memory into
// cluster CTA memory at dst (a peer address), completing on the peer's mbarrier at bar (peer address).
XJ_DEV void bulk_s2peer(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(dst), "r"(smem_u32(src)), "r"(bytes), "r"(bar) : "memory");
}

// D = A.B with C = 0 (the first k-step of a fresh accumulator).
XJ_DEV void mma16816_z(float *d, const uint32_t *a, uint32_t b0, uint32_t b1) {
    const float z = 0.0f;
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
                 : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(z));
}
// The A registers of the two hi/lo k-steps of one 16-wide fragment f (f[0..3] = rows g / g+8 at
// elements (2c, 2c+1) and (2c+8, 2c+9)): k-step s pairs K slots (2j, 2j+1) = (hi, lo) of one element,
// so each register holds that element's code twice.
XJ_DEV void b64_dup(const uint32_t *f, uint32_t (&a)[2][4]) {
    a[0][0] = __byte_perm(f[0], 0u, 0x1010); a[0][1] = __byte_perm(f[1], 0u, 0x1010);
    a[0][2] = __byte_perm(f[0], 0u, 0x3232); a[0][3] = __byte_perm(f[1], 0u, 0x3232);
    a[1][0] = __byte_perm(f[2], 0u, 0x1010); a[1][1] = __byte_perm(f[3], 0u, 0x1010);
    a[1][2] = __byte_perm(f[2], 0u, 0x3232); a[1][3] = __byte_perm(f[3], 0u, 0x3232);
}

// One chunk of this warp's NQ row tiles against the 8-token n-tiles. The K dimension of each MMA holds
// 8 elements as (hi, lo) pairs, so an accumulator sums code * (hi + lo) directly: per element group of
// 16, two k-steps whose B fragments come from one 16-byte load (see b64_pos). wst[q]: tile q's weights
// in the stage; xs: the stage's token rows; xsum: its block sums [4][64]; hh: which half of the
// super-block. Each per-block scale term is applied to the fresh accumulator of its block, as in
// unit_compute_n.
template <int TYPE, int NQ>
XJ_DEV void b64_chunk(const uint8_t *const *wst, int hh, int lane, int T, int ntl, const uint8_t *xs, const float *xsum,
                      float *scw, float (&y)[2][8][4]) {
    using BG = B64Geo<TYPE>;
    const int g = lane >> 2, c = lane & 3;
    const uint8_t *xb = xs + (size_t)g * B64_XROW + c * 16;      // this lane's quad of group 0, token g of n-tile 0
    if constexpr (TYPE == XJ_Q4_K) {
        uint4 q0[NQ], q1[NQ];
#pragma unroll
        for (int q = 0; q < NQ; q++) {
            q0[q] = *reinterpret_cast<const uint4 *>(wst[q] + lane * 16);
            q1[q] = *reinterpret_cast<const uint4 *>(wst[q] + (32 + lane) * 16);
            const int r = lane & 15;
            const uint4 hdr = *reinterpret_cast<const uint4 *>(wst[q] + BG::Q + r * 16);
            const float d = h2f((uint16_t)(hdr.x & 0xffff)), dmin = h2f((uint16_t)(hdr.x >> 16));
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const int sbl = 2 * (lane >> 4) + e, sb = 4 * hh + sbl;
                int s_, m_;
                if (sb < 4) { s_ = byte_of(hdr, 4 + sb) & 63; m_ = byte_of(hdr, 8 + sb) & 63; }
                else {
                    s_ = (byte_of(hdr, 8 + sb) & 0xF) | ((byte_of(hdr, sb) >> 6) << 4);
                    m_ = (byte_of(hdr, 8 + sb) >> 4) | ((byte_of(hdr, 4 + sb) >> 6) << 4);
                }
                const float d1 = d * (float)s_, m1 = dmin * (float)m_;
                float *o = scw + q * 128 + ((sbl * 8 + (r & 7)) * 4 + (r >> 3) * 2);
                o[0] = d1;
                o[1] = 64.0f * d1 + m1;
            }
        }
        __syncwarp();
#pragma unroll
        for (int sbl = 0; sbl < 4; sbl++) {
            uint32_t af[NQ][2][2][4];            // tile, 16-group, k-step
            float4 sc4[NQ];
#pragma unroll
            for (int q = 0; q < NQ; q++) {
#pragma unroll
                for (int e = 0; e < 2; e++) {
                    uint32_t f[4];
                    nib_frag64(word_of(e + 2 * sbl < 4 ? q0[q] : q1[q], (2 * sbl + e) & 3), f);
                    b64_dup(f, af[q][e]);
                }
                sc4[q] = *reinterpret_cast<const float4 *>(scw + q * 128 + (sbl * 8 + g) * 4);
            }
#pragma unroll
            for (int n = 0; n < 8; n++) {
                if (n < ntl) {
                    uint4 b[2] = {make_uint4(0u, 0u, 0u, 0u), make_uint4(0u, 0u, 0u, 0u)};
                    if (8 * n + g < T) {
                        b[0] = *reinterpret_cast<const uint4 *>(xb + (size_t)(8 * n) * B64_XROW + (2 * sbl) * 64);
                        b[1] = *reinterpret_cast<const uint4 *>(xb + (size_t)(8 * n) * B64_XROW + (2 * sbl + 1) * 64);
                    }
                    const float2 S = *reinterpret_cast<const float2 *>(xsum + sbl * B64_T + 8 * n + 2 * c);
#pragma unroll
                    for (int q = 0; q < NQ; q++) {
                        float d4[4];
                        mma16816_z(d4, af[q][0][0], b[0].x, b[0].y);
                        mma16816(d4, af[q][0][1], b[0].z, b[0].w);
                        mma16816(d4, af[q][1][0], b[1].x, b[1].y);
                        mma16816(d4, af[q][1][1], b[1].z, b[1].w);
                        y[q][n][0] = fmaf(sc4[q].x, d4[0], y[q][n][0]); y[q][n][0] = fmaf(-sc4[q].y, S.x, y[q][n][0]);
                        y[q][n][1] = fmaf(sc4[q].x, d4[1], y[q][n][1]); y[q][n][1] = fmaf(-sc4[q].y, S.y, y[q][n][1]);
                        y[q][n][2] = fmaf(sc4[q].z, d4[2], y[q][n][2]); y[q][n][2] = fmaf(-sc4[q].w, S.x, y[q][n][2]);
                        y[q][n][3] = fmaf(sc4[q].z, d4[3], y[q][n][3]); y[q][n][3] = fmaf(-sc4[q].w, S.y, y[q][n][3]);
                    }
                }
            }
        }
        __syncwarp();
    } else if constexpr (TYPE == XJ_Q6_K) {
        uint4 q0[NQ], q1[NQ], hq[NQ];
#pragma unroll
        for (int q = 0; q < NQ; q++) {
            q0[q] = *reinterpret_cast<const uint4 *>(wst[q] + lane * 16);
            q1[q] = *reinterpret_cast<const uint4 *>(wst[q] + (32 + lane) * 16);
            hq[q] = *reinterpret_cast<const uint4 *>(wst[q] + BG::Q + lane * 16);
            const int r = lane & 15;
            const uint4 sc = *reinterpret_cast<const uint4 *>(wst[q] + BG::Q + BG::H + r * 16);
            const float d = h2f(*reinterpret_cast<const uint16_t *>(wst[q] + BG::Q + BG::H + BG::S + r * 2));
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int sl = 4 * (lane >> 4) + e;
                scw[q * 128 + (sl * 8 + (r & 7)) * 2 + (r >> 3)] = d * (float)(int8_t)byte_of(sc, 8 * hh + sl);
            }
        }
        __syncwarp();
#pragma unroll
        for (int sl = 0; sl < 8; sl++) {
            uint32_t af[NQ][2][4];
            float2 sc2[NQ];
#pragma unroll
            for (int q = 0; q < NQ; q++) {
                // code q - 32 = low nibble + (16*high - 32), in [-32, 31]: the fp16 sum is exact
                uint32_t f[4], fh[4];
                nib_frag(word_of(sl < 4 ? q0[q] : q1[q], sl & 3), f);
                uint32_t hw = word_of(hq[q], sl >> 1);
                if (sl & 1) hw >>= 8;
                hi_frag(hw, fh);
#pragma unroll
                for (int k = 0; k < 4; k++) f[k] = hadd2(f[k], fh[k]);
                b64_dup(f, af[q]);
                sc2[q] = *reinterpret_cast<const float2 *>(scw + q * 128 + (sl * 8 + g) * 2);
            }
#pragma unroll
            for (int n = 0; n < 8; n++) {
                if (n < ntl) {
                    uint4 b = make_uint4(0u, 0u, 0u, 0u);
                    if (8 * n + g < T) b = *reinterpret_cast<const uint4 *>(xb + (size_t)(8 * n) * B64_XROW + sl * 64);
#pragma unroll
                    for (int q = 0; q < NQ; q++) {
                        float d4[4];
                        mma16816_z(d4, af[q][0], b.x, b.y);
                        mma16816(d4, af[q][1], b.z, b.w);
                        y[q][n][0] = fmaf(sc2[q].x, d4[0], y[q][n][0]);
                        y[q][n][1] = fmaf(sc2[q].x, d4[1], y[q][n][1]);
                        y[q][n][2] = fmaf(sc2[q].y, d4[2], y[q][n][2]);
                        y[q][n][3] = fmaf(sc2[q].y, d4[3], y[q][n][3]);
                    }
                }
            }
        }
        __syncwarp();
    } else {
#pragma unroll 1
        for (int ui = 0; ui < 4; ui++) {
            uint32_t af[NQ][2][2][4];
            float dg[NQ], dg8[NQ];
#pragma unroll
            for (int q = 0; q < NQ; q++) {
                const uint4 qv = *reinterpret_cast<const uint4 *>(wst[q] + ui * 512 + lane * 16);
                const float dv = lane < 16 ? h2f(*reinterpret_cast<const uint16_t *>(wst[q] + BG::Q + ui * 32 + lane * 2)) : 0.0f;
                dg[q] = __shfl_sync(0xffffffffu, dv, g);
                dg8[q] = __shfl_sync(0xffffffffu, dv, g + 8);
#pragma unroll
                for (int e = 0; e < 2; e++) {
                    uint32_t f[4];
                    q8_frag(word_of(qv, 2 * e), word_of(qv, 2 * e + 1), f);
                    b64_dup(f, af[q][e]);
                }
            }
#pragma unroll
            for (int n = 0; n < 8; n++) {
                if (n < ntl) {
                    uint4 b[2] = {make_uint4(0u, 0u, 0u, 0u), make_uint4(0u, 0u, 0u, 0u)};
                    if (8 * n + g < T) {
                        b[0] = *reinterpret_cast<const uint4 *>(xb + (size_t)(8 * n) * B64_XROW + (2 * ui) * 64);
                        b[1] = *reinterpret_cast<const uint4 *>(xb + (size_t)(8 * n) * B64_XROW + (2 * ui + 1) * 64);
                    }
#pragma unroll
                    for (int q = 0; q < NQ; q++) {
                        float d4[4];
                        mma16816_z(d4, af[q][0][0], b[0].x, b[0].y);
                        mma16816(d4, af[q][0][1], b[0].z, b[0].w);
                        mma16816(d4, af[q][1][0], b[1].x, b[1].y);
                        mma16816(d4, af[q][1][1], b[1].z, b[1].w);
                        y[q][n][0] = fmaf(dg[q], d4[0], y[q][n][0]);
                        y[q][n][1] = fmaf(dg[q], d4[1], y[q][n][1]);
                        y[q][n][2] = fmaf(dg8[q], d4[2], y[q][n][2]);
                        y[q][n][3] = fmaf(dg8[q], d4[3], y[q][n][3]);
                    }
                }
            }
        }
    }
}

template <int TYPE>
__global__ void __launch_bounds__(B64_WARPS * 32, 1) k_gemv_b64(B64Args a) {
    using BG = B64Geo<TYPE>;
    constexpr int WB = b64_wbytes<TYPE>(), SBY = b64_stage<TYPE>();
    constexpr bool KQ = TYPE != XJ_Q8_0;
    constexpr int NTH = B64_WARPS * 32;
    extern __shared__ __align__(128) uint8_t smem[];
    float *scs = reinterpret_cast<float *>(smem + (size_t)B64_STAGES * SBY);
    float *recv = scs + B64_WARPS * 2 * 128;               // [ns][ceil(256/ns)][B64_RS] partials of this CTA's rows
    __shared__ __align__(8) uint64_t bars[B64_STAGES];
    __shared__ __align__(8) uint64_t rbar;                  // partials of this CTA's rows from the other splits
    __shared__ float tok_inv[B64_T];                        // 1 / range scale (a power of two: exact)
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, c = lane & 3;
    const int T = a.T, K = a.K, ntl = (T + 7) / 8, ns = a.nsplit;
    const int blk = blockIdx.x / ns;
    const int split = ns > 1 ? (int)cluster_rank() : 0;       // = blockIdx.x % ns (1-D clusters of ns CTAs)
    int j = 0;
    while (blk >= a.blk_start[j + 1]) j++;
    const MmaJob &jb = a.job[j];
    const Tiled &W = jb.w;
    const int ntiles = (W.N + 15) / 16;
    const int t0 = (blk - a.blk_start[j]) * B64_TILES;
    const int nt = ntiles - t0 < B64_TILES ? ntiles - t0 : B64_TILES;
    const int nch = K / B64_CK;
    const int c0 = (int)((long long)split * nch / ns), c1 = (int)((long long)(split + 1) * nch / ns);
    const int nc = c1 - c0;
    const int nrmax = (B64_ROWS + ns - 1) / ns;
    const uint32_t act_bytes = (uint32_t)b64_rec_bytes(T);
    auto issue_w = [&](int i) {       // warp 0: weights of chunk c0 + i for the block's tiles into stage i % B64_STAGES,
        const int ch = c0 + i;         // one tile per lane (lane 0 also declares the stage's bytes)
        uint8_t *st = smem + (size_t)(i % B64_STAGES) * SBY + B64_ACT;
        uint64_t *bar = &bars[i % B64_STAGES];
        if (lane == 0) mbar_expect_tx(bar, act_bytes + (uint32_t)(nt * WB));
        __syncwarp();
        for (int tl = lane; tl < nt; tl += 32) {
            uint8_t *dst = st + tl * WB;
            const size_t tile = (size_t)(t0 + tl);
            if (KQ) {
                constexpr int QB = Geo<TYPE>::QB, HB = Geo<TYPE>::HB, SB = Geo<TYPE>::SB, DB = Geo<TYPE>::DB;
                const size_t tu = tile * W.nu + (ch >> 1);
                const int hh = ch & 1;
                bulk_g2s(dst, W.q + tu * QB + hh * (QB / 2), QB / 2, bar);
                if (HB) bulk_g2s(dst + BG::Q, W.h + tu * HB + hh * (HB / 2), HB / 2, bar);
                bulk_g2s(dst + BG::Q + BG::H, W.s + tu * SB, SB, bar);
                if (DB) bulk_g2s(dst + BG::Q + BG::H + BG::S, W.d + tu * DB, DB, bar);
            } else {
                const size_t tu = tile * W.nu + (size_t)ch * 4;
                bulk_g2s(dst, W.q + tu * Geo<TYPE>::QB, 4 * Geo<TYPE>::QB, bar);
                bulk_g2s(dst + BG::Q, W.d + tu * Geo<TYPE>::DB, 4 * Geo<TYPE>::DB, bar);
            }
        }
    };
    auto issue_x = [&](int i) {       // activation record of chunk c0 + i (after the predecessor finished)
        bulk_g2s(smem + (size_t)(i % B64_STAGES) * SBY, (const uint8_t *)a.xbuf + (size_t)(c0 + i) * act_bytes, act_bytes,
                 &bars[i % B64_STAGES]);
    };
    const int rb = split * B64_ROWS / ns, nr = (split + 1) * B64_ROWS / ns - rb;   // the rows this CTA finishes
    if (tid == 0) {
        for (int q = 0; q < B64_STAGES; q++) mbar_init(&bars[q], 1);
        mbar_init(&rbar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        if (ns > 1) mbar_expect_tx(&rbar, (uint32_t)((ns - 1) * nr * B64_RS * 4));
    }
    if (ns > 1) cluster_arrive();                          // every CTA's receive barrier is armed before any send
    if (warp == 0) {
        __syncwarp();
        for (int i = 0; i < B64_STAGES && i < nc; i++) issue_w(i);
    }
    griddep_launch();
    griddep_wait();
    if (tid == 0)
        for (int i = 0; i < B64_STAGES && i < nc; i++) issue_x(i);
    if (tid < T) tok_inv[tid] = 1.0f / reinterpret_cast<const float *>((const uint8_t *)a.xbuf + (size_t)nch * act_bytes)[tid];
    const int nq = (warp < nt) + (warp + B64_WARPS < nt);
    float y[2][8][4];                                      // tile q, n-tile n: rows g / g+8 x tokens 8n+2c, 8n+2c+1
#pragma unroll
    for (int q = 0; q < 2; q++)
#pragma unroll
        for (int n = 0; n < 8; n++) y[q][n][0] = y[q][n][1] = y[q][n][2] = y[q][n][3] = 0.0f;
    float *scw = scs + warp * 256;
    for (int i = 0; i < nc; i++) {
        const int slot = i % B64_STAGES;
        uint8_t *st = smem + (size_t)slot * SBY;
        mbar_wait(&bars[slot], (uint32_t)((i / B64_STAGES) & 1), a.err);
        const float *xsum = reinterpret_cast<const float *>(st + (size_t)T * B64_XROW);
        const uint8_t *wst[2] = {st + B64_ACT + warp * WB, st + B64_ACT + (warp + B64_WARPS) * WB};
        const int hh = (c0 + i) & 1;
        if (nq == 2) b64_chunk<TYPE, 2>(wst, hh, lane, T, ntl, st, xsum, scw, y);
        else if (nq == 1) b64_chunk<TYPE, 1>(wst, hh, lane, T, ntl, st, xsum, scw, y);
        __syncthreads();                                   // the stage is free
        if (warp == 0 && i + B64_STAGES < nc) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue_w(i + B64_STAGES);
            if (lane == 0) issue_x(i + B64_STAGES);
        }
    }
    // ---- partial sums of all 256 rows into this CTA's staging area (idle now), [row][B64_RS]
    float *part = reinterpret_cast<float *>(smem);
#pragma unroll
    for (int q = 0; q < 2; q++) {
        if (q < nq) {
#pragma unroll
            for (int h = 0; h < 2; h++) {
                float *dst = part + ((warp + q * B64_WARPS) * 16 + g + 8 * h) * B64_RS;
#pragma unroll
                for (int n = 0; n < 8; n++)
                    if (n < ntl) *reinterpret_cast<float2 *>(dst + 8 * n + 2 * c) = make_float2(y[q][n][2 * h], y[q][n][2 * h + 1]);
            }
        }
    }
    __syncthreads();
    if (ns > 1) {
        // each owner's rows to slot `split` of its receive buffer, one bulk copy per owner
        cluster_wait();                                    // the owners' receive barriers are armed
        if (tid < ns && tid != split) {
            const int o = tid, orb = o * B64_ROWS / ns, onr = (o + 1) * B64_ROWS / ns - orb;
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            bulk_s2peer(peer_addr(recv + (size_t)split * nrmax * B64_RS, (uint32_t)o), part + (size_t)orb * B64_RS,
                        (uint32_t)(onr * B64_RS * 4), peer_addr(&rbar, (uint32_t)o));
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
            asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");   // the source may be reused / freed
        }
        mbar_wait(&rbar, 0u, a.err);                       // every other split's partials of this CTA's rows
    }
    // ---- rows [rb, rb + nr): sum over splits in rank order, epilogue. Thread -> one row, every
    // tstep-th token (consecutive threads take consecutive rows).
    const int epi = jb.epi, ldy = (int)jb.ldy, kc = jb.kc;
    float *yb = jb.y;
    const int tstep = NTH / nr, rl = tid % nr, tt = tid / nr;
    const int row = rb + rl, ch = t0 * 16 + row;
    if (tt < tstep && ch < W.N) {
        const float *own = part + (size_t)row * B64_RS;
        const float *rcv = recv + (size_t)rl * B64_RS;
        auto total = [&](int t) {
            float sv = 0.0f;
#pragma unroll
            for (int r = 0; r < B64_MAXSPLIT; r++)
                if (r < ns) sv += r == split ? own[t] : rcv[(size_t)r * nrmax * B64_RS + t];
            return sv * tok_inv[t];
        };
        if (epi == EPI_CONV) {
            // kc <= 9 (b64_ok): fixed-size, predicated loops keep the state in registers
            float wc[9], wl = 0.0f;
#pragma unroll
            for (int k = 0; k < 9; k++) wc[k] = k < kc ? jb.conv_w[(size_t)ch * kc + k] : 0.0f;
#pragma unroll
            for (int k = 0; k < 9; k++)
                if (k == kc - 1) wl = wc[k];
            for (int t = tt; t < T; t += tstep) {
                float *stt = jb.conv_state + t * jb.conv_bstride + (size_t)ch * (kc - 1);
                float cs[8];
#pragma unroll
                for (int k = 0; k < 8; k++) cs[k] = k < kc - 1 ? stt[k] : 0.0f;
                const float v = total(t);
                float acc = 0.0f;
#pragma unroll
                for (int k = 0; k < 8; k++)
                    if (k < kc - 1) acc = fmaf(cs[k], wc[k], acc);
                acc = fmaf(v, wl, acc);
#pragma unroll
                for (int k = 0; k < 7; k++)
                    if (k < kc - 2) stt[k] = cs[k + 1];
                stt[kc - 2] = v;
                yb[(size_t)t * ldy + ch] = silu_f(acc);
            }
        } else if (epi == EPI_ADD) {
            constexpr int U = 4;
            for (int t0u = tt; t0u < T; t0u += U * tstep) {
                float yv[U];
#pragma unroll
                for (int u = 0; u < U; u++) {
                    const int t = t0u + u * tstep;
                    yv[u] = t < T ? yb[(size_t)t * ldy + ch] : 0.0f;
                }
#pragma unroll
                for (int u = 0; u < U; u++) {
                    const int t = t0u + u * tstep;
                    if (t < T) yb[(size_t)t * ldy + ch] = yv[u] + total(t);
                }
            }
        } else {
            for (int t = tt; t < T; t += tstep) yb[(size_t)t * ldy + ch] = total(t);
        }
    }
}

// ------------------------------------------------------------------ host: launch
constexpr size_t MMA_SMEM_MAX = 200 * 1024;              // 4-token launches
constexpr int MMA_KMAX = MMA_KMAX_PT * MMA_WARPS * 32;   // longest row the prologue stages

inline int ring_bytes(int type) {
    switch (type) {
    case XJ_Q4_K: return stage_bytes<XJ_Q4_K>() * Geo<XJ_Q4_K>::STAGES;
    case XJ_Q6_K: return stage_bytes<XJ_Q6_K>() * Geo<XJ_Q6_K>::STAGES;
    case XJ_Q5_K: return stage_bytes<XJ_Q5_K>() * Geo<XJ_Q5_K>::STAGES;
    case XJ_F16: case XJ_BF16: return stage_bytes<XJ_F16>() * Geo<XJ_F16>::STAGES;
    default: return stage_bytes<XJ_Q8_0>() * Geo<XJ_Q8_0>::STAGES;
    }
}
inline size_t mma_smem_bytes(int type, int T, int K, int tmax = MMA_MAXT) { return MmaSmem(T, K, ring_bytes(type), tmax).bytes; }



// Matrices the tensor-core path can take (at up to MMA_MAXT tokens).
inline bool tiled_ok(int type, int K, int N) {
    if (N < 1 || K > MMA_KMAX) return false;
    if (type == XJ_Q4_K || type == XJ_Q5_K || type == XJ_Q6_K) { if (K % 256) return false; }
    else if (type == XJ_Q8_0 || type == XJ_F16 || type == XJ_BF16) { if (K % 32) return false; }
    else return false;
    return mma_smem_bytes(type, MMA_MAXT, K) <= MMA_SMEM_MAX;
}

// Programmatic dependent launch: the kernel may start while its stream predecessor runs; it calls
// griddepcontrol.wait before touching anything the predecessor writes. g_pdl = 0 launches plainly.
inline int g_pdl = 1;
// CTAs per SM for the standalone kernel: two 16-warp CTAs hide the latency of the unit code's
// dependent chains (one CTA per SM measured 1.1-1.3 TB/s on large matrices, two 2.0-2.5 TB/s).
inline int g_mma_ctas_per_sm = 2;
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = g_pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

// Per-device, once: allow the kernel's dynamic shared memory; returns the SM count.
template <int TYPE, int NT>
inline int mma_setup() {
    constexpr int MAXDEV = 64;
    static int sms[MAXDEV] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= MAXDEV) dev = 0;
    if (!sms[dev]) {
        cudaFuncSetAttribute(k_gemv_mma<TYPE, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)MMA_SMEM_MAX);
        cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    }
    return sms[dev];
}

// One launch for up to 4 same-type matrices sharing the input x[T][K], T <= 4: up to
// g_mma_ctas_per_sm CTAs per SM, each owning a contiguous, balanced range of tiles.
template <int TYPE, int NT>
inline cudaError_t launch_mma_nt(MmaArgs a, cudaStream_t st) {
    const int sms = mma_setup<TYPE, NT>() * (NT == 1 ? g_mma_ctas_per_sm : 1);
    const int tiles = a.tile_start[a.njob];
    const int ctas = tiles < sms ? tiles : sms;
    a.tiles_per_cta = (tiles + ctas - 1) / ctas;
    const dim3 grid((tiles + a.tiles_per_cta - 1) / a.tiles_per_cta), block(MMA_WARPS * 32);
    return launch_pdl(k_gemv_mma<TYPE, NT>, grid, block, mma_smem_bytes(TYPE, a.T, a.K, 4 * NT), st, a);
}
template <int TYPE>
inline cudaError_t launch_mma_t(MmaArgs a, cudaStream_t st) {
    if (a.T <= MMA_MAXT) return launch_mma_nt<TYPE, 1>(a, st);
    return cudaErrorInvalidValue;   // 5..16 tokens: launch_wide
}

// Wide launch (5..16 tokens) on activations prepared by k_prep_xt into xbuf.
template <int TYPE>
inline cudaError_t launch_wide_t(MmaArgs a, const void *xbuf, cudaStream_t st) {
    constexpr int MAXDEV = 64;
    static int sms_dev[MAXDEV] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= MAXDEV) dev = 0;
    const size_t smem = WideSmem(ring_bytes(TYPE)).bytes;
    if (!sms_dev[dev]) {
        cudaFuncSetAttribute(k_gemv_wide<TYPE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        cudaDeviceGetAttribute(&sms_dev[dev], cudaDevAttrMultiProcessorCount, dev);
    }
    const int tiles = a.tile_start[a.njob];
    const int cu = Geo<TYPE>::CU, nsl = (a.job[0].w.nu + cu - 1) / cu;
    const int ctas = tiles < sms_dev[dev] ? tiles : sms_dev[dev];
    a.tiles_per_cta = (tiles + ctas - 1) / ctas;
    if (nsl > 1 && a.tiles_per_cta > WIDE_MAXTILES) a.tiles_per_cta = WIDE_MAXTILES;   // carried accumulators
    const dim3 grid((tiles + a.tiles_per_cta - 1) / a.tiles_per_cta), block(MMA_WARPS * 32);
    return launch_pdl(k_gemv_wide<TYPE>, grid, block, smem, st, a, xbuf);
}
// 64-token launch on activations prepared by k_prep_xt<PREP_B64> into a.xbuf. Blocks of 256 rows; when
// there are fewer blocks than SMs, each block's K chunks are split over a cluster of ns <= B64_MAXSPLIT
// CTAs, ns chosen (per device, type and block count) to minimise waves x chunks per CTA with the
// number of clusters that fit the GPU at once.
template <int TYPE>
inline cudaError_t launch_b64_t(B64Args a, cudaStream_t st) {
    constexpr int MAXDEV = 64;
    static int sms_dev[MAXDEV] = {0};
    static int occ[MAXDEV][B64_MAXSPLIT + 1] = {};      // clusters of ns CTAs resident at once
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= MAXDEV) dev = 0;
    constexpr size_t smem = b64_smem<TYPE>();
    if (!sms_dev[dev]) {
        cudaFuncSetAttribute(k_gemv_b64<TYPE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        cudaFuncSetAttribute(k_gemv_b64<TYPE>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        cudaDeviceGetAttribute(&sms_dev[dev], cudaDevAttrMultiProcessorCount, dev);
        occ[dev][1] = sms_dev[dev];
        for (int ns = 2; ns <= B64_MAXSPLIT; ns++) {
            cudaLaunchConfig_t q{};
            q.gridDim = dim3(ns * 64);
            q.blockDim = dim3(B64_WARPS * 32);
            q.dynamicSmemBytes = smem;
            cudaLaunchAttribute ca[1];
            ca[0].id = cudaLaunchAttributeClusterDimension;
            ca[0].val.clusterDim.x = (unsigned)ns;
            ca[0].val.clusterDim.y = 1;
            ca[0].val.clusterDim.z = 1;
            q.attrs = ca;
            q.numAttrs = 1;
            int n = 0;
            if (cudaOccupancyMaxActiveClusters(&n, k_gemv_b64<TYPE>, &q) != cudaSuccess) { cudaGetLastError(); n = 0; }
            occ[dev][ns] = n;
        }
    }
    a.blk_start[0] = 0;
    for (int j = 0; j < a.njob; j++) a.blk_start[j + 1] = a.blk_start[j] + ((a.job[j].w.N + 15) / 16 + B64_TILES - 1) / B64_TILES;
    const int nblk = a.blk_start[a.njob], nch = a.K / B64_CK;
    // cost in chunk times: waves x (chunks per CTA + ~2 for the start and the split exchange / epilogue)
    constexpr int FIXED = 2;
    int best = 1;
    long long best_cost = (long long)((nblk + occ[dev][1] - 1) / occ[dev][1]) * (nch + FIXED);
    for (int ns = 2; ns <= B64_MAXSPLIT && ns <= nch; ns++) {
        if (occ[dev][ns] < 1) continue;
        const long long cost = (long long)((nblk + occ[dev][ns] - 1) / occ[dev][ns]) * ((nch + ns - 1) / ns + FIXED);
        if (cost < best_cost) { best_cost = cost; best = ns; }
    }
    const int ns = best;
    a.nsplit = ns;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(nblk * ns);
    cfg.blockDim = dim3(B64_WARPS * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    int na = 0;
    if (g_pdl) {
        at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[na].val.programmaticStreamSerializationAllowed = 1;
        na++;
    }
    if (ns > 1) {
        at[na].id = cudaLaunchAttributeClusterDimension;
        at[na].val.clusterDim.x = (unsigned)ns;
        at[na].val.clusterDim.y = 1;
        at[na].val.clusterDim.z = 1;
        na++;
    }
    cfg.attrs = at;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, k_gemv_b64<TYPE>, a);
}
inline cudaError_t launch_b64(const B64Args &a, int type, cudaStream_t st) {
    switch (type) {
    case XJ_Q4_K: return launch_b64_t<XJ_Q4_K>(a, st);
    case XJ_Q6_K: return launch_b64_t<XJ_Q6_K>(a, st);
    case XJ_Q8_0: return launch_b64_t<XJ_Q8_0>(a, st);
    default: return cudaErrorInvalidValue;
    }
}
// Matrices and epilogues the 64-token kernel takes: tiled types with K a multiple of the chunk, and no
// epilogue that runs across tokens (the sequential conv of one sequence's prompt) or picks an argmax.
inline bool b64_ok(const MmaJob &j, int K) {
    if (K % B64_CK || K > MMA_KMAX_PT * MMA_WARPS * 32) return false;
    if (j.w.type != XJ_Q4_K && j.w.type != XJ_Q6_K && j.w.type != XJ_Q8_0) return false;
    if (j.epi == EPI_ARGMAX || (j.epi == EPI_CONV && (!j.conv_bstride || j.kc > 9 || j.conv_ck))) return false;
    return true;
}
inline cudaError_t launch_wide(const MmaArgs &a, int type, const void *xbuf, cudaStream_t st) {
    switch (type) {
    case XJ_Q4_K: return launch_wide_t<XJ_Q4_K>(a, xbuf, st);
    case XJ_Q6_K: return launch_wide_t<XJ_Q6_K>(a, xbuf, st);
    case XJ_Q8_0: return launch_wide_t<XJ_Q8_0>(a, xbuf, st);
    case XJ_Q5_K: return launch_wide_t<XJ_Q5_K>(a, xbuf, st);
    case XJ_F16: return launch_wide_t<XJ_F16>(a, xbuf, st);
    default: return cudaErrorInvalidValue;
    }
}

inline cudaError_t launch_mma(const MmaArgs &a, int type, cudaStream_t st) {
    switch (type) {
    case XJ_Q4_K: return launch_mma_t<XJ_Q4_K>(a, st);
    case XJ_Q6_K: return launch_mma_t<XJ_Q6_K>(a, st);
    case XJ_Q8_0: return launch_mma_t<XJ_Q8_0>(a, st);
    case XJ_Q5_K: return launch_mma_t<XJ_Q5_K>(a, st);
    case XJ_F16: return launch_mma_t<XJ_F16>(a, st);
    default: return cudaErrorInvalidValue;
    }
}

// ------------------------------------------------------------------ host: tiled re-encoding
// Host bytes of the tiled layout for an [N][K] GGUF matrix: q, h, s, d regions. The last tile is padded
// to 16 rows with all-zero blocks (scale 0: every padded row's product is exactly 0).
struct TiledHost {
    std::vector<uint8_t> q, h, s, d;
};

inline uint8_t q4k_code(const uint8_t *blk, int col) {   // Q4_K code of column col (0..255) of a super-block
    const int j = col / 32, l = col % 32;
    const uint8_t b = blk[16 + 32 * (j / 2) + l];
    return (j & 1) ? (b >> 4) : (b & 0xF);
}

inline uint8_t q5k_code(const uint8_t *blk, int col) {   // Q5_K code 0..31 (core/xj_quant.h layout)
    const int j = col / 32, l = col % 32;
    const uint8_t ql = blk[48 + 32 * (j / 2) + l];
    return (uint8_t)(((j & 1) ? (ql >> 4) : (ql & 0xF)) | (((blk[16 + l] >> j) & 1) << 4));
}

inline uint8_t q6k_code(const uint8_t *blk, int col) {   // Q6_K code 0..63 (value + 32)
    const int h = col / 128, r = col % 128, part = r / 32, l = r % 32;
    const uint8_t ql = blk[64 * h + (part & 1) * 32 + l], qh = blk[128 + 32 * h + l];
    return (uint8_t)(((ql >> ((part >> 1) * 4)) & 0xF) | (((qh >> (2 * part)) & 3) << 4));
}

// Column (0..15 within the k-step) / row (0..15 within the tile) of A-fragment register r, half e.
inline int frag_col(int r, int e, int c) { return 2 * c + e + 8 * (r >> 1); }
inline int frag_row(int r, int g) { return g + 8 * (r & 1); }

// F16 / BF16 row r, elements k0..k0+31 -> fp16 values and the block's power-of-two scale (fp16 bits);
// false when a BF16 block cannot be carried exactly (an element more than ~2^29 below the block's
// largest, a non-finite value, or a scale outside fp16).
inline bool h32_block(int type, const uint8_t *row, int k0, uint16_t *v, uint16_t *scale) {
    float f[32], m = 0.0f;
    for (int i = 0; i < 32; i++) {
        uint16_t u;
        memcpy(&u, row + 2 * (k0 + i), 2);
        if (type == XJ_F16) { v[i] = u; continue; }
        const uint32_t w = (uint32_t)u << 16;
        memcpy(&f[i], &w, 4);
        if (!std::isfinite(f[i])) return false;
        m = fabsf(f[i]) > m ? fabsf(f[i]) : m;
    }
    if (type == XJ_F16) { *scale = 0x3C00; return true; }
    const int e = m > 0.0f ? ilogbf(m) - 14 : 0;    // the largest lands in [2^14, 2^15)
    if (e < -24 || e > 15) return false;
    const float inv = ldexpf(1.0f, -e);
    for (int i = 0; i < 32; i++) {
        const float x = f[i] * inv;                 // exact: a power of two
        const __half h = __float2half_rn(x);
        if (__half2float(h) != x) return false;
        v[i] = __half_as_ushort(h);
    }
    *scale = __half_as_ushort(__float2half_rn(ldexpf(1.0f, e)));
    return true;
}

// Re-encodes an [N][K] GGUF matrix into the tiled layout of its type; false if the matrix cannot be
// carried exactly (BF16 only), in which case it stays row-major.
inline bool repack_tiled(int type, const uint8_t *src_rows, int K, int N, TiledHost &o) {
    const int tiles = (N + 15) / 16;
    const bool kq = type == XJ_Q4_K || type == XJ_Q5_K || type == XJ_Q6_K;
    const int bb = type == XJ_Q4_K ? 144 : type == XJ_Q5_K ? 176 : 210;
    const size_t rb0 = type == XJ_Q8_0 ? (size_t)(K / 32) * 34 : kq ? (size_t)(K / 256) * bb : (size_t)K * 2;
    std::vector<uint8_t> padded;
    const uint8_t *src = src_rows;
    if (N % 16) {
        padded.assign((size_t)tiles * 16 * rb0, 0);
        memcpy(padded.data(), src_rows, (size_t)N * rb0);
        src = padded.data();
    }
    if (kq) {
        const int nu = K / 256;
        const size_t rb = (size_t)nu * bb;
        o.q.assign((size_t)tiles * nu * 2048, 0);
        o.s.assign((size_t)tiles * nu * 16 * 16, 0);
        if (type == XJ_Q6_K) { o.h.assign((size_t)tiles * nu * 1024, 0); o.d.assign((size_t)tiles * nu * 16 * 2, 0); }
        if (type == XJ_Q5_K) o.h.assign((size_t)tiles * nu * 512, 0);
        for (int t = 0; t < tiles; t++)
            for (int u = 0; u < nu; u++) {
                const size_t tu = (size_t)t * nu + u;
                const uint8_t *blk[16];
                for (int i = 0; i < 16; i++) blk[i] = src + (size_t)(16 * t + i) * rb + (size_t)u * bb;
                for (int i = 0; i < 16; i++) {
                    if (type != XJ_Q6_K) memcpy(&o.s[(tu * 16 + i) * 16], blk[i], 16);   // d, dmin, scales
                    else { memcpy(&o.s[(tu * 16 + i) * 16], blk[i] + 192, 16); memcpy(&o.d[(tu * 16 + i) * 2], blk[i] + 208, 2); }
                }
                for (int lane = 0; lane < 32; lane++) {
                    const int g = lane >> 2, c = lane & 3;
                    uint32_t h5[4] = {0, 0, 0, 0};   // Q5_K: the lane's high-bit record, 4 k-steps per word
                    for (int s = 0; s < 16; s++) {
                        uint32_t w = 0, hw = 0;
                        for (int r = 0; r < 4; r++)
                            for (int e = 0; e < 2; e++) {
                                const int row = frag_row(r, g), col = 16 * s + frag_col(r, e, c);
                                const uint8_t code = type == XJ_Q4_K ? q4k_code(blk[row], col)
                                                   : type == XJ_Q5_K ? q5k_code(blk[row], col) : q6k_code(blk[row], col);
                                w |= (uint32_t)(code & 0xF) << (4 * r + 16 * e);
                                hw |= (uint32_t)(code >> 4) << (2 * r + 16 * e);
                                if (type == XJ_Q5_K) h5[s >> 2] |= (uint32_t)(code >> 4) << (16 * e + 4 * (s & 3) + r);
                            }
                        memcpy(&o.q[((tu * 4 + s / 4) * 32 + lane) * 16 + (s % 4) * 4], &w, 4);
                        if (type == XJ_Q6_K) {
                            // two k-steps share one word: odd k-step in the upper byte of each half
                            uint32_t cur;
                            uint8_t *p = &o.h[((tu * 2 + s / 8) * 32 + lane) * 16 + ((s / 2) % 4) * 4];
                            memcpy(&cur, p, 4);
                            cur |= hw << ((s & 1) * 8);
                            memcpy(p, &cur, 4);
                        }
                    }
                    if (type == XJ_Q5_K) memcpy(&o.h[(tu * 32 + lane) * 16], h5, 16);
                }
            }
    } else if (type == XJ_Q8_0) {
        const int nu = K / 32;
        const size_t rb = (size_t)nu * 34;
        o.q.assign((size_t)tiles * nu * 512, 0);
        o.d.assign((size_t)tiles * nu * 16 * 2, 0);
        for (int t = 0; t < tiles; t++)
            for (int u = 0; u < nu; u++) {
                const size_t tu = (size_t)t * nu + u;
                for (int i = 0; i < 16; i++) memcpy(&o.d[(tu * 16 + i) * 2], src + (size_t)(16 * t + i) * rb + (size_t)u * 34, 2);
                for (int lane = 0; lane < 32; lane++) {
                    const int g = lane >> 2, c = lane & 3;
                    uint8_t out[16];
                    for (int ss = 0; ss < 2; ss++)
                        for (int hw = 0; hw < 2; hw++)        // word: hw=0 -> a0,a1 ; hw=1 -> a2,a3
                            for (int b = 0; b < 4; b++) {     // byte b: (r = 2*hw + b/2, e = b%2)
                                const int r = 2 * hw + b / 2, e = b % 2;
                                const int row = frag_row(r, g), col = 16 * ss + frag_col(r, e, c);
                                out[ss * 8 + hw * 4 + b] = src[(size_t)(16 * t + row) * rb + (size_t)u * 34 + 2 + col];
                            }
                    memcpy(&o.q[(tu * 32 + lane) * 16], out, 16);
                }
            }
    } else {   // F16 / BF16: fp16 values in fragment order, k-step ss of lane l at 512 ss + 16 l
        const int nu = K / 32;
        const size_t rb = (size_t)K * 2;
        o.q.assign((size_t)tiles * nu * 1024, 0);
        o.d.assign((size_t)tiles * nu * 16 * 2, 0);
        uint16_t v[16][32];
        for (int t = 0; t < tiles; t++)
            for (int u = 0; u < nu; u++) {
                const size_t tu = (size_t)t * nu + u;
                for (int i = 0; i < 16; i++) {
                    uint16_t sc;
                    if (!h32_block(type, src + (size_t)(16 * t + i) * rb, 32 * u, v[i], &sc)) return false;
                    memcpy(&o.d[(tu * 16 + i) * 2], &sc, 2);
                }
                for (int lane = 0; lane < 32; lane++) {
                    const int g = lane >> 2, c = lane & 3;
                    for (int ss = 0; ss < 2; ss++)
                        for (int r = 0; r < 4; r++)
                            for (int e = 0; e < 2; e++) {
                                const int row = frag_row(r, g), col = 16 * ss + frag_col(r, e, c);
                                memcpy(&o.q[tu * 1024 + ss * 512 + lane * 16 + r * 4 + e * 2], &v[row][col], 2);
                            }
                }
            }
    }
    return true;
}

}  // namespace xjk
