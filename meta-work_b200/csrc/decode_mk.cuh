// Persistent decode kernel: every greedy decode step of the whole model (all layers, the LM head and
// the token pick) for any number of steps in ONE cooperative launch.
//
// A decode step at batch 1 is ~150 dependent phases (matrix-vector products, the Gated DeltaNet
// update, attention, the argmax), each of which moves only a few MB. Launched as separate kernels every
// phase pays launch latency and an empty weight pipeline; here one CTA per SM runs the phase program
// in a loop and the phases are separated by a grid barrier instead (a counter in global memory; every
// wait bounded).
//
// Each CTA has 16 consumer warps and one producer warp. The producer walks the same phase program and,
// for every matrix-vector phase, requests this CTA's weight chunks into a shared-memory ring with bulk
// asynchronous copies (one mbarrier per slot for "full", one for "empty"; no multicast). Weights do not
// depend on activations, so the producer runs ahead of the consumers across phase boundaries and the
// grid barriers: the HBM stream of the next phases overlaps the barrier and the small phases.
//
// Phases (one decode step, core/xj_cpu.c:161-291 for the layer math):
//   GEMV   y_j (+)= W_j . f(x) for up to 4 matrices sharing x (the tensor-core unit code of
//          gemv_mma.cuh; f = identity, RMSNorm, SwiGLU, or the Gated DeltaNet output norm); 16-row
//          tiles are dealt to CTAs round-robin; epilogues store, add, causal conv + SiLU, argmax partials
//   GDN    the delta-rule state update of 16 (S=128) value rows of one head per work item, so 128 CTAs
//          share the 16 heads; the per-head gated RMSNorm moves into the next GEMV's prologue
//   ATTN   q/k RMSNorm + RoPE, the new K/V row, and attention over one split of the positions per work
//          item; the last split of a head to finish merges the splits (counter + fence, no barrier)
//   ARGMAX the greedy pick from the LM head's tile partials, the next token's embedding, position + 1
//
// Matrix-vector products give the same bits as the standalone tensor-core kernel (same unit order,
// same prologue arithmetic, same fixed-order reductions). GDN and attention sum in a different order
// than the standalone kernels (more threads per row and per head), within float rounding.
#pragma once
#include "gemv_mma.cuh"

namespace xjk {

constexpr int MK_CWARPS = 16;                    // consumer warps
constexpr int MK_CTHREADS = MK_CWARPS * 32;      // 512
constexpr int MK_THREADS = MK_CTHREADS + 32;     // + the producer warp
constexpr int MK_SLOT = 26880;                   // largest chunk: 8 Q6_K units
constexpr int MK_NS = 6;                         // ring slots
constexpr int MK_KMAX = MMA_KMAX_PT * MK_CTHREADS;
constexpr int MK_XS_BYTES = 2 * (MK_KMAX + 16) * 2;   // hi/lo fp16 columns (also GDN / attention scratch)
using BarC = BarNamed<1, MK_CTHREADS>;           // the consumer warps only

enum { MK_GEMV = 0, MK_GDN = 1, MK_ATTN = 2, MK_ARGMAX = 3 };
enum { PRO_GNORM = 3 };                          // per-head RMSNorm(ssm_norm) * silu(z), core/xj_cpu.c:218-224

struct MkPhase {
    int op;
    // MK_GEMV
    int njob, ntiles;
    int tile_start[5];
    int K, pro, gs;              // gs: PRO_GNORM head size
    const float *x, *x2;         // input; SwiGLU up values or the GNORM gate z
    const float *norm_w;
    float eps;
    MmaJob job[4];
    // MK_GDN / MK_ATTN / MK_ARGMAX
    GdnArgs gdn;
    AttnArgs attn;
    ArgmaxArgs am;
};

struct MkArgs {
    const MkPhase *prog;
    int nphase, nsteps;
    unsigned *bar;               // grid barrier counter, zero at launch
    int *err;                    // 1: weight stream wait gave up, 2: grid barrier wait gave up
    float *apart;                // attention split partials [H][max_split][D + 2]
    int *acnt;                   // per-head split counters, zero at launch
    int max_split;
    int kv_f32;
};

constexpr size_t MK_SMEM = (size_t)MK_NS * MK_SLOT + MK_XS_BYTES + (MK_KMAX / 32) * 4 + MK_CWARPS * 128 * 4 +
                           2 * MK_CWARPS * 16 * 4;

XJ_DEV unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
XJ_DEV unsigned ld_acquire(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
XJ_DEV int ld_volatile(const int *p) { return *(const volatile int *)p; }
// Bounded wait that ignores the grid's error word (used to let copies in flight land before exit).
XJ_DEV bool mk_wait_drain(uint64_t *bar, uint32_t parity) {
    const unsigned long long t0 = globaltimer();
    for (int it = 0; it < (1 << 24); it++) {
        if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer() - t0 > 100000000ull) break;
    }
    return false;
}
XJ_DEV void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(smem_u32(bar)) : "memory");
}

constexpr unsigned long long MK_WAIT_NS = 2000000000ull;   // 2 s: no legitimate wait comes near it

// Wait for an mbarrier phase; gives up (recording `code`) after MK_WAIT_NS (or 2^30 polls, should the
// clock not advance) or as soon as another part of the grid has recorded an error.
XJ_DEV bool mk_wait(uint64_t *bar, uint32_t parity, int *err, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = globaltimer();
    for (int it = 0; it < (1 << 24); it++) {
        for (int i = 0; i < 64; i++)
            if (mbar_try_wait(bar, parity)) return true;
        if (ld_volatile(err)) return false;
        if (globaltimer() - t0 > MK_WAIT_NS) break;
    }
    atomicExch(err, code);
    return false;
}

// All consumer threads of all CTAs: returns false (uniformly) when the grid records an error.
XJ_DEV bool mk_grid_sync(unsigned *bar, unsigned target, int *err, int tid) {
    __shared__ int s_ok;
    BarC::sync();
    if (tid == 0) {
        __threadfence();
        atomicAdd(bar, 1u);
        int ok = 1;
        const unsigned long long t0 = globaltimer();
        for (int it = 0; ld_acquire(bar) < target; it++) {
            if (ld_volatile(err)) { ok = 0; break; }
            if (globaltimer() - t0 > MK_WAIT_NS || it > (1 << 27)) { atomicExch(err, 2); ok = 0; break; }
            __nanosleep(20);
        }
        __threadfence();
        if (ok && ld_volatile(err)) ok = 0;
        s_ok = ok;
    }
    BarC::sync();
    return s_ok != 0;
}

// ------------------------------------------------------------------ matrix-vector phases
XJ_DEV int mk_cu(int type) { return type == XJ_Q4_K ? Geo<XJ_Q4_K>::CU : type == XJ_Q6_K ? Geo<XJ_Q6_K>::CU : Geo<XJ_Q8_0>::CU; }
XJ_DEV int mk_job_of(const MkPhase &p, int tg) {
    int j = 0;
    while (j + 1 < p.njob && tg >= p.tile_start[j + 1]) j++;
    return j;
}

template <int TYPE>
XJ_DEV void mk_issue_t(const Tiled &W, int tile, int u0, int cu, uint8_t *st, uint64_t *bar) {
    using G = Geo<TYPE>;
    const size_t tu0 = (size_t)tile * W.nu + u0;
    mbar_expect_tx(bar, (uint32_t)(cu * unit_bytes<TYPE>()));
    bulk_g2s(st, W.q + tu0 * G::QB, cu * G::QB, bar);
    if (G::HB) bulk_g2s(st + G::CU * G::QB, W.h + tu0 * G::HB, cu * G::HB, bar);
    if (G::SB) bulk_g2s(st + G::CU * (G::QB + G::HB), W.s + tu0 * G::SB, cu * G::SB, bar);
    if (G::DB) bulk_g2s(st + G::CU * (G::QB + G::HB + G::SB), W.d + tu0 * G::DB, cu * G::DB, bar);
}

// f(x) for one token -> exact power-of-two range scale -> fp16 hi/lo columns (B operand) + 32-wide block
// sums; the same arithmetic as k_gemv_mma's prologue at T = 1. Returns the range scale.
XJ_DEV float mk_prologue(const MkPhase &p, __half *xs, float *xsum, int tid) {
    __shared__ float s_ss[MK_CWARPS], s_am[MK_CWARPS];
    __shared__ double s_hg[MK_KMAX / 32];
    const int lane = tid & 31, warp = tid >> 5, K = p.K, xstride = K + 16;
    constexpr int XPT = MMA_KMAX_PT;
    float v[XPT];
    float ss = 0.0f, am = 0.0f;
#pragma unroll
    for (int k = 0; k < XPT; k++) {
        const int i = tid + k * MK_CTHREADS;
        v[k] = 0.0f;
        if (i < K) {
            const float xv = lda(p.x + i);
            if (p.pro == PRO_NORM) { ss = fmaf(xv, xv, ss); am = fmaxf(am, fabsf(xv * p.norm_w[i])); v[k] = xv; }
            else if (p.pro == PRO_SWIGLU) { v[k] = silu_f(xv) * lda(p.x2 + i); am = fmaxf(am, fabsf(v[k])); }
            else if (p.pro == PRO_GNORM) v[k] = xv;
            else { v[k] = xv; am = fmaxf(am, fabsf(xv)); }
        }
    }
    if (p.pro == PRO_GNORM) {
        // o * (1/sqrt(mean_head(o^2) + eps)) * w[j] * silu(z), head sums in double
        const int gs = p.gs;
        double hd[XPT];
#pragma unroll
        for (int k = 0; k < XPT; k++) {
            const int i = tid + k * MK_CTHREADS;   // K is a multiple of 32: warp-uniform
            double d = i < K ? (double)v[k] * v[k] : 0.0;
            if (gs >= 32) {
                d = warp_sum_d(d);
                if (lane == 0 && i < K) s_hg[i >> 5] = d;
            } else {
                for (int o = gs >> 1; o; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
            }
            hd[k] = d;
        }
        if (gs >= 32) BarC::sync();
#pragma unroll
        for (int k = 0; k < XPT; k++) {
            const int i = tid + k * MK_CTHREADS;
            if (i < K) {
                double so = hd[k];
                if (gs >= 32) {
                    so = 0.0;
                    const int c0 = (i / gs) * (gs >> 5);
                    for (int c = 0; c < (gs >> 5); c++) so += s_hg[c0 + c];
                }
                const float sc = 1.0f / sqrtf((float)(so / gs) + p.eps);
                v[k] = v[k] * sc * p.norm_w[i % gs] * silu_f(lda(p.x2 + i));
                am = fmaxf(am, fabsf(v[k]));
            }
        }
    }
    ss = warp_sum(ss);
    am = warp_max(am);
    if (lane == 0) { s_ss[warp] = ss; s_am[warp] = am; }
    BarC::sync();
    double tss = 0;
    float tam = 0.0f;
    for (int w = 0; w < MK_CWARPS; w++) { tss += s_ss[w]; tam = fmaxf(tam, s_am[w]); }
    const float nsc = p.pro == PRO_NORM ? 1.0f / sqrtf((float)(tss / K) + p.eps) : 1.0f;
    const float m = tam * nsc;
    const float sc = ldexpf(1.0f, 14 - (m > 0.0f ? ilogbf(m) : 0));
#pragma unroll
    for (int k = 0; k < XPT; k++) {
        const int i = tid + k * MK_CTHREADS;
        if (i < K) {
            const float val = (p.pro == PRO_NORM ? (v[k] * nsc) * p.norm_w[i] : v[k]) * sc;
            const __half hi = __float2half_rn(val);
            const __half lo = __float2half_rn(val - __half2float(hi));
            const int pos = (i & ~15) + bperm(i & 15);
            xs[pos] = hi;
            xs[xstride + pos] = lo;
            const float bs = warp_sum(__half2float(hi) + __half2float(lo));
            if (lane == 0) xsum[i >> 5] = bs;
        }
    }
    BarC::sync();
    return sc;
}

// Epilogue of one 16-row tile from the per-warp partials red[warp][16] (fixed-order sum over warps).
XJ_DEV void mk_epilogue(const MmaJob &jb, int tile, const float *red, float tscale, int tid) {
    const bool real = tile * 16 + (tid & 15) < jb.w.N;   // rows past N pad the last tile
    if (jb.epi == EPI_CONV) {
        if (tid < 16 && real) {
            const int ch = tile * 16 + tid, kc = jb.kc;
            float s = 0.0f;
#pragma unroll
            for (int w = 0; w < MK_CWARPS; w++) s += red[w * 16 + tid];
            s /= tscale;
            float cs[8];
            float *st = jb.conv_state + (size_t)ch * (kc - 1);
            for (int k = 0; k < kc - 1; k++) cs[k] = __ldcg(st + k);
            const float *wc = jb.conv_w + (size_t)ch * kc;
            float acc = 0.0f;
            for (int k = 0; k < kc - 1; k++) acc = fmaf(cs[k], wc[k], acc);
            acc = fmaf(s, wc[kc - 1], acc);
            for (int k = 0; k < kc - 2; k++) st[k] = cs[k + 1];
            st[kc - 2] = s;
            jb.y[ch] = silu_f(acc);
        }
    } else if (jb.epi == EPI_ARGMAX) {
        if (tid < 32) {
            const int row = tid & 15;
            float s = 0.0f;
#pragma unroll
            for (int w = 0; w < MK_CWARPS; w++) s += red[w * 16 + row];
            s /= tscale;
            if (jb.y && tid < 16 && real) jb.y[(size_t)tile * 16 + row] = s;
            if (!real) s = -INFINITY;
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
    } else if (tid < 16 && real) {
        float s = 0.0f;
#pragma unroll
        for (int w = 0; w < MK_CWARPS; w++) s += red[w * 16 + tid];
        s /= tscale;
        float *yp = jb.y + (size_t)tile * 16 + tid;
        *yp = jb.epi == EPI_ADD ? __ldcg(yp) + s : s;
    }
}

// ------------------------------------------------------------------ Gated DeltaNet rows
// Work item = RPI value rows of one head (T = 1, no checkpoints): the decayed state row, its product
// with k, the delta-rule update and the raw output o[j] = (M[j] . q) / sqrt(S) (core/xj_cpu.c:184-217).
template <int S>
struct GdnGeo {
    static constexpr int TPR = S / 4 < 32 ? S / 4 : 32;                  // threads per state row
    static constexpr int P = S / TPR;                                    // elements per thread (4 or 8)
    static constexpr int RPI = MK_CTHREADS / TPR < S ? MK_CTHREADS / TPR : S;
    static constexpr int IPH = S / RPI;                                  // items per head
};

template <int S>
XJ_DEV void mk_gdn_item(const GdnArgs &a, int item, float *scr, int tid) {
    using Gg = GdnGeo<S>;
    constexpr int TPR = Gg::TPR, P = Gg::P, RPI = Gg::RPI;
    float *qs = scr, *ks = scr + 256;
    double *red = reinterpret_cast<double *>(scr + 512);
    const int hv = item / Gg::IPH, r0 = (item % Gg::IPH) * RPI, hk = hv % a.Hk;
    const int lane = tid & 31, warp = tid >> 5;
    const int j = r0 + tid / TPR, qq = tid % TPR;
    const bool act = tid < RPI * TPR;                                    // warp-uniform
    const float *x = a.qkv;
    // L2 norms of q (threads 0..S-1) and k (threads 256..256+S-1), sums in double
    const float qv = tid < S ? lda(x + hk * S + tid) : 0.0f;
    const float kv = (tid >= 256 && tid - 256 < S) ? lda(x + a.key_dim + hk * S + tid - 256) : 0.0f;
    const double d = warp_sum_d(tid < 256 ? (double)qv * qv : (double)kv * kv);
    if (lane == 0) red[warp] = d;
    BarC::sync();
    double sq = 0, sk2 = 0;
    for (int w = 0; w < 8; w++) { sq += red[w]; sk2 += red[8 + w]; }
    if (tid < S) qs[tid] = qv * (1.0f / sqrtf((float)sq + a.eps));
    if (tid >= 256 && tid - 256 < S) ks[tid - 256] = kv * (1.0f / sqrtf((float)sk2 + a.eps));
    BarC::sync();
    if (act) {
        float *M = a.ssm + ((size_t)hv * S + j) * S + qq * P;
        float row[P];
#pragma unroll
        for (int i = 0; i < P; i += 4) {
            const float4 v4 = __ldcg(reinterpret_cast<const float4 *>(M + i));
            row[i] = v4.x; row[i + 1] = v4.y; row[i + 2] = v4.z; row[i + 3] = v4.w;
        }
        const float b = sigm_f(lda(a.beta + hv));
        const float g = softplus_f(lda(a.alpha + hv) + a.dt[hv]) * a.A[hv];
        const float eg = expf(g);
        float sk = 0.0f;
#pragma unroll
        for (int i = 0; i < P; i++) { row[i] *= eg; sk = fmaf(row[i], ks[qq * P + i], sk); }
#pragma unroll
        for (int o = TPR >> 1; o; o >>= 1) sk += __shfl_xor_sync(0xffffffffu, sk, o);
        const float delta = (lda(x + 2 * a.key_dim + hv * S + j) - sk) * b;
        float acc = 0.0f;
#pragma unroll
        for (int i = 0; i < P; i++) { row[i] = fmaf(ks[qq * P + i], delta, row[i]); acc = fmaf(row[i], qs[qq * P + i], acc); }
#pragma unroll
        for (int o = TPR >> 1; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (qq == 0) a.out[hv * S + j] = acc * (1.0f / sqrtf((float)S));
#pragma unroll
        for (int i = 0; i < P; i += 4) *reinterpret_cast<float4 *>(M + i) = make_float4(row[i], row[i + 1], row[i + 2], row[i + 3]);
    }
    BarC::sync();   // qs / ks / red are reused by the next item
}

// ------------------------------------------------------------------ attention splits
template <typename KV> XJ_DEV float kv_round(float v);
template <> XJ_DEV float kv_round<float>(float v) { return v; }
template <> XJ_DEV float kv_round<__half>(float v) { return __half2float(__float2half_rn(v)); }

// Work item (head h, split sp of nsplit): q head h and its KV head through RMSNorm + NeoX RoPE (the
// arithmetic of attn_prep_slot), the new K/V row stored at position npast by one item per KV head, and
// online-softmax attention over positions [sp*n/nsplit, (sp+1)*n/nsplit) of n = npast + 1 (the new row
// is taken from shared memory, rounded as the cache stores it). One split writes the gated output
// directly; otherwise the last split of the head to finish merges all splits (core/xj_cpu.c:118-150).
template <typename KV, int DPL>
XJ_DEV void mk_attn_item(const AttnArgs &a, int h, int sp, int nsplit, float *apart, int *acnt, float *scr, int tid) {
    __shared__ int s_last;
    const int D = a.D, group = a.H / a.Hkv, kvh = h / group, lane = tid & 31, warp = tid >> 5;
    float *nq = scr, *rq = scr + 256, *nk = scr + 512, *rk = scr + 768, *rv = scr + 1024;
    double *red = reinterpret_cast<double *>(scr + 1280);
    float *sm_m = scr + 1312, *sm_l = scr + 1328, *sm_o = scr + 1344;      // [16][256]
    const int pos = __ldcg(a.npast), n = pos + 1;
    const float qv = tid < D ? lda(a.q + (size_t)h * 2 * D + tid) : 0.0f;
    const float kv = (tid >= 256 && tid - 256 < D) ? lda(a.k + (size_t)kvh * D + tid - 256) : 0.0f;
    const double d = warp_sum_d(tid < 256 ? (double)qv * qv : (double)kv * kv);
    if (lane == 0) red[warp] = d;
    BarC::sync();
    double ssq = 0, ssk = 0;
    for (int w = 0; w < 8; w++) { ssq += red[w]; ssk += red[8 + w]; }
    if (tid < D) nq[tid] = qv * (1.0f / sqrtf((float)(ssq / D) + a.eps)) * a.qn[tid];
    if (tid >= 256 && tid - 256 < D) nk[tid - 256] = kv * (1.0f / sqrtf((float)(ssk / D) + a.eps)) * a.kn[tid - 256];
    BarC::sync();
    {
        const bool isq = tid < 256;
        const int i = isq ? tid : tid - 256;
        if (i < D) {
            const float *src = isq ? nq : nk;
            float r = src[i];
            const int half = a.n_rot / 2;
            if (i < a.n_rot) {
                const int p = i < half ? i : i - half;
                const float theta = (float)pos * powf(a.base, -2.0f * (float)p / (float)a.n_rot);
                const float c = cosf(theta), s = sinf(theta);
                const float x0 = src[p], x1 = src[p + half];
                r = i < half ? x0 * c - x1 * s : x0 * s + x1 * c;
            }
            if (isq) rq[i] = r;
            else {
                const float vv = lda(a.v + (size_t)kvh * D + i);
                rk[i] = kv_round<KV>(r);
                rv[i] = kv_round<KV>(vv);
                if (sp == nsplit - 1 && h % group == 0) {
                    const size_t o = (size_t)pos * a.Hkv * D + (size_t)kvh * D + i;
                    store_kv<KV>((KV *)a.kc + o, r);
                    store_kv<KV>((KV *)a.vc + o, vv);
                }
            }
        }
    }
    BarC::sync();
    // online softmax over this split's positions, 16 warps interleaved
    const int j0 = (int)((long long)sp * n / nsplit), j1 = (int)((long long)(sp + 1) * n / nsplit);
    const int kvd = a.Hkv * D;
    const float scale = 1.0f / sqrtf((float)D);
    const KV *kc = (const KV *)a.kc, *vc = (const KV *)a.vc;
    const bool on = lane * DPL < D;
    float qr[DPL], o[DPL];
#pragma unroll
    for (int e = 0; e < DPL; e++) { qr[e] = on ? rq[lane * DPL + e] : 0.0f; o[e] = 0.0f; }
    float m = -INFINITY, l = 0.0f;
    for (int j = j0 + warp; j < j1; j += MK_CWARPS) {
        float kr[DPL], vr[DPL];
        if (j == pos) {
#pragma unroll
            for (int e = 0; e < DPL; e++) { kr[e] = on ? rk[lane * DPL + e] : 0.0f; vr[e] = on ? rv[lane * DPL + e] : 0.0f; }
        } else {
            const KV *kp = kc + (size_t)j * kvd + (size_t)kvh * D + lane * DPL;
            const KV *vp = vc + (size_t)j * kvd + (size_t)kvh * D + lane * DPL;
#pragma unroll
            for (int e = 0; e < DPL; e++) { kr[e] = on ? load_kv(kp + e) : 0.0f; vr[e] = on ? load_kv(vp + e) : 0.0f; }
        }
        float s = 0.0f;
#pragma unroll
        for (int e = 0; e < DPL; e++) s = fmaf(qr[e], kr[e], s);
        s = warp_sum(s) * scale;
        const float mn = fmaxf(m, s);
        const float corr = expf(m - mn), p = expf(s - mn);
        l = l * corr + p;
#pragma unroll
        for (int e = 0; e < DPL; e++) o[e] = fmaf(p, vr[e], o[e] * corr);
        m = mn;
    }
    if (lane == 0) { sm_m[warp] = m; sm_l[warp] = l; }
#pragma unroll
    for (int e = 0; e < DPL; e++) sm_o[warp * 256 + lane * DPL + e] = o[e];
    BarC::sync();
    float *part = apart + ((size_t)h * nsplit + sp) * (D + 2);
    const float *gate = a.q + (size_t)h * 2 * D + D;
    if (tid < D) {
        float M = -INFINITY;
        for (int w = 0; w < MK_CWARPS; w++) M = fmaxf(M, sm_m[w]);
        float L = 0.0f, acc = 0.0f;
        for (int w = 0; w < MK_CWARPS; w++) {
            const float c = sm_m[w] == -INFINITY ? 0.0f : expf(sm_m[w] - M);
            L += sm_l[w] * c;
            acc = fmaf(sm_o[w * 256 + tid], c, acc);
        }
        if (nsplit == 1) a.out[(size_t)h * D + tid] = (acc / L) * sigm_f(lda(gate + tid));
        else {
            part[tid] = acc;
            if (tid == 0) { part[D] = M; part[D + 1] = L; }
            __threadfence();
        }
    }
    if (nsplit > 1) {
        BarC::sync();
        if (tid == 0) {
            __threadfence();
            const int old = atomicAdd(acnt + h, 1);
            s_last = old == nsplit - 1;
        }
        BarC::sync();
        if (s_last) {
            __threadfence();
            if (tid < D) {
                const float *p0 = apart + (size_t)h * nsplit * (D + 2);
                float M = -INFINITY;
                for (int s = 0; s < nsplit; s++) M = fmaxf(M, __ldcg(p0 + (size_t)s * (D + 2) + D));
                float L = 0.0f, acc = 0.0f;
                for (int s = 0; s < nsplit; s++) {
                    const float *ps = p0 + (size_t)s * (D + 2);
                    const float c = expf(__ldcg(ps + D) - M);
                    L += __ldcg(ps + D + 1) * c;
                    acc = fmaf(__ldcg(ps + tid), c, acc);
                }
                a.out[(size_t)h * D + tid] = (acc / L) * sigm_f(lda(gate + tid));
            }
            if (tid == 0) atomicExch(acnt + h, 0);
        }
    }
    BarC::sync();   // scratch is reused by the next item
}

XJ_DEV int mk_nsplit(int n, int H, int max_split) {
    int ns = (n + 31) / 32;
    if (ns > max_split) ns = max_split;
    return ns < 1 ? 1 : ns;
}

template <typename KV>
XJ_DEV void mk_attn_phase(const MkArgs &A, const AttnArgs &a, float *scr, int tid) {
    const int n = __ldcg(a.npast) + 1, nsplit = mk_nsplit(n, a.H, A.max_split);
    const int items = a.H * nsplit;
    for (int it = blockIdx.x; it < items; it += gridDim.x) {
        const int h = it / nsplit, sp = it % nsplit;
        switch ((a.D + 31) / 32) {
        case 1: mk_attn_item<KV, 1>(a, h, sp, nsplit, A.apart, A.acnt, scr, tid); break;
        case 2: mk_attn_item<KV, 2>(a, h, sp, nsplit, A.apart, A.acnt, scr, tid); break;
        case 4: mk_attn_item<KV, 4>(a, h, sp, nsplit, A.apart, A.acnt, scr, tid); break;
        default: mk_attn_item<KV, 8>(a, h, sp, nsplit, A.apart, A.acnt, scr, tid); break;
        }
    }
}

template <int S>
XJ_DEV void mk_gdn_phase(const GdnArgs &a, float *scr, int tid) {
    const int items = a.Hv * GdnGeo<S>::IPH;
    for (int it = blockIdx.x; it < items; it += gridDim.x) mk_gdn_item<S>(a, it, scr, tid);
}

// ------------------------------------------------------------------ the kernel
__global__ void __launch_bounds__(MK_THREADS, 1) k_decode_persistent(MkArgs A) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t full[MK_NS], empty[MK_NS];
    __shared__ unsigned s_issued;
    uint8_t *ring = smem;
    __half *xs = reinterpret_cast<__half *>(smem + (size_t)MK_NS * MK_SLOT);
    float *xsum = reinterpret_cast<float *>(smem + (size_t)MK_NS * MK_SLOT + MK_XS_BYTES);
    float *scs = xsum + MK_KMAX / 32;
    float *red = scs + MK_CWARPS * 128;
    float *scr = reinterpret_cast<float *>(xs);     // GDN / attention scratch (xs is dead between GEMVs)
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, cta = blockIdx.x;
    if (tid == 0) {
        for (int s = 0; s < MK_NS; s++) { mbar_init(&full[s], 1); mbar_init(&empty[s], MK_CWARPS); }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        s_issued = 0;
    }
    __syncthreads();
    unsigned consumed = 0, drain_from = 0xffffffffu;

    if (warp == MK_CWARPS) {
        // ---------------- producer: this CTA's weight chunks of every GEMV phase, in program order
        if (lane == 0) {
            unsigned i = 0;
            bool ok = true;
            for (int step = 0; ok && step < A.nsteps; step++)
                for (int ph = 0; ok && ph < A.nphase; ph++) {
                    const MkPhase &p = A.prog[ph];
                    if (p.op != MK_GEMV) continue;
                    for (int tg = cta; ok && tg < p.ntiles; tg += G) {
                        const int j = mk_job_of(p, tg);
                        const Tiled &W = p.job[j].w;
                        const int tile = tg - p.tile_start[j], CU = mk_cu(W.type);
                        for (int u0 = 0; u0 < W.nu; u0 += CU, i++) {
                            const int slot = i % MK_NS;
                            if (i >= MK_NS && !mk_wait(&empty[slot], ((i / MK_NS) - 1) & 1, A.err, 1)) { ok = false; break; }
                            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                            const int cu = W.nu - u0 < CU ? W.nu - u0 : CU;
                            uint8_t *st = ring + (size_t)slot * MK_SLOT;
                            if (W.type == XJ_Q4_K) mk_issue_t<XJ_Q4_K>(W, tile, u0, cu, st, &full[slot]);
                            else if (W.type == XJ_Q6_K) mk_issue_t<XJ_Q6_K>(W, tile, u0, cu, st, &full[slot]);
                            else mk_issue_t<XJ_Q8_0>(W, tile, u0, cu, st, &full[slot]);
                            *(volatile unsigned *)&s_issued = i + 1;
                        }
                    }
                }
        }
        __syncwarp();
    } else {
        // ---------------- consumers
        const int g = lane >> 2, c = lane & 3;
        float *scw = scs + warp * 128;
        unsigned nbar = 0;
        int rb = 0;
        for (int step = 0; step < A.nsteps; step++) {
            bool ok = true;
            for (int ph = 0; ph < A.nphase; ph++) {
                const MkPhase &p = A.prog[ph];
                if (p.op == MK_GEMV && cta < p.ntiles) {
                    const float tsc = mk_prologue(p, xs, xsum, tid);
                    const int xstride = p.K + 16;
                    const bool bcol = g < 2;
                    const __half *xb = xs + (size_t)g * xstride + 4 * c;
                    const float *xsum_t = c == 0 ? xsum : nullptr;
                    for (int tg = cta; tg < p.ntiles; tg += G) {
                        const int j = mk_job_of(p, tg);
                        const MmaJob &jb = p.job[j];
                        const Tiled &W = jb.w;
                        const int tile = tg - p.tile_start[j], CU = mk_cu(W.type);
                        float yg = 0.0f, yg8 = 0.0f;
                        for (int u0 = 0; u0 < W.nu; u0 += CU, consumed++) {
                            const int slot = consumed % MK_NS;
                            const bool got = mk_wait(&full[slot], (consumed / MK_NS) & 1, A.err, 1);
                            const uint8_t *st = ring + (size_t)slot * MK_SLOT;
                            const int cu = W.nu - u0 < CU ? W.nu - u0 : CU;
                            if (W.type == XJ_Q4_K) {
                                const int ui = warp >> 1;
                                if (ui < cu) unit_compute<XJ_Q4_K>(st, ui, u0 + ui, warp & 1, lane, bcol, xb, xsum_t, scw, yg, yg8);
                            } else if (W.type == XJ_Q6_K) {
                                const int ui = warp >> 1;
                                if (ui < cu) unit_compute<XJ_Q6_K>(st, ui, u0 + ui, warp & 1, lane, bcol, xb, xsum_t, scw, yg, yg8);
                            } else {
#pragma unroll
                                for (int k = 0; k < Geo<XJ_Q8_0>::CU / MK_CWARPS; k++) {
                                    const int ui = warp + k * MK_CWARPS;
                                    if (ui < cu) unit_compute<XJ_Q8_0>(st, ui, u0 + ui, 0, lane, bcol, xb, xsum_t, scw, yg, yg8);
                                }
                            }
                            __syncwarp();
                            if (lane == 0 && got) mbar_arrive(&empty[slot]);
                            if (!got && drain_from == 0xffffffffu) drain_from = consumed;
                        }
                        float *rr = red + rb * (MK_CWARPS * 16);
                        if (c == 0) { rr[warp * 16 + g] = yg; rr[warp * 16 + g + 8] = yg8; }
                        BarC::sync();
                        mk_epilogue(jb, tile, rr, tsc, tid);
                        rb ^= 1;
                    }
                } else if (p.op == MK_GDN) {
                    switch (p.gs) {
                    case 16: mk_gdn_phase<16>(p.gdn, scr, tid); break;
                    case 32: mk_gdn_phase<32>(p.gdn, scr, tid); break;
                    case 64: mk_gdn_phase<64>(p.gdn, scr, tid); break;
                    case 128: mk_gdn_phase<128>(p.gdn, scr, tid); break;
                    case 256: mk_gdn_phase<256>(p.gdn, scr, tid); break;
                    default: break;
                    }
                } else if (p.op == MK_ATTN) {
                    if (A.kv_f32) mk_attn_phase<float>(A, p.attn, scr, tid);
                    else mk_attn_phase<__half>(A, p.attn, scr, tid);
                } else if (p.op == MK_ARGMAX) {
                    if (cta == 0) argmax_final_dev<BarC>(p.am, tid, MK_CTHREADS);
                }
                if (step == A.nsteps - 1 && ph == A.nphase - 1) break;
                nbar++;
                if (!mk_grid_sync(A.bar, nbar * (unsigned)G, A.err, tid)) { ok = false; break; }
            }
            if (!ok) break;
        }
    }
    __syncthreads();
    // chunks requested but never consumed (only after an error): let their copies land before exiting
    if (tid == 0) {
        const unsigned issued = s_issued;
        for (unsigned i = drain_from < consumed ? drain_from : consumed; i < issued; i++)
            if (!mk_wait_drain(&full[i % MK_NS], (i / MK_NS) & 1)) break;
    }
}

}  // namespace xjk
