// Persistent decode kernel: every greedy decode step of the whole model (all layers, the LM head and
// the token pick) for any number of steps in ONE cooperative launch.
//
// A decode step at batch 1 is ~150 dependent phases (matrix-vector products, the Gated DeltaNet
// update, attention, the argmax), each of which moves only a few MB. Launched as separate kernels every
// phase pays launch latency and an empty weight pipeline; here one CTA per SM runs the phase program
// in a loop and the phases are separated by a grid barrier instead (a counter in global memory; every
// wait bounded).
//
// Each CTA has 16 compute warps, one producer warp and one epilogue warp. The producer walks the same
// phase program and, for every matrix-vector phase, requests this CTA's weight chunks into a
// shared-memory ring with bulk asynchronous copies (one mbarrier per slot for "full", one for "empty";
// no multicast). Weights do not depend on activations, so the producer runs ahead of the consumers
// across phase boundaries and the grid barriers: the HBM stream of the next phases overlaps the barrier
// and the small phases. The compute warps hand each tile's partial rows to the epilogue warp through a
// small ring of buffers (mbarriers again) and go straight on to the next tile.
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
//   SAMPLE (a sampler set) a top-k / top-p / temperature draw from the LM head's logits, keyed by the
//          position (sample_row_dev, the session sampler's arithmetic), then as ARGMAX
//
// Matrix-vector products give the same bits as the standalone tensor-core kernel (same unit order,
// same prologue arithmetic, same fixed-order reductions). GDN and attention sum in a different order
// than the standalone kernels (more threads per row and per head), within float rounding.
#pragma once
#include "gemv_mma.cuh"
#include "sample.cuh"

namespace xjk {

constexpr int MK_CWARPS = 16;                    // consumer (compute) warps
constexpr int MK_CTHREADS = MK_CWARPS * 32;      // 512
constexpr int MK_EWARP = MK_CWARPS + 1;          // the epilogue warp (after the producer warp)
constexpr int MK_THREADS = MK_CTHREADS + 64;     // + the producer and the epilogue warp
constexpr int MK_NR = 4;                         // tile partial buffers between compute and epilogue warps
constexpr int MK_SLOT = 26880;                   // largest chunk: 8 Q6_K units
constexpr int MK_NS = 3;                         // ring slots (3 measured faster than 2, 4 or 6)
constexpr int MK_KMAX = MMA_KMAX_PT * MK_CTHREADS;
constexpr int MK_XS_BYTES = 2 * (MK_KMAX + 16) * 2;   // hi/lo fp16 columns (also GDN / attention scratch)
constexpr int MK_MAX_SPLIT = 64;                      // attention splits per KV head
using BarC = BarNamed<1, MK_CTHREADS>;           // the compute warps only
using BarP = BarNamed<2, MK_CTHREADS + 32>;      // compute + epilogue warps (descriptor hand-over, phase ends)

enum { MK_GEMV = 0, MK_GDN = 1, MK_ATTN = 2, MK_ARGMAX = 3, MK_SAMPLE = 4 };
enum { PRO_GNORM = 3,                             // per-head RMSNorm(ssm_norm) * silu(z), core/xj_cpu.c:218-224
       PRO_GNORM_S = 4,                           // the same with x2 = silu(z) already (MK_EPI_SILU)
       PRO_SWIGLU_S = 5 };                        // x * up with x = silu(gate) already (MK_EPI_SILU)
enum { MK_EPI_SILU = 4 };                         // store silu(row) (GDN gate rows z, FFN gate rows)

struct alignas(16) MkPhase {
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
    ArgmaxArgs am;               // MK_ARGMAX, MK_SAMPLE: where the pick goes
    SampleArgs sa;               // MK_SAMPLE: the LM head's logits and the sampler settings
};

// One GEMV phase as the producer streams it (the weight regions of each job's tiled layout).
struct alignas(16) MkStream {
    int ntiles, njob, ph;         // ph: index of the phase in the program
    int tile_start[5];
    int type[4], nu[4];
    const uint8_t *q[4], *h[4], *s[4], *d[4];
    // side data of this phase and of the non-GEMV phase after it (norm and conv weights, recurrent
    // state), prefetched into L2 when the producer reaches this phase: a 1/G slice per CTA
    const uint8_t *pf[6];
    unsigned pf_bytes[6];
};

struct MkArgs {
    const MkPhase *prog;
    const MkStream *stream;      // the GEMV phases of prog, in order
    int nphase, nstream, nsteps;
    unsigned long long *trace;   // optional, per CTA and phase of the last step (ns): start, end, time the
                                 // consumers waited for weights, first and last chunk request, end of
                                 // the prologue, end of the first tile, tiles
    unsigned *bar;               // grid barrier counter, zero at launch
    int *err;                    // 1: weight stream wait gave up, 2: grid barrier wait gave up
    float *apart;                // attention split partials [H][max_split][D + 2]
    int *acnt;                   // per-head split counters, zero at launch
    int max_split;
    int kv_f32;
    int *diag;                   // first wait that gave up: kind, cta, tid, step, phase, index, extra
};

constexpr size_t MK_SMEM = (size_t)MK_NS * MK_SLOT + MK_XS_BYTES + 2 * (MK_KMAX / 32) * 4 + MK_CWARPS * 128 * 4 +
                           MK_NR * MK_CWARPS * 16 * 4;

XJ_DEV unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
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

// Where the first wait that gave up was (read by the host after an error).
XJ_DEV void mk_record(int *diag, int kind, int step, int ph, int idx, int extra) {
    if (diag && atomicCAS(diag, 0, kind) == 0) {
        diag[1] = blockIdx.x; diag[2] = threadIdx.x; diag[3] = step; diag[4] = ph; diag[5] = idx; diag[6] = extra;
        __threadfence();
    }
}

// Wait for an mbarrier phase; gives up (recording `code`) after MK_WAIT_NS (or 2^26 polls, should the
// clock not advance) or once another part of the grid has recorded an error. mbarrier.try_wait suspends
// the thread in hardware until the phase completes (or a short time limit), so the loop polls it back to
// back and wakes as soon as the phase completes. The grid's error word is a global load of about a
// microsecond: it is issued every 16 polls and its value read 16 polls later, so the wait never stalls on
// it; the same polls read the clock and, if `nap` is set, sleep that many ns.
// The polling part, out of line: the fast path (the phase already complete) stays a single try_wait in
// the callers' loops, which keeps the unit loop's code short.
__device__ __noinline__ bool mk_wait_slow(uint64_t *bar, uint32_t parity, int *err, int code, int *diag, int step,
                                          int ph, int idx, int nap) {
    const unsigned long long t0 = globaltimer();
    int ev = ld_volatile(err);
    for (int it = 1; it < (1 << 26); it++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 15) == 0) {
            if (ev) return false;
            ev = ld_volatile(err);
            if (globaltimer() - t0 > MK_WAIT_NS) break;
            if (nap) __nanosleep(nap);
        }
    }
    mk_record(diag, code == 1 ? 10 + (int)parity : code, step, ph, idx, (int)(globaltimer() - t0) / 1000);
    atomicExch(err, code);
    return false;
}
XJ_DEV bool mk_wait(uint64_t *bar, uint32_t parity, int *err, int code, int *diag = nullptr, int step = 0,
                    int ph = 0, int idx = 0, int nap = 0) {
    if (mbar_try_wait(bar, parity)) return true;
    return mk_wait_slow(bar, parity, err, code, diag, step, ph, idx, nap);
}

// All compute and epilogue threads of all CTAs: returns false (uniformly within the CTA) when the grid
// records an error. Ordering: the CTA barrier orders every participating thread's writes before thread
// 0's release add, and thread 0's acquire load before the other threads' reads after the second CTA
// barrier (release and acquire are cumulative in the PTX memory model), so no separate fences are
// needed; the add returns nothing, so the arriving CTA does not wait for it. Thread 0 polls the counter
// back to back (one acquire load in flight); the error word is loaded alongside every 16 polls and its
// value used at the next check, so it adds no round trip to the barrier. A CTA that passes a barrier
// while another records an error stops at its next wait instead (every wait also reads the error word).
XJ_DEV bool mk_grid_sync(unsigned *bar, unsigned target, int *err, int tid, int *diag, int step, int ph) {
    __shared__ int s_ok;
    BarP::sync();
    if (tid == 0) {
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" :: "l"(bar) : "memory");
        int ok = 1, ev = ld_volatile(err);
        const unsigned long long t0 = globaltimer();
        for (unsigned it = 1; ld_acquire(bar) < target; it++) {
            if ((it & 15) == 0) {
                if (ev) { ok = 0; break; }
                ev = ld_volatile(err);
                if (globaltimer() - t0 > MK_WAIT_NS || it > (1u << 24)) {
                    mk_record(diag, 2, step, ph, (int)target, (int)ld_acquire(bar));
                    atomicExch(err, 2);
                    ok = 0;
                    break;
                }
            }
        }
        if (ev) ok = 0;
        s_ok = ok;
    }
    BarP::sync();
    return s_ok != 0;
}

// Asynchronous 16-byte global -> shared copies (L2 only) for the phase descriptors.
XJ_DEV void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(smem_u32(dst)), "l"(src) : "memory");
}
XJ_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
XJ_DEV void prefetch_l2(const void *p, unsigned bytes) {   // p 16-byte aligned, bytes a multiple of 16
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" :: "l"(p), "r"(bytes) : "memory");
}
XJ_DEV void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// Threads tid < bytes/16 start copying `bytes` (a multiple of 16) from src to dst.
XJ_DEV void copy_desc_async(void *dst, const void *src, int bytes, int tid) {
    if (tid < bytes / 16) {
        cp_async16(reinterpret_cast<uint8_t *>(dst) + tid * 16, reinterpret_cast<const uint8_t *>(src) + tid * 16);
        cp_async_commit();
    }
}

// ------------------------------------------------------------------ matrix-vector phases
XJ_DEV int mk_cu(int type) {
    return type == XJ_Q4_K ? Geo<XJ_Q4_K>::CU : type == XJ_Q5_K ? Geo<XJ_Q5_K>::CU : type == XJ_Q6_K ? Geo<XJ_Q6_K>::CU
         : type == XJ_F16 ? Geo<XJ_F16>::CU : Geo<XJ_Q8_0>::CU;
}
static_assert(stage_bytes<XJ_Q5_K>() <= 26880 && stage_bytes<XJ_F16>() <= 26880 && stage_bytes<XJ_Q6_K>() <= 26880,
              "every type's chunk fits a ring slot");
XJ_DEV int mk_job_of(const MkPhase &p, int tg) {
    int j = 0;
    while (j + 1 < p.njob && tg >= p.tile_start[j + 1]) j++;
    return j;
}

template <int TYPE>
XJ_DEV void mk_issue_t(const MkStream &S, int j, int tile, int u0, int cu, uint8_t *st, uint64_t *bar) {
    using G = Geo<TYPE>;
    const size_t tu0 = (size_t)tile * S.nu[j] + u0;
    mbar_expect_tx(bar, (uint32_t)(cu * unit_bytes<TYPE>()));
    bulk_g2s(st, S.q[j] + tu0 * G::QB, cu * G::QB, bar);
    if (G::HB) bulk_g2s(st + G::CU * G::QB, S.h[j] + tu0 * G::HB, cu * G::HB, bar);
    if (G::SB) bulk_g2s(st + G::CU * (G::QB + G::HB), S.s[j] + tu0 * G::SB, cu * G::SB, bar);
    if (G::DB) bulk_g2s(st + G::CU * (G::QB + G::HB + G::SB), S.d[j] + tu0 * G::DB, cu * G::DB, bar);
}

// f(x) for one token -> fp16 hi/lo columns (B operand) with a power-of-two range scale per 32-element
// block, the block sums and the blocks' inverse scales. Thread t takes the 4 consecutive elements
// 2048r + 4t .. +3 (r < 3): one vector load per operand (all issued before the first use, so the
// prologue costs one memory round trip), two half2 stores per column; a block is 8 consecutive lanes,
// so its largest magnitude, scale and sum are warp shuffles. Only RMSNorm needs a CTA-wide sum (of
// squares, in double as core/xj_cpu.c:56-61 does; a different summation order changes it only near
// 1e-16 relative, far below the float scale derived from it).
//
// Scaling a block by a power of two is exact and the unit code multiplies the block's weight scales by
// the inverse (exact again), so every product and partial sum equals the one computed with one scale
// for the whole vector (as the standalone kernels do) times a power of two: the results are the same
// bits unless an element is small enough (about 2^-17 of the vector's largest) that its fp16 low part
// turns subnormal under the whole-vector scale.
XJ_DEV float4 ldcg4(const float *p) { return __ldcg(reinterpret_cast<const float4 *>(p)); }
XJ_DEV float4 ld4(const float *p) { return *reinterpret_cast<const float4 *>(p); }
XJ_DEV float f4(const float4 &v, int e) { return e == 0 ? v.x : e == 1 ? v.y : e == 2 ? v.z : v.w; }
XJ_DEV void f4set(float4 &v, int e, float x) { if (e == 0) v.x = x; else if (e == 1) v.y = x; else if (e == 2) v.z = x; else v.w = x; }

XJ_DEV void mk_prologue(const MkPhase &p, __half *xs, float *xsum, float *xinv, int tid) {
    __shared__ double s_ss[MK_CWARPS];
    __shared__ double s_hd[MK_KMAX / 128];
    const int lane = tid & 31, warp = tid >> 5, K = p.K, xstride = K + 16, pro = p.pro, gs = p.gs;
    const float *px = p.x, *px2 = p.x2, *pw = p.norm_w;
    const float eps = p.eps;
    constexpr int NG = MK_KMAX / (4 * MK_CTHREADS);   // groups of 2048 elements
    const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
    const bool gn = pro == PRO_GNORM || pro == PRO_GNORM_S;
    float4 v[NG], w[NG], v2[NG];
#pragma unroll
    for (int r = 0; r < NG; r++) {
        const int i = r * 4 * MK_CTHREADS + 4 * tid;
        const bool in = i < K;
        v[r] = in ? ldcg4(px + i) : z4;
        w[r] = in && pro == PRO_NORM ? ld4(pw + i) : in && gn ? ld4(pw + i % gs) : z4;
        v2[r] = in && (pro == PRO_SWIGLU || pro == PRO_SWIGLU_S || gn) ? ldcg4(px2 + i) : z4;
    }
    double ss = 0.0;
#pragma unroll
    for (int r = 0; r < NG; r++) {
        if (r * 4 * MK_CTHREADS + 4 * tid >= K) continue;
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const float xv = f4(v[r], e);
            if (pro == PRO_NORM) ss += (double)xv * xv;
            else if (pro == PRO_SWIGLU) f4set(v[r], e, silu_f(xv) * f4(v2[r], e));
            else if (pro == PRO_SWIGLU_S) f4set(v[r], e, xv * f4(v2[r], e));
        }
    }
    if (gn) {
        // o * (1/sqrt(mean_head(o^2) + eps)) * w[j] * silu(z): head sums (in double) over the
        // gs/4 lanes of a head, across warps through shared memory for heads wider than 128
        double hd[NG];
#pragma unroll
        for (int r = 0; r < NG; r++) {
            double d = 0.0;
#pragma unroll
            for (int e = 0; e < 4; e++) d += (double)f4(v[r], e) * f4(v[r], e);
            if (gs <= 128) {
                for (int o = gs >> 3; o; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
            } else {
                d = warp_sum_d(d);
                const int i = r * 4 * MK_CTHREADS + 4 * tid;
                if (lane == 0 && i < K) s_hd[i >> 7] = d;
            }
            hd[r] = d;
        }
        if (gs > 128) BarC::sync();
#pragma unroll
        for (int r = 0; r < NG; r++) {
            const int i = r * 4 * MK_CTHREADS + 4 * tid;
            if (i >= K) continue;
            double so = hd[r];
            if (gs > 128) {
                so = 0.0;
                for (int c = 0; c < (gs >> 7); c++) so += s_hd[(i / gs) * (gs >> 7) + c];
            }
            const float sc = 1.0f / sqrtf((float)(so / gs) + eps);
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const float z = f4(v2[r], e);
                f4set(v[r], e, f4(v[r], e) * sc * f4(w[r], e) * (pro == PRO_GNORM_S ? z : silu_f(z)));
            }
        }
    }
    float nsc = 1.0f;
    if (pro == PRO_NORM) {
        ss = warp_sum_d(ss);
        if (lane == 0) s_ss[warp] = ss;
        BarC::sync();
        double tss = lane < MK_CWARPS ? s_ss[lane] : 0.0;
        tss = warp_sum_d(tss);
        nsc = 1.0f / sqrtf((float)(tss / K) + eps);
    }
#pragma unroll
    for (int r = 0; r < NG; r++) {
        const int i = r * 4 * MK_CTHREADS + 4 * tid;
        if (r * 4 * MK_CTHREADS >= K) break;          // uniform: whole groups beyond K
        float val[4], m = 0.0f;
#pragma unroll
        for (int e = 0; e < 4; e++) {
            val[e] = pro == PRO_NORM ? (f4(v[r], e) * nsc) * f4(w[r], e) : f4(v[r], e);
            m = fmaxf(m, fabsf(val[e]));
        }
        // the block's largest magnitude (8 lanes; K is a multiple of 32, so a block is all in or all out)
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
        const int ex = m > 0.0f ? ilogbf(m) : 14;
        const float sc = ldexpf(1.0f, 14 - ex);
        float bs = 0.0f;
        __half hi[4], lo[4];
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const float vs = val[e] * sc;
            hi[e] = __float2half_rn(vs);
            lo[e] = __float2half_rn(vs - __half2float(hi[e]));
            bs += __half2float(hi[e]) + __half2float(lo[e]);
        }
        // block sums of the 32 elements of 8 consecutive lanes
        bs += __shfl_xor_sync(0xffffffffu, bs, 1);
        bs += __shfl_xor_sync(0xffffffffu, bs, 2);
        bs += __shfl_xor_sync(0xffffffffu, bs, 4);
        if (i < K) {
            const int pos = (i & ~15) + bperm(i & 15);       // elements i, i+1 -> pos, pos+1; i+2, i+3 -> pos+4, pos+5
            *reinterpret_cast<__half2 *>(xs + pos) = __halves2half2(hi[0], hi[1]);
            *reinterpret_cast<__half2 *>(xs + pos + 4) = __halves2half2(hi[2], hi[3]);
            *reinterpret_cast<__half2 *>(xs + xstride + pos) = __halves2half2(lo[0], lo[1]);
            *reinterpret_cast<__half2 *>(xs + xstride + pos + 4) = __halves2half2(lo[2], lo[3]);
            if ((lane & 7) == 0) { xsum[i >> 5] = bs; xinv[i >> 5] = ldexpf(1.0f, ex - 14); }
        }
    }
    BarC::sync();
}

// ------------------------------------------------------------------ K-quant units at T = 1
// One warp's half of a Q4_K / Q6_K unit (16 rows x 128 codes: k-steps 8*HH .. 8*HH+7 of the super-block)
// from a staged chunk, with unit_compute_n's arithmetic for the token's columns (lanes c = 0: columns 0
// and 1 = hi and lo). Leaner than unit_compute_n at T = 1: the half index HH is a compile-time constant,
// so each header byte is one byte-permute; and no lane predicate guards the operand loads: lanes whose
// B-fragment column is not the token's (g >= 2) read the token's own columns again and lanes c != 0
// read its block sums, which only changes D columns and partial rows that are never stored.
XJ_DEV uint32_t byte_sel(uint32_t w, int j) { return __byte_perm(w, 0u, 0x4440u | (uint32_t)j); }   // byte j of w

template <int HH>
XJ_DEV void mk_q4k(const uint8_t *stage, int ui, int u, int lane, const __half *xb, const float *xsum, const float *xinv,
                   float *scw, float &yg, float &yg8) {
    using G = Geo<XJ_Q4_K>;
    const int g = lane >> 2;
    const uint8_t *qs = stage + ui * G::QB;
    const uint8_t *ss = stage + G::CU * G::QB + ui * G::SB;
    const uint4 q0 = *reinterpret_cast<const uint4 *>(qs + ((2 * HH) * 32 + lane) * 16);
    const uint4 q1 = *reinterpret_cast<const uint4 *>(qs + ((2 * HH + 1) * 32 + lane) * 16);
    {   // (d*sc, 64*d*sc + dmin*m) for row r, sub-blocks 4HH + 2*(lane>>4) + {0,1} (core/xj_quant.h:49-52)
        const int r = lane & 15;
        const uint4 hdr = *reinterpret_cast<const uint4 *>(ss + r * 16);
        const float d = h2f((uint16_t)(hdr.x & 0xffff)), dmin = h2f((uint16_t)(hdr.x >> 16));
#pragma unroll
        for (int e = 0; e < 2; e++) {
            const int sbl = 2 * (lane >> 4) + e;          // sub-block within this half = header byte index
            int s_, m_;
            if (HH == 0) { s_ = (int)(byte_sel(hdr.y, sbl) & 63); m_ = (int)(byte_sel(hdr.z, sbl) & 63); }
            else {
                const uint32_t b8 = byte_sel(hdr.w, sbl), b0 = byte_sel(hdr.y, sbl), b4 = byte_sel(hdr.z, sbl);
                s_ = (int)((b8 & 0xF) | ((b0 >> 6) << 4));
                m_ = (int)((b8 >> 4) | ((b4 >> 6) << 4));
            }
            const float d1 = d * (float)s_, m1 = dmin * (float)m_;
            const float iv = xinv[u * 8 + 4 * HH + sbl];   // the activation block's inverse range scale
            float *o = scw + ((sbl * 8 + (r & 7)) * 4 + (r >> 3) * 2);
            o[0] = d1 * iv;
            o[1] = (64.0f * d1 + m1) * iv;
        }
    }
    __syncwarp();
    const int kb = u * 256;
    const __half *xk = xb + kb + 128 * HH;
    const float *sk = xsum + (kb >> 5) + 4 * HH;
#pragma unroll
    for (int sbl = 0; sbl < 4; sbl++) {
        float d4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int e = 0; e < 2; e++) {
            uint32_t af[4];
            nib_frag64(word_of(e + 2 * sbl < 4 ? q0 : q1, (2 * sbl + e) & 3), af);
            const uint2 bv = *reinterpret_cast<const uint2 *>(xk + 16 * (2 * sbl + e));
            mma16816(d4, af, bv.x, bv.y);
        }
        const float4 sc4 = *reinterpret_cast<const float4 *>(scw + (sbl * 8 + g) * 4);
        const float S = sk[sbl];
        yg = fmaf(sc4.x, d4[0] + d4[1], yg);
        yg = fmaf(-sc4.y, S, yg);
        yg8 = fmaf(sc4.z, d4[2] + d4[3], yg8);
        yg8 = fmaf(-sc4.w, S, yg8);
    }
    __syncwarp();
}

// Q5_K: mk_q4k with the high bit of every code from the 1-bit plane (codes 64 + q, q < 32).
template <int HH>
XJ_DEV void mk_q5k(const uint8_t *stage, int ui, int u, int lane, const __half *xb, const float *xsum, const float *xinv,
                   float *scw, float &yg, float &yg8) {
    using G = Geo<XJ_Q5_K>;
    const int g = lane >> 2;
    const uint8_t *qs = stage + ui * G::QB;
    const uint8_t *ss = stage + G::CU * (G::QB + G::HB) + ui * G::SB;
    // this half's two words of the lane's high-bit record (k-steps 8HH .. 8HH+3, 8HH+4 .. 8HH+7)
    const uint2 hq = *reinterpret_cast<const uint2 *>(stage + G::CU * G::QB + ui * G::HB + lane * 16 + HH * 8);
    const uint4 q0 = *reinterpret_cast<const uint4 *>(qs + ((2 * HH) * 32 + lane) * 16);
    const uint4 q1 = *reinterpret_cast<const uint4 *>(qs + ((2 * HH + 1) * 32 + lane) * 16);
    {   // (d*sc, 64*d*sc + dmin*m) for row r, sub-blocks 4HH + 2*(lane>>4) + {0,1} (core/xj_quant.h:49-52)
        const int r = lane & 15;
        const uint4 hdr = *reinterpret_cast<const uint4 *>(ss + r * 16);
        const float d = h2f((uint16_t)(hdr.x & 0xffff)), dmin = h2f((uint16_t)(hdr.x >> 16));
#pragma unroll
        for (int e = 0; e < 2; e++) {
            const int sbl = 2 * (lane >> 4) + e;          // sub-block within this half = header byte index
            int s_, m_;
            if (HH == 0) { s_ = (int)(byte_sel(hdr.y, sbl) & 63); m_ = (int)(byte_sel(hdr.z, sbl) & 63); }
            else {
                const uint32_t b8 = byte_sel(hdr.w, sbl), b0 = byte_sel(hdr.y, sbl), b4 = byte_sel(hdr.z, sbl);
                s_ = (int)((b8 & 0xF) | ((b0 >> 6) << 4));
                m_ = (int)((b8 >> 4) | ((b4 >> 6) << 4));
            }
            const float d1 = d * (float)s_, m1 = dmin * (float)m_;
            const float iv = xinv[u * 8 + 4 * HH + sbl];   // the activation block's inverse range scale
            float *o = scw + ((sbl * 8 + (r & 7)) * 4 + (r >> 3) * 2);
            o[0] = d1 * iv;
            o[1] = (64.0f * d1 + m1) * iv;
        }
    }
    __syncwarp();
    const int kb = u * 256;
    const __half *xk = xb + kb + 128 * HH;
    const float *sk = xsum + (kb >> 5) + 4 * HH;
#pragma unroll
    for (int sbl = 0; sbl < 4; sbl++) {
        float d4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int e = 0; e < 2; e++) {
            uint32_t af[4];
            nib5_frag64(word_of(e + 2 * sbl < 4 ? q0 : q1, (2 * sbl + e) & 3), e + 2 * sbl < 4 ? hq.x : hq.y, (2 * sbl + e) & 3, af);
            const uint2 bv = *reinterpret_cast<const uint2 *>(xk + 16 * (2 * sbl + e));
            mma16816(d4, af, bv.x, bv.y);
        }
        const float4 sc4 = *reinterpret_cast<const float4 *>(scw + (sbl * 8 + g) * 4);
        const float S = sk[sbl];
        yg = fmaf(sc4.x, d4[0] + d4[1], yg);
        yg = fmaf(-sc4.y, S, yg);
        yg8 = fmaf(sc4.z, d4[2] + d4[3], yg8);
        yg8 = fmaf(-sc4.w, S, yg8);
    }
    __syncwarp();
}

template <int HH>
XJ_DEV void mk_q6k(const uint8_t *stage, int ui, int u, int lane, const __half *xb, const float *xinv, float *scw,
                   float &yg, float &yg8) {
    using G = Geo<XJ_Q6_K>;
    const int g = lane >> 2;
    const uint8_t *qs = stage + ui * G::QB;
    const uint8_t *hs = stage + G::CU * G::QB + ui * G::HB;
    const uint8_t *ss = stage + G::CU * (G::QB + G::HB) + ui * G::SB;
    const uint8_t *ds = stage + G::CU * (G::QB + G::HB + G::SB) + ui * G::DB;
    const uint4 q0 = *reinterpret_cast<const uint4 *>(qs + ((2 * HH) * 32 + lane) * 16);
    const uint4 q1 = *reinterpret_cast<const uint4 *>(qs + ((2 * HH + 1) * 32 + lane) * 16);
    const uint4 hq = *reinterpret_cast<const uint4 *>(hs + (HH * 32 + lane) * 16);
    {   // d*sc for row r, k-steps 8HH + 4*(lane>>4) + {0..3} (core/xj_quant.h:106-118)
        const int r = lane & 15;
        const uint4 sc = *reinterpret_cast<const uint4 *>(ss + r * 16);
        const float d = h2f(*reinterpret_cast<const uint16_t *>(ds + r * 2));
        const uint32_t wsel = (lane >> 4) ? (HH ? sc.w : sc.y) : (HH ? sc.z : sc.x);   // bytes 8HH + 4*(lane>>4) ..
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const int sl = 4 * (lane >> 4) + e;
            const float ds = d * (float)(int)(int8_t)(wsel >> (8 * e));
            scw[(sl * 8 + (r & 7)) * 2 + (r >> 3)] = ds * xinv[u * 8 + 4 * HH + (sl >> 1)];
        }
    }
    __syncwarp();
    const __half *xk = xb + u * 256 + 128 * HH;
#pragma unroll
    for (int sl = 0; sl < 8; sl++) {
        float d4[4] = {0.f, 0.f, 0.f, 0.f};
        uint32_t af[4], ah[4];
        nib_frag(word_of(sl < 4 ? q0 : q1, sl & 3), af);
        uint32_t hw = word_of(hq, sl >> 1);
        if (sl & 1) hw >>= 8;
        hi_frag(hw, ah);
        const uint2 bv = *reinterpret_cast<const uint2 *>(xk + 16 * sl);
        mma16816(d4, af, bv.x, bv.y);
        mma16816(d4, ah, bv.x, bv.y);
        const float2 sc2 = *reinterpret_cast<const float2 *>(scw + (sl * 8 + g) * 2);
        yg = fmaf(sc2.x, d4[0] + d4[1], yg);
        yg8 = fmaf(sc2.y, d4[2] + d4[3], yg8);
    }
    __syncwarp();
}

// One Q8_0 unit (16 rows x 32 codes) at T = 1, unit_compute_n's arithmetic with the block's scale
// multiplied by the activation block's inverse range scale.
XJ_DEV void mk_q80(const uint8_t *stage, int ui, int u, int lane, bool bcol, const __half *xb, const float *xinv,
                   float &yg, float &yg8) {
    using G = Geo<XJ_Q8_0>;
    const int g = lane >> 2;
    const uint8_t *qs = stage + ui * G::QB;
    const uint8_t *ds = stage + G::CU * G::QB + ui * G::DB;
    const uint4 q = *reinterpret_cast<const uint4 *>(qs + lane * 16);
    const float dv = lane < 16 ? h2f(*reinterpret_cast<const uint16_t *>(ds + lane * 2)) : 0.0f;
    const float iv = xinv[u];
    const float dg = __shfl_sync(0xffffffffu, dv, g) * iv, dg8 = __shfl_sync(0xffffffffu, dv, g + 8) * iv;
    float d4[4] = {0.f, 0.f, 0.f, 0.f};
    const int kb = u * 32;
#pragma unroll
    for (int e = 0; e < 2; e++) {
        uint32_t af[4];
        q8_frag(word_of(q, 2 * e), word_of(q, 2 * e + 1), af);
        uint2 bv = make_uint2(0u, 0u);
        if (bcol) bv = *reinterpret_cast<const uint2 *>(xb + kb + 16 * e);
        mma16816(d4, af, bv.x, bv.y);
    }
    yg = fmaf(dg, d4[0] + d4[1], yg);
    yg8 = fmaf(dg8, d4[2] + d4[3], yg8);
}

// One F16 unit (16 rows x 32 elements, the fp16 values are the A fragments) at T = 1: mk_q80 without
// the code conversion; the row-block scale (1 for F16, a power of two for BF16) times the activation
// block's inverse range scale.
XJ_DEV void mk_h32(const uint8_t *stage, int ui, int u, int lane, bool bcol, const __half *xb, const float *xinv,
                   float &yg, float &yg8) {
    using G = Geo<XJ_F16>;
    const int g = lane >> 2;
    const uint8_t *qs = stage + ui * G::QB;
    const uint8_t *ds = stage + G::CU * G::QB + ui * G::DB;
    const uint4 q0 = *reinterpret_cast<const uint4 *>(qs + lane * 16);
    const uint4 q1 = *reinterpret_cast<const uint4 *>(qs + 512 + lane * 16);
    const float dv = lane < 16 ? h2f(*reinterpret_cast<const uint16_t *>(ds + lane * 2)) : 0.0f;
    const float iv = xinv[u];
    const float dg = __shfl_sync(0xffffffffu, dv, g) * iv, dg8 = __shfl_sync(0xffffffffu, dv, g + 8) * iv;
    const uint32_t af[2][4] = {{q0.x, q0.y, q0.z, q0.w}, {q1.x, q1.y, q1.z, q1.w}};
    float d4[4] = {0.f, 0.f, 0.f, 0.f};
    const int kb = u * 32;
#pragma unroll
    for (int e = 0; e < 2; e++) {
        uint2 bv = make_uint2(0u, 0u);
        if (bcol) bv = *reinterpret_cast<const uint2 *>(xb + kb + 16 * e);
        mma16816(d4, af[e], bv.x, bv.y);
    }
    yg = fmaf(dg, d4[0] + d4[1], yg);
    yg8 = fmaf(dg8, d4[2] + d4[3], yg8);
}

// Global operands of a tile's epilogue, loaded when the tile starts so the load latency overlaps the
// tile's tensor-core work (threads tid < 16, one output row each).
constexpr int MK_KC = 4;   // longest causal conv the persistent kernel takes (the models' conv_k)
struct EpiPre {
    float y;                // EPI_ADD: current value of the output row
    float cs[MK_KC - 1];    // EPI_CONV: the channel's rolling state (kc - 1 values)
    float wc[MK_KC];        // EPI_CONV: the channel's kc conv weights
};

XJ_DEV void mk_epi_load(const MmaJob &jb, int tile, int tid, EpiPre &e) {
    const int row = tile * 16 + tid;
    if (tid >= 16 || row >= jb.w.N) return;
    if (jb.epi == EPI_ADD) e.y = __ldcg(jb.y + row);
    else if (jb.epi == EPI_CONV) {
        const int kc = jb.kc;
        const float *st = jb.conv_state + (size_t)row * (kc - 1);
        const float *wc = jb.conv_w + (size_t)row * kc;
#pragma unroll
        for (int k = 0; k < MK_KC - 1; k++) e.cs[k] = k < kc - 1 ? __ldcg(st + k) : 0.0f;
#pragma unroll
        for (int k = 0; k < MK_KC; k++) e.wc[k] = k < kc ? wc[k] : 0.0f;
    }
}

// Running greedy pick of one CTA over its LM-head tiles (warp 0): best value, runner-up, lowest index.
struct ArgRun {
    float b = -INFINITY, b2 = -INFINITY;
    int bi = 0x7fffffff;
};

// Epilogue of one 16-row tile from the per-warp partials red[warp][16] (fixed-order sum over warps).
XJ_DEV void mk_epilogue(const MmaJob &jb, int tile, const float *red, int tid, const EpiPre &e, ArgRun &ar) {
    const bool real = tile * 16 + (tid & 15) < jb.w.N;   // rows past N pad the last tile
    if (jb.epi == EPI_CONV) {
        if (tid < 16 && real) {
            const int ch = tile * 16 + tid, kc = jb.kc;
            float s = 0.0f;
#pragma unroll
            for (int w = 0; w < MK_CWARPS; w++) s += red[w * 16 + tid];
            float acc = 0.0f;
#pragma unroll
            for (int k = 0; k < MK_KC - 1; k++)
                if (k < kc - 1) acc = fmaf(e.cs[k], e.wc[k], acc);
            float wl = e.wc[0];
#pragma unroll
            for (int k = 1; k < MK_KC; k++)
                if (k == kc - 1) wl = e.wc[k];
            acc = fmaf(s, wl, acc);
            float *st = jb.conv_state + (size_t)ch * (kc - 1);
#pragma unroll
            for (int k = 0; k < MK_KC - 2; k++)
                if (k < kc - 2) st[k] = e.cs[k + 1];
            st[kc - 2] = s;
            jb.y[ch] = silu_f(acc);
        }
    } else if (jb.epi == EPI_ARGMAX) {
        if (tid < 32) {
            const int row = tid & 15;
            float s = 0.0f;
#pragma unroll
            for (int w = 0; w < MK_CWARPS; w++) s += red[w * 16 + row];
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
            // merge the tile into the CTA's running pick (same rule as argmax_final_dev)
            if (b > ar.b || (b == ar.b && bi < ar.bi)) { ar.b2 = fmaxf(fmaxf(ar.b, ar.b2), b2); ar.b = b; ar.bi = bi; }
            else ar.b2 = fmaxf(ar.b2, b);
        }
    } else if (tid < 16 && real) {
        float s = 0.0f;
#pragma unroll
        for (int w = 0; w < MK_CWARPS; w++) s += red[w * 16 + tid];
        jb.y[(size_t)tile * 16 + tid] = jb.epi == EPI_ADD ? e.y + s : jb.epi == MK_EPI_SILU ? silu_f(s) : s;
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
    // every global operand first (one memory round trip): q, k, the state row slice, v, gates
    const float qv = tid < S ? lda(x + hk * S + tid) : 0.0f;
    const float kv = (tid >= 256 && tid - 256 < S) ? lda(x + a.key_dim + hk * S + tid - 256) : 0.0f;
    float *M = a.ssm + ((size_t)hv * S + (act ? j : 0)) * S + qq * P;
    float row[P];
#pragma unroll
    for (int i = 0; i < P; i += 4) {
        float4 v4 = make_float4(0.f, 0.f, 0.f, 0.f);
        if (act) v4 = __ldcg(reinterpret_cast<const float4 *>(M + i));
        row[i] = v4.x; row[i + 1] = v4.y; row[i + 2] = v4.z; row[i + 3] = v4.w;
    }
    const float vj = act ? lda(x + 2 * a.key_dim + hv * S + j) : 0.0f;
    const float bb = lda(a.beta + hv), al = lda(a.alpha + hv), dt = a.dt[hv], Ah = a.A[hv];
    // L2 norms of q (threads 0..S-1) and k (threads 256..256+S-1), sums in double
    const double d = warp_sum_d(tid < 256 ? (double)qv * qv : (double)kv * kv);
    if (lane == 0) red[warp] = d;
    BarC::sync();
    double sq = 0, sk2 = 0;
    for (int w = 0; w < 8; w++) { sq += red[w]; sk2 += red[8 + w]; }
    if (tid < S) qs[tid] = qv * (1.0f / sqrtf((float)sq + a.eps));
    if (tid >= 256 && tid - 256 < S) ks[tid - 256] = kv * (1.0f / sqrtf((float)sk2 + a.eps));
    BarC::sync();
    if (act) {
        const float b = sigm_f(bb);
        const float g = softplus_f(al + dt) * Ah;
        const float eg = expf(g);
        float sk = 0.0f;
#pragma unroll
        for (int i = 0; i < P; i++) { row[i] *= eg; sk = fmaf(row[i], ks[qq * P + i], sk); }
#pragma unroll
        for (int o = TPR >> 1; o; o >>= 1) sk += __shfl_xor_sync(0xffffffffu, sk, o);
        const float delta = (vj - sk) * b;
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

// Cache positions per round of an attention item: the round's K and V rows (8 KB each) sit in the
// activation staging area, which is dead between matrix-vector phases.
template <typename KV> constexpr int mk_attn_pe() { return 8192 / (int)sizeof(KV); }
__host__ __device__ inline int mk_attn_rows(int D, int kvsz) { const int r = 8192 / kvsz / D; return r < 64 ? r : 64; }
// Bytes of the staging area an attention item uses (the rows, queries, scores, the new row, the
// rotation table; the split merge's weights fit in the rows' place).
__host__ __device__ inline int mk_attn_scratch(int group, int D, int kvsz) {
    return 16384 + 4 * (group * D + group * mk_attn_rows(D, kvsz) + 3 * D);
}
// Splits per KV head for n positions: one round per split while the items fit the grid.
XJ_DEV int mk_nsplit(int n, int D, int kvsz, int max_split) {
    const int P = mk_attn_rows(D, kvsz);
    int ns = (n + P - 1) / P;
    if (ns > max_split) ns = max_split;
    return ns < 1 ? 1 : ns;
}

XJ_DEV float kv_f(float v) { return v; }
XJ_DEV float kv_f(__half v) { return __half2float(v); }
template <typename KV> XJ_DEV KV kv_from(float v);
template <> XJ_DEV float kv_from<float>(float v) { return v; }
template <> XJ_DEV __half kv_from<__half>(float v) { return __float2half_rn(v); }

constexpr int MK_GQA = 8;    // query heads per KV head the persistent attention takes

// Work item (KV head kvh, split sp of nsplit): every query head of the GQA group over positions
// [sp*n/nsplit, (sp+1)*n/nsplit) of n = npast + 1, so the group's query heads share one read of each
// cached row. The round's cache rows are requested first; meanwhile warps 0..group-1 put the query
// heads and warp `group` the new K row through RMSNorm + NeoX RoPE (attn_prep_slot's arithmetic; the
// new K/V row enters the round's rows from there, rounded as the cache stores it, and the last split
// stores it at position npast). Per round: scores (warp per position, lanes over the head dim), the
// softmax statistics (warp per query head), then o = sum p v (thread per (head, dim)). One split writes
// the gated output directly; otherwise each split leaves (o, m, l) per query head and the last split of
// the KV head to finish merges them (acquire/release counter, core/xj_cpu.c:118-150).
template <typename KV, int DPL>
XJ_DEV void mk_attn_item(const AttnArgs &a, int n, int kvh, int sp, int nsplit, float *apart, int *acnt, float *scr,
                         int tid, unsigned long long *trow) {
    constexpr int PE = mk_attn_pe<KV>();
    constexpr int OPT = (MK_GQA * 32 * DPL + MK_CTHREADS - 1) / MK_CTHREADS;   // (head, dim) pairs per thread
    __shared__ float st_m[MK_GQA], st_l[MK_GQA], st_c[MK_GQA];
    __shared__ int s_last;
    const int D = a.D, group = a.H / a.Hkv, lane = tid & 31, warp = tid >> 5;
    const int P = mk_attn_rows(D, (int)sizeof(KV)), kvd = a.Hkv * D;
    KV *sk = reinterpret_cast<KV *>(scr);                       // [P][D]
    KV *sv = reinterpret_cast<KV *>(reinterpret_cast<uint8_t *>(scr) + 8192);
    float *rq = scr + 4096;                                     // [group][D] normed + rotated queries
    float *ps = rq + group * D;                                 // [group][P] scores, then probabilities
    float *rkn = ps + group * P;                                // [D] the new K row (normed, then rotated)
    float *rvn = rkn + D;                                       // [D] the new V row
    const int pos = n - 1;
    if (trow) trow[5] = globaltimer();
    const int j0 = (int)((long long)sp * n / nsplit), j1 = (int)((long long)(sp + 1) * n / nsplit);
    const float scale = 1.0f / sqrtf((float)D);
    const KV *kc = (const KV *)a.kc + (size_t)kvh * D, *vc = (const KV *)a.vc + (size_t)kvh * D;
    // this thread's (head, dim) pairs: gates and running outputs
    float gate[OPT], o[OPT];
#pragma unroll
    for (int k = 0; k < OPT; k++) {
        const int t = tid + k * MK_CTHREADS, hq = t / D, d = t - hq * D;
        gate[k] = hq < group ? lda(a.q + (size_t)(kvh * group + hq) * 2 * D + D + d) : 0.0f;
        o[k] = 0.0f;
    }
    if (tid < MK_GQA) { st_m[tid] = -INFINITY; st_l[tid] = 0.0f; }
    for (int r0 = j0; r0 < j1; r0 += P) {
        const int np = j1 - r0 < P ? j1 - r0 : P;
        // the round's cached rows straight into shared memory (16-byte asynchronous copies, 8 elements
        // per piece for fp16), all requested before any use
        const int nchunk = np * D / 8;
        for (int c = tid; c < nchunk; c += MK_CTHREADS) {
            const int e = c * 8, j = e / D, d = e - j * D;
            if (r0 + j == pos) continue;
#pragma unroll
            for (int i = 0; i < (int)sizeof(KV) / 2; i++) {
                cp_async16(reinterpret_cast<uint4 *>(sk + e) + i, reinterpret_cast<const uint4 *>(kc + (size_t)(r0 + j) * kvd + d) + i);
                cp_async16(reinterpret_cast<uint4 *>(sv + e) + i, reinterpret_cast<const uint4 *>(vc + (size_t)(r0 + j) * kvd + d) + i);
            }
        }
        cp_async_commit();
        if (r0 == j0) {
            // query heads (warps < group) and the new K row (warp group): RMSNorm, then NeoX RoPE with
            // the rotation table (cos, sin of every pair) computed once per item by threads p < n_rot/2
            const int half = a.n_rot / 2;
            float *tab = rvn + D;                                   // [half][2]
            for (int p = tid; p < half; p += MK_CTHREADS) {
                const float theta = (float)pos * powf(a.base, -2.0f * (float)p / (float)a.n_rot);
                tab[2 * p] = cosf(theta);
                tab[2 * p + 1] = sinf(theta);
            }
            const bool isq = warp < group;
            float *buf = isq ? rq + warp * D : rkn;
            if (warp <= group) {
                const float *src = isq ? a.q + (size_t)(kvh * group + warp) * 2 * D : a.k + (size_t)kvh * D;
                const float *nw = isq ? a.qn : a.kn;
                float x[8];
                double ssq = 0.0;
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    const int i = lane + 32 * e;
                    x[e] = i < D ? lda(src + i) : 0.0f;
                    ssq += (double)x[e] * x[e];
                }
                ssq = warp_sum_d(ssq);
                const float sc = 1.0f / sqrtf((float)(ssq / D) + a.eps);
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    const int i = lane + 32 * e;
                    if (i < D) buf[i] = x[e] * sc * nw[i];
                }
            }
            BarC::sync();
            if (trow) trow[6] = globaltimer();
            if (warp <= group) {
                // each lane rotates whole pairs (p, p + half) in place
                for (int p = lane; p < half; p += 32) {
                    const float c = tab[2 * p], sn = tab[2 * p + 1];
                    const float x0 = buf[p], x1 = buf[p + half];
                    buf[p] = x0 * c - x1 * sn;
                    buf[p + half] = x0 * sn + x1 * c;
                }
                if (!isq && sp == nsplit - 1) {
                    __syncwarp();
                    const bool mine = pos < r0 + P;     // the new row is in this round
                    for (int i = lane; i < D; i += 32) {
                        const float kr0 = rkn[i], vv = lda(a.v + (size_t)kvh * D + i);
                        rvn[i] = vv;
                        const size_t og = (size_t)pos * kvd + (size_t)kvh * D + i;
                        store_kv<KV>((KV *)a.kc + og, kr0);
                        store_kv<KV>((KV *)a.vc + og, vv);
                        if (mine) { sk[(pos - r0) * D + i] = kv_from<KV>(kr0); sv[(pos - r0) * D + i] = kv_from<KV>(vv); }
                    }
                }
            }
        }
        if (r0 != j0 && pos >= r0 && pos < r0 + np)
            // the new row in a later round of the last split (round j0 had it from the RoPE warp)
            for (int i = tid; i < D; i += MK_CTHREADS) {
                sk[(pos - r0) * D + i] = kv_from<KV>(rkn[i]);
                sv[(pos - r0) * D + i] = kv_from<KV>(rvn[i]);
            }
        cp_async_wait_all();
        BarC::sync();
        if (trow && r0 == j0) trow[8] = globaltimer();
        // scores: warp w takes positions w, w + 16, ...; lanes DPL consecutive dims
        for (int j = warp; j < np; j += MK_CWARPS) {
            float kv[DPL];
#pragma unroll
            for (int e = 0; e < DPL; e++) {
                const int i = lane * DPL + e;
                kv[e] = i < D ? kv_f(sk[j * D + i]) : 0.0f;
            }
            for (int h0 = 0; h0 < group; h0 += 4) {   // four query heads' reductions interleaved
                float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                for (int e = 0; e < DPL; e++) {
                    const int i = lane * DPL + e;
#pragma unroll
                    for (int q = 0; q < 4; q++)
                        if (h0 + q < group && i < D) acc[q] = fmaf(rq[(h0 + q) * D + i], kv[e], acc[q]);
                }
#pragma unroll
                for (int q = 0; q < 4; q++)
                    if (h0 + q < group) {
                        const float sc = warp_sum(acc[q]) * scale;
                        if (lane == 0) ps[(h0 + q) * P + j] = sc;
                    }
            }
        }
        BarC::sync();
        // softmax statistics of the round per query head (warp hq), probabilities in place
        if (warp < group) {
            float s0 = lane < np ? ps[warp * P + lane] : -INFINITY;
            float s1 = lane + 32 < np ? ps[warp * P + lane + 32] : -INFINITY;
            const float mr = warp_max(fmaxf(s0, s1)), mo = st_m[warp], mn = fmaxf(mo, mr);
            const float p0 = lane < np ? expf(s0 - mn) : 0.0f, p1 = lane + 32 < np ? expf(s1 - mn) : 0.0f;
            if (lane < np) ps[warp * P + lane] = p0;
            if (lane + 32 < np) ps[warp * P + lane + 32] = p1;
            const float psum = warp_sum(p0 + p1);
            const float corr = mo == -INFINITY ? 0.0f : expf(mo - mn);
            __syncwarp();
            if (lane == 0) { st_c[warp] = corr; st_l[warp] = st_l[warp] * corr + psum; st_m[warp] = mn; }
        }
        BarC::sync();
#pragma unroll
        for (int k = 0; k < OPT; k++) {
            const int t = tid + k * MK_CTHREADS, hq = t / D, d = t - hq * D;
            if (hq >= group) continue;
            float acc = o[k] * st_c[hq];
            for (int j = 0; j < np; j++) acc = fmaf(ps[hq * P + j], kv_f(sv[j * D + d]), acc);
            o[k] = acc;
        }
        BarC::sync();   // the round's rows and scores are overwritten by the next round
    }
    const size_t hstride = (size_t)nsplit * (D + 2);
    if (trow) trow[9] = globaltimer();
    if (nsplit == 1) {
#pragma unroll
        for (int k = 0; k < OPT; k++) {
            const int t = tid + k * MK_CTHREADS, hq = t / D, d = t - hq * D;
            if (hq < group) a.out[(size_t)(kvh * group + hq) * D + d] = (o[k] / st_l[hq]) * sigm_f(gate[k]);
        }
        BarC::sync();   // the statistics are reset by the next item
        return;
    }
#pragma unroll
    for (int k = 0; k < OPT; k++) {
        const int t = tid + k * MK_CTHREADS, hq = t / D, d = t - hq * D;
        if (hq < group) {
            float *part = apart + (size_t)(kvh * group + hq) * hstride + (size_t)sp * (D + 2);
            part[d] = o[k];
            if (d == 0) { part[D] = st_m[hq]; part[D + 1] = st_l[hq]; }
        }
    }
    BarC::sync();
    if (tid == 0) {
        // release: the CTA's partials (ordered before this by the barrier); acquire: the other splits'
        int old;
        asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(old) : "l"(acnt + kvh) : "memory");
        s_last = old == nsplit - 1;
        if (trow) trow[10] = globaltimer();
    }
    BarC::sync();
    if (!s_last) return;
    // merge: per query head (warp hq, lanes over splits) the weights c_s = exp(m_s - M) and L from one
    // read of every split's (m, l); then o = sum_s c_s o_s / L by (head, dim) thread
    float *cs = scr;                     // [group][nsplit]
    if (warp < group) {
        const float *p0 = apart + (size_t)(kvh * group + warp) * hstride;
        float mv[MK_MAX_SPLIT / 32], lv[MK_MAX_SPLIT / 32];
        float M = -INFINITY;
#pragma unroll
        for (int k = 0; k < MK_MAX_SPLIT / 32; k++) {
            const int s_ = lane + 32 * k;
            mv[k] = s_ < nsplit ? __ldcg(p0 + (size_t)s_ * (D + 2) + D) : -INFINITY;
            lv[k] = s_ < nsplit ? __ldcg(p0 + (size_t)s_ * (D + 2) + D + 1) : 0.0f;
            M = fmaxf(M, mv[k]);
        }
        M = warp_max(M);
        float L = 0.0f;
#pragma unroll
        for (int k = 0; k < MK_MAX_SPLIT / 32; k++) {
            const int s_ = lane + 32 * k;
            if (s_ < nsplit) {
                const float c = expf(mv[k] - M);
                cs[warp * nsplit + s_] = c;
                L = fmaf(lv[k], c, L);
            }
        }
        L = warp_sum(L);
        if (lane == 0) st_l[warp] = L;
    }
    BarC::sync();
#pragma unroll
    for (int k = 0; k < OPT; k++) {
        const int t = tid + k * MK_CTHREADS, hq = t / D, d = t - hq * D;
        if (hq >= group) continue;
        const float *p0 = apart + (size_t)(kvh * group + hq) * hstride;
        float acc = 0.0f;
#pragma unroll 4
        for (int s_ = 0; s_ < nsplit; s_++) acc = fmaf(cs[hq * nsplit + s_], __ldcg(p0 + (size_t)s_ * (D + 2) + d), acc);
        a.out[(size_t)(kvh * group + hq) * D + d] = (acc / st_l[hq]) * sigm_f(gate[k]);
    }
    if (tid == 0) { atomicExch(acnt + kvh, 0); if (trow) trow[11] = globaltimer(); }
    BarC::sync();   // scratch is reused by the next item
}

template <typename KV>
XJ_DEV void mk_attn_phase(const MkArgs &A, const AttnArgs &a, int n, float *scr, int tid, unsigned long long *trow) {
    if (trow)
        for (int i = 5; i < 12; i++) trow[i] = 0;
    const int nsplit = mk_nsplit(n, a.D, (int)sizeof(KV), A.max_split);
    const int items = a.Hkv * nsplit;
    for (int it = blockIdx.x; it < items; it += gridDim.x) {
        const int kvh = it / nsplit, sp = it % nsplit;
        // lanes take DPL consecutive dims of the head (DPL * 32 >= D; dims past D are masked)
        if (a.D <= 64) mk_attn_item<KV, 2>(a, n, kvh, sp, nsplit, A.apart, A.acnt, scr, tid, it == (int)blockIdx.x ? trow : nullptr);
        else if (a.D <= 128) mk_attn_item<KV, 4>(a, n, kvh, sp, nsplit, A.apart, A.acnt, scr, tid, it == (int)blockIdx.x ? trow : nullptr);
        else mk_attn_item<KV, 8>(a, n, kvh, sp, nsplit, A.apart, A.acnt, scr, tid, it == (int)blockIdx.x ? trow : nullptr);
    }
}

template <int S>
XJ_DEV void mk_gdn_phase(const GdnArgs &a, float *scr, int tid) {
    const int items = a.Hv * GdnGeo<S>::IPH;
    for (int it = blockIdx.x; it < items; it += gridDim.x) mk_gdn_item<S>(a, it, scr, tid);
}

// The SAMPLE phase on CTA 0's compute warps: k_sample_final's pick with 512 threads, its sampler state
// in the activation staging area and the scale scratch after it (dead outside matrix-vector phases).
constexpr size_t MK_SCRATCH_BYTES = MK_XS_BYTES + 2 * (MK_KMAX / 32) * 4 + MK_CWARPS * 128 * 4 + MK_NR * MK_CWARPS * 16 * 4;
static_assert(sizeof(SampleSmem) <= MK_SCRATCH_BYTES, "the sampler state fits the phase scratch");
XJ_DEV void mk_sample_phase(const SampleArgs &a, const ArgmaxArgs &g, SampleSmem &S, int tid) {
    const int pos = ld_volatile(g.npast);
    float mg = 0.0f;
    const int id = sample_row_dev<BarC>(a.logits, a.n, a.temp, a.top_k, a.top_p, sample_uniform(a.seed, (unsigned long long)pos),
                                        S, tid, MK_CTHREADS, &mg);
    if (tid == 0) {
        const int s = *g.step;
        g.out_tok[s] = id;
        if (g.margin) g.margin[s] = mg;
        *g.cur = id;
        *g.step = s + 1;
        *g.npast = pos + 1;
    }
    const DevMat &emb = g.emb;
    for (int e0 = tid * 8; e0 < emb.K; e0 += MK_CTHREADS * 8) {
        float y[8];
        if (id >= 0 && id < emb.N) dequant8(emb.type, emb.p + id * emb.ld, e0, y);
        else {
#pragma unroll
            for (int l = 0; l < 8; l++) y[l] = 0.0f;
        }
#pragma unroll
        for (int l = 0; l < 8; l++) g.x[e0 + l] = y[l];
    }
}

// ------------------------------------------------------------------ the kernel
// FULL: the Q5_K / F16 / Q8_0 unit code, the SAMPLE phase and the phase trace are compiled in. The lean
// variant (Q4_K and Q6_K matrices, the greedy pick, no trace) is what a Q4_K_M model decodes with: the
// extra code in the unit loop and the phase switch measurably slows the whole step even where it never
// runs.
template <bool FULL>
__global__ void __launch_bounds__(MK_THREADS, 1) k_decode_persistent(MkArgs A) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t full[MK_NS], empty[MK_NS];
    __shared__ __align__(8) uint64_t rfull[MK_NR], rfree[MK_NR];   // tile partials: ready / consumed
    __shared__ unsigned s_issued;
    __shared__ MkPhase sph[2];     // consumers: this phase's descriptor and the next one (prefetched)
    __shared__ MkStream sst[2];    // producer: same for its GEMV stream
    uint8_t *ring = smem;
    __half *xs = reinterpret_cast<__half *>(smem + (size_t)MK_NS * MK_SLOT);
    float *xsum = reinterpret_cast<float *>(smem + (size_t)MK_NS * MK_SLOT + MK_XS_BYTES);
    float *xinv = xsum + MK_KMAX / 32;   // per 32-element activation block: 1 / its range scale
    float *scs = xinv + MK_KMAX / 32;
    float *red = scs + MK_CWARPS * 128;
    float *scr = reinterpret_cast<float *>(xs);     // GDN / attention scratch (xs is dead between GEMVs)
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, cta = blockIdx.x;
    if (tid == 0) {
        for (int s = 0; s < MK_NS; s++) { mbar_init(&full[s], 1); mbar_init(&empty[s], MK_CWARPS); }
        for (int s = 0; s < MK_NR; s++) { mbar_init(&rfull[s], MK_CWARPS); mbar_init(&rfree[s], 1); }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        s_issued = 0;
    }
    __syncthreads();
    unsigned consumed = 0, drain_from = 0xffffffffu;

    if (warp == MK_CWARPS) {
        // ---------------- producer: this CTA's weight chunks of every GEMV phase, in program order
        copy_desc_async(&sst[0], &A.stream[0], (int)sizeof(MkStream), lane);
        cp_async_wait_all();
        __syncwarp();
        unsigned i = 0;
        int gk = 0;                 // GEMV phases streamed so far
        bool ok = true;
        for (int step = 0; ok && step < A.nsteps; step++)
            for (int k = 0; ok && k < A.nstream; k++, gk++) {
                const MkStream &S = sst[gk & 1];
                const int kn = k + 1 < A.nstream ? k + 1 : 0;
                copy_desc_async(&sst[(gk + 1) & 1], &A.stream[kn], (int)sizeof(MkStream), lane);
                unsigned long long *trp = FULL && A.trace && step == A.nsteps - 1 ? A.trace + ((size_t)cta * A.nphase + S.ph) * 12 : nullptr;
                if (lane < 6 && S.pf[lane]) {
                    // this CTA's slice of the side-data range (16-byte granules)
                    const unsigned bytes = S.pf_bytes[lane];
                    const unsigned chunk = ((bytes + G - 1) / G + 15u) & ~15u, off = (unsigned)cta * chunk;
                    if (off < bytes) prefetch_l2(S.pf[lane] + off, bytes - off < chunk ? bytes - off : chunk);
                }
                if (lane == 0) {
                    for (int tg = cta; ok && tg < S.ntiles; tg += G) {
                        int j = 0;
                        while (j + 1 < S.njob && tg >= S.tile_start[j + 1]) j++;
                        const int type = S.type[j], nu = S.nu[j];
                        const int tile = tg - S.tile_start[j], CU = mk_cu(type);
                        for (int u0 = 0; u0 < nu; u0 += CU, i++) {
                            const int slot = i % MK_NS;
                            if (i >= MK_NS && !mk_wait(&empty[slot], ((i / MK_NS) - 1) & 1, A.err, 1, A.diag, step, k, (int)i, 128)) { ok = false; break; }
                            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                            const int cu = nu - u0 < CU ? nu - u0 : CU;
                            uint8_t *st = ring + (size_t)slot * MK_SLOT;
                            if (type == XJ_Q4_K) mk_issue_t<XJ_Q4_K>(S, j, tile, u0, cu, st, &full[slot]);
                            else if (type == XJ_Q6_K) mk_issue_t<XJ_Q6_K>(S, j, tile, u0, cu, st, &full[slot]);
                            else if (FULL && type == XJ_Q5_K) mk_issue_t<XJ_Q5_K>(S, j, tile, u0, cu, st, &full[slot]);
                            else if (FULL && type == XJ_F16) mk_issue_t<XJ_F16>(S, j, tile, u0, cu, st, &full[slot]);
                            else if (FULL) mk_issue_t<XJ_Q8_0>(S, j, tile, u0, cu, st, &full[slot]);
                            *(volatile unsigned *)&s_issued = i + 1;
                            if (trp) {
                                const unsigned long long now = globaltimer();
                                if (tg == cta && u0 == 0) trp[3] = now;
                                trp[4] = now;
                            }
                        }
                    }
                }
                ok = __shfl_sync(0xffffffffu, ok, 0);
                cp_async_wait_all();
                __syncwarp();
            }
        cp_async_wait_all();
        __syncwarp();
    } else {
        // ---------------- compute warps (warp < MK_CWARPS) and the epilogue warp (warp == MK_EWARP)
        // Per tile the compute warps leave their partial rows in one of MK_NR buffers and go on to the
        // next tile; the epilogue warp sums the partials (fixed warp order), applies the epilogue and
        // hands the buffer back. So no CTA-wide barrier separates the tiles of a phase.
        const bool ew = warp == MK_EWARP;
        const int g = lane >> 2, c = lane & 3;
        float *scw = scs + (ew ? 0 : warp) * 128;
        unsigned nbar = 0, ntile = 0;   // ntile: GEMV tiles of this CTA so far (counted alike by both roles)
        int attn_n0 = -1;               // attention: positions at step 0 (npast + 1), once read
        int gp = 0;                 // gp: phases run so far (selects the descriptor buffer)
        if (!ew) copy_desc_async(&sph[0], &A.prog[0], (int)sizeof(MkPhase), tid);
        cp_async_wait_all();
        BarP::sync();
        for (int step = 0; step < A.nsteps; step++) {
            bool ok = true;
            for (int ph = 0; ph < A.nphase; ph++, gp++) {
                const MkPhase &p = sph[gp & 1];
                const int pn = ph + 1 < A.nphase ? ph + 1 : 0;
                if (!ew) copy_desc_async(&sph[(gp + 1) & 1], &A.prog[pn], (int)sizeof(MkPhase), tid);
                const bool last_step = FULL && A.trace && step == A.nsteps - 1;   // tracing: the full variant
                const bool tr = last_step && tid == 0, tre = last_step && tid == MK_EWARP * 32;
                unsigned long long *trow = FULL && A.trace ? A.trace + ((size_t)cta * A.nphase + ph) * 12 : nullptr;
                unsigned long long wait_ns = 0;
                if (tr) trow[0] = globaltimer();
                if (p.op == MK_GEMV && cta < p.ntiles && ew) {
                    // ---- epilogues of this CTA's tiles, in the compute warps' order
                    ArgRun ar;
                    int ntile_done = 0;
                    for (int tg = cta; tg < p.ntiles; tg += G, ntile++, ntile_done++) {
                        const int j = mk_job_of(p, tg);
                        const MmaJob &jb = p.job[j];
                        const int tile = tg - p.tile_start[j];
                        EpiPre e;
                        mk_epi_load(jb, tile, lane, e);    // overlaps the wait for the partials
                        const int b = (int)(ntile % MK_NR);
                        if (!mk_wait(&rfull[b], (ntile / MK_NR) & 1, A.err, 3, A.diag, step, ph, (int)ntile, 32)) continue;
                        if (tre && ntile_done == 0) trow[10] = globaltimer();
                        mk_epilogue(jb, tile, red + b * (MK_CWARPS * 16), lane, e, ar);
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&rfree[b]);
                        if (tre && ntile_done == 0) { trow[11] = globaltimer(); trow[6] = trow[11]; }
                    }
                    if (lane == 0 && p.job[0].epi == EPI_ARGMAX) {
                        // one greedy-pick partial per CTA (CTA c holds tiles c, c + G, ...)
                        p.job[0].pbest[cta] = ar.b; p.job[0].psecond[cta] = ar.b2; p.job[0].pidx[cta] = ar.bi;
                    }
                } else if (p.op == MK_GEMV && cta < p.ntiles) {
                    mk_prologue(p, xs, xsum, xinv, tid);
                    if (tr) trow[5] = globaltimer();
                    int ntile_done = 0;
                    const int xstride = p.K + 16;
                    const bool bcol = g < 2;
                    const __half *xb = xs + (size_t)g * xstride + 4 * c;
                    const __half *xb2 = xs + (size_t)(g & 1) * xstride + 4 * c;   // always a staged column
                    for (int tg = cta; tg < p.ntiles; tg += G, ntile++, ntile_done++) {
                        const int j = mk_job_of(p, tg);
                        const Tiled &W = p.job[j].w;
                        const int CU = mk_cu(W.type);
                        float yg = 0.0f, yg8 = 0.0f;
                        for (int u0 = 0; u0 < W.nu; u0 += CU, consumed++) {
                            const int slot = consumed % MK_NS;
                            const unsigned long long w0 = tr ? globaltimer() : 0;
                            const bool got = mk_wait(&full[slot], (consumed / MK_NS) & 1, A.err, 1, A.diag, step, ph, (int)consumed, 32);
                            if (tr) { const unsigned long long w1 = globaltimer(); wait_ns += w1 - w0; if (ntile_done == 0 && u0 == 0) trow[8] = w1; }
                            const uint8_t *st = ring + (size_t)slot * MK_SLOT;
                            const int cu = W.nu - u0 < CU ? W.nu - u0 : CU;
                            if (W.type == XJ_Q4_K) {
                                const int ui = warp >> 1;
                                if (ui < cu) {
                                    if (warp & 1) mk_q4k<1>(st, ui, u0 + ui, lane, xb2, xsum, xinv, scw, yg, yg8);
                                    else mk_q4k<0>(st, ui, u0 + ui, lane, xb2, xsum, xinv, scw, yg, yg8);
                                }
                            } else if (W.type == XJ_Q6_K) {
                                const int ui = warp >> 1;
                                if (ui < cu) {
                                    if (warp & 1) mk_q6k<1>(st, ui, u0 + ui, lane, xb2, xinv, scw, yg, yg8);
                                    else mk_q6k<0>(st, ui, u0 + ui, lane, xb2, xinv, scw, yg, yg8);
                                }
                            } else if (FULL && W.type == XJ_Q5_K) {
                                const int ui = warp >> 1;
                                if (ui < cu) {
                                    if (warp & 1) mk_q5k<1>(st, ui, u0 + ui, lane, xb2, xsum, xinv, scw, yg, yg8);
                                    else mk_q5k<0>(st, ui, u0 + ui, lane, xb2, xsum, xinv, scw, yg, yg8);
                                }
                            } else if (FULL && W.type == XJ_F16) {
                                static_assert(Geo<XJ_F16>::CU == MK_CWARPS, "one F16 unit per warp");
                                if (warp < cu) mk_h32(st, warp, u0 + warp, lane, bcol, xb, xinv, yg, yg8);
                            } else if (FULL) {
#pragma unroll
                                for (int k = 0; k < Geo<XJ_Q8_0>::CU / MK_CWARPS; k++) {
                                    const int ui = warp + k * MK_CWARPS;
                                    if (ui < cu) mk_q80(st, ui, u0 + ui, lane, bcol, xb, xinv, yg, yg8);
                                }
                            }
                            __syncwarp();
                            if (lane == 0 && got) mbar_arrive(&empty[slot]);
                            if (!got && drain_from == 0xffffffffu) drain_from = consumed;
                        }
                        // hand the tile's partial rows to the epilogue warp (its buffer free again first)
                        const int b = (int)(ntile % MK_NR);
                        if (ntile >= MK_NR && lane == 0)
                            mk_wait(&rfree[b], ((ntile / MK_NR) - 1) & 1, A.err, 3, A.diag, step, ph, (int)ntile, 32);
                        __syncwarp();
                        float *rr = red + b * (MK_CWARPS * 16);
                        if (c == 0) { rr[warp * 16 + g] = yg; rr[warp * 16 + g + 8] = yg8; }
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&rfull[b]);
                        if (tr && ntile_done == 0) trow[9] = globaltimer();
                    }
                    if (tr) trow[7] = ntile_done;
                } else if (!ew && p.op == MK_GDN) {
                    switch (p.gs) {
                    case 16: mk_gdn_phase<16>(p.gdn, scr, tid); break;
                    case 32: mk_gdn_phase<32>(p.gdn, scr, tid); break;
                    case 64: mk_gdn_phase<64>(p.gdn, scr, tid); break;
                    case 128: mk_gdn_phase<128>(p.gdn, scr, tid); break;
                    case 256: mk_gdn_phase<256>(p.gdn, scr, tid); break;
                    default: break;
                    }
                } else if (!ew && p.op == MK_ATTN) {
                    // positions attended: read once per launch (every step adds one)
                    if (attn_n0 < 0) attn_n0 = __ldcg(p.attn.npast) + 1 - step;
                    if (A.kv_f32) mk_attn_phase<float>(A, p.attn, attn_n0 + step, scr, tid, tr ? trow : nullptr);
                    else mk_attn_phase<__half>(A, p.attn, attn_n0 + step, scr, tid, tr ? trow : nullptr);
                } else if (!ew && p.op == MK_ARGMAX) {
                    if (cta == 0) argmax_final_dev<BarC>(p.am, tid, MK_CTHREADS);
                } else if (FULL && !ew && p.op == MK_SAMPLE) {
                    if (cta == 0) mk_sample_phase(p.sa, p.am, *reinterpret_cast<SampleSmem *>(xs), tid);
                }
                if (tr) {
                    trow[1] = globaltimer();
                    trow[2] = wait_ns;
                }
                cp_async_wait_all();   // the next descriptor has landed (visible after the barrier below)
                if (step == A.nsteps - 1 && ph == A.nphase - 1) break;
                nbar++;
                if (!mk_grid_sync(A.bar, nbar * (unsigned)G, A.err, tid, A.diag, step, ph)) { ok = false; break; }
            }
            if (!ok) break;
        }
        cp_async_wait_all();
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
