// Layer kernels of the xj CUDA backend (everything except the fast GEMV paths, gemv_mma.cuh).
//
// Token positions are read from device memory (*npast), so a decode step does not depend on any
// host-side scalar and can be captured once as a CUDA graph and replayed.
#pragma once
#include "common.cuh"

namespace xjk {

// Kernels in this header have internal linkage (static): each translation unit that includes it
// gets its own copies. Programmatic dependent launch: every kernel waits for its stream predecessor's results before
// touching activations or state (a no-op when launched without the programmatic attribute).
XJ_DEV void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
XJ_DEV void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" :::); }

constexpr int MAXT = 16;   // tokens per forward handled by the CUDA-core GEMV

// Barriers for the device functions below: the whole block (standalone kernels), or a named
// barrier over the first N threads (the persistent decode kernel, whose last warp streams weights).
struct BarBlock { XJ_DEV static void sync() { __syncthreads(); } };
template <int ID, int N> struct BarNamed {
    XJ_DEV static void sync() { asm volatile("bar.sync %0, %1;" :: "n"(ID), "n"(N) : "memory"); }
};

// Sum over nthr threads (tid < nthr) in double; `red` holds one double per warp. All get the result.
template <class Bar>
XJ_DEV double group_sum_d(double v, double *red, int tid, int nthr) {
    const int lane = tid & 31, w = tid >> 5, nw = (nthr + 31) >> 5;
    v = warp_sum_d(v);
    Bar::sync();
    if (lane == 0) red[w] = v;
    Bar::sync();
    double t = 0;
    for (int i = 0; i < nw; i++) t += red[i];
    return t;
}

// Activations written by other blocks are read through L2 only (never a stale L1 line).
XJ_DEV float lda(const float *p) { return __ldcg(p); }

// ---------------------------------------------------------------- dequant / embed
// out[r][K] = rows [row0, row0+nrows) of W in fp32 (bit-exact with core/xj_quant.h).
static __global__ void k_dequant(DevMat w, int row0, int nrows, float *out) {
    griddep_wait();
    const long long total = (long long)nrows * (w.K / 8);
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const int r = (int)(i / (w.K / 8)), e0 = (int)(i % (w.K / 8)) * 8;
        float y[8];
        dequant8(w.type, w.p + (row0 + r) * w.ld, e0, y);
        float *o = out + (size_t)r * w.K + e0;
#pragma unroll
        for (int l = 0; l < 8; l++) o[l] = y[l];
    }
}

// x[t] = row tok[t] of the embedding table; out-of-range ids give zeros (core/xj_cpu.c:369-373).
static __global__ void k_embed(DevMat w, const int32_t *tok, int T, float *x, int ldx) {
    griddep_wait();
    griddep_launch();   // successors may start their prologue; they wait for this grid before reading
    const int t = blockIdx.y;
    if (t >= T) return;
    const int id = tok[t];
    for (int e0 = (blockIdx.x * blockDim.x + threadIdx.x) * 8; e0 < w.K; e0 += gridDim.x * blockDim.x * 8) {
        float y[8];
        if (id >= 0 && id < w.N) dequant8(w.type, w.p + id * w.ld, e0, y);
        else {
#pragma unroll
            for (int l = 0; l < 8; l++) y[l] = 0.0f;
        }
#pragma unroll
        for (int l = 0; l < 8; l++) x[(size_t)t * ldx + e0 + l] = y[l];
    }
}

// ---------------------------------------------------------------- norms
// y[r] = x[r] * w / sqrt(mean(x[r]^2) + eps), sum in double (core/xj_cpu.c:56-61). One block per row.
static __global__ void k_rmsnorm(const float *x, long long ldx, const float *w, float *y, long long ldy, int n, float eps) {
    griddep_wait();
    griddep_launch();   // successors may start their prologue; they wait for this grid before reading
    __shared__ double red[32];
    const float *xr = x + blockIdx.x * ldx;
    float *yr = y + blockIdx.x * ldy;
    double ss = 0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss += (double)xr[i] * xr[i];
    ss = block_sum_d(ss, red);
    const float sc = 1.0f / sqrtf((float)(ss / n) + eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x) yr[i] = xr[i] * sc * (w ? w[i] : 1.0f);
}

// ---------------------------------------------------------------- generic GEMV
// y[t][r] (+)= dot(W[r], x[t]) for up to 4 matrices sharing the input x[T][K]: one warp per row,
// each lane dequantises 8 consecutive elements at a time with the reference formulas and keeps T fp32
// partial sums. Used for every type when XJC_OPT_GEMV=1 and for the small/odd types otherwise.
struct GemvJob {
    DevMat w;
    float *y;
    long long ldy;       // floats between tokens in y
    int accumulate;      // y += W x (residual add, core/xj_cpu.c:268,275)
};
struct GemvArgs {
    GemvJob job[4];
    int njob;
    int row_start[5];    // prefix sums of rows over jobs
    const float *x;
    long long ldx;
    int T;
};

static __global__ void __launch_bounds__(256) k_gemv_generic(GemvArgs a) {
    griddep_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int grow = blockIdx.x * 8 + warp;
    if (grow >= a.row_start[a.njob]) return;
    int j = 0;
    while (grow >= a.row_start[j + 1]) j++;
    const GemvJob &jb = a.job[j];
    const int r = grow - a.row_start[j];
    const int K = jb.w.K, T = a.T;
    const uint8_t *row = jb.w.p + r * jb.w.ld;
    float acc[MAXT];
#pragma unroll
    for (int t = 0; t < MAXT; t++) acc[t] = 0.0f;
    for (int e0 = lane * 8; e0 < K; e0 += 256) {
        float wv[8];
        dequant8(jb.w.type, row, e0, wv);
#pragma unroll
        for (int t = 0; t < MAXT; t++) {
            if (t < T) {
                const float4 *xp = reinterpret_cast<const float4 *>(a.x + t * a.ldx + e0);
                float4 x0 = __ldg(xp), x1 = __ldg(xp + 1);
                float s = acc[t];
                s = fmaf(wv[0], x0.x, s); s = fmaf(wv[1], x0.y, s); s = fmaf(wv[2], x0.z, s); s = fmaf(wv[3], x0.w, s);
                s = fmaf(wv[4], x1.x, s); s = fmaf(wv[5], x1.y, s); s = fmaf(wv[6], x1.z, s); s = fmaf(wv[7], x1.w, s);
                acc[t] = s;
            }
        }
    }
#pragma unroll
    for (int t = 0; t < MAXT; t++) {
        if (t < T) {
            float s = warp_sum(acc[t]);
            if (lane == 0) {
                float *yp = jb.y + t * jb.ldy + r;
                *yp = jb.accumulate ? *yp + s : s;
            }
        }
    }
}

// ---------------------------------------------------------------- Gated DeltaNet
// Causal depthwise conv (kernel KC) with a rolling state, then SiLU, in place on qkv[T][CD]
// (core/xj_cpu.c:172-182). One thread per channel, tokens in order. With ck != nullptr the state
// after token t (t < T-1) is saved to ck[t][CD][KC-1] (core/xj_cpu.c:220).
static __global__ void k_conv_silu(float *qkv, long long ldq, int T, int CD, int KC, float *state, const float *cw, float *ck) {
    griddep_wait();
    griddep_launch();   // successors may start their prologue; they wait for this grid before reading
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= CD) return;
    float cs[8];
    const float *wc = cw + (size_t)c * KC;
    for (int k = 0; k < KC - 1; k++) cs[k] = state[(size_t)c * (KC - 1) + k];
    for (int t = 0; t < T; t++) {
        float *xp = qkv + t * ldq + c;
        float acc = 0.0f;
        for (int k = 0; k < KC - 1; k++) acc = fmaf(cs[k], wc[k], acc);
        acc = fmaf(*xp, wc[KC - 1], acc);
        for (int k = 0; k < KC - 2; k++) cs[k] = cs[k + 1];
        cs[KC - 2] = *xp;
        *xp = silu_f(acc);
        if (ck && t < T - 1)
            for (int k = 0; k < KC - 1; k++) ck[((size_t)t * CD + c) * (KC - 1) + k] = cs[k];
    }
    for (int k = 0; k < KC - 1; k++) state[(size_t)c * (KC - 1) + k] = cs[k];
}

struct GdnArgs {
    const float *qkv; long long ldq;
    const float *z; long long ldz;
    const float *beta, *alpha; long long ldg;
    const float *dt, *A, *nw;
    float *ssm, *ck_ssm, *out; long long ldo;
    int T, Hk, Hv, key_dim;
    float eps;
};

// Gated DeltaNet for value head hv over T tokens, 4*S threads (tid < 4*S); thread (j, q) keeps key
// dims {16m + 4q + e : m < S/16, e < 4} of row j of the head's state M in registers, so the four
// threads of a row read and write 64 contiguous bytes per access (core/xj_cpu.c:194-219):
//   q, k <- L2-normalised key head hv % Hk;  b = sigmoid(beta);  g = softplus(alpha + dt) * A
//   M *= exp(g);  delta_j = (v_j - M_j.k) * b;  M_j += delta_j k;  o_j = M_j.q / sqrt(S)
//   out = rmsnorm(o) * norm_w * silu(z)
// State layout [Hv][S(j)][S(i)] as the CPU oracle.
// ck_ssm != nullptr saves M after token t < T-1 into ck_ssm[t][Hv][S][S].
template <int S, class Bar>
XJ_DEV void gdn_head(const GdnArgs &a, int hv, int tid) {
    constexpr int P = S / 4, NT = 4 * S;
    __shared__ float qs[S], ks[S];
    __shared__ double red[32], red2[32];
    const int hk = hv % a.Hk;
    const int j = tid >> 2, qq = tid & 3, lane = tid & 31, w = tid >> 5;
    // this token's operands first (independent of the state), then the state slice
    const float dtv = a.dt[hv], Av = a.A[hv], nwj = a.nw[j];
    const float *x = a.qkv;
    float qv = tid < S ? lda(x + hk * S + tid) : 0.0f, kv = tid < S ? lda(x + a.key_dim + hk * S + tid) : 0.0f;
    float vj = lda(x + 2 * a.key_dim + hv * S + j), zj = lda(a.z + hv * S + j);
    float bt = lda(a.beta + hv), al = lda(a.alpha + hv);
    float row[P];                       // row[4m + e] = M[j][16m + 4qq + e]
    float *M = a.ssm + (size_t)hv * S * S + (size_t)j * S + 4 * qq;
#pragma unroll
    for (int i = 0; i < P; i += 4) {
        const float4 v4 = __ldcg(reinterpret_cast<const float4 *>(M + 4 * i));
        row[i] = v4.x; row[i + 1] = v4.y; row[i + 2] = v4.z; row[i + 3] = v4.w;
    }
    const float qscale = 1.0f / sqrtf((float)S);
    for (int t = 0; t < a.T; t++) {
        if (t > 0) {
            x = a.qkv + t * a.ldq;
            qv = tid < S ? lda(x + hk * S + tid) : 0.0f;
            kv = tid < S ? lda(x + a.key_dim + hk * S + tid) : 0.0f;
            vj = lda(x + 2 * a.key_dim + hv * S + j);
            zj = lda(a.z + t * a.ldz + hv * S + j);
            bt = lda(a.beta + t * a.ldg + hv);
            al = lda(a.alpha + t * a.ldg + hv);
        }
        // L2 norms of q and k (sums in double, core/xj_cpu.c:185-193): both in one pass, each with the
        // warp-then-warps order of group_sum_d
        double sq = warp_sum_d((double)qv * qv), sk2 = warp_sum_d((double)kv * kv);
        Bar::sync();
        if (lane == 0) { red[w] = sq; red2[w] = sk2; }
        Bar::sync();
        sq = 0.0; sk2 = 0.0;
        for (int i = 0; i < NT / 32; i++) sq += red[i];
        for (int i = 0; i < NT / 32; i++) sk2 += red2[i];
        if (tid < S) {
            qs[tid] = qv * (1.0f / sqrtf((float)sq + a.eps));
            ks[tid] = kv * (1.0f / sqrtf((float)sk2 + a.eps));
        }
        Bar::sync();
        const float b = sigm_f(bt);
        const float g = softplus_f(al + dtv) * Av;
        const float eg = expf(g);
        float sk = 0.0f;
#pragma unroll
        for (int i = 0; i < P; i++) { row[i] *= eg; sk = fmaf(row[i], ks[4 * (i & ~3) + 4 * qq + (i & 3)], sk); }
        sk += __shfl_xor_sync(0xffffffffu, sk, 1);
        sk += __shfl_xor_sync(0xffffffffu, sk, 2);
        const float delta = (vj - sk) * b;
        float acc = 0.0f;
#pragma unroll
        for (int i = 0; i < P; i++) {
            const int col = 4 * (i & ~3) + 4 * qq + (i & 3);
            row[i] = fmaf(ks[col], delta, row[i]);
            acc = fmaf(row[i], qs[col], acc);
        }
        acc += __shfl_xor_sync(0xffffffffu, acc, 1);
        acc += __shfl_xor_sync(0xffffffffu, acc, 2);
        const float o = acc * qscale;
        const double so = group_sum_d<Bar>(qq == 0 ? (double)o * o : 0.0, red, tid, NT);
        if (qq == 0) {
            const float sc = 1.0f / sqrtf((float)(so / S) + a.eps);
            a.out[t * a.ldo + hv * S + j] = o * sc * nwj * silu_f(zj);
        }
        if (a.ck_ssm && t < a.T - 1) {
            float *C = a.ck_ssm + ((size_t)t * a.Hv + hv) * S * S + (size_t)j * S + 4 * qq;
#pragma unroll
            for (int i = 0; i < P; i += 4) *reinterpret_cast<float4 *>(C + 4 * i) = make_float4(row[i], row[i + 1], row[i + 2], row[i + 3]);
        }
        Bar::sync();
    }
#pragma unroll
    for (int i = 0; i < P; i += 4) *reinterpret_cast<float4 *>(M + 4 * i) = make_float4(row[i], row[i + 1], row[i + 2], row[i + 3]);
}

// ---------------------------------------------------------------- chunked Gated DeltaNet (prompts)
// The recurrence of gdn_head over T tokens, chunk by chunk (GC_C tokens), for prompt forwards without
// checkpoints. Each value row j of a head's state evolves on its own, so a head's S rows are split
// over S / 16 CTAs. Within a chunk with state M0 at its start, cumulative log decay G_i = g_1 + .. + g_i
// (g = softplus(alpha + dt) * A <= 0) and normalised q, k:
//   u_i = b_i (v_i - e^G_i M0 k_i) - sum_{l<i} b_i e^(G_i - G_l) (k_i . k_l) u_l     (forward substitution)
//   o_i = (e^G_i M0 q_i + sum_{l<=i} e^(G_i - G_l) (q_i . k_l) u_l) / sqrt(S)
//   M_C = e^G_C M0 + sum_l e^(G_C - G_l) u_l k_l^T
// which is the token-by-token update M = e^g M; u = (v - M k) b; M += u k^T; o = M q / sqrt(S) of
// core/xj_cpu.c:194-219 regrouped. The substitution is solved once per chunk and value head, for all
// chunks at once, as a triangular inverse (k_gdn_chunk_solve), which leaves the walk over chunks
// (k_gdn_chunk) three small matrix products per chunk. fp32 values, products as 3xTF32 on tensor cores,
// sums in another order: results agree with the sequential kernel to rounding. The gated RMSNorm of the
// outputs is a separate pass (k_gdn_gnorm).
constexpr int GC_C = 64;          // tokens per chunk
constexpr int GC_MIN_T = 32;      // forwards of at least this many tokens take the chunked path

// Grid (Hk, nchunks), 256 threads: q, k of key head hk for the chunk's tokens, L2-normalised (sums in
// double, core/xj_cpu.c:185-193) into qn, kn [T][Hk][S]; kk[i][l] = k_i . k_l (l < i) and
// qk[i][l] = q_i . k_l (l <= i) into [Hk][nchunks][GC_C][GC_C].
template <int S>
__global__ void __launch_bounds__(256) k_gdn_chunk_prep(GdnArgs a, float *qn, float *kn, float *kk, float *qk) {
    griddep_wait();
    griddep_launch();   // successors may start their prologue; they wait for this grid before reading
    extern __shared__ __align__(16) float gsm[];
    constexpr int CP = GC_C + 4;                           // transposed rows [S][CP]
    float *qt = gsm, *kt = gsm + S * CP;
    const int hk = blockIdx.x, ch = blockIdx.y, t0 = ch * GC_C, n = a.T - t0 < GC_C ? a.T - t0 : GC_C;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // normalise: one warp per token
    for (int i = warp; i < GC_C; i += 8) {
        const int t = t0 + i;
        float qv[S / 32], kv[S / 32];
        double sq = 0.0, sk = 0.0;
#pragma unroll
        for (int e = 0; e < S / 32; e++) {
            const int c = lane + 32 * e;
            qv[e] = i < n ? lda(a.qkv + (size_t)t * a.ldq + hk * S + c) : 0.0f;
            kv[e] = i < n ? lda(a.qkv + (size_t)t * a.ldq + a.key_dim + hk * S + c) : 0.0f;
            sq += (double)qv[e] * qv[e];
            sk += (double)kv[e] * kv[e];
        }
        sq = warp_sum_d(sq);
        sk = warp_sum_d(sk);
        const float rq = 1.0f / sqrtf((float)sq + a.eps), rk = 1.0f / sqrtf((float)sk + a.eps);
#pragma unroll
        for (int e = 0; e < S / 32; e++) {
            const int c = lane + 32 * e;
            const float q = qv[e] * rq, k = kv[e] * rk;
            qt[c * CP + i] = q;
            kt[c * CP + i] = k;
            if (i < n) {
                qn[((size_t)t * a.Hk + hk) * S + c] = q;
                kn[((size_t)t * a.Hk + hk) * S + c] = k;
            }
        }
    }
    __syncthreads();
    // 4x4 output blocks: thread (bi, bl) = (tid / 16, tid % 16) takes rows 4bi.., columns 4bl..
    const int bi = tid >> 4, bl = tid & 15;
    if (bl > bi) return;                                   // strictly above the diagonal: unused
    float ak[4][4] = {}, aq[4][4] = {};
    for (int c = 0; c < S; c++) {
        const float4 ki = *reinterpret_cast<const float4 *>(kt + c * CP + 4 * bi);
        const float4 qi = *reinterpret_cast<const float4 *>(qt + c * CP + 4 * bi);
        const float4 kl = *reinterpret_cast<const float4 *>(kt + c * CP + 4 * bl);
        const float kiv[4] = {ki.x, ki.y, ki.z, ki.w}, qiv[4] = {qi.x, qi.y, qi.z, qi.w}, klv[4] = {kl.x, kl.y, kl.z, kl.w};
#pragma unroll
        for (int x = 0; x < 4; x++)
#pragma unroll
            for (int y = 0; y < 4; y++) {
                ak[x][y] = fmaf(kiv[x], klv[y], ak[x][y]);
                aq[x][y] = fmaf(qiv[x], klv[y], aq[x][y]);
            }
    }
    float *KK = kk + ((size_t)hk * gridDim.y + ch) * GC_C * GC_C, *QK = qk + ((size_t)hk * gridDim.y + ch) * GC_C * GC_C;
#pragma unroll
    for (int x = 0; x < 4; x++)
#pragma unroll
        for (int y = 0; y < 4; y++) {
            KK[(4 * bi + x) * GC_C + 4 * bl + y] = ak[x][y];
            QK[(4 * bi + x) * GC_C + 4 * bl + y] = aq[x][y];
        }
}

template <int S> constexpr size_t gdn_prep_smem() { return (size_t)2 * S * (GC_C + 4) * 4; }

// The chunk-parallel half of the recurrence. Per value head and chunk, with A[i][l] = b_i e^(G_i - G_l)
// (k_i . k_l) for l < i, the substitution above is (I + A) u = b (v - e^G M0 k), so with
//   W = (I + A)^-1 diag(b e^G) K,   U0 = (I + A)^-1 diag(b) V                      (state-independent)
// u = U0 - W M0^T. Substituting into o and M_C:
//   o = O0 + Q' M0^T,  Q' = diag(e^G) Q - D W,  O0 = D U0,  D[i][l] = e^(G_i - G_l) (q_i . k_l), l <= i
//   M_C = e^G_C M0 + u^T Kd,  Kd[l] = e^(G_C - G_l) k_l
// so the walk over chunks (k_gdn_chunk) is three small matrix products per chunk and this kernel runs
// every chunk at once. Tokens past the prompt count as g = 0, b = 0, q = k = v = 0 (they change nothing).
// Scratch wx, all [T][Hv][S]: W, Q', Kd, U0, O0; then e^(G_C) per [Hv][chunk].
inline size_t gc_wx_floats(int T, int Hv, int S) { return (size_t)5 * T * Hv * S + (size_t)Hv * ((T + GC_C - 1) / GC_C); }
// fp32 x = hi + lo with hi, lo tf32 (round to nearest): products of the two parts (hi*hi + hi*lo +
// lo*hi, the lo*lo term dropped) carry about the precision of an fp32 product ("3xTF32").
XJ_DEV uint32_t tf32_of(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return r;
}
XJ_DEV void tf32_split(float x, uint32_t &hi, uint32_t &lo) {
    hi = tf32_of(x);
    lo = tf32_of(x - __uint_as_float(hi));
}
// D (16 x 8, f32) += A (16 x 8, tf32, row) . B (8 x 8, tf32, col); fragments in the PTX ISA's m16n8k8
// layout (lane = 4 g + c: a = A[g][c], A[g+8][c], A[g][c+4], A[g+8][c+4]; b = B[c][g], B[c+4][g];
// d = D[g][2c], D[g][2c+1], D[g+8][2c], D[g+8][2c+1]).
XJ_DEV void mma_tf32(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// The two small terms into ds, the large one into d (two accumulators: shorter dependent MMA chains).
XJ_DEV void mma_3xtf32(float (&d)[4], float (&ds)[4], const uint32_t (&ah)[4], const uint32_t (&al)[4], uint32_t bh0,
                       uint32_t bh1, uint32_t bl0, uint32_t bl1) {
    mma_tf32(ds, al, bh0, bh1);
    mma_tf32(d, ah, bh0, bh1);
    mma_tf32(ds, ah, bl0, bl1);
}

template <int S> constexpr size_t gdn_solve_smem() { return ((size_t)3 * GC_C * (GC_C + 4) + 3 * GC_C * (S + 4)) * 4; }

// Grid (Hv, nchunks), 2S threads (S / 16 warps): the chunk's operands into shared memory, Kd, then
// T = (I + A)^-1 by forward substitution (S / 32 threads per column), then the four products W, U0, Q',
// O0 on tensor cores.
template <int S>
__global__ void __launch_bounds__(2 * S) k_gdn_chunk_solve(GdnArgs a, const float *qn, const float *kn, const float *kk,
                                                           const float *qk, float *wx) {
    griddep_wait();
    griddep_launch();   // successors may start their prologue; they wait for this grid before reading
    constexpr int CP = GC_C + 4, SP = S + 4, NT = 2 * S;
    extern __shared__ __align__(16) float gsm[];
    float *Am = gsm, *Dm = Am + GC_C * CP;                  // [C][CP]: A (l < i), D (l <= i)
    float *Tm = Dm + GC_C * CP;                             // [C][CP]: (I + A)^-1
    float *Xk = Tm + GC_C * CP, *Xv = Xk + GC_C * SP, *Xq = Xv + GC_C * SP;   // [C][SP]: k, v, q rows of the chunk
    __shared__ float G[GC_C], bv[GC_C], eG[GC_C];
    const int hv = blockIdx.x, hk = hv % a.Hk, ch = blockIdx.y, nch = gridDim.y;
    const int t0 = ch * GC_C, n = a.T - t0 < GC_C ? a.T - t0 : GC_C;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const size_t plane = (size_t)a.T * a.Hv * S;
    // every global operand first, loads batched ahead of the stores (each loop's trip count is fixed)
    {
        constexpr int NR = GC_C * (S / 4) / NT;            // 16-byte pieces per thread and array
        float4 rk[NR], rq[NR];
        float rv[4 * NR];
#pragma unroll
        for (int r = 0; r < NR; r++) {
            const int x = tid + r * NT, i = x / (S / 4), c4 = (x % (S / 4)) * 4;
            const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
            const size_t o = ((size_t)(t0 + i) * a.Hk + hk) * S + c4;
            rk[r] = i < n ? __ldcg(reinterpret_cast<const float4 *>(kn + o)) : z4;
            rq[r] = i < n ? __ldcg(reinterpret_cast<const float4 *>(qn + o)) : z4;
            const float *vp = a.qkv + (size_t)(t0 + i) * a.ldq + 2 * a.key_dim + hv * S + c4;   // 4-byte aligned only
#pragma unroll
            for (int e = 0; e < 4; e++) rv[4 * r + e] = i < n ? lda(vp + e) : 0.0f;
        }
#pragma unroll
        for (int r = 0; r < NR; r++) {
            const int x = tid + r * NT, i = x / (S / 4), c4 = (x % (S / 4)) * 4;
            *reinterpret_cast<float4 *>(Xk + i * SP + c4) = rk[r];
            *reinterpret_cast<float4 *>(Xq + i * SP + c4) = rq[r];
            *reinterpret_cast<float4 *>(Xv + i * SP + c4) = make_float4(rv[4 * r], rv[4 * r + 1], rv[4 * r + 2], rv[4 * r + 3]);
        }
    }
    if (warp == 0) {
        // g, b per token; G by a sequential prefix sum (fp32)
        const float dtv = a.dt[hv], Av = a.A[hv];
        for (int i = lane; i < GC_C; i += 32) {
            const int t = t0 + i;
            G[i] = i < n ? softplus_f(lda(a.alpha + (size_t)t * a.ldg + hv) + dtv) * Av : 0.0f;
            bv[i] = i < n ? sigm_f(lda(a.beta + (size_t)t * a.ldg + hv)) : 0.0f;
        }
        __syncwarp();
        if (lane == 0) {
            float acc = 0.0f;
            for (int i = 0; i < GC_C; i++) { acc += G[i]; G[i] = acc; }
        }
        __syncwarp();
        for (int i = lane; i < GC_C; i += 32) eG[i] = expf(G[i]);
    }
    {
        // the chunk's k.k and q.k products (16-byte rows; the never-written upper blocks are masked)
        const float *KKg = kk + ((size_t)hk * nch + ch) * GC_C * GC_C, *QKg = qk + ((size_t)hk * nch + ch) * GC_C * GC_C;
        constexpr int NQ = GC_C * GC_C / 4 / NT;
        float4 rkk[NQ], rqk[NQ];
#pragma unroll
        for (int r = 0; r < NQ; r++) {
            const int x = (tid + r * NT) * 4;
            rkk[r] = __ldcg(reinterpret_cast<const float4 *>(KKg + x));
            rqk[r] = __ldcg(reinterpret_cast<const float4 *>(QKg + x));
        }
        __syncthreads();                                   // G, bv, eG
#pragma unroll
        for (int r = 0; r < NQ; r++) {
            const int x = (tid + r * NT) * 4, i = x / GC_C, l0 = x % GC_C;
            const float kv4[4] = {rkk[r].x, rkk[r].y, rkk[r].z, rkk[r].w}, qv4[4] = {rqk[r].x, rqk[r].y, rqk[r].z, rqk[r].w};
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int l = l0 + e;
                const float d = l <= i ? expf(G[i] - G[l]) : 0.0f;
                Am[i * CP + l] = l < i ? bv[i] * d * kv4[e] : 0.0f;
                Dm[i * CP + l] = l <= i ? d * qv4[e] : 0.0f;
            }
        }
    }
    __syncthreads();
    if (tid < S) {
        // Kd = e^(G_C - G_l) k_l, before the W threads overwrite the k rows
        float *kd = wx + 2 * plane;
        for (int i = 0; i < n; i++) kd[((size_t)(t0 + i) * a.Hv + hv) * S + tid] = expf(G[GC_C - 1] - G[i]) * Xk[i * SP + tid];
    }
    __syncthreads();
    // T = (I + A)^-1 (unit lower triangular), row by row: T[i][cc] = -sum_{cc <= l < i} A[i][l] T[l][cc];
    // TPC consecutive lanes per column split the sum (column cc's rows are written and read by its own
    // lanes only, so a warp barrier orders them)
    {
        constexpr int TPC = NT / GC_C;
        const int cc = tid / TPC, q = tid % TPC;
        for (int i = 0; i < GC_C; i++) {
            float s0 = 0.0f, s1 = 0.0f;
            const float *ar = Am + i * CP;
            int l = cc + q;
            for (; l + TPC < i; l += 2 * TPC) {
                s0 = fmaf(ar[l], Tm[l * CP + cc], s0);
                s1 = fmaf(ar[l + TPC], Tm[(l + TPC) * CP + cc], s1);
            }
            if (l < i) s0 = fmaf(ar[l], Tm[l * CP + cc], s0);
            float sum = s0 + s1;
#pragma unroll
            for (int o = TPC >> 1; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
            if (q == 0) Tm[i * CP + cc] = cc < i ? -sum : (cc == i ? 1.0f : 0.0f);
            __syncwarp();
        }
    }
    __syncthreads();
    // W = T diag(b e^G) K and U0 = T diag(b) V on tensor cores (mma.sync m16n8k8 tf32, 3xTF32): task
    // (product pr, 16-token tile mt); the row scales go into T's columns as the A fragments are formed.
    // Every warp holds its tasks' whole rows (64 accumulators a thread) until all warps have read the k
    // and v rows, then the results replace them in place.
    {
        constexpr int NWS = NT / 32, TPW = 8 / NWS, NTL = S / 8;
        const int g = lane >> 2, cq = lane & 3;
        float acc[TPW][NTL][4] = {};
#pragma unroll
        for (int tt = 0; tt < TPW; tt++) {
            const int task = warp + tt * NWS, pr = task >> 2, mt = task & 3;
            const float *Xs = pr ? Xv : Xk;
            for (int k0 = 0; k0 < 16 * mt + 16; k0 += 8) {
                const float sc0 = pr ? bv[k0 + cq] : bv[k0 + cq] * eG[k0 + cq];
                const float sc1 = pr ? bv[k0 + cq + 4] : bv[k0 + cq + 4] * eG[k0 + cq + 4];
                uint32_t ah[4], al[4];
                const int o0 = (16 * mt + g) * CP + k0 + cq, o1 = o0 + 8 * CP;
                tf32_split(Tm[o0] * sc0, ah[0], al[0]);
                tf32_split(Tm[o1] * sc0, ah[1], al[1]);
                tf32_split(Tm[o0 + 4] * sc1, ah[2], al[2]);
                tf32_split(Tm[o1 + 4] * sc1, ah[3], al[3]);
#pragma unroll
                for (int j = 0; j < NTL; j++) {
                    const int col = 8 * j + g;
                    uint32_t bh0, bl0, bh1, bl1;
                    tf32_split(Xs[(k0 + cq) * SP + col], bh0, bl0);
                    tf32_split(Xs[(k0 + cq + 4) * SP + col], bh1, bl1);
                    mma_tf32(acc[tt][j], al, bh0, bh1);
                    mma_tf32(acc[tt][j], ah, bl0, bl1);
                    mma_tf32(acc[tt][j], ah, bh0, bh1);
                }
            }
        }
        __syncthreads();                                   // every k and v row has been read
#pragma unroll
        for (int tt = 0; tt < TPW; tt++) {
            const int task = warp + tt * NWS, pr = task >> 2, mt = task & 3;
            float *Xs = pr ? Xv : Xk;
            float *dst = wx + (pr ? 3 * plane : 0);
#pragma unroll
            for (int j = 0; j < NTL; j++)
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const int i = 16 * mt + g + 8 * (e >> 1), col = 8 * j + 2 * cq + (e & 1);
                    Xs[i * SP + col] = acc[tt][j][e];
                    if (i < n) dst[((size_t)(t0 + i) * a.Hv + hv) * S + col] = acc[tt][j][e];
                }
        }
    }
    __syncthreads();                                       // every column of W and U0 is final
    // Q' = e^G q - D W and O0 = D U0 on tensor cores (mma.sync m16n8k8 tf32, 3xTF32): task (product pr,
    // 16-token tile mt) per warp in turn, 8 column tiles at a time; D is lower triangular, so the k-steps
    // stop at the tile's diagonal block
    {
        constexpr int NWS = NT / 32, NTL = S / 8, NB = NTL < 8 ? NTL : 8;
        const int g = lane >> 2, cq = lane & 3;
        for (int task = warp; task < 8; task += NWS) {
            const int pr = task >> 2, mt = task & 3;
            const float *Xs = pr ? Xv : Xk;
            float *dst = wx + (pr ? 4 * plane : plane);
            for (int nb = 0; nb < NTL; nb += NB) {
                float acc[NB][4] = {};
                for (int k0 = 0; k0 < 16 * mt + 16; k0 += 8) {
                    uint32_t ah[4], al[4];
                    const int o0 = (16 * mt + g) * CP + k0 + cq, o1 = o0 + 8 * CP;
                    tf32_split(Dm[o0], ah[0], al[0]);
                    tf32_split(Dm[o1], ah[1], al[1]);
                    tf32_split(Dm[o0 + 4], ah[2], al[2]);
                    tf32_split(Dm[o1 + 4], ah[3], al[3]);
#pragma unroll
                    for (int j = 0; j < NB; j++) {
                        const int col = 8 * (nb + j) + g;
                        uint32_t bh0, bl0, bh1, bl1;
                        tf32_split(Xs[(k0 + cq) * SP + col], bh0, bl0);
                        tf32_split(Xs[(k0 + cq + 4) * SP + col], bh1, bl1);
                        mma_tf32(acc[j], al, bh0, bh1);
                        mma_tf32(acc[j], ah, bl0, bl1);
                        mma_tf32(acc[j], ah, bh0, bh1);
                    }
                }
#pragma unroll
                for (int j = 0; j < NB; j++)
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const int i = 16 * mt + g + 8 * (e >> 1), col = 8 * (nb + j) + 2 * cq + (e & 1);
                        if (i < n)
                            dst[((size_t)(t0 + i) * a.Hv + hv) * S + col] = pr ? acc[j][e] : eG[i] * Xq[i * SP + col] - acc[j][e];
                    }
            }
        }
    }
    if (tid == 0) wx[5 * plane + (size_t)hv * nch + ch] = eG[GC_C - 1];
}

constexpr int GC_RP = 20;         // row stride (floats) of the walk's U0 / O0 column tiles (16-byte rows)
constexpr int GC_UP = GC_C + 4;   // row stride of u^T (16 state rows x the chunk's tokens)
template <int S> constexpr size_t gdn_chunk_smem() {
    return ((size_t)5 * GC_C * (S + 4) + 2 * 16 * (S + 4) + 4 * GC_C * GC_RP + 2 * 16 * GC_UP) * 4;
}
// 16 bytes global -> shared, asynchronously (zeros when !valid; src must still be a mapped address).
XJ_DEV void gc_cp16(float *dst, const float *src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" :: "r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src),
                 "r"(valid ? 16 : 0) : "memory");
}
XJ_DEV void gc_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> XJ_DEV void gc_wait() { asm volatile("cp.async.wait_group %0;" :: "n"(N) : "memory"); }

// Grid (Hv, S / 16), 256 threads (8 warps): rows [16 r, 16 r + 16) of value head hv's state over all
// chunks, on tensor cores (mma.sync m16n8k8 tf32, 3xTF32 for fp32-level products). Per chunk, from the
// solve kernel's rows:
//   u = U0 - W M0^T, o = O0 + Q' M0^T   ([64 tokens x S] x [S x 16 rows]: warp w takes tokens 16 (w % 4)..
//                                         of W (w < 4) or of Q' (w >= 4), both 8-row tiles)
//   M = e^G_C M0 + u^T Kd               ([16 rows x 64 tokens] x [64 x S]: warp w < S / 16 takes state
//                                         columns 16 w .. 16 w + 15 and keeps them as its accumulators)
// The state's hi / lo tf32 parts and those of u^T go through shared memory once per chunk (every warp
// reads them). Raw outputs o (scaled by 1/sqrt(S), before the gated norm) to out[t][hv*S + j]. The rows
// do not depend on the state, so they are copied in ahead: W, Q', U0, O0 of chunk c + 1 (double-
// buffered) while chunk c computes, Kd of chunk c + 1 while chunk c + 1 computes u and o (one commit
// group each, waited for in issue order).
template <int S>
__global__ void __launch_bounds__(256) k_gdn_chunk(GdnArgs a, const float *wx) {
    griddep_wait();
    griddep_launch();   // successors may start their prologue; they wait for this grid before reading
    constexpr int SP = S + 4, RP = GC_RP, UP = GC_UP, NW3 = S / 16;
    extern __shared__ __align__(16) float gsm[];
    float *Wb = gsm, *Qb = Wb + 2 * GC_C * SP, *Kc = Qb + 2 * GC_C * SP;   // [2][C][SP], [2][C][SP], [C][SP]
    float *Mh = Kc + GC_C * SP, *Ml = Mh + 16 * SP;                      // [16][SP]: the state rows, tf32 hi / lo
    float *Ub = Ml + 16 * SP, *Ob = Ub + 2 * GC_C * RP;                  // [2][C][RP]: U0, O0 (the CTA's rows)
    float *Th = Ob + 2 * GC_C * RP, *Tl = Th + 16 * UP;                  // [16][UP]: u^T, tf32 hi / lo
    const int hv = blockIdx.x, r0 = blockIdx.y * 16;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, c = lane & 3;
    const int nch = (a.T + GC_C - 1) / GC_C;
    const size_t plane = (size_t)a.T * a.Hv * S;
    const float *Wg = wx, *Qg = wx + plane, *Kg = wx + 2 * plane, *Ug = wx + 3 * plane, *Og = wx + 4 * plane;
    const float *eGCg = wx + 5 * plane;
    auto stage_wq = [&](int ch, int b) {
        const int t0 = ch * GC_C, n = a.T - t0 < GC_C ? a.T - t0 : GC_C;
        for (int x = tid; x < GC_C * (S / 4); x += 256) {
            const int i = x / (S / 4), cc = (x % (S / 4)) * 4;
            const size_t o = i < n ? ((size_t)(t0 + i) * a.Hv + hv) * S + cc : 0;
            gc_cp16(Wb + (b * GC_C + i) * SP + cc, Wg + o, i < n);
            gc_cp16(Qb + (b * GC_C + i) * SP + cc, Qg + o, i < n);
        }
        for (int x = tid; x < GC_C * 4; x += 256) {
            const int i = x >> 2, q = (x & 3) * 4;
            const size_t o = i < n ? ((size_t)(t0 + i) * a.Hv + hv) * S + r0 + q : 0;
            gc_cp16(Ub + (b * GC_C + i) * RP + q, Ug + o, i < n);
            gc_cp16(Ob + (b * GC_C + i) * RP + q, Og + o, i < n);
        }
        gc_commit();
    };
    auto stage_k = [&](int ch) {
        const int t0 = ch * GC_C, n = a.T - t0 < GC_C ? a.T - t0 : GC_C;
        for (int x = tid; x < GC_C * (S / 4); x += 256) {
            const int i = x / (S / 4), cc = (x % (S / 4)) * 4;
            const size_t o = i < n ? ((size_t)(t0 + i) * a.Hv + hv) * S + cc : 0;
            gc_cp16(Kc + i * SP + cc, Kg + o, i < n);
        }
        gc_commit();
    };
    // the state columns of warp w < NW3 as m16n8 accumulators: tile j holds rows g, g + 8 and columns
    // 16 w + 8 j + 2 c, + 1
    float st[2][4];
    float *Mbase = a.ssm + (size_t)hv * S * S + (size_t)r0 * S;
    auto put_state = [&]() {   // hi / lo parts into Mh / Ml
#pragma unroll
        for (int j = 0; j < 2; j++)
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int o = (g + 8 * h) * SP + 16 * warp + 8 * j + 2 * c;
                uint32_t h0, l0, h1, l1;
                tf32_split(st[j][2 * h], h0, l0);
                tf32_split(st[j][2 * h + 1], h1, l1);
                *reinterpret_cast<float2 *>(Mh + o) = make_float2(__uint_as_float(h0), __uint_as_float(h1));
                *reinterpret_cast<float2 *>(Ml + o) = make_float2(__uint_as_float(l0), __uint_as_float(l1));
            }
    };
    if (warp < NW3) {
#pragma unroll
        for (int j = 0; j < 2; j++)
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const float2 v = __ldcg(reinterpret_cast<const float2 *>(Mbase + (size_t)(g + 8 * h) * S + 16 * warp + 8 * j + 2 * c));
                st[j][2 * h] = v.x;
                st[j][2 * h + 1] = v.y;
            }
        put_state();
    }
    const float qscale = 1.0f / sqrtf((float)S);
    const int mt = warp & 3, pr = warp >> 2;            // products: token tile mt of W (pr 0) or Q' (pr 1)
    stage_wq(0, 0);
    stage_k(0);
    for (int ch = 0; ch < nch; ch++) {
        const int t0 = ch * GC_C, n = a.T - t0 < GC_C ? a.T - t0 : GC_C, b = ch & 1;
        const float *Xc = (pr ? Qb : Wb) + (b * GC_C + 16 * mt) * SP;
        const float *Uc = Ub + b * GC_C * RP, *Oc = Ob + b * GC_C * RP;
        gc_wait<1>();                                      // this chunk's W, Q', U0, O0 (Kd may be in flight)
        const float eGC = __ldcg(eGCg + (size_t)hv * nch + ch);
        __syncthreads();
        if (ch + 1 < nch) stage_wq(ch + 1, b ^ 1);         // that buffer's last reader was chunk ch - 1
        // [16 tokens x S] x [S x 16 rows]; accumulators per k-step parity and term size, summed after
        float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        {
            float pa[2][2][2][4] = {};
#pragma unroll 2
            for (int k0 = 0; k0 < S; k0 += 16) {
#pragma unroll
                for (int p = 0; p < 2; p++) {
                    const int k = k0 + 8 * p;
                    uint32_t ah[4], al[4];
                    tf32_split(Xc[g * SP + k + c], ah[0], al[0]);
                    tf32_split(Xc[(g + 8) * SP + k + c], ah[1], al[1]);
                    tf32_split(Xc[g * SP + k + c + 4], ah[2], al[2]);
                    tf32_split(Xc[(g + 8) * SP + k + c + 4], ah[3], al[3]);
#pragma unroll
                    for (int j = 0; j < 2; j++) {
                        const int o = (8 * j + g) * SP + k + c;
                        mma_3xtf32(pa[p][0][j], pa[p][1][j], ah, al, __float_as_uint(Mh[o]), __float_as_uint(Mh[o + 4]),
                                   __float_as_uint(Ml[o]), __float_as_uint(Ml[o + 4]));
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < 2; j++)
#pragma unroll
                for (int e = 0; e < 4; e++) acc[j][e] = (pa[0][1][j][e] + pa[1][1][j][e]) + (pa[0][0][j][e] + pa[1][0][j][e]);
        }
#pragma unroll
        for (int j = 0; j < 2; j++)
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int tok = 16 * mt + g + 8 * (e >> 1), row = 8 * j + 2 * c + (e & 1);
                if (pr == 0) {
                    uint32_t h, l;
                    tf32_split(Uc[tok * RP + row] - acc[j][e], h, l);
                    Th[row * UP + tok] = __uint_as_float(h);
                    Tl[row * UP + tok] = __uint_as_float(l);
                } else if (tok < n) {
                    a.out[(size_t)(t0 + tok) * a.ldo + hv * S + r0 + row] = (Oc[tok * RP + row] + acc[j][e]) * qscale;
                }
            }
        // this chunk's Kd (issued before the next chunk's W, Q', U0, O0, if any)
        if (ch + 1 < nch) gc_wait<1>();
        else gc_wait<0>();
        __syncthreads();
        // M = e^G_C M + u^T Kd: [16 rows x 64 tokens] x [64 tokens x 16 columns] per warp (rows and columns
        // of u and Kd past the prompt are zero)
        if (warp < NW3) {
            float sm[2][4] = {};                           // the small terms of the 3xTF32 products
#pragma unroll
            for (int j = 0; j < 2; j++)
#pragma unroll
                for (int e = 0; e < 4; e++) st[j][e] *= eGC;
#pragma unroll 2
            for (int k0 = 0; k0 < GC_C; k0 += 8) {
                uint32_t ah[4], al[4];
                const int o0 = g * UP + k0 + c, o1 = (g + 8) * UP + k0 + c;
                ah[0] = __float_as_uint(Th[o0]); ah[1] = __float_as_uint(Th[o1]);
                ah[2] = __float_as_uint(Th[o0 + 4]); ah[3] = __float_as_uint(Th[o1 + 4]);
                al[0] = __float_as_uint(Tl[o0]); al[1] = __float_as_uint(Tl[o1]);
                al[2] = __float_as_uint(Tl[o0 + 4]); al[3] = __float_as_uint(Tl[o1 + 4]);
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    const int col = 16 * warp + 8 * j + g;
                    uint32_t bh0, bl0, bh1, bl1;
                    tf32_split(Kc[(k0 + c) * SP + col], bh0, bl0);
                    tf32_split(Kc[(k0 + c + 4) * SP + col], bh1, bl1);
                    mma_3xtf32(st[j], sm[j], ah, al, bh0, bh1, bl0, bl1);
                }
            }
#pragma unroll
            for (int j = 0; j < 2; j++)
#pragma unroll
                for (int e = 0; e < 4; e++) st[j][e] += sm[j][e];
        }
        __syncthreads();                                   // Kc, u^T and the old state parts are consumed
        if (warp < NW3) put_state();
        if (ch + 1 < nch) stage_k(ch + 1);
    }
    gc_wait<0>();
    if (warp < NW3)
#pragma unroll
        for (int j = 0; j < 2; j++)
#pragma unroll
            for (int h = 0; h < 2; h++)
                *reinterpret_cast<float2 *>(Mbase + (size_t)(g + 8 * h) * S + 16 * warp + 8 * j + 2 * c) =
                    make_float2(st[j][2 * h], st[j][2 * h + 1]);
}

// Grid (T, Hv), S threads (S <= 1024): out[t][hv*S + j] = o * rsqrt(mean_j o^2 + eps) * norm_w[j] * silu(z),
// in place on the raw outputs of k_gdn_chunk (the gated RMSNorm of gdn_head, sum in double).
template <int S>
__global__ void __launch_bounds__(S) k_gdn_gnorm(GdnArgs a) {
    griddep_wait();
    griddep_launch();   // successors may start their prologue; they wait for this grid before reading
    __shared__ double red[32];
    const int t = blockIdx.x, hv = blockIdx.y, j = threadIdx.x;
    float *op = a.out + (size_t)t * a.ldo + hv * S + j;
    const float o = *op;
    const double so = group_sum_d<BarBlock>((double)o * o, red, j, S);
    const float sc = 1.0f / sqrtf((float)(so / S) + a.eps);
    *op = o * sc * a.nw[j] * silu_f(lda(a.z + (size_t)t * a.ldz + hv * S + j));
}

// One block of 4*S threads per value head.
template <int S>
__global__ void __launch_bounds__(4 * S) k_gdn(GdnArgs a) {
    griddep_wait();
    griddep_launch();   // successors may start their prologue; they wait for this grid before reading
    gdn_head<S, BarBlock>(a, blockIdx.x, threadIdx.x);
}

// ---------------------------------------------------------------- gated full attention
template <typename KV>
XJ_DEV void store_kv(KV *p, float v);
template <> XJ_DEV void store_kv<float>(float *p, float v) { *p = v; }
template <> XJ_DEV void store_kv<__half>(__half *p, float v) { *p = __float2half_rn(v); }
// KV rows may have been written by another block this step: read them through L2.
XJ_DEV float load_kv(const float *p) { return __ldcg(p); }
XJ_DEV float load_kv(const __half *p) { return __half2float(__ushort_as_half(__ldcg(reinterpret_cast<const unsigned short *>(p)))); }

struct AttnArgs {
    const float *q; long long ldq;       // [T][H][q(D) | gate(D)]
    const float *k, *v; long long ldkv;  // [T][Hkv*D]
    const float *qn, *kn;                // per-head RMSNorm weights
    float *qrot;                         // [T][H][D]
    void *kc, *vc;                       // [n_ctx][Hkv*D]
    const int *npast;
    float *out; long long ldo;           // [T][H*D]
    int H, Hkv, D, n_rot;
    float base, eps;
};

// Token t, head slot `slot` (q heads, then KV heads): q heads get RMSNorm(q_norm) + NeoX RoPE into
// qrot[t][h][D]; KV heads get RMSNorm(k_norm) + RoPE and are stored with v at position npast+t
// (core/xj_cpu.c:107-116). Threads tid < ceil32(D) take part (Bar spans exactly those).
template <typename KV, class Bar>
XJ_DEV void attn_prep_slot(const AttnArgs &a, int slot, int t, int tid) {
    __shared__ float sh[256];
    __shared__ double red[32];
    const int D = a.D, nthr = (D + 31) / 32 * 32;
    const int pos = __ldcg(a.npast) + t;
    const bool isq = slot < a.H;
    const int hh = isq ? slot : slot - a.H;
    const float *src = isq ? a.q + t * a.ldq + (size_t)hh * 2 * D : a.k + t * a.ldkv + (size_t)hh * D;
    const float xi = tid < D ? lda(src + tid) : 0.0f;
    const double ss = group_sum_d<Bar>((double)xi * xi, red, tid, nthr);
    const float sc = 1.0f / sqrtf((float)(ss / D) + a.eps);
    const float *nw = isq ? a.qn : a.kn;
    if (tid < D) sh[tid] = xi * sc * nw[tid];
    Bar::sync();
    float r = tid < D ? sh[tid] : 0.0f;
    const int half = a.n_rot / 2;
    if (tid < a.n_rot) {
        const int p = tid < half ? tid : tid - half;
        const float theta = (float)pos * powf(a.base, -2.0f * (float)p / (float)a.n_rot);
        const float c = cosf(theta), s = sinf(theta);
        const float x0 = sh[p], x1 = sh[p + half];
        r = tid < half ? x0 * c - x1 * s : x0 * s + x1 * c;
    }
    if (tid < D) {
        if (isq) a.qrot[((size_t)t * a.H + hh) * D + tid] = r;
        else {
            const size_t o = (size_t)pos * a.Hkv * D + (size_t)hh * D + tid;
            store_kv<KV>((KV *)a.kc + o, r);
            store_kv<KV>((KV *)a.vc + o, lda(a.v + t * a.ldkv + (size_t)hh * D + tid));
        }
    }
    Bar::sync();   // sh / red are reused by the caller's next slot
}

// Grid (H + Hkv, T), ceil32(D) threads.
template <typename KV>
static __global__ void k_attn_prep(AttnArgs a) {
    griddep_wait();
    griddep_launch();   // successors may start their prologue; they wait for this grid before reading
    attn_prep_slot<KV, BarBlock>(a, blockIdx.x, blockIdx.y, threadIdx.x);
}

// Attention of query (t, h) over positions 0..npast+t of its KV head, online softmax, then the
// sigmoid output gate: out[t][h*D + i] = (sum_j p_j v_j[i]) * sigmoid(gate[i]) (core/xj_cpu.c:118-150).
// 4 warps (tid < 128); lanes split the head dim (D <= 256).
template <typename KV, int DPL, class Bar>
XJ_DEV void attn_head(const AttnArgs &a, int h, int t, int tid) {
    __shared__ float sm_m[4], sm_l[4];
    __shared__ float sm_o[4][256];
    const int warp = tid >> 5, lane = tid & 31, D = a.D;
    const int n = __ldcg(a.npast) + t + 1, kvh = h / (a.H / a.Hkv), kvd = a.Hkv * D;
    const float scale = 1.0f / sqrtf((float)D);
    const KV *kc = (const KV *)a.kc, *vc = (const KV *)a.vc;
    float qv[DPL], o[DPL];
    const float *qp = a.qrot + ((size_t)t * a.H + h) * D;
    const bool on = lane * DPL < D;   // head dims below 32 leave the upper lanes idle
#pragma unroll
    for (int d = 0; d < DPL; d++) { qv[d] = on ? lda(qp + lane * DPL + d) : 0.0f; o[d] = 0.0f; }
    float m = -INFINITY, l = 0.0f;
    for (int j = warp; j < n; j += 4) {
        const KV *kr = kc + (size_t)j * kvd + (size_t)kvh * D + lane * DPL;
        float s = 0.0f;
        if (on) {
#pragma unroll
            for (int d = 0; d < DPL; d++) s = fmaf(qv[d], load_kv(kr + d), s);
        }
        s = warp_sum(s) * scale;
        const float mn = fmaxf(m, s);
        const float corr = expf(m - mn), p = expf(s - mn);
        l = l * corr + p;
        if (on) {
            const KV *vr = vc + (size_t)j * kvd + (size_t)kvh * D + lane * DPL;
#pragma unroll
            for (int d = 0; d < DPL; d++) o[d] = fmaf(p, load_kv(vr + d), o[d] * corr);
        }
        m = mn;
    }
    if (lane == 0) { sm_m[warp] = m; sm_l[warp] = l; }
#pragma unroll
    for (int d = 0; d < DPL; d++) sm_o[warp][lane * DPL + d] = o[d];   // lane*DPL + d < 32*DPL <= 256
    Bar::sync();
    if (warp == 0) {
        float M = fmaxf(fmaxf(sm_m[0], sm_m[1]), fmaxf(sm_m[2], sm_m[3]));
        float L = 0.0f, c[4];
#pragma unroll
        for (int w = 0; w < 4; w++) { c[w] = sm_m[w] == -INFINITY ? 0.0f : expf(sm_m[w] - M); L += sm_l[w] * c[w]; }
        const float *gate = a.q + t * a.ldq + (size_t)h * 2 * D + D;
#pragma unroll
        for (int d = 0; d < DPL; d++) {
            const int i = lane * DPL + d;
            if (i >= D) break;
            float acc = 0.0f;
#pragma unroll
            for (int w = 0; w < 4; w++) acc = fmaf(sm_o[w][i], c[w], acc);
            a.out[t * a.ldo + (size_t)h * D + i] = (acc / L) * sigm_f(lda(gate + i));
        }
    }
    Bar::sync();   // sm_* are reused by the caller's next head
}

// Grid (H, T), 128 threads.
template <typename KV, int DPL>
static __global__ void __launch_bounds__(128) k_attn(AttnArgs a) {
    griddep_wait();
    griddep_launch();   // successors may start their prologue; they wait for this grid before reading
    attn_head<KV, DPL, BarBlock>(a, blockIdx.x, blockIdx.y, threadIdx.x);
}

// ---------------------------------------------------------------- FFN / misc
// out = silu(g) * u (core/xj_cpu.c:273).
static __global__ void k_swiglu(const float *g, const float *u, float *out, long long n) {
    griddep_wait();
    griddep_launch();   // successors may start their prologue; they wait for this grid before reading
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        out[i] = silu_f(g[i]) * u[i];
}

static __global__ void k_advance(int *npast, int T) {
    griddep_wait();
    griddep_launch();   // successors may start their prologue; they wait for this grid before reading
    if (threadIdx.x == 0 && blockIdx.x == 0) *npast += T;
}

// Positions of B sequences: npast[b] += T.
static __global__ void k_advance_batch(int *npast, int B, int T) {
    griddep_wait();
    griddep_launch();   // successors may start their prologue; they wait for this grid before reading
    for (int b = threadIdx.x; b < B; b += blockDim.x) npast[b] += T;
}

// Greedy pick over logits[V]: largest value, lowest index on ties (core/xj_spec.c:12-16); also the
// gap to the runner-up. Writes the id to out_tok[*step] and to *cur (the next step's input), the gap
// to margin[*step], then advances *step. One block of 1024 threads.
static __global__ void __launch_bounds__(1024) k_argmax(const float *logits, int V, int32_t *out_tok, float *margin,
                                                 int32_t *cur, int *step) {
    __shared__ float sv[32], sv2[32];
    __shared__ int si[32];
    griddep_wait();
    float b = -INFINITY, b2 = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
        const float v = logits[i];
        if (v > b || (v == b && i < bi)) { b2 = fmaxf(b2, b); b = v; bi = i; }
        else b2 = fmaxf(b2, v);
    }
    // warp reduce (value desc, index asc), keeping the runner-up value
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, b, o), ov2 = __shfl_xor_sync(0xffffffffu, b2, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > b || (ov == b && oi < bi)) { b2 = fmaxf(b, ov2); b = ov; bi = oi; }
        else b2 = fmaxf(b2, ov);
    }
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) { sv[w] = b; sv2[w] = b2; si[w] = bi; }
    __syncthreads();
    if (w == 0) {
        const int nw = blockDim.x >> 5;
        b = lane < nw ? sv[lane] : -INFINITY;
        b2 = lane < nw ? sv2[lane] : -INFINITY;
        bi = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, b, o), ov2 = __shfl_xor_sync(0xffffffffu, b2, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > b || (ov == b && oi < bi)) { b2 = fmaxf(b, ov2); b = ov; bi = oi; }
            else b2 = fmaxf(b2, ov);
        }
        if (lane == 0) {
            const int s = *step;
            out_tok[s] = bi;
            if (margin) margin[s] = b - b2;
            *cur = bi;
            *step = s + 1;
        }
    }
}

// Per 16-row tile of logits[V]: best value, runner-up, lowest best index (the partials the fused
// LM-head epilogue produces, for heads that are not on the tensor-core path). One warp per tile.
static __global__ void k_argmax_rows(const float *logits, int V, float *pbest, float *psecond, int *pidx) {
    griddep_wait();
    const int tile = blockIdx.x, row = threadIdx.x & 15, r = tile * 16 + row;
    float b = r < V ? logits[r] : -INFINITY, b2 = -INFINITY;
    int bi = r < V ? r : 0x7fffffff;
#pragma unroll
    for (int o = 8; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, b, o), ov2 = __shfl_xor_sync(0xffffffffu, b2, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > b || (ov == b && oi < bi)) { b2 = fmaxf(b, ov2); b = ov; bi = oi; }
        else b2 = fmaxf(b2, ov);
    }
    if (threadIdx.x == 0) { pbest[tile] = b; psecond[tile] = b2; pidx[tile] = bi; }
}

struct ArgmaxArgs {
    const float *pbest, *psecond;
    const int *pidx;
    int ntiles;
    int32_t *out_tok;
    float *margin;
    int32_t *cur;
    int *step;
    DevMat emb;
    float *x;
    int *npast;
};

// Greedy pick from the LM head's per-tile partials (best, runner-up, lowest index of each 16 rows):
// token = largest value, lowest index on ties (core/xj_spec.c:12-16). Writes out_tok[*step], the
// runner-up gap to margin[*step], the token to *cur, then the token's embedding row into x (the next
// decode step's input, core/xj_cpu.c:369-373), advances *npast by one and *step by one.
// nthr threads (a multiple of 32, at most 1024); Bar spans exactly those.
template <class Bar>
XJ_DEV void argmax_final_dev(const ArgmaxArgs &a, int tid, int nthr) {
    __shared__ float sv[32], sv2[32];
    __shared__ int si[32];
    __shared__ int s_tok;
    float b = -INFINITY, b2 = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = tid; i < a.ntiles; i += nthr) {
        const float v = __ldcg(a.pbest + i), v2 = __ldcg(a.psecond + i);
        const int vi = __ldcg(a.pidx + i);
        if (v > b || (v == b && vi < bi)) { b2 = fmaxf(fmaxf(b, b2), v2); b = v; bi = vi; }
        else b2 = fmaxf(b2, v);                      // the tile's runner-up is <= its best
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, b, o), ov2 = __shfl_xor_sync(0xffffffffu, b2, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > b || (ov == b && oi < bi)) { b2 = fmaxf(b, ov2); b = ov; bi = oi; }
        else b2 = fmaxf(b2, ov);
    }
    const int w = tid >> 5, lane = tid & 31;
    if (lane == 0) { sv[w] = b; sv2[w] = b2; si[w] = bi; }
    Bar::sync();
    if (w == 0) {
        const int nw = nthr >> 5;
        b = lane < nw ? sv[lane] : -INFINITY;
        b2 = lane < nw ? sv2[lane] : -INFINITY;
        bi = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, b, o), ov2 = __shfl_xor_sync(0xffffffffu, b2, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > b || (ov == b && oi < bi)) { b2 = fmaxf(b, ov2); b = ov; bi = oi; }
            else b2 = fmaxf(b2, ov);
        }
        if (lane == 0) {
            const int s = *a.step;
            a.out_tok[s] = bi;
            if (a.margin) a.margin[s] = b - b2;
            *a.cur = bi;
            *a.step = s + 1;
            *a.npast += 1;
            s_tok = bi;
        }
    }
    Bar::sync();
    const int id = s_tok;
    const DevMat &emb = a.emb;
    for (int e0 = tid * 8; e0 < emb.K; e0 += nthr * 8) {
        float y[8];
        if (id >= 0 && id < emb.N) dequant8(emb.type, emb.p + id * emb.ld, e0, y);
        else {
#pragma unroll
            for (int l = 0; l < 8; l++) y[l] = 0.0f;
        }
#pragma unroll
        for (int l = 0; l < 8; l++) a.x[e0 + l] = y[l];
    }
}

// One block of 1024 threads.
static __global__ void __launch_bounds__(1024) k_argmax_final(ArgmaxArgs a) {
    griddep_wait();
    griddep_launch();   // successors may start their prologue; they wait for this grid before reading
    argmax_final_dev<BarBlock>(a, threadIdx.x, blockDim.x);
}

// ---------------------------------------------------------------- batch of independent sequences
// One token of each of B sequences per launch: the single-sequence device functions with the
// operands of sequence b = blockIdx.y (its activation row, recurrent state, KV cache, position,
// output slots). The arithmetic per sequence is exactly the single-sequence kernels' at T = 1.

// Grid (Hv, B), 4*S threads; state of sequence b at ssm + b*state_stride.
template <int S>
__global__ void __launch_bounds__(4 * S, 2) k_gdn_batch(GdnArgs a, long long state_stride) {
    griddep_wait();
    griddep_launch();   // successors may start their prologue; they wait for this grid before reading
    const int b = blockIdx.y;
    GdnArgs c = a;
    c.qkv += b * a.ldq; c.z += b * a.ldz; c.beta += b * a.ldg; c.alpha += b * a.ldg;
    c.ssm += b * state_stride; c.out += b * a.ldo; c.T = 1; c.ck_ssm = nullptr;
    gdn_head<S, BarBlock>(c, blockIdx.x, threadIdx.x);
}

// ---------------------------------------------------------------- several tokens of every sequence
// B sequences x T tokens in one forward, rows b*T + t (speculative verify of a batch, chunked prefill of
// a batch); per token the arithmetic of the one-token kernels.

// Grid (Hv, B), 4*S threads: the T tokens of sequence b in order through its own state (gdn_head's token
// loop, as for a single-sequence prompt). ck_ssm (may be null): state after token t < T-1 at
// ck_ssm + b*ck_stride + t*Hv*S*S.
template <int S>
__global__ void __launch_bounds__(4 * S, 2) k_gdn_batch_multi(GdnArgs a, long long state_stride, long long ck_stride) {
    griddep_wait();
    griddep_launch();   // successors may start their prologue; they wait for this grid before reading
    const int b = blockIdx.y;
    const long long r = (long long)b * a.T;      // the sequence's first row
    GdnArgs c = a;
    c.qkv += r * a.ldq; c.z += r * a.ldz; c.beta += r * a.ldg; c.alpha += r * a.ldg;
    c.ssm += b * state_stride; c.out += r * a.ldo;
    c.ck_ssm = a.ck_ssm ? a.ck_ssm + b * ck_stride : nullptr;
    gdn_head<S, BarBlock>(c, blockIdx.x, threadIdx.x);
}

// The conv + SiLU of T tokens of each of B sequences (rows b*T + t) from their raw projections, with the
// arithmetic of the GEMV conv epilogue (y = silu(sum_k state_k w_k + raw w_last), core/xj_cpu.c:167-176).
// y_t depends only on the raw projections of tokens t - kc + 1 .. t (the conv state stands for the
// tokens before the forward), so every token is computed at once. Grid (ceil(CD / 128), B, ceil(T /
// GC_CT)), 128 threads: channel ch of sequence b, tokens t0 .. t0 + GC_CT - 1. ck (may be null): the
// state after token t < T-1 at ck[b][t][CD][kc-1]. kc <= 9. The state is only read here; k_conv_state
// then moves it past the forward's tokens.
constexpr int GC_CT = 16;
static __global__ void __launch_bounds__(128) k_conv_tokens(const float *raw, long long ldr, float *y, long long ldy,
                                                            const float *state, const float *w, int CD, int kc, int T,
                                                            float *ck) {
    griddep_wait();
    griddep_launch();   // successors may start their prologue; they wait for this grid before reading
    const int ch = blockIdx.x * blockDim.x + threadIdx.x, b = blockIdx.y, t0 = blockIdx.z * GC_CT;
    if (ch >= CD) return;
    const float *st = state + ((size_t)b * CD + ch) * (kc - 1);
    float wc[9], win[GC_CT + 8];       // win[j]: raw value of token t0 - (kc - 1) + j
#pragma unroll
    for (int k = 0; k < 9; k++) wc[k] = k < kc ? w[(size_t)ch * kc + k] : 0.0f;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const int tt = t0 - (kc - 1) + j;
        win[j] = j >= kc - 1 ? 0.0f : tt >= 0 ? raw[((size_t)b * T + tt) * ldr + ch] : st[tt + kc - 1];
    }
#pragma unroll
    for (int i = 0; i < GC_CT; i++) {
        const int t = t0 + i;
        const float v = t < T ? raw[((size_t)b * T + t) * ldr + ch] : 0.0f;
#pragma unroll
        for (int j = 0; j < 9; j++)
            if (j == kc - 1) win[i + j] = v;
    }
#pragma unroll
    for (int i = 0; i < GC_CT; i++) {
        const int t = t0 + i;
        if (t >= T) break;
        float acc = 0.0f;
#pragma unroll
        for (int k = 0; k < 8; k++)
            if (k < kc - 1) acc = fmaf(win[i + k], wc[k], acc);
        float wl = wc[0], xl = win[i];
#pragma unroll
        for (int k = 1; k < 9; k++)
            if (k == kc - 1) { wl = wc[k]; xl = win[i + k]; }
        acc = fmaf(xl, wl, acc);
        y[((size_t)b * T + t) * ldy + ch] = silu_f(acc);
        if (ck && t < T - 1)
#pragma unroll
            for (int k = 0; k < 8; k++)
                if (k < kc - 1) ck[(((size_t)b * (T - 1) + t) * CD + ch) * (kc - 1) + k] = win[i + 1 + k];
    }
}

// Grid (ceil(CD / 128), B), 128 threads: the conv state of channel ch of sequence b after the forward's
// T tokens (the last kc - 1 raw projections, older state entries when T < kc - 1).
static __global__ void __launch_bounds__(128) k_conv_state(const float *raw, long long ldr, float *state, int CD, int kc,
                                                           int T) {
    griddep_wait();
    griddep_launch();   // successors may start their prologue; they wait for this grid before reading
    const int ch = blockIdx.x * blockDim.x + threadIdx.x, b = blockIdx.y;
    if (ch >= CD) return;
    float *st = state + ((size_t)b * CD + ch) * (kc - 1);
    for (int k = 0; k < kc - 1; k++) {                     // ascending: st[k + T] is read before it is written
        const int tt = T - (kc - 1) + k;
        st[k] = tt >= 0 ? raw[((size_t)b * T + tt) * ldr + ch] : st[k + T];
    }
}

// Grid (blocks, B), 256 threads: sequence b keeps the first keep[b] (1..T) tokens of its last T-token
// forward: its n-float state becomes the copy taken after token keep[b]-1, at
// ck + b*ck_bstride + (keep[b]-1)*ck_slot (nothing to do when keep[b] == T: the state is current).
static __global__ void __launch_bounds__(256) k_batch_keep_state(float *state, long long n, const float *ck, long long ck_bstride,
                                                                 long long ck_slot, const int *keep, int T) {
    griddep_wait();
    griddep_launch();   // successors may start their prologue; they wait for this grid before reading
    const int b = blockIdx.y, kb = keep[b];
    if (kb >= T || kb < 1) return;
    const float *src = ck + b * ck_bstride + (kb - 1) * ck_slot;
    float *dst = state + b * n;
    const long long i0 = (long long)blockIdx.x * blockDim.x + threadIdx.x, step = (long long)gridDim.x * blockDim.x;
    if ((n & 3) == 0 && (ck_bstride & 3) == 0 && (ck_slot & 3) == 0)
        for (long long i = i0; i < n / 4; i += step)
            reinterpret_cast<float4 *>(dst)[i] = __ldcg(reinterpret_cast<const float4 *>(src) + i);
    else
        for (long long i = i0; i < n; i += step) dst[i] = __ldcg(src + i);
}

// npast[b] -= T - keep[b] (the tokens a sequence did not keep); one block.
static __global__ void k_batch_keep_pos(int *npast, const int *keep, int T, int B) {
    griddep_wait();
    griddep_launch();   // successors may start their prologue; they wait for this grid before reading
    for (int b = threadIdx.x; b < B; b += blockDim.x) npast[b] -= T - keep[b];
}

// Greedy acceptance of one speculative round for every sequence (one thread each), the rule of
// core/xj_spec.c:131-209: drafts d[b*ldd + i] (i < k), target picks p[b*(k+1) + t] after token t of the
// verified [last, d_0 .. d_(k-1)]; a = the longest prefix with d_i == p_i; the round emits d_0 .. d_(a-1)
// and p_a into out[b][n[b]..] (at most n_gen in all), keeps a + 1 tokens of the verify forward
// (keep[b]) and feeds p_a next (next[b]). stats[0] += k (drafted), stats[1] += a (accepted).
static __global__ void k_spec_accept_batch(const int32_t *d, int ldd, const int32_t *p, int k, int B, int32_t *out,
                                           long long out_stride, int *n, int n_gen, int *keep, int32_t *next,
                                           unsigned long long *stats) {
    griddep_wait();
    griddep_launch();   // successors may start their prologue; they wait for this grid before reading
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    const int32_t *db = d + (size_t)b * ldd, *pb = p + (size_t)b * (k + 1);
    int a = 0;
    while (a < k && db[a] == pb[a]) a++;
    int c = n[b];
    for (int i = 0; i <= a && c < n_gen; i++, c++) out[b * out_stride + c] = i < a ? db[i] : pb[a];
    n[b] = c;
    keep[b] = a + 1;
    next[b] = pb[a];
    atomicAdd(&stats[0], (unsigned long long)k);
    atomicAdd(&stats[1], (unsigned long long)a);
}

// The verify rows of a speculative round: row b*(k+1) = last[b], row b*(k+1) + 1 + i = d[b*ldd + i].
static __global__ void k_spec_rows(const int32_t *last, const int32_t *d, int ldd, int k, int B, int32_t *rows) {
    griddep_wait();
    griddep_launch();   // successors may start their prologue; they wait for this grid before reading
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= B * (k + 1)) return;
    const int b = i / (k + 1), t = i % (k + 1);
    rows[i] = t == 0 ? last[b] : d[(size_t)b * ldd + t - 1];
}

template <typename KV>
XJ_DEV AttnArgs attn_seq(const AttnArgs &a, const int *npast_b, long long kv_stride, int b) {
    AttnArgs c = a;
    c.q += b * a.ldq; c.k += b * a.ldkv; c.v += b * a.ldkv;
    c.qrot += (size_t)b * a.H * a.D;
    c.kc = (KV *)a.kc + b * kv_stride; c.vc = (KV *)a.vc + b * kv_stride;
    c.npast = npast_b + b;
    c.out += b * a.ldo;
    return c;
}

// Grid (H + Hkv, B), ceil32(D) threads; KV cache of sequence b at kc/vc + b*kv_stride elements.
template <typename KV>
static __global__ void k_attn_prep_batch(AttnArgs a, const int *npast_b, long long kv_stride) {
    griddep_wait();
    griddep_launch();   // successors may start their prologue; they wait for this grid before reading
    attn_prep_slot<KV, BarBlock>(attn_seq<KV>(a, npast_b, kv_stride, blockIdx.y), blockIdx.x, 0, threadIdx.x);
}

// Grid (H, B), 128 threads.
template <typename KV, int DPL>
static __global__ void __launch_bounds__(128) k_attn_batch(AttnArgs a, const int *npast_b, long long kv_stride) {
    griddep_wait();
    griddep_launch();   // successors may start their prologue; they wait for this grid before reading
    attn_head<KV, DPL, BarBlock>(attn_seq<KV>(a, npast_b, kv_stride, blockIdx.y), blockIdx.x, 0, threadIdx.x);
}

// Grid (ceil(ntiles/16), B), 256 threads: per-tile (16-row) argmax partials of each sequence's logits row.
static __global__ void __launch_bounds__(256) k_argmax_rows_batch(const float *logits, int V, float *pbest, float *psecond,
                                                                   int *pidx, int ntiles) {
    griddep_wait();
    griddep_launch();   // successors may start their prologue; they wait for this grid before reading
    // 16 tiles per block, one per half-warp (the shuffles below stay inside a half-warp)
    const int b = blockIdx.y, tile = blockIdx.x * 16 + (threadIdx.x >> 4), row = threadIdx.x & 15, r = tile * 16 + row;
    const float *lg = logits + (size_t)b * V;
    float v = r < V ? lg[r] : -INFINITY, v2 = -INFINITY;
    int vi = r < V ? r : 0x7fffffff;
#pragma unroll
    for (int o = 8; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o), ov2 = __shfl_xor_sync(0xffffffffu, v2, o);
        const int oi = __shfl_xor_sync(0xffffffffu, vi, o);
        if (ov > v || (ov == v && oi < vi)) { v2 = fmaxf(v, ov2); v = ov; vi = oi; }
        else v2 = fmaxf(v2, ov);
    }
    if (row == 0 && tile < ntiles) {
        const size_t o = (size_t)b * ntiles + tile;
        pbest[o] = v; psecond[o] = v2; pidx[o] = vi;
    }
}

// Grid (B), 1024 threads: the greedy pick of each sequence (argmax_final_dev on its partials),
// written to out_tok[b*out_stride + step_b], with the next token's embedding into row b of x.
static __global__ void __launch_bounds__(1024) k_argmax_final_batch(ArgmaxArgs a, long long out_stride, int E) {
    griddep_wait();
    griddep_launch();   // successors may start their prologue; they wait for this grid before reading
    const int b = blockIdx.x;
    ArgmaxArgs c = a;
    c.pbest += (size_t)b * a.ntiles; c.psecond += (size_t)b * a.ntiles; c.pidx += (size_t)b * a.ntiles;
    c.out_tok += b * out_stride;
    if (c.margin) c.margin += b * out_stride;
    c.cur += b; c.step += b; c.x += (size_t)b * E; c.npast += b;
    argmax_final_dev<BarBlock>(c, threadIdx.x, blockDim.x);
}

// Grid (T), 1024 threads: ids[t] = argmax of logits row t, the lowest index among equal maxima (the
// strict '>' of core/xj_spec.c:12-16).
static __global__ void __launch_bounds__(1024) k_argmax_pick_rows(const float *logits, int V, int32_t *ids) {
    griddep_wait();
    griddep_launch();   // successors may start their prologue; they wait for this grid before reading
    __shared__ float sb[32];
    __shared__ int si[32];
    const float *lg = logits + (size_t)blockIdx.x * V;
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
        const float v = lg[i];
        if (v > best) { best = v; bi = i; }
    }
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) { sb[w] = best; si[w] = bi; }
    __syncthreads();
    if (w == 0) {
        best = lane < (int)(blockDim.x >> 5) ? sb[lane] : -INFINITY;
        bi = lane < (int)(blockDim.x >> 5) ? si[lane] : 0x7fffffff;
        for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
        }
        if (lane == 0) ids[blockIdx.x] = bi == 0x7fffffff ? 0 : bi;
    }
}

}  // namespace xjk
