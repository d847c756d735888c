// xj_cuda_stage_new: the CUDA implementation of the runtime's stage vtable (include/xj_abi.h).
//
// State machine and error behaviour follow the reference CPU stage (src/xiaoju-pipe/core/xj_cpu.c):
//   forward   :244-280  (T checks, keep one-shot, ck_start/ck_T, n_past += T)
//   logits    :282-291  (output_norm or the MTP shared_head_norm, then the LM head)
//   rollback  :293-319  (KV-only stages truncate; recurrent stages restore checkpoint j)
//   reset     :321-330  (zero conv + recurrent state, n_past = 0)
//   ctor      :375-418  (layer-range / MTP-range validation)
// and the device-side structure follows the Metal stage's (metal/xj_metal.m:422-534): weights are
// uploaded once per stage, the KV cache is fp16 (fp32 on request), recurrent state fp32, and one
// forward is one stream of kernels with a single host synchronisation at the end.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <vector>

#include "../../include/xj_cuda.h"
#include "kernels.cuh"
#include "gemv_mma.cuh"
#include "sample.cuh"
#include "decode_mk.cuh"
#include "tc_gemm.cuh"

using namespace xjk;

namespace {

int g_opt_kv_f32 = 0;
int g_opt_gemv = 0;
int g_opt_persist = 1;
int g_opt_trace = 0;
int g_opt_tc = 1;

void seterr(char *err, size_t errlen, const char *fmt, ...) {
    if (!err || !errlen) return;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(err, errlen, fmt, ap);
    va_end(ap);
}

struct Layer {
    bool rec = false;
    float *attn_norm = nullptr, *post_norm = nullptr;
    DevMat ffn_gate{}, ffn_up{}, ffn_down{};
    // Gated DeltaNet
    DevMat qkv{}, gate{}, beta{}, alpha{}, out{};
    float *conv_w = nullptr, *dt = nullptr, *A = nullptr, *ssm_norm = nullptr;
    float *conv = nullptr, *ssm = nullptr, *ck_conv = nullptr, *ck_ssm = nullptr;
    // full attention
    bool fused = false;
    DevMat wqkv{}, wq{}, wk{}, wv{}, wo{};
    float *q_norm = nullptr, *k_norm = nullptr;
    void *kc = nullptr, *vc = nullptr;
};

struct Impl {
    int dev = 0;
    cudaStream_t st = nullptr;
    cudaEvent_t ev[3] = {};
    std::vector<Layer> L;
    std::map<const void *, DevMat> uploaded;   // host weight pointer -> device copy
    std::vector<void *> allocs;
    bool kv_f32 = false;
    int gemv_mode = 0;
    int n_ck = 0;
    size_t state_bytes = 0;
    DevMat tok_embd{}, output{}, mtp_eh{};
    float *output_norm = nullptr, *mtp_enorm = nullptr, *mtp_hnorm = nullptr, *mtp_head_norm = nullptr;
    // activations (device)
    float *x = nullptr, *xin = nullptr, *h = nullptr, *qkvb = nullptr, *z = nullptr, *beta = nullptr, *alpha = nullptr;
    float *o = nullptr, *qrot = nullptr, *g = nullptr, *u = nullptr, *logits = nullptr;
    float *q = nullptr, *k = nullptr, *v = nullptr, *hn = nullptr;
    void *wide_buf = nullptr;   // activations of a wide (5..16-token) GEMV launch, prepared by k_prep_xt<PREP_WIDE>
    void *b64_buf = nullptr;    // activations of a 64-token GEMV launch (stages taking more than 16 tokens)
    void *tc_buf = nullptr;     // the same in the tensor-core operand layout (k_gemm_tc), tc_nchunk chunks
    int tc_nchunk = 0;
    // chunked GDN (prompt forwards of >= GC_MIN_T tokens): normalised q, k and the chunk products
    float *gc_qn = nullptr, *gc_kn = nullptr, *gc_kk = nullptr, *gc_qk = nullptr, *gc_wx = nullptr;
    float *conv_raw = nullptr;    // [max_batch][conv_dim] raw qkv projections of prompts of 17+ tokens
    float *pbest = nullptr, *psecond = nullptr;
    int *pidx = nullptr;
    int *derr = nullptr;       // device error word: set when a kernel's bounded wait gives up
    int *npast = nullptr, *step = nullptr;
    int32_t *tok = nullptr, *cur = nullptr, *out_tok = nullptr;
    float *margin = nullptr;
    int out_cap = 0;
    // pinned host staging
    float *hx = nullptr, *hlogits = nullptr;
    // decode-step graph
    cudaGraphExec_t step_graph = nullptr;
    int step_kernels = 0;
    // persistent decode kernel: phase program (device), barrier counter, attention split scratch
    int mk_state = 0;          // 0: not built, 1: built, -1: this stage cannot use it
    bool mk_full = false, mkf_full = false;   // the program needs the full kernel variant (Q5_K / F16 / Q8_0 / sampling)
    MkPhase *mk_prog = nullptr;
    MkStream *mk_stream = nullptr;
    int mk_nphase = 0, mk_nstream = 0, mk_ctas = 0, mk_max_split = 1;
    // the layers-only program (one-token vtable forward): same kernel, no head or pick
    int mkf_state = 0;
    MkPhase *mkf_prog = nullptr;
    MkStream *mkf_stream = nullptr;
    int mkf_nphase = 0, mkf_nstream = 0;
    unsigned long long *mk_trace = nullptr;   // per CTA and phase: start, end (last step of a traced launch)
    std::vector<int> mk_ops;
    unsigned *mk_bar = nullptr;
    int *mk_diag = nullptr;
    float *mk_apart = nullptr;
    int *mk_acnt = nullptr;
    // recurrent-state snapshot (draft stage of speculative decoding): conv and GDN state per layer
    std::vector<float *> snap_conv, snap_ssm;
    int snap_np = -1;
    long long nlaunch = 0;                   // kernels launched on the stage stream so far
    long long last_launches[2] = {0, 0};     // last xj_cuda_decode: prompt, decode steps
    // sampler of xj_cuda_decode (xj_cuda_set_sampler): temperature <= 0 = greedy
    float samp_temp = 0.0f;
    double samp_top_p = 0.95;
    int samp_top_k = 40;
    unsigned long long samp_seed = 0;
};

Impl *I(xj_stage *s) { return (Impl *)s->impl; }

#define CK(call) do { cudaError_t e_ = (call); if (e_ != cudaSuccess) { seterr(err, errlen, "CUDA error %s at %s:%d", cudaGetErrorString(e_), __FILE__, __LINE__); return -1; } } while (0)

struct DevGuard {
    int prev = -1;
    explicit DevGuard(int d) { cudaGetDevice(&prev); if (prev != d) cudaSetDevice(d); }
    ~DevGuard() { int cur; cudaGetDevice(&cur); if (prev >= 0 && cur != prev) cudaSetDevice(prev); }
};

template <typename T>
int dalloc(Impl *im, T **p, size_t n, char *err, size_t errlen) {
    void *q = nullptr;
    cudaError_t e = cudaMalloc(&q, n ? n * sizeof(T) : 16);
    if (e != cudaSuccess) { seterr(err, errlen, "cudaMalloc(%zu bytes) failed: %s", n * sizeof(T), cudaGetErrorString(e)); return -1; }
    im->allocs.push_back(q);
    *p = (T *)q;
    return 0;
}

uint64_t row_bytes(uint32_t type, int64_t n) {
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

template <typename T>
int dput(Impl *im, const std::vector<T> &v, const uint8_t **dst, char *err, size_t errlen) {
    if (v.empty()) { *dst = nullptr; return 0; }
    uint8_t *p;
    if (dalloc(im, &p, v.size() * sizeof(T), err, errlen)) return -1;
    CK(cudaMemcpy(p, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice));
    *dst = p;
    return 0;
}

// Upload one weight once per host pointer: in the tensor-core tiled layout when the fast GEMV can
// take it, and/or in the GGUF row-major layout (always for the embedding table, which is read by row,
// and for everything the fast path cannot take).
int upload(Impl *im, const xj_w &w, DevMat *out, char *err, size_t errlen, bool need_rowmajor = false) {
    if (!w.data || !w.nbytes) { seterr(err, errlen, "weight is not mapped"); return -1; }
    DevMat d{nullptr, (int)w.type, (int)w.ne0, (int)w.ne1, (long long)row_bytes(w.type, w.ne0)};
    auto it = im->uploaded.find(w.data);
    if (it != im->uploaded.end()) d = it->second;
    bool want_tiled = im->gemv_mode == 0 && w.ne1 > 1 && tiled_ok((int)w.type, (int)w.ne0, (int)w.ne1);
    if (want_tiled && !d.tq) {
        TiledHost th;
        // a BF16 matrix whose values do not all fit the scaled fp16 layout stays row-major
        if (!repack_tiled((int)w.type, (const uint8_t *)w.data, (int)w.ne0, (int)w.ne1, th)) want_tiled = false;
        else if (dput(im, th.q, &d.tq, err, errlen) || dput(im, th.h, &d.th, err, errlen) ||
                 dput(im, th.s, &d.ts, err, errlen) || dput(im, th.d, &d.td, err, errlen)) return -1;
    }
    if ((need_rowmajor || !want_tiled) && !d.p) {
        uint8_t *p;
        if (dalloc(im, &p, (size_t)w.nbytes, err, errlen)) return -1;
        CK(cudaMemcpy(p, w.data, (size_t)w.nbytes, cudaMemcpyHostToDevice));
        d.p = p;
    }
    im->uploaded[w.data] = d;
    *out = d;
    return 0;
}

int upload_f32(Impl *im, const xj_w &w, float **out, char *err, size_t errlen) {
    if (w.type != XJ_F32) { seterr(err, errlen, "expected an F32 tensor"); return -1; }
    DevMat d;
    if (upload(im, w, &d, err, errlen)) return -1;
    *out = (float *)d.p;
    return 0;
}

// ------------------------------------------------------------------ launches
// One matrix of a GEMV group: y (+)= W f(x), with an epilogue (see gemv_mma.cuh).
struct Job {
    DevMat w;
    float *y;
    long long ldy;
    int epi = EPI_STORE;
    float *conv_state = nullptr;
    const float *conv_w = nullptr;
    float *conv_ck = nullptr;
    int kc = 0;
    long long conv_bstride = 0;   // batch of sequences: token t's conv state at conv_state + t*conv_bstride
    float *pbest = nullptr, *psecond = nullptr;
    int *pidx = nullptr;
};

template <typename... KArgs, typename... Args>
void launch(Impl *im, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, Args... args) {
    launch_pdl(kern, grid, block, smem, im->st, args...);
    im->nlaunch++;
}

// Activations of the 64-token GEMV: 64 tokens at the longest K.
// ntok: the most tokens of one forward (the tensor-core operand buffer holds that many, in 64-token chunks)
int alloc_b64(Impl *im, int ntok, char *err, size_t errlen) {
    const int nchunk = (ntok + TC_T - 1) / TC_T;
    if (dalloc(im, (uint8_t **)&im->b64_buf, b64_x_bytes(B64_T, MMA_KMAX), err, errlen) ||
        dalloc(im, (uint8_t **)&im->tc_buf, (size_t)nchunk * TC_XSTRIDE, err, errlen))
        return -1;
    im->tc_nchunk = nchunk;
    // the block-sum planes' unused columns stay zero (the tensor cores multiply them)
    CK(cudaMemset(im->tc_buf, 0, (size_t)nchunk * TC_XSTRIDE));
    return 0;
}

void rmsnorm(Impl *im, const float *x, long long ldx, const float *w, float *y, long long ldy, int n, int rows, float eps) {
    launch(im, k_rmsnorm, dim3(rows), dim3(256), 0, x, ldx, w, y, ldy, n, eps);
}

// y_j[t] (+)= W_j . f(x[t]) for a group of matrices sharing the input x[T][K]; f = identity, RMSNorm
// (norm_w) or SwiGLU silu(x) * x2. Tiled matrices go to the tensor-core kernel (one launch per weight
// type, f and the epilogues fused); the rest to the generic kernel with f and the epilogues as passes.
void gemv(Impl *im, const float *x, const float *x2, long long ldx, int T, int pro, const float *norm_w, float eps,
          std::initializer_list<Job> jobs) {
    const int K = jobs.begin()->w.K;
    std::vector<Job> fast, slow;
    for (const Job &j : jobs) {
        // a tiled matrix has no row-major copy: it always takes the tensor-core kernel
        if (j.w.tq && !(j.epi == EPI_ARGMAX && T != 1)) fast.push_back(j);
        else slow.push_back(j);
    }
    // group the fast matrices by weight type (one launch per group, at most 4 matrices each)
    std::vector<MmaArgs> groups;
    std::vector<int> gtype;
    std::vector<char> done(fast.size(), 0);
    for (size_t i = 0; i < fast.size(); i++) {
        if (done[i]) continue;
        MmaArgs m{};
        m.ldx = ldx; m.K = K; m.pro = pro; m.norm_w = norm_w; m.eps = eps; m.err = im->derr;
        const int type = tiled_type(fast[i].w.type);
        m.tile_start[0] = 0;
        for (size_t k = i; k < fast.size() && m.njob < 4; k++) {
            if (done[k] || tiled_type(fast[k].w.type) != type) continue;
            const Job &f = fast[k];
            MmaJob &mj = m.job[m.njob];
            mj.w = tiled_of(f.w); mj.y = f.y; mj.ldy = f.ldy; mj.epi = f.epi;
            mj.conv_state = f.conv_state; mj.conv_w = f.conv_w; mj.conv_ck = f.conv_ck; mj.kc = f.kc;
            mj.conv_bstride = f.conv_bstride;
            mj.pbest = f.pbest; mj.psecond = f.psecond; mj.pidx = f.pidx;
            m.tile_start[m.njob + 1] = m.tile_start[m.njob] + (f.w.N + 15) / 16;
            m.njob++;
            done[k] = 1;
        }
        groups.push_back(m);
        gtype.push_back(type);
    }
    // more than 16 tokens and every matrix fit for it: 64-token launches (weights streamed once per 64
    // tokens; each token's result depends only on the matrix shapes, not on the other tokens)
    bool use64 = T > MMA_WIDE_T && im->b64_buf && !groups.empty();
    for (const MmaArgs &m : groups)
        for (int j = 0; j < m.njob; j++) use64 = use64 && b64_ok(m.job[j], K);
    bool usetc = use64 && g_opt_tc && im->tc_buf;
    for (const MmaArgs &m : groups)
        for (int j = 0; j < m.njob; j++) usetc = usetc && tc_ok(m.job[j], K);
    if (usetc) {
        // tcgen05 tensor cores: weights decoded to fp16 pairs in shared memory, accumulators in TMEM
        // every token's operands in one launch when the buffer holds all chunks, else chunk by chunk
        const bool all = (T + TC_T - 1) / TC_T <= im->tc_nchunk;
        if (all)
            launch(im, k_prep_xt<PREP_TC>, dim3(T), dim3(MMA_WARPS * 32), 0, x, x2, ldx, K, pro, norm_w, eps, im->tc_buf, T);
        for (int t0 = 0; t0 < T; t0 += TC_T) {
            const int Tc = T - t0 < TC_T ? T - t0 : TC_T;
            if (!all)
                launch(im, k_prep_xt<PREP_TC>, dim3(Tc), dim3(MMA_WARPS * 32), 0, (const float *)(x + t0 * ldx),
                       (const float *)(x2 ? x2 + t0 * ldx : nullptr), ldx, K, pro, norm_w, eps, im->tc_buf, Tc);
            for (size_t gi = 0; gi < groups.size(); gi++) {
                const MmaArgs &m = groups[gi];
                B64Args b{};
                b.njob = m.njob; b.T = Tc; b.K = K;
                b.xbuf = all ? (void *)((uint8_t *)im->tc_buf + (size_t)(t0 / TC_T) * TC_XSTRIDE) : im->tc_buf;
                b.err = im->derr;
                for (int j = 0; j < m.njob; j++) {
                    b.job[j] = m.job[j];
                    if (b.job[j].y) b.job[j].y = m.job[j].y + t0 * m.job[j].ldy;
                    if (b.job[j].conv_bstride) b.job[j].conv_state = m.job[j].conv_state + t0 * m.job[j].conv_bstride;
                }
                launch_tc(b, gtype[gi], im->st);
                im->nlaunch++;
            }
        }
        groups.clear();
    } else if (use64) {
        for (int t0 = 0; t0 < T; t0 += B64_T) {
            const int Tc = T - t0 < B64_T ? T - t0 : B64_T;
            launch(im, k_prep_xt<PREP_B64>, dim3(Tc), dim3(MMA_WARPS * 32), 0, (const float *)(x + t0 * ldx),
                   (const float *)(x2 ? x2 + t0 * ldx : nullptr), ldx, K, pro, norm_w, eps, im->b64_buf, Tc);
            for (size_t gi = 0; gi < groups.size(); gi++) {
                const MmaArgs &m = groups[gi];
                B64Args b{};
                b.njob = m.njob; b.T = Tc; b.K = K;
                b.xbuf = im->b64_buf; b.err = im->derr;
                for (int j = 0; j < m.njob; j++) {
                    b.job[j] = m.job[j];
                    if (b.job[j].y) b.job[j].y = m.job[j].y + t0 * m.job[j].ldy;
                    if (b.job[j].conv_bstride) b.job[j].conv_state = m.job[j].conv_state + t0 * m.job[j].conv_bstride;
                }
                launch_b64(b, gtype[gi], im->st);
                im->nlaunch++;
            }
        }
        groups.clear();
    }
    // tokens in chunks of 16 (wide launches on activations prepared once per chunk) or, for 4 tokens or
    // fewer, one launch; each token's result does not depend on the chunking (the conv epilogue carries
    // its state across chunks, its checkpoints are indexed by absolute token)
    const int tch = T > MMA_MAXT ? MMA_WIDE_T : MMA_MAXT;
    for (int t0 = 0; t0 < T; t0 += tch) {
        const int Tc = T - t0 < tch ? T - t0 : tch;
        const bool wide = Tc > MMA_MAXT;
        if (wide && !groups.empty()) {
            launch(im, k_prep_xt<PREP_WIDE>, dim3(Tc), dim3(MMA_WARPS * 32), 0, (const float *)(x + t0 * ldx),
                   (const float *)(x2 ? x2 + t0 * ldx : nullptr), ldx, K, pro, norm_w, eps, im->wide_buf, Tc);
        }
        for (size_t gi = 0; gi < groups.size(); gi++) {
            const MmaArgs &m = groups[gi];
            MmaArgs c = m;
            c.T = Tc;
            c.x = x + t0 * ldx;
            c.x2 = x2 ? x2 + t0 * ldx : nullptr;
            for (int j = 0; j < c.njob; j++) {
                if (c.job[j].y) c.job[j].y = m.job[j].y + t0 * m.job[j].ldy;
                if (c.job[j].conv_bstride) c.job[j].conv_state = m.job[j].conv_state + t0 * m.job[j].conv_bstride;
                if (c.job[j].conv_ck) {
                    // the chunk saves the states after its tokens t0..t0+Tc-2; the one after t0+Tc-1
                    // (when that is not the last token) is saved by the next chunk as its "previous" state
                    c.job[j].conv_ck = m.job[j].conv_ck + (size_t)t0 * m.job[j].w.N * (m.job[j].kc - 1);
                }
            }
            if (wide) launch_wide(c, gtype[gi], im->wide_buf, im->st);
            else launch_mma(c, gtype[gi], im->st);
            im->nlaunch++;
            for (int j = 0; j < c.njob; j++)
                if (m.job[j].conv_ck && !m.job[j].conv_bstride && t0 + Tc < T) {
                    // state after token t0+Tc-1 = current conv state: copy it into its checkpoint slot
                    const size_t n = (size_t)m.job[j].w.N * (m.job[j].kc - 1);
                    cudaMemcpyAsync(m.job[j].conv_ck + (size_t)(t0 + Tc - 1) * n, m.job[j].conv_state, n * 4,
                                    cudaMemcpyDeviceToDevice, im->st);
                }
        }
    }
    if (slow.empty()) return;
    if (pro == PRO_NORM) {
        rmsnorm(im, x, ldx, norm_w, im->hn, K, K, T, eps);
        x = im->hn;
        ldx = K;
    } else if (pro == PRO_SWIGLU) {
        for (int t = 0; t < T; t++)
            launch(im, k_swiglu, dim3((K + 255) / 256), dim3(256), 0, (const float *)(x + t * ldx),
                   (const float *)(x2 + t * ldx), im->hn + (size_t)t * K, (long long)K);
        x = im->hn;
        ldx = K;
    }
    GemvArgs a{};
    a.x = x; a.ldx = ldx; a.T = T;
    for (size_t i0 = 0; i0 < slow.size(); i0 += 4) {
        a.njob = 0;
        a.row_start[0] = 0;
        for (size_t i = i0; i < slow.size() && a.njob < 4; i++) {
            a.job[a.njob] = {slow[i].w, slow[i].y, slow[i].ldy, slow[i].epi == EPI_ADD ? 1 : 0};
            a.row_start[a.njob + 1] = a.row_start[a.njob] + slow[i].w.N;
            a.njob++;
        }
        for (int t0 = 0; t0 < T; t0 += MAXT) {
            GemvArgs b = a;
            b.T = T - t0 < MAXT ? T - t0 : MAXT;
            b.x = x + t0 * ldx;
            for (int j = 0; j < b.njob; j++) b.job[j].y = a.job[j].y + t0 * a.job[j].ldy;
            launch(im, k_gemv_generic, dim3((b.row_start[b.njob] + 7) / 8), dim3(256), 0, b);
        }
    }
    for (const Job &j : slow) {
        if (j.epi == EPI_CONV)
            launch(im, k_conv_silu, dim3((j.w.N + 127) / 128), dim3(128), 0, j.y, j.ldy, T, j.w.N, j.kc, j.conv_state,
                   j.conv_w, j.conv_ck);
        else if (j.epi == EPI_ARGMAX)
            launch(im, k_argmax_rows, dim3((j.w.N + 15) / 16), dim3(32), 0, (const float *)j.y, j.w.N, j.pbest, j.psecond, j.pidx);
    }
}

GdnArgs gdn_args(Impl *im, const xj_hparams *hp, Layer &Ly, int T, bool ck) {
    GdnArgs g;
    g.qkv = im->qkvb; g.ldq = hp->conv_dim; g.z = im->z; g.ldz = hp->d_inner;
    g.beta = im->beta; g.alpha = im->alpha; g.ldg = hp->h_v;
    g.dt = Ly.dt; g.A = Ly.A; g.nw = Ly.ssm_norm;
    g.ssm = Ly.ssm; g.ck_ssm = ck ? Ly.ck_ssm : nullptr; g.out = im->o; g.ldo = hp->d_inner;
    g.T = T; g.Hk = hp->h_k; g.Hv = hp->h_v; g.key_dim = hp->key_dim; g.eps = hp->eps;
    return g;
}

// Chunked GDN over T tokens (no checkpoints): prep (per key head and chunk), the chunk-parallel solve
// (per value head and chunk), the state walk (per value head and 16-row block), gated RMSNorm.
// Scratch: qn, kn [T][Hk][S], kk, qk [Hk][chunks][GC_C][GC_C], wx gc_wx_floats(T, Hv, S).
template <int S>
void launch_gdn_chunked(Impl *im, const GdnArgs &g, float *qn, float *kn, float *kk, float *qk, float *wx) {
    static bool attr[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr[dev & 63]) {
        cudaFuncSetAttribute(k_gdn_chunk_prep<S>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gdn_prep_smem<S>());
        cudaFuncSetAttribute(k_gdn_chunk_solve<S>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gdn_solve_smem<S>());
        cudaFuncSetAttribute(k_gdn_chunk<S>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gdn_chunk_smem<S>());
        attr[dev & 63] = true;
    }
    const int nch = (g.T + GC_C - 1) / GC_C;
    launch(im, k_gdn_chunk_prep<S>, dim3(g.Hk, nch), dim3(256), gdn_prep_smem<S>(), g, qn, kn, kk, qk);
    launch(im, k_gdn_chunk_solve<S>, dim3(g.Hv, nch), dim3(2 * S), gdn_solve_smem<S>(), g, (const float *)qn,
           (const float *)kn, (const float *)kk, (const float *)qk, wx);
    launch(im, k_gdn_chunk<S>, dim3(g.Hv, S / 16), dim3(256), gdn_chunk_smem<S>(), g, (const float *)wx);
    launch(im, k_gdn_gnorm<S>, dim3(g.T, g.Hv), dim3(S), 0, g);
}
bool gdn_chunked_ok(const xj_hparams *hp) { return hp->s_v == hp->s_k && (hp->s_k == 32 || hp->s_k == 64 || hp->s_k == 128); }

void launch_gdn(Impl *im, const xj_hparams *hp, Layer &Ly, int T, bool ck) {
    const GdnArgs g = gdn_args(im, hp, Ly, T, ck);
    if (!ck && T >= GC_MIN_T && im->gc_qn && gdn_chunked_ok(hp)) {
        switch (hp->s_k) {
        case 32: launch_gdn_chunked<32>(im, g, im->gc_qn, im->gc_kn, im->gc_kk, im->gc_qk, im->gc_wx); return;
        case 64: launch_gdn_chunked<64>(im, g, im->gc_qn, im->gc_kn, im->gc_kk, im->gc_qk, im->gc_wx); return;
        default: launch_gdn_chunked<128>(im, g, im->gc_qn, im->gc_kn, im->gc_kk, im->gc_qk, im->gc_wx); return;
        }
    }
    switch (hp->s_k) {
    case 16: launch(im, k_gdn<16>, dim3(hp->h_v), dim3(64), 0, g); break;
    case 32: launch(im, k_gdn<32>, dim3(hp->h_v), dim3(128), 0, g); break;
    case 64: launch(im, k_gdn<64>, dim3(hp->h_v), dim3(256), 0, g); break;
    case 128: launch(im, k_gdn<128>, dim3(hp->h_v), dim3(512), 0, g); break;
    case 256: launch(im, k_gdn<256>, dim3(hp->h_v), dim3(1024), 0, g); break;
    default: break;
    }
}

AttnArgs attn_args(Impl *im, const xj_hparams *hp, Layer &Ly, const float *q, long long ldq, const float *k,
                   const float *v, long long ldkv) {
    AttnArgs a;
    a.q = q; a.ldq = ldq; a.k = k; a.v = v; a.ldkv = ldkv;
    a.qn = Ly.q_norm; a.kn = Ly.k_norm; a.qrot = im->qrot; a.kc = Ly.kc; a.vc = Ly.vc; a.npast = im->npast;
    a.out = im->o; a.ldo = (long long)hp->n_head * hp->head_dim;
    a.H = hp->n_head; a.Hkv = hp->n_head_kv; a.D = hp->head_dim; a.n_rot = hp->n_rot;
    a.base = hp->rope_base; a.eps = hp->eps;
    return a;
}

template <typename KV>
void launch_attn(Impl *im, const xj_hparams *hp, Layer &Ly, int T, const float *q, long long ldq, const float *k,
                 const float *v, long long ldkv) {
    const AttnArgs a = attn_args(im, hp, Ly, q, ldq, k, v, ldkv);
    const int H = hp->n_head, Hkv = hp->n_head_kv, D = hp->head_dim;
    launch(im, k_attn_prep<KV>, dim3(H + Hkv, T), dim3((D + 31) / 32 * 32), 0, a);
    // lanes cover the head dim DPL elements each: DPL = 1, 2, 4 or 8 (head dims up to 256)
    const int dpl = (D + 31) / 32;
    if (dpl == 1) launch(im, k_attn<KV, 1>, dim3(H, T), dim3(128), 0, a);
    else if (dpl == 2) launch(im, k_attn<KV, 2>, dim3(H, T), dim3(128), 0, a);
    else if (dpl <= 4) launch(im, k_attn<KV, 4>, dim3(H, T), dim3(128), 0, a);
    else launch(im, k_attn<KV, 8>, dim3(H, T), dim3(128), 0, a);
}

// All layers of the stage on im->x[T][E] (device) at positions *npast .. *npast+T-1, then a last kernel
// moves *npast forward by `advance` (the decode step's argmax kernel does its own +1).
void run_layers(xj_stage *s, int T, bool keep, int advance) {
    Impl *im = I(s);
    const xj_hparams *hp = &s->m->hp;
    const int E = hp->n_embd, FF = hp->n_ff;
    const float eps = hp->eps;
    for (int il = s->l0; il < s->l1; il++) {
        Layer &Ly = im->L[il - s->l0];
        if (Ly.rec) {
            const int CD = hp->conv_dim, DI = hp->d_inner, Hv = hp->h_v, kc = hp->conv_k;
            if (T > MMA_WIDE_T && kc <= 9 && im->conv_raw) {
                // more than 16 tokens: the raw projections from the 17..64-token kernels (their epilogue
                // has no conv carried across one sequence's tokens), then the conv over all tokens at once
                gemv(im, im->x, nullptr, E, T, PRO_NORM, Ly.attn_norm, eps,
                     {{Ly.qkv, im->conv_raw, CD}, {Ly.gate, im->z, DI}, {Ly.beta, im->beta, Hv}, {Ly.alpha, im->alpha, Hv}});
                launch(im, k_conv_tokens, dim3((CD + 127) / 128, 1, (T + GC_CT - 1) / GC_CT), dim3(128), 0,
                       (const float *)im->conv_raw, (long long)CD, im->qkvb, (long long)CD, (const float *)Ly.conv,
                       (const float *)Ly.conv_w, CD, kc, T, keep ? Ly.ck_conv : (float *)nullptr);
                launch(im, k_conv_state, dim3((CD + 127) / 128, 1), dim3(128), 0, (const float *)im->conv_raw,
                       (long long)CD, Ly.conv, CD, kc, T);
            } else {
                Job qkv{Ly.qkv, im->qkvb, CD};
                qkv.epi = EPI_CONV; qkv.conv_state = Ly.conv; qkv.conv_w = Ly.conv_w; qkv.kc = kc;
                qkv.conv_ck = keep ? Ly.ck_conv : nullptr;
                gemv(im, im->x, nullptr, E, T, PRO_NORM, Ly.attn_norm, eps,
                     {qkv, {Ly.gate, im->z, DI}, {Ly.beta, im->beta, Hv}, {Ly.alpha, im->alpha, Hv}});
            }
            launch_gdn(im, hp, Ly, T, keep);
            Job out{Ly.out, im->x, E};
            out.epi = EPI_ADD;
            gemv(im, im->o, nullptr, DI, T, PRO_NONE, nullptr, eps, {out});
        } else {
            const int H = hp->n_head, Hkv = hp->n_head_kv, D = hp->head_dim, nq = 2 * H * D, nk = Hkv * D;
            const float *q, *k, *v;
            long long ldq, ldkv;
            if (Ly.fused) {
                gemv(im, im->x, nullptr, E, T, PRO_NORM, Ly.attn_norm, eps, {{Ly.wqkv, im->qkvb, nq + 2 * nk}});
                q = im->qkvb; k = im->qkvb + nq; v = im->qkvb + nq + nk; ldq = ldkv = nq + 2 * nk;
            } else {
                gemv(im, im->x, nullptr, E, T, PRO_NORM, Ly.attn_norm, eps,
                     {{Ly.wq, im->q, nq}, {Ly.wk, im->k, nk}, {Ly.wv, im->v, nk}});
                q = im->q; k = im->k; v = im->v; ldq = nq; ldkv = nk;
            }
            if (im->kv_f32) launch_attn<float>(im, hp, Ly, T, q, ldq, k, v, ldkv);
            else launch_attn<__half>(im, hp, Ly, T, q, ldq, k, v, ldkv);
            Job o{Ly.wo, im->x, E};
            o.epi = EPI_ADD;
            gemv(im, im->o, nullptr, (long long)H * D, T, PRO_NONE, nullptr, eps, {o});
        }
        gemv(im, im->x, nullptr, E, T, PRO_NORM, Ly.post_norm, eps, {{Ly.ffn_gate, im->g, FF}, {Ly.ffn_up, im->u, FF}});
        Job down{Ly.ffn_down, im->x, E};
        down.epi = EPI_ADD;
        gemv(im, im->g, im->u, FF, T, PRO_SWIGLU, nullptr, eps, {down});
    }
    if (advance) launch(im, k_advance, dim3(1), dim3(32), 0, im->npast, advance);
}

// MTP prefix (core/xj_cpu.c:253-261): x[T][E] = eh_proj([enorm(emb) | hnorm(hid)]), input in im->xin[T][2E].
void run_mtp_prefix(xj_stage *s, int T) {
    Impl *im = I(s);
    const xj_hparams *hp = &s->m->hp;
    const int E = hp->n_embd;
    rmsnorm(im, im->xin, 2 * E, im->mtp_enorm, im->h, 2 * E, E, T, hp->eps);
    rmsnorm(im, im->xin + E, 2 * E, im->mtp_hnorm, im->h + E, 2 * E, E, T, hp->eps);
    gemv(im, im->h, nullptr, 2 * E, T, PRO_NONE, nullptr, hp->eps, {{im->mtp_eh, im->x, E}});
}

// Output norm + LM head: logits[T][V] (core/xj_cpu.c:282-291).
void head(xj_stage *s, const float *x, int T) {
    Impl *im = I(s);
    const xj_hparams *hp = &s->m->hp;
    gemv(im, x, nullptr, hp->n_embd, T, PRO_NORM, s->mtp ? im->mtp_head_norm : im->output_norm, hp->eps,
         {{im->output, im->logits, im->output.N}});
}

ArgmaxArgs argmax_args(Impl *im) {
    ArgmaxArgs a;
    a.pbest = im->pbest; a.psecond = im->psecond; a.pidx = im->pidx; a.ntiles = (im->output.N + 15) / 16;
    a.out_tok = im->out_tok; a.margin = im->margin; a.cur = im->cur; a.step = im->step;
    a.emb = im->tok_embd; a.x = im->x; a.npast = im->npast;
    return a;
}

// Output norm + LM head for one row with the greedy pick fused (per-tile partials, then one small
// kernel that also embeds the picked token into x and advances the position).
void head_argmax(xj_stage *s, const float *x) {
    Impl *im = I(s);
    const xj_hparams *hp = &s->m->hp;
    Job h{im->output, im->logits, im->output.N};
    h.epi = EPI_ARGMAX; h.pbest = im->pbest; h.psecond = im->psecond; h.pidx = im->pidx;
    gemv(im, x, nullptr, hp->n_embd, 1, PRO_NORM, im->output_norm, hp->eps, {h});
    launch(im, k_argmax_final, dim3(1), dim3(1024), 0, argmax_args(im));
}

// The pick after the last row x: greedy (head_argmax), or with a sampler set, the LM head's logits and a
// top-k / top-p draw (k_sample_final) that also embeds the picked token and advances the position.
void head_pick(xj_stage *s, const float *x) {
    Impl *im = I(s);
    if (im->samp_temp <= 0.0f) { head_argmax(s, x); return; }
    const xj_hparams *hp = &s->m->hp;
    gemv(im, x, nullptr, hp->n_embd, 1, PRO_NORM, im->output_norm, hp->eps, {{im->output, im->logits, im->output.N}});
    SampleArgs a{};
    a.logits = im->logits; a.ld = im->output.N; a.n = im->output.N;
    a.temp = im->samp_temp; a.top_p = im->samp_top_p; a.top_k = im->samp_top_k; a.seed = im->samp_seed;
    launch(im, k_sample_final, dim3(1), dim3(SAMPLE_THREADS), 0, a, argmax_args(im));
}

int sync_check(Impl *im, char *err, size_t errlen) {
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaStreamSynchronize(im->st);
    if (e != cudaSuccess) { seterr(err, errlen, "GPU error: %s", cudaGetErrorString(e)); return -1; }
    int flag = 0;
    if (im->derr && cudaMemcpy(&flag, im->derr, sizeof(int), cudaMemcpyDeviceToHost) == cudaSuccess && flag) {
        cudaMemset(im->derr, 0, sizeof(int));
        seterr(err, errlen, "a bounded wait on the GPU gave up (%s)",
               flag == 2 ? "grid barrier" : flag == 3 ? "tile partial hand-over" : "weight stream");
        return -1;
    }
    return 0;
}

// Checkpoint slots for speculative rollback (core/xj_cpu.c:228-242).
int ensure_ck(xj_stage *s, int n, char *err, size_t errlen) {
    Impl *im = I(s);
    const xj_hparams *hp = &s->m->hp;
    if (n <= im->n_ck) return 0;
    for (auto &Ly : im->L) {
        if (!Ly.rec) continue;
        float *a, *b;
        if (dalloc(im, &a, (size_t)n * hp->conv_dim * (hp->conv_k - 1), err, errlen)) return -1;
        if (dalloc(im, &b, (size_t)n * hp->h_v * hp->s_v * hp->s_k, err, errlen)) return -1;
        Ly.ck_conv = a; Ly.ck_ssm = b;
    }
    im->n_ck = n;
    return 0;
}

// ------------------------------------------------------------------ vtable
int mk_build(xj_stage *s, bool fwd, char *err, size_t errlen);
int mk_launch(xj_stage *s, int n, bool fwd, char *err, size_t errlen);

int cuda_forward(xj_stage *s, float *x, int T, char *err, size_t errlen) {
    Impl *im = I(s);
    DevGuard dg(im->dev);
    const int E = s->m->hp.n_embd;
    if (T <= 0 || T > s->max_batch) { seterr(err, errlen, "%d tokens in one forward exceeds the limit %d", T, s->max_batch); s->keep = 0; return -1; }
    if (s->n_past + T > s->n_ctx) { seterr(err, errlen, "context is full (%d)", s->n_ctx); s->keep = 0; return -1; }
    if (s->keep && ensure_ck(s, T - 1, err, errlen)) { s->keep = 0; return -1; }
    s->ck_start = s->n_past;
    s->ck_T = s->keep ? T : 0;
    const bool keep = s->keep != 0;
    const int in_w = s->mtp ? 2 * E : E;
    memcpy(im->hx, x, sizeof(float) * (size_t)T * in_w);
    if (cudaMemcpyAsync(s->mtp ? im->xin : im->x, im->hx, sizeof(float) * (size_t)T * in_w, cudaMemcpyHostToDevice, im->st) != cudaSuccess) {
        seterr(err, errlen, "host-to-device copy failed"); s->keep = 0; return -1;
    }
    if (s->mtp) run_mtp_prefix(s, T);
    // one token without checkpoints: the layers-only program of the persistent kernel, then the position
    char why[256];
    if (T == 1 && !keep && !s->mtp && g_opt_persist && mk_build(s, true, why, sizeof why) == 1) {
        if (mk_launch(s, 1, true, err, errlen)) { s->keep = 0; return -1; }
        launch(im, k_advance, dim3(1), dim3(32), 0, im->npast, 1);
    } else {
        run_layers(s, T, keep, T);
    }
    cudaMemcpyAsync(im->hx, im->x, sizeof(float) * (size_t)T * E, cudaMemcpyDeviceToHost, im->st);
    if (sync_check(im, err, errlen)) { s->keep = 0; return -1; }
    memcpy(x, im->hx, sizeof(float) * (size_t)T * E);
    s->n_past += T;
    s->keep = 0;
    return 0;
}

int cuda_logits(xj_stage *s, const float *x, int T, float *logits, char *err, size_t errlen) {
    Impl *im = I(s);
    DevGuard dg(im->dev);
    const int E = s->m->hp.n_embd, V = im->output.N;
    if (!s->has_head) { seterr(err, errlen, "this stage has no output head"); return -1; }
    if (T < 1 || T > s->max_batch) { seterr(err, errlen, "%d tokens for the output head exceeds the limit", T); return -1; }
    memcpy(im->hx, x, sizeof(float) * (size_t)T * E);
    CK(cudaMemcpyAsync(im->xin, im->hx, sizeof(float) * (size_t)T * E, cudaMemcpyHostToDevice, im->st));
    head(s, im->xin, T);
    cudaMemcpyAsync(im->hlogits, im->logits, sizeof(float) * (size_t)T * V, cudaMemcpyDeviceToHost, im->st);
    if (sync_check(im, err, errlen)) return -1;
    memcpy(logits, im->hlogits, sizeof(float) * (size_t)T * V);
    return 0;
}

int cuda_rollback(xj_stage *s, int n_past, char *err, size_t errlen) {
    Impl *im = I(s);
    DevGuard dg(im->dev);
    const xj_hparams *hp = &s->m->hp;
    if (n_past == s->n_past) { s->ck_T = 0; return 0; }
    bool recurrent = false;
    for (auto &Ly : im->L) if (Ly.rec) recurrent = true;
    if (!recurrent) {
        if (n_past < 0 || n_past > s->n_past) { seterr(err, errlen, "cannot roll back to position %d", n_past); return -1; }
    } else {
        const int j = n_past - s->ck_start - 1;
        if (!s->ck_T || s->n_past != s->ck_start + s->ck_T || j < 0 || j >= s->ck_T - 1) {
            seterr(err, errlen, "cannot roll back to position %d (checkpoints %d+%d, now %d)", n_past, s->ck_start, s->ck_T, s->n_past);
            return -1;
        }
        const size_t nc = (size_t)hp->conv_dim * (hp->conv_k - 1), ns = (size_t)hp->h_v * hp->s_v * hp->s_k;
        for (auto &Ly : im->L) {
            if (!Ly.rec) continue;
            CK(cudaMemcpyAsync(Ly.conv, Ly.ck_conv + (size_t)j * nc, nc * 4, cudaMemcpyDeviceToDevice, im->st));
            CK(cudaMemcpyAsync(Ly.ssm, Ly.ck_ssm + (size_t)j * ns, ns * 4, cudaMemcpyDeviceToDevice, im->st));
        }
        s->ck_T = 0;
    }
    int np = n_past;
    CK(cudaMemcpyAsync(im->npast, &np, sizeof(int), cudaMemcpyHostToDevice, im->st));
    if (sync_check(im, err, errlen)) return -1;
    s->n_past = n_past;
    return 0;
}

void cuda_reset(xj_stage *s) {
    Impl *im = I(s);
    DevGuard dg(im->dev);
    const xj_hparams *hp = &s->m->hp;
    for (auto &Ly : im->L) {
        if (!Ly.rec) continue;
        cudaMemsetAsync(Ly.conv, 0, sizeof(float) * hp->conv_dim * (hp->conv_k - 1), im->st);
        cudaMemsetAsync(Ly.ssm, 0, sizeof(float) * (size_t)hp->h_v * hp->s_v * hp->s_k, im->st);
    }
    cudaMemsetAsync(im->npast, 0, sizeof(int), im->st);
    cudaStreamSynchronize(im->st);
    s->n_past = 0;
}

void cuda_destroy(xj_stage *s) {
    if (!s) return;
    Impl *im = I(s);
    if (im) {
        DevGuard dg(im->dev);
        if (im->st) cudaStreamSynchronize(im->st);
        if (im->step_graph) cudaGraphExecDestroy(im->step_graph);
        for (void *p : im->allocs) cudaFree(p);
        if (im->hx) cudaFreeHost(im->hx);
        if (im->hlogits) cudaFreeHost(im->hlogits);
        for (auto &e : im->ev) if (e) cudaEventDestroy(e);
        if (im->st) cudaStreamDestroy(im->st);
        delete im;
    }
    free(s);
}

size_t scratch_floats(const xj_hparams *hp) {
    size_t n = (size_t)hp->n_ff;
    const size_t qkv = 2 * (size_t)hp->n_head * hp->head_dim + 2 * (size_t)hp->n_head_kv * hp->head_dim;
    if (qkv > n) n = qkv;
    if ((size_t)hp->conv_dim > n) n = hp->conv_dim;
    if ((size_t)hp->n_embd * 2 > n) n = 2 * (size_t)hp->n_embd;
    return n;
}

int build(xj_stage *s, char *err, size_t errlen) {
    Impl *im = I(s);
    const xj_model *m = s->m;
    const xj_hparams *hp = &m->hp;
    const int E = hp->n_embd, B = s->max_batch;
    CK(cudaStreamCreateWithFlags(&im->st, cudaStreamNonBlocking));
    for (auto &e : im->ev) CK(cudaEventCreate(&e));
    im->kv_f32 = g_opt_kv_f32 != 0;
    im->gemv_mode = g_opt_gemv;
    im->L.resize((size_t)(s->l1 - s->l0));
    for (int il = s->l0; il < s->l1; il++) {
        const xj_layer &X = m->layers[il];
        Layer &Ly = im->L[il - s->l0];
        Ly.rec = il < hp->n_layer && X.recurrent;
        if (upload_f32(im, X.attn_norm, &Ly.attn_norm, err, errlen) || upload_f32(im, X.post_norm, &Ly.post_norm, err, errlen) ||
            upload(im, X.ffn_gate, &Ly.ffn_gate, err, errlen) || upload(im, X.ffn_up, &Ly.ffn_up, err, errlen) ||
            upload(im, X.ffn_down, &Ly.ffn_down, err, errlen)) return -1;
        if (Ly.rec) {
            if (upload(im, X.ssm_qkv, &Ly.qkv, err, errlen) || upload(im, X.ssm_gate, &Ly.gate, err, errlen) ||
                upload(im, X.ssm_beta, &Ly.beta, err, errlen) || upload(im, X.ssm_alpha, &Ly.alpha, err, errlen) ||
                upload(im, X.ssm_out, &Ly.out, err, errlen) || upload_f32(im, X.ssm_conv1d, &Ly.conv_w, err, errlen) ||
                upload_f32(im, X.ssm_dt, &Ly.dt, err, errlen) || upload_f32(im, X.ssm_a, &Ly.A, err, errlen) ||
                upload_f32(im, X.ssm_norm, &Ly.ssm_norm, err, errlen)) return -1;
            const size_t nc = (size_t)hp->conv_dim * (hp->conv_k - 1), ns = (size_t)hp->h_v * hp->s_v * hp->s_k;
            if (dalloc(im, &Ly.conv, nc, err, errlen) || dalloc(im, &Ly.ssm, ns, err, errlen)) return -1;
            CK(cudaMemset(Ly.conv, 0, nc * 4));
            CK(cudaMemset(Ly.ssm, 0, ns * 4));
            im->state_bytes += (nc + ns) * 4;
        } else {
            Ly.fused = X.wqkv.nbytes != 0;
            if (Ly.fused) { if (upload(im, X.wqkv, &Ly.wqkv, err, errlen)) return -1; }
            else if (upload(im, X.wq, &Ly.wq, err, errlen) || upload(im, X.wk, &Ly.wk, err, errlen) ||
                     upload(im, X.wv, &Ly.wv, err, errlen)) return -1;
            if (upload(im, X.wo, &Ly.wo, err, errlen) || upload_f32(im, X.q_norm, &Ly.q_norm, err, errlen) ||
                upload_f32(im, X.k_norm, &Ly.k_norm, err, errlen)) return -1;
            const size_t n = (size_t)s->n_ctx * hp->n_head_kv * hp->head_dim, es = im->kv_f32 ? 4 : 2;
            uint8_t *a, *b;
            if (dalloc(im, &a, n * es, err, errlen) || dalloc(im, &b, n * es, err, errlen)) return -1;
            Ly.kc = a; Ly.vc = b;
            im->state_bytes += 2 * n * es;
        }
    }
    if (s->mtp) {
        if (upload(im, m->mtp_eh, &im->mtp_eh, err, errlen) || upload_f32(im, m->mtp_enorm, &im->mtp_enorm, err, errlen) ||
            upload_f32(im, m->mtp_hnorm, &im->mtp_hnorm, err, errlen) ||
            upload_f32(im, m->mtp_head_norm, &im->mtp_head_norm, err, errlen)) return -1;
    }
    if (s->has_head) {
        if (upload(im, m->output, &im->output, err, errlen) || upload_f32(im, m->output_norm, &im->output_norm, err, errlen)) return -1;
    }
    const size_t sf = scratch_floats(hp) * (size_t)B;
    const size_t V = s->has_head ? (size_t)m->output.ne1 : 1;
    if (dalloc(im, &im->x, (size_t)B * E, err, errlen) || dalloc(im, &im->xin, (size_t)B * 2 * E, err, errlen) ||
        dalloc(im, &im->h, (size_t)B * 2 * E, err, errlen) || dalloc(im, &im->qkvb, sf, err, errlen) ||
        dalloc(im, &im->z, sf, err, errlen) || dalloc(im, &im->beta, (size_t)B * hp->h_v + 16, err, errlen) ||
        dalloc(im, &im->alpha, (size_t)B * hp->h_v + 16, err, errlen) || dalloc(im, &im->o, sf, err, errlen) ||
        dalloc(im, &im->qrot, (size_t)B * hp->n_head * hp->head_dim, err, errlen) || dalloc(im, &im->g, sf, err, errlen) ||
        dalloc(im, &im->u, sf, err, errlen) || dalloc(im, &im->q, sf, err, errlen) || dalloc(im, &im->k, sf, err, errlen) ||
        dalloc(im, &im->v, sf, err, errlen) || dalloc(im, &im->logits, V * (size_t)B, err, errlen) ||
        dalloc(im, &im->hn, sf, err, errlen) ||
        dalloc(im, (uint8_t **)&im->wide_buf, wide_x_bytes(MMA_WIDE_T, MMA_KMAX), err, errlen) ||
        dalloc(im, &im->npast, 4, err, errlen) || dalloc(im, &im->step, 4, err, errlen) ||
        dalloc(im, &im->derr, 4, err, errlen) ||
        dalloc(im, &im->tok, (size_t)B, err, errlen) || dalloc(im, &im->cur, 4, err, errlen)) return -1;
    if (B > MMA_WIDE_T && (alloc_b64(im, B, err, errlen) ||
                           (hp->conv_dim > 0 && dalloc(im, &im->conv_raw, (size_t)B * hp->conv_dim, err, errlen)))) return -1;
    if (B >= GC_MIN_T && gdn_chunked_ok(hp)) {
        const size_t nch = (size_t)(B + GC_C - 1) / GC_C;
        if (dalloc(im, &im->gc_qn, (size_t)B * hp->key_dim, err, errlen) || dalloc(im, &im->gc_kn, (size_t)B * hp->key_dim, err, errlen) ||
            dalloc(im, &im->gc_kk, (size_t)hp->h_k * nch * GC_C * GC_C, err, errlen) ||
            dalloc(im, &im->gc_qk, (size_t)hp->h_k * nch * GC_C * GC_C, err, errlen) ||
            dalloc(im, &im->gc_wx, gc_wx_floats(B, hp->h_v, hp->s_v), err, errlen)) return -1;
    }
    if (s->has_head) {
        const size_t nt = (size_t)(m->output.ne1 + 15) / 16;
        if (dalloc(im, &im->pbest, nt, err, errlen) || dalloc(im, &im->psecond, nt, err, errlen) ||
            dalloc(im, &im->pidx, nt, err, errlen)) return -1;
    }
    CK(cudaMemset(im->npast, 0, 16));
    CK(cudaMemset(im->derr, 0, sizeof(int)));
    CK(cudaMallocHost(&im->hx, sizeof(float) * (size_t)B * 2 * E));
    CK(cudaMallocHost(&im->hlogits, sizeof(float) * V * (size_t)B));
    im->state_bytes += sizeof(float) * (sf * 7 + (size_t)B * 4 * E + V * B);
    CK(cudaDeviceSynchronize());
    return 0;
}

int count_kernels(cudaGraph_t g) {
    size_t n = 0;
    if (cudaGraphGetNodes(g, nullptr, &n) != cudaSuccess || !n) return 0;
    std::vector<cudaGraphNode_t> nodes(n);
    cudaGraphGetNodes(g, nodes.data(), &n);
    int k = 0;
    for (auto nd : nodes) {
        cudaGraphNodeType t;
        if (cudaGraphNodeGetType(nd, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) k++;
    }
    return k;
}

// One decode step on device: x = embed(*cur); layers; head on the last row; argmax -> out_tok[*step], *cur.
void decode_step(xj_stage *s) {
    Impl *im = I(s);
    run_layers(s, 1, false, 0);
    head_pick(s, im->x);
}

// ------------------------------------------------------------------ persistent decode kernel
// The phase program of one decode step: the same layer sequence as decode_step (run_layers at T = 1,
// then the head with the fused greedy pick), expressed for k_decode_persistent. Returns false when a
// matrix is not in the tiled layout (the persistent kernel has only the tensor-core GEMV).
bool mk_gemv(std::vector<MkPhase> &prog, std::vector<MkStream> &stream, int K, int pro, const float *x,
             const float *x2, const float *norm_w, float eps, int gs, std::initializer_list<Job> jobs) {
    MkPhase p{};
    MkStream ms{};
    p.op = MK_GEMV; p.K = K; p.pro = pro; p.x = x; p.x2 = x2; p.norm_w = norm_w; p.eps = eps; p.gs = gs;
    if (K > MK_KMAX || K % 32) return false;
    p.tile_start[0] = 0;
    for (const Job &f : jobs) {
        if (!f.w.tq || p.njob == 4 || f.w.K != K) return false;
        MmaJob &mj = p.job[p.njob];
        mj.w = tiled_of(f.w); mj.y = f.y; mj.ldy = f.ldy; mj.epi = f.epi;
        mj.conv_state = f.conv_state; mj.conv_w = f.conv_w; mj.conv_ck = nullptr; mj.kc = f.kc;
        mj.pbest = f.pbest; mj.psecond = f.psecond; mj.pidx = f.pidx;
        ms.type[p.njob] = mj.w.type; ms.nu[p.njob] = mj.w.nu;
        ms.q[p.njob] = mj.w.q; ms.h[p.njob] = mj.w.h; ms.s[p.njob] = mj.w.s; ms.d[p.njob] = mj.w.d;
        p.tile_start[p.njob + 1] = p.tile_start[p.njob] + (f.w.N + 15) / 16;
        p.njob++;
    }
    p.ntiles = p.tile_start[p.njob];
    ms.ntiles = p.ntiles; ms.njob = p.njob; ms.ph = (int)prog.size();
    for (int j = 0; j < 5; j++) ms.tile_start[j] = p.tile_start[j];
    prog.push_back(p);
    stream.push_back(ms);
    return true;
}

// 1: built, -1: unsupported for this stage, with the reason in err.
// fwd: the layers-only program of a one-token forward (no head, no pick: the caller advances the
// position); otherwise a whole greedy decode step.
int mk_build(xj_stage *s, bool fwd, char *err, size_t errlen) {
    Impl *im = I(s);
    int &state = fwd ? im->mkf_state : im->mk_state;
    if (state) return state;
    const xj_hparams *hp = &s->m->hp;
    const int E = hp->n_embd, FF = hp->n_ff;
    const float eps = hp->eps;
    std::vector<MkPhase> prog;
    std::vector<MkStream> stream;
    const int group = hp->n_head / hp->n_head_kv;
    bool ok = hp->s_k == hp->s_v && hp->head_dim <= 256 && hp->n_head % hp->n_head_kv == 0 && hp->conv_k <= MK_KC &&
              group <= MK_GQA && mk_attn_scratch(group, hp->head_dim, im->kv_f32 ? 4 : 2) <= MK_XS_BYTES;
    for (int il = s->l0; ok && il < s->l1; il++) {
        Layer &Ly = im->L[il - s->l0];
        if (Ly.rec) {
            const int CD = hp->conv_dim, DI = hp->d_inner, Hv = hp->h_v;
            Job qkv{Ly.qkv, im->qkvb, CD};
            qkv.epi = EPI_CONV; qkv.conv_state = Ly.conv; qkv.conv_w = Ly.conv_w; qkv.kc = hp->conv_k;
            // the gate rows z are stored as silu(z) (MK_EPI_SILU): only the gated norm below reads them
            Job zj{Ly.gate, im->z, DI};
            zj.epi = MK_EPI_SILU;
            ok = ok && mk_gemv(prog, stream, E, PRO_NORM, im->x, nullptr, Ly.attn_norm, eps, 0,
                               {qkv, zj, {Ly.beta, im->beta, Hv}, {Ly.alpha, im->alpha, Hv}});
            MkPhase g{};
            g.op = MK_GDN; g.gdn = gdn_args(im, hp, Ly, 1, false); g.gs = hp->s_k;
            prog.push_back(g);
            Job out{Ly.out, im->x, E};
            out.epi = EPI_ADD;
            ok = ok && mk_gemv(prog, stream, DI, PRO_GNORM_S, im->o, im->z, Ly.ssm_norm, eps, hp->s_k, {out});
        } else {
            const int H = hp->n_head, Hkv = hp->n_head_kv, D = hp->head_dim, nq = 2 * H * D, nk = Hkv * D;
            const float *q, *k, *v;
            long long ldq, ldkv;
            if (Ly.fused) {
                ok = ok && mk_gemv(prog, stream, E, PRO_NORM, im->x, nullptr, Ly.attn_norm, eps, 0, {{Ly.wqkv, im->qkvb, nq + 2 * nk}});
                q = im->qkvb; k = im->qkvb + nq; v = im->qkvb + nq + nk; ldq = ldkv = nq + 2 * nk;
            } else {
                ok = ok && mk_gemv(prog, stream, E, PRO_NORM, im->x, nullptr, Ly.attn_norm, eps, 0,
                                   {{Ly.wq, im->q, nq}, {Ly.wk, im->k, nk}, {Ly.wv, im->v, nk}});
                q = im->q; k = im->k; v = im->v; ldq = nq; ldkv = nk;
            }
            MkPhase a{};
            a.op = MK_ATTN; a.attn = attn_args(im, hp, Ly, q, ldq, k, v, ldkv);
            prog.push_back(a);
            Job o{Ly.wo, im->x, E};
            o.epi = EPI_ADD;
            ok = ok && mk_gemv(prog, stream, H * D, PRO_NONE, im->o, nullptr, nullptr, eps, 0, {o});
        }
        // the gate rows are stored as silu(gate) (MK_EPI_SILU), once, instead of in every CTA's prologue
        Job gate{Ly.ffn_gate, im->g, FF};
        gate.epi = MK_EPI_SILU;
        ok = ok && mk_gemv(prog, stream, E, PRO_NORM, im->x, nullptr, Ly.post_norm, eps, 0, {gate, {Ly.ffn_up, im->u, FF}});
        Job down{Ly.ffn_down, im->x, E};
        down.epi = EPI_ADD;
        ok = ok && mk_gemv(prog, stream, FF, PRO_SWIGLU_S, im->g, im->u, nullptr, eps, 0, {down});
    }
    // with a sampler set, the LM head also writes its logits for the SAMPLE phase
    const bool samp = im->samp_temp > 0.0f;
    if (!fwd) {
        Job h{im->output, samp ? im->logits : nullptr, im->output.N};
        h.epi = EPI_ARGMAX; h.pbest = im->pbest; h.psecond = im->psecond; h.pidx = im->pidx;
        ok = ok && mk_gemv(prog, stream, E, PRO_NORM, im->x, nullptr, im->output_norm, eps, 0, {h});
    }
    if (!ok) { state = -1; seterr(err, errlen, "persistent decode needs every matrix in the tiled layout"); return -1; }
    if (!fwd) {
        MkPhase am{};
        am.op = samp ? MK_SAMPLE : MK_ARGMAX; am.am = argmax_args(im);
        if (samp) {
            SampleArgs &a = am.sa;
            a.logits = im->logits; a.ld = im->output.N; a.n = im->output.N;
            a.temp = im->samp_temp; a.top_p = im->samp_top_p; a.top_k = im->samp_top_k; a.seed = im->samp_seed;
        }
        prog.push_back(am);
    }
    // side data each GEMV phase (and the GDN / attention phase after it) reads, for the producer's
    // L2 prefetch
    for (MkStream &ms : stream) {
        int n = 0;
        auto add = [&](const void *ptr, size_t bytes) {
            if (ptr && bytes >= 16 && n < 6) { ms.pf[n] = (const uint8_t *)ptr; ms.pf_bytes[n] = (unsigned)(bytes & ~(size_t)15); n++; }
        };
        const MkPhase &g = prog[ms.ph];
        if (g.pro == PRO_NORM) add(g.norm_w, (size_t)g.K * 4);
        if (g.pro == PRO_GNORM || g.pro == PRO_GNORM_S) add(g.norm_w, (size_t)g.gs * 4);
        for (int j = 0; j < g.njob; j++)
            if (g.job[j].epi == EPI_CONV) {
                add(g.job[j].conv_w, (size_t)g.job[j].w.N * g.job[j].kc * 4);
                add(g.job[j].conv_state, (size_t)g.job[j].w.N * (g.job[j].kc - 1) * 4);
            }
        if (ms.ph + 1 < (int)prog.size() && prog[ms.ph + 1].op == MK_GDN) {
            const GdnArgs &d = prog[ms.ph + 1].gdn;
            add(d.ssm, (size_t)d.Hv * hp->s_k * hp->s_k * 4);
            add(d.dt, (size_t)d.Hv * 4);
            add(d.A, (size_t)d.Hv * 4);
        }
        if (ms.ph + 1 < (int)prog.size() && prog[ms.ph + 1].op == MK_ATTN) {
            const AttnArgs &t = prog[ms.ph + 1].attn;
            add(t.qn, (size_t)t.D * 4);
            add(t.kn, (size_t)t.D * 4);
        }
    }

    // one CTA per SM, all resident (cooperative launch)
    int sms = 0, per_sm = 0, coop = 0;
    CK(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, im->dev));
    CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, im->dev));
    CK(cudaFuncSetAttribute(k_decode_persistent<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)MK_SMEM));
    CK(cudaFuncSetAttribute(k_decode_persistent<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)MK_SMEM));
    CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_decode_persistent<true>, MK_THREADS, MK_SMEM));
    int per_sm_lean = 0;
    CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm_lean, k_decode_persistent<false>, MK_THREADS, MK_SMEM));
    if (per_sm_lean < per_sm) per_sm = per_sm_lean;
    if (!coop || per_sm < 1) { state = -1; seterr(err, errlen, "cooperative launch of the persistent decode kernel is not possible"); return -1; }
    im->mk_ctas = sms;
    // the head phase leaves one greedy-pick partial per CTA that holds LM-head tiles
    if (!fwd) prog.back().am.ntiles = prog[prog.size() - 2].ntiles < sms ? prog[prog.size() - 2].ntiles : sms;
    // attention splits per KV head: at most one work item (KV head, split) per CTA
    int ms = sms / hp->n_head_kv;
    if (ms > MK_MAX_SPLIT) ms = MK_MAX_SPLIT;
    im->mk_max_split = ms > 0 ? ms : 1;
    // scratch shared by both programs (barrier counter, wait record, attention split partials)
    if (!im->mk_bar &&
        (dalloc(im, &im->mk_bar, 4, err, errlen) || dalloc(im, &im->mk_diag, 8, err, errlen) ||
         dalloc(im, &im->mk_acnt, (size_t)hp->n_head, err, errlen) ||
         dalloc(im, &im->mk_apart, (size_t)hp->n_head * im->mk_max_split * (hp->head_dim + 2), err, errlen))) return -1;
    // the program's size is fixed for a stage: a rebuild (after the output buffers moved) reuses these
    MkPhase *&dprog = fwd ? im->mkf_prog : im->mk_prog;
    MkStream *&dstream = fwd ? im->mkf_stream : im->mk_stream;
    if (!dprog && (dalloc(im, &dprog, prog.size(), err, errlen) || dalloc(im, &dstream, stream.size(), err, errlen))) return -1;
    if (!fwd && !im->mk_trace && dalloc(im, &im->mk_trace, (size_t)sms * prog.size() * 12, err, errlen)) return -1;
    CK(cudaMemcpy(dprog, prog.data(), prog.size() * sizeof(MkPhase), cudaMemcpyHostToDevice));
    CK(cudaMemcpy(dstream, stream.data(), stream.size() * sizeof(MkStream), cudaMemcpyHostToDevice));
    // a pageable host-to-device cudaMemcpy may return before its DMA lands, and the stage stream does
    // not wait for the legacy stream: the program must be complete before the kernel reads it
    CK(cudaDeviceSynchronize());
    if (fwd) {
        im->mkf_nphase = (int)prog.size();
        im->mkf_nstream = (int)stream.size();
    } else {
        im->mk_nphase = (int)prog.size();
        im->mk_nstream = (int)stream.size();
        im->mk_ops.clear();
        for (const MkPhase &q : prog) im->mk_ops.push_back(q.op);
    }
    bool full = false;
    for (const MkStream &q : stream)
        for (int j = 0; j < q.njob; j++) full = full || !(q.type[j] == XJ_Q4_K || q.type[j] == XJ_Q6_K);
    for (const MkPhase &q : prog) full = full || q.op == MK_SAMPLE;
    (fwd ? im->mkf_full : im->mk_full) = full;
    state = 1;
    return 1;
}

// n decode steps in one cooperative launch (k_decode_persistent).
int mk_launch(xj_stage *s, int n, bool fwd, char *err, size_t errlen) {
    Impl *im = I(s);
    MkArgs a{};
    if (fwd) { a.prog = im->mkf_prog; a.stream = im->mkf_stream; a.nphase = im->mkf_nphase; a.nstream = im->mkf_nstream; }
    else { a.prog = im->mk_prog; a.stream = im->mk_stream; a.nphase = im->mk_nphase; a.nstream = im->mk_nstream; }
    a.nsteps = n;
    a.trace = g_opt_trace && !fwd ? im->mk_trace : nullptr;
    a.bar = im->mk_bar; a.err = im->derr; a.apart = im->mk_apart; a.acnt = im->mk_acnt;
    a.max_split = im->mk_max_split; a.kv_f32 = im->kv_f32 ? 1 : 0; a.diag = im->mk_diag;
    CK(cudaMemsetAsync(im->mk_bar, 0, sizeof(unsigned), im->st));
    CK(cudaMemsetAsync(im->mk_diag, 0, sizeof(int) * 8, im->st));
    CK(cudaMemsetAsync(im->mk_acnt, 0, sizeof(int) * (size_t)s->m->hp.n_head, im->st));
    void *args[] = {&a};
    const bool full = (fwd ? im->mkf_full : im->mk_full) || a.trace;   // the phase trace is in the full variant
    const void *kern = full ? (const void *)k_decode_persistent<true> : (const void *)k_decode_persistent<false>;
    CK(cudaLaunchCooperativeKernel(kern, dim3(im->mk_ctas), dim3(MK_THREADS), args, MK_SMEM, im->st));
    return 0;
}

// ------------------------------------------------------------------ batch of independent sequences
// B sequences decoded in lockstep, one token of each per step (the reference has no multi-sequence API;
// this is additive). Weights and activation buffers are those of an ordinary stage with max_batch = B;
// each sequence has its own KV caches, Gated-DeltaNet and conv states and position. Matrix-vector
// products take the B tokens as one batch (each token's column is computed independently, so a
// sequence's result is bitwise the single-sequence one); attention, GDN and the greedy pick run one
// CUDA block per (head, sequence).
struct BatchImpl {
    xj_stage *s = nullptr;
    int B = 0, n_ctx = 0, n_past = 0;
    std::vector<float *> ssm, conv;        // per layer: [B][h_v][s_v][s_k], [B][conv_dim][conv_k-1]
    std::vector<void *> kc, vc;            // per layer: [B][n_ctx][n_head_kv * head_dim]
    int *npast = nullptr, *step = nullptr, *np_scratch = nullptr;
    int32_t *cur = nullptr, *prompts = nullptr, *out_tok = nullptr;
    float *margin = nullptr, *pbest = nullptr, *psecond = nullptr;
    int *pidx = nullptr;
    int ntiles = 0, out_cap = 0, prompt_cap = 0;
    cudaGraphExec_t step_graph = nullptr;
    int step_kernels = 0;
    long long last_launches[2] = {0, 0};
    bool async_rows = false;               // *_rows calls return without waiting for the stream
    // several tokens per sequence in one forward (xj_cuda_batch_new_spec): chunked prefill, speculative
    // verify. Rows b*T + t. Buffers of B*tmax rows; checkpoints allocated on the first verify.
    int tmax = 1;
    float *conv_raw = nullptr;             // [B*tmax][conv_dim] raw qkv projections
    int32_t *rows_tok = nullptr, *picks = nullptr;   // [B*tmax]
    float *x_multi = nullptr, *x_last = nullptr;     // [B*tmax][E], [B][E]
    std::vector<float *> ck_ssm, ck_conv;  // per layer: [B][tmax-1][state] after each verified token
    // speculative rounds (target side): acceptance per sequence
    int *keep = nullptr, *nout = nullptr;
    int32_t *next = nullptr, *spec_out = nullptr;
    int spec_out_cap = 0;
    unsigned long long *spec_stats = nullptr;
    // draft side: the recurrent state after each of the first k drafting steps, per layer [k][B][state]
    std::vector<float *> snap_ssm, snap_conv;
    int snap_k = 0;
};

// Layers of the batch's stage on rows x[0..nr) = sequences r0..r0+nr-1 (their own states and positions).
void run_layers_batch(BatchImpl *bi, float *x, int r0, int nr) {
    xj_stage *s = bi->s;
    Impl *im = I(s);
    const xj_hparams *hp = &s->m->hp;
    const int E = hp->n_embd, FF = hp->n_ff, B = nr;
    const float eps = hp->eps;
    const int *npast = bi->npast + r0;
    for (int il = s->l0; il < s->l1; il++) {
        Layer &Ly = im->L[il - s->l0];
        const int li = il - s->l0;
        if (Ly.rec) {
            const int CD = hp->conv_dim, DI = hp->d_inner, Hv = hp->h_v;
            Job qkv{Ly.qkv, im->qkvb, CD};
            qkv.epi = EPI_CONV; qkv.conv_state = bi->conv[li] + (size_t)r0 * hp->conv_dim * (hp->conv_k - 1); qkv.conv_w = Ly.conv_w; qkv.kc = hp->conv_k;
            qkv.conv_bstride = (long long)CD * (hp->conv_k - 1);
            gemv(im, x, nullptr, E, B, PRO_NORM, Ly.attn_norm, eps,
                 {qkv, {Ly.gate, im->z, DI}, {Ly.beta, im->beta, Hv}, {Ly.alpha, im->alpha, Hv}});
            GdnArgs g = gdn_args(im, hp, Ly, 1, false);
            g.ssm = bi->ssm[li] + (size_t)r0 * hp->h_v * hp->s_v * hp->s_k;
            const long long ss = (long long)hp->h_v * hp->s_v * hp->s_k;
            switch (hp->s_k) {
            case 16: launch(im, k_gdn_batch<16>, dim3(Hv, B), dim3(64), 0, g, ss); break;
            case 32: launch(im, k_gdn_batch<32>, dim3(Hv, B), dim3(128), 0, g, ss); break;
            case 64: launch(im, k_gdn_batch<64>, dim3(Hv, B), dim3(256), 0, g, ss); break;
            case 128: launch(im, k_gdn_batch<128>, dim3(Hv, B), dim3(512), 0, g, ss); break;
            default: launch(im, k_gdn_batch<256>, dim3(Hv, B), dim3(1024), 0, g, ss); break;
            }
            Job out{Ly.out, x, E};
            out.epi = EPI_ADD;
            gemv(im, im->o, nullptr, DI, B, PRO_NONE, nullptr, eps, {out});
        } else {
            const int H = hp->n_head, Hkv = hp->n_head_kv, D = hp->head_dim, nq = 2 * H * D, nk = Hkv * D;
            const float *q, *k, *v;
            long long ldq, ldkv;
            if (Ly.fused) {
                gemv(im, x, nullptr, E, B, PRO_NORM, Ly.attn_norm, eps, {{Ly.wqkv, im->qkvb, nq + 2 * nk}});
                q = im->qkvb; k = im->qkvb + nq; v = im->qkvb + nq + nk; ldq = ldkv = nq + 2 * nk;
            } else {
                gemv(im, x, nullptr, E, B, PRO_NORM, Ly.attn_norm, eps,
                     {{Ly.wq, im->q, nq}, {Ly.wk, im->k, nk}, {Ly.wv, im->v, nk}});
                q = im->q; k = im->k; v = im->v; ldq = nq; ldkv = nk;
            }
            AttnArgs a = attn_args(im, hp, Ly, q, ldq, k, v, ldkv);
            const long long kvs = (long long)bi->n_ctx * nk;
            const size_t kvoff = (size_t)r0 * kvs * (im->kv_f32 ? 4 : 2);
            a.kc = (uint8_t *)bi->kc[li] + kvoff; a.vc = (uint8_t *)bi->vc[li] + kvoff;
            const int dpl = (D + 31) / 32;
            if (im->kv_f32) {
                launch(im, k_attn_prep_batch<float>, dim3(H + Hkv, B), dim3((D + 31) / 32 * 32), 0, a, npast, kvs);
                if (dpl == 1) launch(im, k_attn_batch<float, 1>, dim3(H, B), dim3(128), 0, a, npast, kvs);
                else if (dpl == 2) launch(im, k_attn_batch<float, 2>, dim3(H, B), dim3(128), 0, a, npast, kvs);
                else if (dpl <= 4) launch(im, k_attn_batch<float, 4>, dim3(H, B), dim3(128), 0, a, npast, kvs);
                else launch(im, k_attn_batch<float, 8>, dim3(H, B), dim3(128), 0, a, npast, kvs);
            } else {
                launch(im, k_attn_prep_batch<__half>, dim3(H + Hkv, B), dim3((D + 31) / 32 * 32), 0, a, npast, kvs);
                if (dpl == 1) launch(im, k_attn_batch<__half, 1>, dim3(H, B), dim3(128), 0, a, npast, kvs);
                else if (dpl == 2) launch(im, k_attn_batch<__half, 2>, dim3(H, B), dim3(128), 0, a, npast, kvs);
                else if (dpl <= 4) launch(im, k_attn_batch<__half, 4>, dim3(H, B), dim3(128), 0, a, npast, kvs);
                else launch(im, k_attn_batch<__half, 8>, dim3(H, B), dim3(128), 0, a, npast, kvs);
            }
            Job o{Ly.wo, x, E};
            o.epi = EPI_ADD;
            gemv(im, im->o, nullptr, (long long)H * D, B, PRO_NONE, nullptr, eps, {o});
        }
        gemv(im, x, nullptr, E, B, PRO_NORM, Ly.post_norm, eps, {{Ly.ffn_gate, im->g, FF}, {Ly.ffn_up, im->u, FF}});
        Job down{Ly.ffn_down, x, E};
        down.epi = EPI_ADD;
        gemv(im, im->g, im->u, FF, B, PRO_SWIGLU, nullptr, eps, {down});
    }
}

// Layers of the batch's stage on T tokens of every sequence at once (rows b*T + t of x, T <= tmax): the
// one-token kernels per token (the same arithmetic), the conv through its own kernel so each sequence's
// tokens pass its rolling state in order, attention token by token (token t at position npast[b] + t).
// ck: checkpoints of each sequence's GDN and conv state after tokens t < T-1 (speculative verify).
// Positions advance by `advance` at the end.
void run_layers_batch_multi(BatchImpl *bi, float *x, int T, bool ck, int advance) {
    xj_stage *s = bi->s;
    Impl *im = I(s);
    const xj_hparams *hp = &s->m->hp;
    const int E = hp->n_embd, FF = hp->n_ff, B = bi->B, R = B * T;
    const float eps = hp->eps;
    for (int il = s->l0; il < s->l1; il++) {
        Layer &Ly = im->L[il - s->l0];
        const int li = il - s->l0;
        if (Ly.rec) {
            const int CD = hp->conv_dim, DI = hp->d_inner, Hv = hp->h_v, kc = hp->conv_k;
            gemv(im, x, nullptr, E, R, PRO_NORM, Ly.attn_norm, eps,
                 {{Ly.qkv, bi->conv_raw, CD}, {Ly.gate, im->z, DI}, {Ly.beta, im->beta, Hv}, {Ly.alpha, im->alpha, Hv}});
            launch(im, k_conv_tokens, dim3((CD + 127) / 128, B, (T + GC_CT - 1) / GC_CT), dim3(128), 0,
                   (const float *)bi->conv_raw, (long long)CD, im->qkvb, (long long)CD, (const float *)bi->conv[li],
                   (const float *)Ly.conv_w, CD, kc, T, ck ? bi->ck_conv[li] : (float *)nullptr);
            launch(im, k_conv_state, dim3((CD + 127) / 128, B), dim3(128), 0, (const float *)bi->conv_raw, (long long)CD,
                   bi->conv[li], CD, kc, T);
            GdnArgs g = gdn_args(im, hp, Ly, T, false);
            g.ssm = bi->ssm[li];
            g.ck_ssm = ck ? bi->ck_ssm[li] : nullptr;
            const long long ss = (long long)hp->h_v * hp->s_v * hp->s_k, cks = (long long)(T - 1) * ss;
            switch (hp->s_k) {
            case 16: launch(im, k_gdn_batch_multi<16>, dim3(Hv, B), dim3(64), 0, g, ss, cks); break;
            case 32: launch(im, k_gdn_batch_multi<32>, dim3(Hv, B), dim3(128), 0, g, ss, cks); break;
            case 64: launch(im, k_gdn_batch_multi<64>, dim3(Hv, B), dim3(256), 0, g, ss, cks); break;
            default: launch(im, k_gdn_batch_multi<128>, dim3(Hv, B), dim3(512), 0, g, ss, cks); break;
            }
            Job out{Ly.out, x, E};
            out.epi = EPI_ADD;
            gemv(im, im->o, nullptr, DI, R, PRO_NONE, nullptr, eps, {out});
        } else {
            const int H = hp->n_head, Hkv = hp->n_head_kv, D = hp->head_dim, nq = 2 * H * D, nk = Hkv * D;
            const float *q, *k, *v;
            long long ldq, ldkv;
            if (Ly.fused) {
                gemv(im, x, nullptr, E, R, PRO_NORM, Ly.attn_norm, eps, {{Ly.wqkv, im->qkvb, nq + 2 * nk}});
                q = im->qkvb; k = im->qkvb + nq; v = im->qkvb + nq + nk; ldq = ldkv = nq + 2 * nk;
            } else {
                gemv(im, x, nullptr, E, R, PRO_NORM, Ly.attn_norm, eps,
                     {{Ly.wq, im->q, nq}, {Ly.wk, im->k, nk}, {Ly.wv, im->v, nk}});
                q = im->q; k = im->k; v = im->v; ldq = nq; ldkv = nk;
            }
            const long long kvs = (long long)bi->n_ctx * nk;
            const int dpl = (D + 31) / 32;
            for (int t = 0; t < T; t++) {
                // token t of every sequence: rows t, t + T, ... (strides of T rows), position npast[b]
                AttnArgs a = attn_args(im, hp, Ly, q + t * ldq, ldq * T, k + t * ldkv, v + t * ldkv, ldkv * T);
                a.out = im->o + (size_t)t * H * D;
                a.ldo = (long long)T * H * D;
                a.kc = bi->kc[li]; a.vc = bi->vc[li];
                if (im->kv_f32) {
                    launch(im, k_attn_prep_batch<float>, dim3(H + Hkv, B), dim3((D + 31) / 32 * 32), 0, a, (const int *)bi->npast, kvs);
                    if (dpl == 1) launch(im, k_attn_batch<float, 1>, dim3(H, B), dim3(128), 0, a, (const int *)bi->npast, kvs);
                    else if (dpl == 2) launch(im, k_attn_batch<float, 2>, dim3(H, B), dim3(128), 0, a, (const int *)bi->npast, kvs);
                    else if (dpl <= 4) launch(im, k_attn_batch<float, 4>, dim3(H, B), dim3(128), 0, a, (const int *)bi->npast, kvs);
                    else launch(im, k_attn_batch<float, 8>, dim3(H, B), dim3(128), 0, a, (const int *)bi->npast, kvs);
                } else {
                    launch(im, k_attn_prep_batch<__half>, dim3(H + Hkv, B), dim3((D + 31) / 32 * 32), 0, a, (const int *)bi->npast, kvs);
                    if (dpl == 1) launch(im, k_attn_batch<__half, 1>, dim3(H, B), dim3(128), 0, a, (const int *)bi->npast, kvs);
                    else if (dpl == 2) launch(im, k_attn_batch<__half, 2>, dim3(H, B), dim3(128), 0, a, (const int *)bi->npast, kvs);
                    else if (dpl <= 4) launch(im, k_attn_batch<__half, 4>, dim3(H, B), dim3(128), 0, a, (const int *)bi->npast, kvs);
                    else launch(im, k_attn_batch<__half, 8>, dim3(H, B), dim3(128), 0, a, (const int *)bi->npast, kvs);
                }
                launch(im, k_advance_batch, dim3(1), dim3(256), 0, bi->npast, B, 1);
            }
            launch(im, k_advance_batch, dim3(1), dim3(256), 0, bi->npast, B, -T);
            Job o{Ly.wo, x, E};
            o.epi = EPI_ADD;
            gemv(im, im->o, nullptr, (long long)H * D, R, PRO_NONE, nullptr, eps, {o});
        }
        gemv(im, x, nullptr, E, R, PRO_NORM, Ly.post_norm, eps, {{Ly.ffn_gate, im->g, FF}, {Ly.ffn_up, im->u, FF}});
        Job down{Ly.ffn_down, x, E};
        down.epi = EPI_ADD;
        gemv(im, im->g, im->u, FF, R, PRO_SWIGLU, nullptr, eps, {down});
    }
    if (advance) launch(im, k_advance_batch, dim3(1), dim3(256), 0, bi->npast, B, advance);
}

// Prompts of every sequence (host [B][n]) through the batch in chunks of up to tmax tokens per
// sequence, continuing from the sequences' positions, which advance by n. copy_last: the last prompt
// token's activation row of each sequence into x_last [B][E] (for the head). Queued on the stage stream;
// the ids go through bi->prompts (capacity B*n, grown here).
int batch_prefill(BatchImpl *bi, const int32_t *prompts, int n, bool copy_last, char *err, size_t errlen) {
    xj_stage *s = bi->s;
    Impl *im = I(s);
    const int B = bi->B, E = s->m->hp.n_embd, tm = bi->tmax;
    if (n > bi->prompt_cap) {
        CK(cudaStreamSynchronize(im->st));
        if (dalloc(im, &bi->prompts, (size_t)B * n, err, errlen)) return -1;
        bi->prompt_cap = n;
    }
    // chunk-major ids: chunk [i0, i0 + Tc) holds B*Tc ids at offset i0*B, rows b*Tc + t
    std::vector<int32_t> h((size_t)B * n);
    for (int i0 = 0; i0 < n; i0 += tm) {
        const int Tc = n - i0 < tm ? n - i0 : tm;
        for (int b = 0; b < B; b++)
            for (int t = 0; t < Tc; t++) h[(size_t)i0 * B + (size_t)b * Tc + t] = prompts[(size_t)b * n + i0 + t];
    }
    CK(cudaMemcpyAsync(bi->prompts, h.data(), h.size() * sizeof(int32_t), cudaMemcpyHostToDevice, im->st));
    CK(cudaStreamSynchronize(im->st));   // h is a host temporary
    for (int i0 = 0; i0 < n; i0 += tm) {
        const int Tc = n - i0 < tm ? n - i0 : tm;
        launch(im, k_embed, dim3((E / 8 + 127) / 128, B * Tc), dim3(128), 0, im->tok_embd,
               (const int32_t *)(bi->prompts + (size_t)i0 * B), B * Tc, im->x, E);
        run_layers_batch_multi(bi, im->x, Tc, false, Tc);
        if (copy_last && i0 + Tc == n)
            CK(cudaMemcpy2DAsync(bi->x_last, sizeof(float) * E, im->x + (size_t)(Tc - 1) * E, sizeof(float) * E * Tc,
                                 sizeof(float) * E, B, cudaMemcpyDeviceToDevice, im->st));
    }
    bi->n_past += n;
    return 0;
}

// LM head and greedy pick of R rows of x: ids[r] (lowest id on equal logits).
void head_pick_rows(BatchImpl *bi, const float *x, int R, int32_t *ids) {
    xj_stage *s = bi->s;
    Impl *im = I(s);
    const xj_hparams *hp = &s->m->hp;
    const int V = im->output.N;
    gemv(im, x, nullptr, hp->n_embd, R, PRO_NORM, im->output_norm, hp->eps, {{im->output, im->logits, V}});
    launch(im, k_argmax_pick_rows, dim3(R), dim3(1024), 0, (const float *)im->logits, V, ids);
}

// Output norm + LM head for rows x[0..nr) = sequences r0.., then each sequence's greedy pick: out_tok of
// sequence r0+i at its step, the token into cur[i], its embedding into row i of emb_x, emb_np[i] + 1.
// The whole-batch decode passes x itself and the positions; a pipeline's last stage passes scratch.
void head_batch(BatchImpl *bi, const float *x, int r0, int nr, int32_t *cur, float *emb_x, int *emb_np) {
    xj_stage *s = bi->s;
    Impl *im = I(s);
    const xj_hparams *hp = &s->m->hp;
    const int V = im->output.N, B = nr;
    gemv(im, x, nullptr, hp->n_embd, B, PRO_NORM, im->output_norm, hp->eps, {{im->output, im->logits, V}});
    launch(im, k_argmax_rows_batch, dim3((bi->ntiles + 15) / 16, B), dim3(256), 0, (const float *)im->logits, V, bi->pbest, bi->psecond,
           bi->pidx, bi->ntiles);
    ArgmaxArgs a;
    a.pbest = bi->pbest; a.psecond = bi->psecond; a.pidx = bi->pidx; a.ntiles = bi->ntiles;
    a.out_tok = bi->out_tok + (size_t)r0 * bi->out_cap; a.margin = bi->margin + (size_t)r0 * bi->out_cap;
    a.cur = cur; a.step = bi->step + r0;
    a.emb = im->tok_embd; a.x = emb_x; a.npast = emb_np;
    launch(im, k_argmax_final_batch, dim3(B), dim3(1024), 0, a, (long long)bi->out_cap, hp->n_embd);
}

int batch_reset_state(BatchImpl *bi, char *err, size_t errlen) {
    Impl *im = I(bi->s);
    const xj_hparams *hp = &bi->s->m->hp;
    const size_t ns = (size_t)bi->B * hp->h_v * hp->s_v * hp->s_k, nc = (size_t)bi->B * hp->conv_dim * (hp->conv_k - 1);
    for (float *p : bi->ssm) if (p) CK(cudaMemsetAsync(p, 0, ns * 4, im->st));     // GDN layers only
    for (float *p : bi->conv) if (p) CK(cudaMemsetAsync(p, 0, nc * 4, im->st));
    CK(cudaMemsetAsync(bi->npast, 0, sizeof(int) * bi->B, im->st));
    CK(cudaStreamSynchronize(im->st));
    bi->n_past = 0;
    return 0;
}

}  // namespace

extern "C" {

const char *xj_cuda_device_name(void) {
    static char name[256];
    int d = 0;
    cudaDeviceProp p;
    if (cudaGetDevice(&d) != cudaSuccess || cudaGetDeviceProperties(&p, d) != cudaSuccess) return "CUDA";
    snprintf(name, sizeof name, "%s", p.name);
    return name;
}

int xj_cuda_set_options(int which, int value) {
    switch (which) {
    case XJC_OPT_KV_F32: g_opt_kv_f32 = value; return 0;
    case XJC_OPT_GEMV: g_opt_gemv = value; return 0;
    case XJC_OPT_PDL: g_pdl = value ? 1 : 0; return 0;
    case XJC_OPT_PERSIST: g_opt_persist = value; return 0;
    case XJC_OPT_TRACE: g_opt_trace = value; return 0;
    case XJC_OPT_TC: g_opt_tc = value ? 1 : 0; return 0;
    case XJC_OPT_GEMV_CTAS: if (value < 1 || value > 2) return -1; g_mma_ctas_per_sm = value; return 0;
    default: return -1;
    }
}

xj_stage *xj_cuda_stage_new(const xj_model *m, int l0, int l1, int n_ctx, int max_batch, bool has_head, char *err,
                            size_t errlen) {
    const xj_hparams *hp = &m->hp;
    const bool mtp = m->has_mtp && l0 == hp->n_layer && l1 == hp->n_layer + 1;
    if (l0 < 0 || (l1 > hp->n_layer && !mtp) || l0 > l1) { seterr(err, errlen, "bad layer range [%d,%d)", l0, l1); return nullptr; }
    if (hp->head_dim > 256 || hp->head_dim % 8) { seterr(err, errlen, "head dim %d not supported", hp->head_dim); return nullptr; }
    if (hp->s_k != 16 && hp->s_k != 32 && hp->s_k != 64 && hp->s_k != 128 && hp->s_k != 256) {
        seterr(err, errlen, "linear-attention head dim %d not supported", hp->s_k); return nullptr;
    }
    if (hp->conv_k < 2 || hp->conv_k > 9) { seterr(err, errlen, "conv kernel %d not supported", hp->conv_k); return nullptr; }
    if (n_ctx <= 0 || max_batch <= 0) { seterr(err, errlen, "n_ctx and max_batch must be positive"); return nullptr; }
    for (int il = l0; il < l1; il++) {
        const xj_layer &X = m->layers[il];
        if (!X.ffn_down.data) { seterr(err, errlen, "layer %d weights are not mapped", il); return nullptr; }
        // every matrix-vector product reads its input 8 elements at a time
        const xj_w *mats[] = {&X.ffn_gate, &X.ffn_up, &X.ffn_down, &X.ssm_qkv, &X.ssm_gate, &X.ssm_beta, &X.ssm_alpha,
                              &X.ssm_out, &X.wqkv, &X.wq, &X.wk, &X.wv, &X.wo};
        for (const xj_w *w : mats)
            if (w->nbytes && w->ne0 % 8) { seterr(err, errlen, "layer %d: row length %lld is not a multiple of 8", il, (long long)w->ne0); return nullptr; }
    }
    if (n_ctx > (1 << 24)) { seterr(err, errlen, "n_ctx %d too large", n_ctx); return nullptr; }
    if (has_head && !m->output.data) { seterr(err, errlen, "output head is not mapped"); return nullptr; }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) { seterr(err, errlen, "no CUDA device"); return nullptr; }
    xj_stage *s = (xj_stage *)calloc(1, sizeof(xj_stage));
    Impl *im = new Impl();
    im->dev = dev;
    s->m = m; s->l0 = l0; s->l1 = l1; s->n_ctx = n_ctx; s->max_batch = max_batch; s->has_head = has_head; s->mtp = mtp;
    s->backend = "cuda";
    s->forward = cuda_forward; s->logits = cuda_logits; s->rollback = cuda_rollback; s->reset = cuda_reset;
    s->destroy = cuda_destroy;
    s->impl = im;
    if (build(s, err, errlen)) { cuda_destroy(s); return nullptr; }
    return s;
}

int xj_cuda_decode(xj_stage *s, const int32_t *prompt, int n_prompt, int n_gen, int32_t *out, float *margins,
                   float *gpu_ms, char *err, size_t errlen) {
    if (!s || s->backend == nullptr || strcmp(s->backend, "cuda") != 0) { seterr(err, errlen, "not a CUDA stage"); return -1; }
    Impl *im = I(s);
    DevGuard dg(im->dev);
    const xj_model *m = s->m;
    const int E = m->hp.n_embd;
    if (s->mtp || s->l0 != 0 || s->l1 != m->hp.n_layer || !s->has_head) {
        seterr(err, errlen, "decode needs a stage over all layers with the head"); return -1;
    }
    if (n_prompt <= 0 || n_gen <= 0) { seterr(err, errlen, "need at least one prompt token and one generated token"); return -1; }
    if (s->n_past + n_prompt + n_gen - 1 > s->n_ctx) { seterr(err, errlen, "context is full (%d)", s->n_ctx); return -1; }
    if (!im->tok_embd.p) {
        if (upload(im, m->tok_embd, &im->tok_embd, err, errlen, true)) return -1;
        CK(cudaDeviceSynchronize());   // the upload's DMA must land before the stage stream reads it
    }
    if (n_gen > im->out_cap) {
        // the step graph and the persistent kernel's program write through these pointers: rebuild them
        if (im->step_graph) { cudaGraphExecDestroy(im->step_graph); im->step_graph = nullptr; }
        if (im->mk_state == 1) im->mk_state = 0;
        const int cap = n_gen > 4096 ? n_gen : 4096;
        if (dalloc(im, &im->out_tok, (size_t)cap, err, errlen) || dalloc(im, &im->margin, (size_t)cap, err, errlen)) return -1;
        im->out_cap = cap;
    }
    CK(cudaMemsetAsync(im->step, 0, sizeof(int), im->st));
    int persist = 0;
    if (g_opt_persist) {   // the persistent kernel picks greedily or samples (a sampler set)
        char why[256];
        persist = mk_build(s, false, why, sizeof why) == 1;
    }
    CK(cudaEventRecord(im->ev[0], im->st));
    const long long nl0 = im->nlaunch;
    const int B = s->max_batch;
    // with the persistent kernel the prompt's last token is its first step (it picks out[0]); otherwise
    // the last prompt chunk ends with the head and the greedy pick
    const int n_pre = persist ? n_prompt - 1 : n_prompt;
    for (int i = 0; i < n_pre; i += B) {
        const int T = n_pre - i < B ? n_pre - i : B;
        CK(cudaMemcpyAsync(im->tok, prompt + i, sizeof(int32_t) * T, cudaMemcpyHostToDevice, im->st));
        launch(im, k_embed, dim3((E / 8 + 127) / 128, T), dim3(128), 0, im->tok_embd, (const int32_t *)im->tok, T, im->x, E);
        const bool last = !persist && i + T == n_prompt;
        run_layers(s, T, false, last ? T - 1 : T);
        if (last) head_pick(s, im->x + (size_t)(T - 1) * E);   // picks out[0], embeds it, position +1
    }
    if (persist) {
        CK(cudaMemcpyAsync(im->tok, prompt + n_prompt - 1, sizeof(int32_t), cudaMemcpyHostToDevice, im->st));
        launch(im, k_embed, dim3((E / 8 + 127) / 128, 1), dim3(128), 0, im->tok_embd, (const int32_t *)im->tok, 1, im->x, E);
    }
    CK(cudaEventRecord(im->ev[1], im->st));
    im->last_launches[0] = im->nlaunch - nl0;
    im->last_launches[1] = 0;
    if (persist) {
        // every step in the persistent kernel (step 0 = the last prompt token); segments of at most 8192
        // steps keep the grid barrier's 32-bit counter far from wrapping
        for (int done = 0; done < n_gen; done += 8192) {
            if (mk_launch(s, n_gen - done < 8192 ? n_gen - done : 8192, false, err, errlen)) return -1;
            im->last_launches[1]++;
        }
    } else if (n_gen > 1) {
        if (!im->step_graph) {
            cudaGraph_t g;
            CK(cudaStreamBeginCapture(im->st, cudaStreamCaptureModeThreadLocal));
            decode_step(s);
            CK(cudaStreamEndCapture(im->st, &g));
            im->step_kernels = count_kernels(g);
            cudaError_t e = cudaGraphInstantiate(&im->step_graph, g, 0);
            cudaGraphDestroy(g);
            if (e != cudaSuccess) { seterr(err, errlen, "graph instantiate: %s", cudaGetErrorString(e)); im->step_graph = nullptr; return -1; }
        }
        for (int i = 1; i < n_gen; i++) CK(cudaGraphLaunch(im->step_graph, im->st));
        im->last_launches[1] = (long long)(n_gen - 1) * im->step_kernels;
    }
    CK(cudaEventRecord(im->ev[2], im->st));
    CK(cudaMemcpyAsync(out, im->out_tok, sizeof(int32_t) * n_gen, cudaMemcpyDeviceToHost, im->st));
    if (margins) CK(cudaMemcpyAsync(margins, im->margin, sizeof(float) * n_gen, cudaMemcpyDeviceToHost, im->st));
    if (sync_check(im, err, errlen)) {
        int d[8] = {0};
        if (persist && im->mk_diag && cudaMemcpy(d, im->mk_diag, sizeof d, cudaMemcpyDeviceToHost) == cudaSuccess && d[0]) {
            const size_t n = strlen(err);
            snprintf(err + n, errlen > n ? errlen - n : 0,
                     " [persistent kernel: wait kind %d, cta %d, thread %d, step %d, phase %d, index %d, extra %d]",
                     d[0], d[1], d[2], d[3], d[4], d[5], d[6]);
        }
        return -1;
    }
    if (gpu_ms) {
        cudaEventElapsedTime(&gpu_ms[0], im->ev[0], im->ev[1]);
        cudaEventElapsedTime(&gpu_ms[1], im->ev[1], im->ev[2]);
    }
    s->n_past += n_prompt + n_gen - 1;
    return 0;
}

// Diagnostic GEMV on host buffers: y[t][n] = W[n] . x[t] with the decode-path kernels (path 0 = fastest
// available, 1 = generic), or average device time per launch over `iters` launches rotating through
// `copies` device copies of W (so L2 cannot serve the weights) when ms != nullptr.
static int gemv_diag(int type, const void *w, int k, int n, const float *x, int t, float *y, int path, int copies,
                     int iters, float *ms, char *err, size_t errlen) {
    if (t < 1 || t > B64_T) { seterr(err, errlen, "t must be in 1..%d", B64_T); return -1; }
    if (k % 8) { seterr(err, errlen, "k must be a multiple of 8"); return -1; }
    Impl tmp;
    Impl *im = &tmp;
    im->gemv_mode = path;
    CK(cudaStreamCreateWithFlags(&im->st, cudaStreamNonBlocking));
    int rc = -1;
    float *dx = nullptr, *dy = nullptr;
    std::vector<DevMat> mats;
    const uint64_t nbytes = row_bytes((uint32_t)type, k) * (uint64_t)n;
    if (!nbytes) { seterr(err, errlen, "unsupported type %d", type); goto done; }
    if (copies < 1) copies = 1;
    {
        std::vector<uint8_t> buf((const uint8_t *)w, (const uint8_t *)w + nbytes);
        for (int c = 0; c < copies; c++) {
            xj_w hw{};
            if (c) buf[0] ^= 0;   // identical bytes, distinct device copies
            hw.data = buf.data() + 0; hw.nbytes = nbytes; hw.type = (uint32_t)type; hw.ne0 = k; hw.ne1 = n;
            im->uploaded.clear();
            DevMat d;
            if (upload(im, hw, &d, err, errlen)) goto done;
            mats.push_back(d);
        }
    }
    if (dalloc(im, &dx, (size_t)t * k, err, errlen) || dalloc(im, &dy, (size_t)t * n, err, errlen) ||
        dalloc(im, &im->hn, (size_t)t * k, err, errlen) || dalloc(im, &im->derr, 1, err, errlen) ||
        dalloc(im, (uint8_t **)&im->wide_buf, wide_x_bytes(MMA_WIDE_T, MMA_KMAX), err, errlen) ||
        (t > MMA_WIDE_T && alloc_b64(im, t, err, errlen))) goto done;
    cudaMemset(im->derr, 0, sizeof(int));
    if (cudaMemcpy(dx, x, sizeof(float) * (size_t)t * k, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaDeviceSynchronize() != cudaSuccess) { seterr(err, errlen, "copy failed"); goto done; }
    gemv(im, dx, nullptr, k, t, PRO_NONE, nullptr, 0.0f, {{mats[0], dy, n}});
    if (ms) {
        cudaEvent_t e0, e1;
        cudaEventCreate(&e0); cudaEventCreate(&e1);
        for (int i = 0; i < 3; i++) gemv(im, dx, nullptr, k, t, PRO_NONE, nullptr, 0.0f, {{mats[i % copies], dy, n}});
        cudaEventRecord(e0, im->st);
        for (int i = 0; i < iters; i++) gemv(im, dx, nullptr, k, t, PRO_NONE, nullptr, 0.0f, {{mats[i % copies], dy, n}});
        cudaEventRecord(e1, im->st);
        cudaEventSynchronize(e1);
        cudaEventElapsedTime(ms, e0, e1);
        *ms /= iters;
        cudaEventDestroy(e0); cudaEventDestroy(e1);
    }
    if (y && cudaMemcpyAsync(y, dy, sizeof(float) * (size_t)t * n, cudaMemcpyDeviceToHost, im->st) != cudaSuccess) {
        seterr(err, errlen, "copy failed"); goto done;
    }
    if (sync_check(im, err, errlen)) goto done;
    rc = 0;
done:
    cudaStreamSynchronize(im->st);
    for (void *p : im->allocs) cudaFree(p);
    im->allocs.clear();
    cudaStreamDestroy(im->st);
    return rc;
}

int xj_cuda_gemv(int type, const void *w, int k, int n, const float *x, int t, float *y, int path, char *err, size_t errlen) {
    return gemv_diag(type, w, k, n, x, t, y, path, 1, 0, nullptr, err, errlen);
}

int xj_cuda_gemv_time(int type, const void *w, int k, int n, int t, int copies, int iters, int path, float *ms,
                      char *err, size_t errlen) {
    std::vector<float> x((size_t)t * k, 0.5f);
    return gemv_diag(type, w, k, n, x.data(), t, nullptr, path, copies, iters, ms, err, errlen);
}

// ------------------------------------------------------------------ speculative decoding with a draft model
// Tokens -> embeddings -> layers on the device (no output head); n_past += T.
static int feed_tokens(xj_stage *s, const int32_t *toks, int T, bool keep, char *err, size_t errlen) {
    Impl *im = I(s);
    const int E = s->m->hp.n_embd;
    if (T < 1 || T > s->max_batch || s->n_past + T > s->n_ctx) { seterr(err, errlen, "cannot feed %d tokens", T); return -1; }
    if (keep && ensure_ck(s, T - 1, err, errlen)) return -1;
    s->ck_start = s->n_past;
    s->ck_T = keep ? T : 0;
    CK(cudaMemcpyAsync(im->tok, toks, sizeof(int32_t) * T, cudaMemcpyHostToDevice, im->st));
    launch(im, k_embed, dim3((E / 8 + 127) / 128, T), dim3(128), 0, im->tok_embd, (const int32_t *)im->tok, T, im->x, E);
    run_layers(s, T, keep, T);
    return 0;
}

// Recurrent state (conv + GDN state of every layer) and position of a stage: save / restore. KV rows
// beyond a restored position are simply overwritten later.
static int snapshot(xj_stage *s, char *err, size_t errlen) {
    Impl *im = I(s);
    const xj_hparams *hp = &s->m->hp;
    const size_t nc = (size_t)hp->conv_dim * (hp->conv_k - 1), ns = (size_t)hp->h_v * hp->s_v * hp->s_k;
    if (im->snap_conv.empty()) {
        im->snap_conv.assign(im->L.size(), nullptr);
        im->snap_ssm.assign(im->L.size(), nullptr);
        for (size_t li = 0; li < im->L.size(); li++) {
            if (!im->L[li].rec) continue;
            if (dalloc(im, &im->snap_conv[li], nc, err, errlen) || dalloc(im, &im->snap_ssm[li], ns, err, errlen)) return -1;
        }
    }
    for (size_t li = 0; li < im->L.size(); li++) {
        if (!im->L[li].rec) continue;
        CK(cudaMemcpyAsync(im->snap_conv[li], im->L[li].conv, nc * 4, cudaMemcpyDeviceToDevice, im->st));
        CK(cudaMemcpyAsync(im->snap_ssm[li], im->L[li].ssm, ns * 4, cudaMemcpyDeviceToDevice, im->st));
    }
    im->snap_np = s->n_past;
    return 0;
}
static int restore(xj_stage *s, char *err, size_t errlen) {
    Impl *im = I(s);
    const xj_hparams *hp = &s->m->hp;
    const size_t nc = (size_t)hp->conv_dim * (hp->conv_k - 1), ns = (size_t)hp->h_v * hp->s_v * hp->s_k;
    if (im->snap_np < 0) { seterr(err, errlen, "no snapshot"); return -1; }
    for (size_t li = 0; li < im->L.size(); li++) {
        if (!im->L[li].rec) continue;
        CK(cudaMemcpyAsync(im->L[li].conv, im->snap_conv[li], nc * 4, cudaMemcpyDeviceToDevice, im->st));
        CK(cudaMemcpyAsync(im->L[li].ssm, im->snap_ssm[li], ns * 4, cudaMemcpyDeviceToDevice, im->st));
    }
    int np = im->snap_np;
    CK(cudaMemcpyAsync(im->npast, &np, sizeof(int), cudaMemcpyHostToDevice, im->st));
    CK(cudaStreamSynchronize(im->st));   // np is a host local
    s->n_past = im->snap_np;
    s->ck_T = 0;
    return 0;
}

int xj_cuda_spec_decode(xj_stage *target, xj_stage *draft, const int32_t *prompt, int n_prompt, int n_gen, int k,
                        int32_t *out, long long *stats, char *err, size_t errlen) {
    for (xj_stage *s : {target, draft})
        if (!s || !s->backend || strcmp(s->backend, "cuda") != 0 || s->mtp || s->l0 != 0 || s->l1 != s->m->hp.n_layer ||
            !s->has_head) {
            seterr(err, errlen, "speculative decoding needs two CUDA stages over all layers with the head");
            return -1;
        }
    if (target == draft) { seterr(err, errlen, "the draft must be its own stage"); return -1; }
    if (target->m->hp.n_vocab != draft->m->hp.n_vocab) { seterr(err, errlen, "draft and target vocabularies differ"); return -1; }
    if (k < 1 || k + 1 > target->max_batch || k + 1 > draft->max_batch) {
        seterr(err, errlen, "k must be in 1..max_batch-1 of both stages"); return -1;
    }
    if (n_prompt < 1 || n_gen < 1) { seterr(err, errlen, "need at least one prompt token and one generated token"); return -1; }
    if (target->n_past + n_prompt + n_gen + k > target->n_ctx || draft->n_past + n_prompt + n_gen + k > draft->n_ctx) {
        seterr(err, errlen, "context is too short for %d + %d tokens", n_prompt, n_gen); return -1;
    }
    Impl *ti = I(target), *di = I(draft);
    long long st[4] = {0, 0, 0, 0};   // verify forwards, drafted, accepted, draft re-feeds
    // the prompt through both models; the target picks out[0]
    int32_t first = 0;
    if (xj_cuda_decode(target, prompt, n_prompt, 1, out, nullptr, nullptr, err, errlen)) return -1;
    if (xj_cuda_decode(draft, prompt, n_prompt, 1, &first, nullptr, nullptr, err, errlen)) return -1;
    const int V = target->m->hp.n_vocab;
    int produced = 1;
    std::vector<int32_t> toks(k + 1), ids(k + 1), dr(k);
    while (produced < n_gen) {
        const int32_t last = out[produced - 1];           // emitted, not yet fed to either model
        const int kk = k < n_gen - produced ? k : n_gen - produced;
        // draft kk tokens greedily from its state before `last`
        {
            DevGuard dg(di->dev);
            if (snapshot(draft, err, errlen)) return -1;
        }
        if (xj_cuda_decode(draft, &last, 1, kk, dr.data(), nullptr, nullptr, err, errlen)) return -1;
        st[1] += kk;
        // the target verifies [last, d0 .. d_{kk-1}] in one forward (checkpoints kept for the rollback)
        const int T = kk + 1;
        toks[0] = last;
        for (int i = 0; i < kk; i++) toks[i + 1] = dr[i];
        {
            DevGuard dg(ti->dev);
            const int P = target->n_past;
            if (feed_tokens(target, toks.data(), T, true, err, errlen)) return -1;
            head(target, ti->x, T);
            launch(ti, k_argmax_pick_rows, dim3(T), dim3(1024), 0, (const float *)ti->logits, V, ti->out_tok);
            CK(cudaMemcpyAsync(ids.data(), ti->out_tok, sizeof(int32_t) * T, cudaMemcpyDeviceToHost, ti->st));
            if (sync_check(ti, err, errlen)) return -1;
            target->n_past = P + T;
            st[0]++;
            int a = 0;
            while (a < kk && ids[a] == dr[a]) a++;
            st[2] += a;
            // emit the accepted drafts, then the target's own pick after them when there is room; every
            // emitted token but the final one of the call is fed
            const bool pick = produced + a < n_gen;
            for (int i = 0; i < a; i++) out[produced++] = dr[i];
            if (pick) out[produced++] = ids[a];
            const int fed = pick ? a + 1 : a;                  // last, d0 .. d_{fed-2}
            if (fed < T && cuda_rollback(target, P + fed, err, errlen)) return -1;
            // the draft consumed last, d0 .. d_{kk-2} (kk tokens): bring it to `fed` tokens
            DevGuard dd(di->dev);
            if (fed == kk + 1) {
                if (feed_tokens(draft, &dr[kk - 1], 1, false, err, errlen)) return -1;
                draft->n_past += 1;
                st[3]++;
            } else if (fed < kk) {
                if (restore(draft, err, errlen)) return -1;
                if (feed_tokens(draft, toks.data(), fed, false, err, errlen)) return -1;
                draft->n_past += fed;
                st[3]++;
            }
            if (sync_check(di, err, errlen)) return -1;
        }
    }
    if (stats) for (int i = 0; i < 4; i++) stats[i] = st[i];
    return 0;
}

// Gated DeltaNet decode step on synthetic operands: B sequences x Hv heads of an
// S x S fp32 state, one token each, with the batch kernel of batched decode (k_gdn_batch; B = 1 is the
// single-sequence case). The states rotate over enough copies that the last-level cache cannot serve
// them (>= 256 MiB in total); *ms = average device time per launch over `iters` launches.
int xj_cuda_gdn_time(int S, int Hv, int B, int iters, float *ms, char *err, size_t errlen) {
    if (S != 16 && S != 32 && S != 64 && S != 128) { seterr(err, errlen, "S must be 16, 32, 64 or 128"); return -1; }
    if (Hv < 1 || B < 1 || iters < 1 || !ms) { seterr(err, errlen, "need Hv, B, iters >= 1 and ms"); return -1; }
    Impl tmp;
    Impl *im = &tmp;
    int rc = -1;
    const size_t state = (size_t)B * Hv * S * S;                 // floats per copy
    const int copies = (int)std::max<size_t>(1, ((size_t)256 << 20) / (state * 4) + 1);
    const int key_dim = Hv * S, ldq = 2 * key_dim + Hv * S;
    float *ssm = nullptr, *qkv = nullptr, *z = nullptr, *ba = nullptr, *par = nullptr, *out = nullptr;
    if (cudaStreamCreateWithFlags(&im->st, cudaStreamNonBlocking) != cudaSuccess) { seterr(err, errlen, "no stream"); return -1; }
    if (dalloc(im, &ssm, state * copies, err, errlen) || dalloc(im, &qkv, (size_t)B * ldq, err, errlen) ||
        dalloc(im, &z, (size_t)B * Hv * S, err, errlen) || dalloc(im, &ba, (size_t)2 * B * Hv, err, errlen) ||
        dalloc(im, &par, (size_t)2 * Hv + S, err, errlen) || dalloc(im, &out, (size_t)B * Hv * S, err, errlen)) goto done;
    {
        // small deterministic operands: decays below 1, state and inputs of unit scale
        std::vector<float> h((size_t)B * ldq);
        for (size_t i = 0; i < h.size(); i++) h[i] = (float)((i * 2654435761u) % 2001) / 1000.0f - 1.0f;
        std::vector<float> hp(2 * Hv + S);
        for (int i = 0; i < Hv; i++) { hp[i] = 0.5f; hp[Hv + i] = -1.0f; }
        for (int i = 0; i < S; i++) hp[2 * Hv + i] = 1.0f;
        if (cudaMemcpy(qkv, h.data(), h.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(z, h.data(), (size_t)B * Hv * S * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(ba, h.data(), (size_t)2 * B * Hv * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(par, hp.data(), hp.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemset(ssm, 0, state * copies * 4) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
            seterr(err, errlen, "setup failed");
            goto done;
        }
    }
    {
        GdnArgs g{};
        g.qkv = qkv; g.ldq = ldq; g.z = z; g.ldz = Hv * S; g.beta = ba; g.alpha = ba + (size_t)B * Hv; g.ldg = Hv;
        g.dt = par; g.A = par + Hv; g.nw = par + 2 * Hv; g.ck_ssm = nullptr; g.out = out; g.ldo = Hv * S;
        g.T = 1; g.Hk = Hv; g.Hv = Hv; g.key_dim = key_dim; g.eps = 1e-6f;
        const long long sstride = (long long)Hv * S * S;
        auto run = [&](int i) {
            g.ssm = ssm + (size_t)(i % copies) * state;
            switch (S) {
            case 16: launch(im, k_gdn_batch<16>, dim3(Hv, B), dim3(64), 0, g, sstride); break;
            case 32: launch(im, k_gdn_batch<32>, dim3(Hv, B), dim3(128), 0, g, sstride); break;
            case 64: launch(im, k_gdn_batch<64>, dim3(Hv, B), dim3(256), 0, g, sstride); break;
            default: launch(im, k_gdn_batch<128>, dim3(Hv, B), dim3(512), 0, g, sstride); break;
            }
        };
        for (int i = 0; i < 3; i++) run(i);
        cudaEvent_t e0, e1;
        cudaEventCreate(&e0); cudaEventCreate(&e1);
        cudaEventRecord(e0, im->st);
        for (int i = 0; i < iters; i++) run(i + 3);
        cudaEventRecord(e1, im->st);
        cudaEventSynchronize(e1);
        cudaEventElapsedTime(ms, e0, e1);
        *ms /= iters;
        cudaEventDestroy(e0); cudaEventDestroy(e1);
    }
    if (cudaStreamSynchronize(im->st) != cudaSuccess || cudaGetLastError() != cudaSuccess) { seterr(err, errlen, "GDN launch failed"); goto done; }
    rc = 0;
done:
    cudaStreamSynchronize(im->st);
    for (void *p : im->allocs) cudaFree(p);
    im->allocs.clear();
    cudaStreamDestroy(im->st);
    return rc;
}

// Gated DeltaNet over a prompt of T tokens (prefill): the chunked kernels against the
// token-by-token kernel on the same synthetic operands (Hk key heads, Hv value heads, S x S state from a
// nonzero start). res[0] = max |o_chunked - o_seq| / max |o_seq| (after the gated norm), res[1] = the same
// for the final state, res[2] / res[3] = device ms of the chunked / token-by-token path.
int xj_cuda_gdn_prefill_check(int S, int Hk, int Hv, int T, float *res, char *err, size_t errlen) {
    if (S != 32 && S != 64 && S != 128) { seterr(err, errlen, "S must be 32, 64 or 128"); return -1; }
    if (Hk < 1 || Hv < Hk || Hv % Hk || T < 1 || !res) { seterr(err, errlen, "need 1 <= Hk, Hk | Hv, T >= 1 and res"); return -1; }
    Impl tmp;
    Impl *im = &tmp;
    int rc = -1;
    const int key_dim = Hk * S, ldq = 2 * key_dim + Hv * S, nch = (T + GC_C - 1) / GC_C;
    const size_t ns = (size_t)Hv * S * S;
    float *qkv = nullptr, *z = nullptr, *ba = nullptr, *par = nullptr, *o1 = nullptr, *o2 = nullptr, *m1 = nullptr, *m2 = nullptr;
    float *qn = nullptr, *kn = nullptr, *kk = nullptr, *qk = nullptr, *wx = nullptr;
    std::vector<float> h1, h2, s1, s2;
    if (cudaStreamCreateWithFlags(&im->st, cudaStreamNonBlocking) != cudaSuccess) { seterr(err, errlen, "no stream"); return -1; }
    if (dalloc(im, &qkv, (size_t)T * ldq, err, errlen) || dalloc(im, &z, (size_t)T * Hv * S, err, errlen) ||
        dalloc(im, &ba, (size_t)2 * T * Hv, err, errlen) || dalloc(im, &par, (size_t)2 * Hv + S, err, errlen) ||
        dalloc(im, &o1, (size_t)T * Hv * S, err, errlen) || dalloc(im, &o2, (size_t)T * Hv * S, err, errlen) ||
        dalloc(im, &m1, ns, err, errlen) || dalloc(im, &m2, ns, err, errlen) ||
        dalloc(im, &qn, (size_t)T * key_dim, err, errlen) || dalloc(im, &kn, (size_t)T * key_dim, err, errlen) ||
        dalloc(im, &kk, (size_t)Hk * nch * GC_C * GC_C, err, errlen) || dalloc(im, &qk, (size_t)Hk * nch * GC_C * GC_C, err, errlen) ||
        dalloc(im, &wx, gc_wx_floats(T, Hv, S), err, errlen))
        goto done;
    {
        // deterministic operands: q, k, v, z ~ U(-1, 1); beta, alpha logits ~ U(-2, 2); dt = 0.5;
        // A = -exp(U(-1, 1)) (decays below 1); norm weights 1 + U(-0.1, 0.1); start state ~ U(-0.1, 0.1)
        uint64_t x = 0x9E3779B97F4A7C15ull;
        auto u = [&]() { x ^= x << 13; x ^= x >> 7; x ^= x << 17; return (float)((x >> 11) * (1.0 / 9007199254740992.0)) * 2.0f - 1.0f; };
        std::vector<float> q((size_t)T * ldq), zz((size_t)T * Hv * S), bb((size_t)2 * T * Hv), pp(2 * Hv + S), mm(ns);
        for (auto &v : q) v = u();
        for (auto &v : zz) v = u();
        for (auto &v : bb) v = 2.0f * u();
        for (int i = 0; i < Hv; i++) { pp[i] = 0.5f; pp[Hv + i] = -expf(u()); }
        for (int i = 0; i < S; i++) pp[2 * Hv + i] = 1.0f + 0.1f * u();
        for (auto &v : mm) v = 0.1f * u();
        if (cudaMemcpy(qkv, q.data(), q.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(z, zz.data(), zz.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(ba, bb.data(), bb.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(par, pp.data(), pp.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(m1, mm.data(), ns * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(m2, mm.data(), ns * 4, cudaMemcpyHostToDevice) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
            seterr(err, errlen, "setup failed");
            goto done;
        }
    }
    {
        GdnArgs g{};
        g.qkv = qkv; g.ldq = ldq; g.z = z; g.ldz = Hv * S; g.beta = ba; g.alpha = ba + (size_t)T * Hv; g.ldg = Hv;
        g.dt = par; g.A = par + Hv; g.nw = par + 2 * Hv; g.ck_ssm = nullptr; g.ldo = Hv * S;
        g.T = T; g.Hk = Hk; g.Hv = Hv; g.key_dim = key_dim; g.eps = 1e-6f;
        cudaEvent_t e[3];
        for (auto &ev : e) cudaEventCreate(&ev);
        GdnArgs gs = g, gc = g;
        gs.ssm = m1; gs.out = o1;
        gc.ssm = m2; gc.out = o2;
        cudaEventRecord(e[0], im->st);
        switch (S) {
        case 32: launch(im, k_gdn<32>, dim3(Hv), dim3(128), 0, gs); break;
        case 64: launch(im, k_gdn<64>, dim3(Hv), dim3(256), 0, gs); break;
        default: launch(im, k_gdn<128>, dim3(Hv), dim3(512), 0, gs); break;
        }
        cudaEventRecord(e[1], im->st);
        switch (S) {
        case 32: launch_gdn_chunked<32>(im, gc, qn, kn, kk, qk, wx); break;
        case 64: launch_gdn_chunked<64>(im, gc, qn, kn, kk, qk, wx); break;
        default: launch_gdn_chunked<128>(im, gc, qn, kn, kk, qk, wx); break;
        }
        cudaEventRecord(e[2], im->st);
        if (cudaStreamSynchronize(im->st) != cudaSuccess || cudaGetLastError() != cudaSuccess) {
            seterr(err, errlen, "GDN launch failed");
            for (auto &ev : e) cudaEventDestroy(ev);
            goto done;
        }
        cudaEventElapsedTime(&res[3], e[0], e[1]);
        cudaEventElapsedTime(&res[2], e[1], e[2]);
        for (auto &ev : e) cudaEventDestroy(ev);
        h1.resize((size_t)T * Hv * S); h2.resize(h1.size()); s1.resize(ns); s2.resize(ns);
        cudaMemcpy(h1.data(), o1, h1.size() * 4, cudaMemcpyDeviceToHost);
        cudaMemcpy(h2.data(), o2, h2.size() * 4, cudaMemcpyDeviceToHost);
        cudaMemcpy(s1.data(), m1, ns * 4, cudaMemcpyDeviceToHost);
        cudaMemcpy(s2.data(), m2, ns * 4, cudaMemcpyDeviceToHost);
        auto rel = [](const std::vector<float> &a, const std::vector<float> &b) {
            double d = 0.0, mx = 0.0;
            for (size_t i = 0; i < a.size(); i++) { d = std::max(d, (double)fabsf(a[i] - b[i])); mx = std::max(mx, (double)fabsf(a[i])); }
            return (float)(mx > 0 ? d / mx : d);
        };
        res[0] = rel(h1, h2);
        res[1] = rel(s1, s2);
    }
    rc = 0;
done:
    cudaStreamSynchronize(im->st);
    for (void *p : im->allocs) cudaFree(p);
    im->allocs.clear();
    cudaStreamDestroy(im->st);
    return rc;
}

// Gated DeltaNet recurrence on caller operands (host buffers), for parity against a host restatement of
// core/xj_cpu.c:194-219. path 0: the token-by-token kernel over T tokens of one sequence (k_gdn, the
// prompt path below 32 tokens and the checkpointing verify path); 1: the chunked prefill kernels;
// 2: the batch decode kernel with T independent sequences of one token each (state [T][Hv][S][S]).
// qkv [T][2*Hk*S + Hv*S] after the convolution and SiLU; z [T][Hv*S] raw gate; beta, alpha [T][Hv]
// logits; dt, A [Hv]; norm_w [S]; state in/out; out [T][Hv*S] after the gated RMSNorm.
int xj_cuda_gdn_run(int path, int S, int Hk, int Hv, int T, const float *qkv, const float *z, const float *beta,
                    const float *alpha, const float *dt, const float *A, const float *norm_w, float eps, float *state,
                    float *out, char *err, size_t errlen) {
    if (path < 0 || path > 2) { seterr(err, errlen, "path must be 0, 1 or 2"); return -1; }
    if (S != 16 && S != 32 && S != 64 && S != 128) { seterr(err, errlen, "S must be 16, 32, 64 or 128"); return -1; }
    if (path == 1 && S == 16) { seterr(err, errlen, "the chunked path needs S = 32, 64 or 128"); return -1; }
    if (Hk < 1 || Hv < Hk || Hv % Hk || T < 1) { seterr(err, errlen, "need 1 <= Hk, Hk | Hv and T >= 1"); return -1; }
    if (!qkv || !z || !beta || !alpha || !dt || !A || !norm_w || !state || !out) { seterr(err, errlen, "null buffer"); return -1; }
    Impl tmp;
    Impl *im = &tmp;
    int rc = -1;
    const int key_dim = Hk * S, ldq = 2 * key_dim + Hv * S, nch = (T + GC_C - 1) / GC_C;
    const size_t ns = (size_t)Hv * S * S * (path == 2 ? T : 1);
    float *dq = nullptr, *dz = nullptr, *dba = nullptr, *dpar = nullptr, *dm = nullptr, *dout = nullptr;
    float *qn = nullptr, *kn = nullptr, *kk = nullptr, *qk = nullptr, *wx = nullptr;
    if (cudaStreamCreateWithFlags(&im->st, cudaStreamNonBlocking) != cudaSuccess) { seterr(err, errlen, "no stream"); return -1; }
    if (dalloc(im, &dq, (size_t)T * ldq, err, errlen) || dalloc(im, &dz, (size_t)T * Hv * S, err, errlen) ||
        dalloc(im, &dba, (size_t)2 * T * Hv, err, errlen) || dalloc(im, &dpar, (size_t)2 * Hv + S, err, errlen) ||
        dalloc(im, &dm, ns, err, errlen) || dalloc(im, &dout, (size_t)T * Hv * S, err, errlen))
        goto done;
    if (path == 1 && (dalloc(im, &qn, (size_t)T * key_dim, err, errlen) || dalloc(im, &kn, (size_t)T * key_dim, err, errlen) ||
                      dalloc(im, &kk, (size_t)Hk * nch * GC_C * GC_C, err, errlen) ||
                      dalloc(im, &qk, (size_t)Hk * nch * GC_C * GC_C, err, errlen) ||
                      dalloc(im, &wx, gc_wx_floats(T, Hv, S), err, errlen)))
        goto done;
    if (cudaMemcpy(dq, qkv, (size_t)T * ldq * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(dz, z, (size_t)T * Hv * S * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(dba, beta, (size_t)T * Hv * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(dba + (size_t)T * Hv, alpha, (size_t)T * Hv * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(dpar, dt, (size_t)Hv * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(dpar + Hv, A, (size_t)Hv * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(dpar + 2 * Hv, norm_w, (size_t)S * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(dm, state, ns * 4, cudaMemcpyHostToDevice) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
        seterr(err, errlen, "upload failed");
        goto done;
    }
    {
        GdnArgs g{};
        g.qkv = dq; g.ldq = ldq; g.z = dz; g.ldz = Hv * S; g.beta = dba; g.alpha = dba + (size_t)T * Hv; g.ldg = Hv;
        g.dt = dpar; g.A = dpar + Hv; g.nw = dpar + 2 * Hv; g.ck_ssm = nullptr; g.ssm = dm; g.out = dout; g.ldo = Hv * S;
        g.T = T; g.Hk = Hk; g.Hv = Hv; g.key_dim = key_dim; g.eps = eps;
        if (path == 0) {
            switch (S) {
            case 16: launch(im, k_gdn<16>, dim3(Hv), dim3(64), 0, g); break;
            case 32: launch(im, k_gdn<32>, dim3(Hv), dim3(128), 0, g); break;
            case 64: launch(im, k_gdn<64>, dim3(Hv), dim3(256), 0, g); break;
            default: launch(im, k_gdn<128>, dim3(Hv), dim3(512), 0, g); break;
            }
        } else if (path == 1) {
            switch (S) {
            case 32: launch_gdn_chunked<32>(im, g, qn, kn, kk, qk, wx); break;
            case 64: launch_gdn_chunked<64>(im, g, qn, kn, kk, qk, wx); break;
            default: launch_gdn_chunked<128>(im, g, qn, kn, kk, qk, wx); break;
            }
        } else {
            const long long sstride = (long long)Hv * S * S;
            g.T = 1;
            switch (S) {
            case 16: launch(im, k_gdn_batch<16>, dim3(Hv, T), dim3(64), 0, g, sstride); break;
            case 32: launch(im, k_gdn_batch<32>, dim3(Hv, T), dim3(128), 0, g, sstride); break;
            case 64: launch(im, k_gdn_batch<64>, dim3(Hv, T), dim3(256), 0, g, sstride); break;
            default: launch(im, k_gdn_batch<128>, dim3(Hv, T), dim3(512), 0, g, sstride); break;
            }
        }
        if (cudaStreamSynchronize(im->st) != cudaSuccess || cudaGetLastError() != cudaSuccess) {
            seterr(err, errlen, "GDN launch failed");
            goto done;
        }
    }
    if (cudaMemcpy(out, dout, (size_t)T * Hv * S * 4, cudaMemcpyDeviceToHost) != cudaSuccess ||
        cudaMemcpy(state, dm, ns * 4, cudaMemcpyDeviceToHost) != cudaSuccess) {
        seterr(err, errlen, "download failed");
        goto done;
    }
    rc = 0;
done:
    cudaStreamSynchronize(im->st);
    for (void *p : im->allocs) cudaFree(p);
    im->allocs.clear();
    cudaStreamDestroy(im->st);
    return rc;
}

int xj_cuda_set_sampler(xj_stage *s, float temperature, int top_k, double top_p, unsigned long long seed, char *err,
                        size_t errlen) {
    if (!s || s->backend == nullptr || strcmp(s->backend, "cuda") != 0) { seterr(err, errlen, "not a CUDA stage"); return -1; }
    if (top_k < 1 || top_k > SAMPLE_KMAX) { seterr(err, errlen, "top_k must be in 1..%d", SAMPLE_KMAX); return -1; }
    if (!(top_p > 0.0 && top_p <= 1.0)) { seterr(err, errlen, "top_p must be in (0, 1]"); return -1; }
    Impl *im = I(s);
    DevGuard dg(im->dev);
    const bool was = im->samp_temp > 0.0f, now = temperature > 0.0f;
    im->samp_temp = now ? temperature : 0.0f;
    im->samp_top_k = top_k;
    im->samp_top_p = top_p;
    im->samp_seed = seed;
    // the decode program of the persistent kernel holds the pick phase and the sampler settings
    if (im->mk_state == 1 && (was || now)) im->mk_state = 0;
    // the cached decode-step graph holds the pick kernel and its arguments
    if (im->step_graph && (was || now)) {
        cudaStreamSynchronize(im->st);
        cudaGraphExecDestroy(im->step_graph);
        im->step_graph = nullptr;
    }
    return 0;
}

int xj_cuda_sample_logits(const float *logits, int rows, int n_vocab, float temperature, int top_k, double top_p,
                          unsigned long long seed, unsigned long long counter0, int32_t *out, float *margins, char *err,
                          size_t errlen) {
    if (!logits || !out || rows < 1 || n_vocab < 1) { seterr(err, errlen, "need logits, out, rows >= 1 and n_vocab >= 1"); return -1; }
    if (top_k < 1 || top_k > SAMPLE_KMAX) { seterr(err, errlen, "top_k must be in 1..%d", SAMPLE_KMAX); return -1; }
    if (!(top_p > 0.0 && top_p <= 1.0)) { seterr(err, errlen, "top_p must be in (0, 1]"); return -1; }
    Impl tmp;
    Impl *im = &tmp;
    int rc = -1;
    float *dl = nullptr, *dm = nullptr;
    int32_t *dout = nullptr;
    if (cudaStreamCreateWithFlags(&im->st, cudaStreamNonBlocking) != cudaSuccess) { seterr(err, errlen, "no stream"); return -1; }
    if (dalloc(im, &dl, (size_t)rows * n_vocab, err, errlen) || dalloc(im, &dm, (size_t)rows, err, errlen) ||
        dalloc(im, &dout, (size_t)rows, err, errlen))
        goto done;
    if (cudaMemcpy(dl, logits, (size_t)rows * n_vocab * 4, cudaMemcpyHostToDevice) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
        seterr(err, errlen, "upload failed");
        goto done;
    }
    {
        SampleArgs a{};
        a.logits = dl; a.ld = n_vocab; a.n = n_vocab; a.temp = temperature; a.top_k = top_k; a.top_p = top_p;
        a.seed = seed; a.counter0 = counter0; a.out = dout; a.margin = dm;
        launch(im, k_sample_rows, dim3(rows), dim3(SAMPLE_THREADS), 0, a);
        if (cudaStreamSynchronize(im->st) != cudaSuccess || cudaGetLastError() != cudaSuccess) { seterr(err, errlen, "sampling launch failed"); goto done; }
    }
    if (cudaMemcpy(out, dout, (size_t)rows * 4, cudaMemcpyDeviceToHost) != cudaSuccess ||
        (margins && cudaMemcpy(margins, dm, (size_t)rows * 4, cudaMemcpyDeviceToHost) != cudaSuccess)) {
        seterr(err, errlen, "download failed");
        goto done;
    }
    rc = 0;
done:
    cudaStreamSynchronize(im->st);
    for (void *p : im->allocs) cudaFree(p);
    im->allocs.clear();
    cudaStreamDestroy(im->st);
    return rc;
}

int xj_cuda_graph_kernels(const xj_stage *s) {
    const Impl *im = (const Impl *)s->impl;
    return im ? im->step_kernels : 0;
}

int xj_cuda_phase_trace(const xj_stage *s, double *out, int cap) {
    Impl *im = (Impl *)s->impl;
    if (!im || im->mk_state != 1 || !g_opt_trace) return -1;
    DevGuard dg(im->dev);
    const int np = im->mk_nphase, G = im->mk_ctas;
    std::vector<unsigned long long> t((size_t)G * np * 12);
    if (cudaMemcpy(t.data(), im->mk_trace, t.size() * 8, cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    for (int ph = 0; ph < np && ph < cap; ph++) {
        unsigned long long s0 = ~0ull, e1 = 0;
        double wmax = 0, wsum = 0, wait = 0, lead = 0, pro = 0, first = 0, f1 = 0, f2 = 0, f3 = 0, f4 = 0;
        int nlead = 0, ntl = 0;
        const bool attn = im->mk_ops[ph] == MK_ATTN;
        double at[6] = {0, 0, 0, 0, 0, 0};
        int nat = 0, nmerge = 0;
        for (int c = 0; c < G; c++) {
            const unsigned long long *r = &t[((size_t)c * np + ph) * 12];
            if (attn && r[5] && r[10]) {
                // an attention item: position read, queries normed, rows staged, rounds, split counter, merge
                at[0] += ((double)r[5] - (double)r[0]) * 1e-3;
                at[1] += ((double)r[6] - (double)r[5]) * 1e-3;
                at[2] += ((double)r[8] - (double)r[6]) * 1e-3;
                at[3] += ((double)r[9] - (double)r[8]) * 1e-3;
                at[4] += ((double)r[10] - (double)r[9]) * 1e-3;
                nat++;
                if (r[11]) { at[5] += ((double)r[11] - (double)r[10]) * 1e-3; nmerge++; }
            }
            if (!attn && r[7]) {
                pro += ((double)r[5] - (double)r[0]) * 1e-3;
                first += ((double)r[6] - (double)r[5]) * 1e-3;
                f1 += ((double)r[8] - (double)r[5]) * 1e-3;    // prologue end -> first chunk ready
                f2 += ((double)r[9] - (double)r[8]) * 1e-3;    // tensor-core work of the first tile (warp 0)
                f3 += ((double)r[10] - (double)r[9]) * 1e-3;   // warp 0's hand-over -> all partials with the epilogue warp
                f4 += ((double)r[11] - (double)r[10]) * 1e-3;  // epilogue (epilogue warp)
                ntl++;
            }
            if (r[0] < s0) s0 = r[0];
            if (r[1] > e1) e1 = r[1];
            const double w = r[1] > r[0] ? (double)(r[1] - r[0]) * 1e-3 : 0.0;
            wsum += w;
            if (w > wmax) wmax = w;
            wait += (double)r[2] * 1e-3;
            if (r[3]) { lead += ((double)r[0] - (double)r[3]) * 1e-3; nlead++; }
        }
        double *o = out + (size_t)ph * 13;
        o[0] = im->mk_ops[ph];
        o[1] = wmax;
        o[2] = wsum / G;
        o[3] = e1 > s0 ? (double)(e1 - s0) * 1e-3 : 0.0;
        o[4] = (double)s0 * 1e-3;
        o[5] = wait / G;
        o[6] = nlead ? lead / nlead : 0.0;
        o[7] = ntl ? pro / ntl : 0.0;
        o[8] = ntl ? first / ntl : 0.0;
        o[9] = ntl ? f1 / ntl : 0.0;
        o[10] = ntl ? f2 / ntl : 0.0;
        o[11] = ntl ? f3 / ntl : 0.0;
        o[12] = ntl ? f4 / ntl : 0.0;
        if (attn) {
            for (int i = 0; i < 5; i++) o[7 + i] = nat ? at[i] / nat : 0.0;
            o[12] = nmerge ? at[5] / nmerge : 0.0;
        }
    }
    return np;
}

long long xj_cuda_last_decode_launches(const xj_stage *s, long long *launches) {
    const Impl *im = (const Impl *)s->impl;
    if (!im) return 0;
    if (launches) { launches[0] = im->last_launches[0]; launches[1] = im->last_launches[1]; }
    return im->last_launches[0] + im->last_launches[1];
}

int xj_cuda_dequant_rows(int type, const void *src, int k, int n_rows, float *out, char *err, size_t errlen) {
    const uint64_t rb = row_bytes((uint32_t)type, k);
    if (!rb || k % 8 || n_rows <= 0) { seterr(err, errlen, "unsupported type %d or row length %d", type, k); return -1; }
    uint8_t *d_src = nullptr;
    float *d_out = nullptr;
    cudaError_t e = cudaMalloc(&d_src, rb * n_rows);
    if (e == cudaSuccess) e = cudaMalloc(&d_out, sizeof(float) * (size_t)k * n_rows);
    if (e == cudaSuccess) e = cudaMemcpy(d_src, src, rb * n_rows, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) {
        DevMat w{d_src, type, k, n_rows, (long long)rb};
        k_dequant<<<148, 256>>>(w, 0, n_rows, d_out);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpy(out, d_out, sizeof(float) * (size_t)k * n_rows, cudaMemcpyDeviceToHost);
    cudaFree(d_src);
    cudaFree(d_out);
    if (e != cudaSuccess) { seterr(err, errlen, "CUDA error: %s", cudaGetErrorString(e)); return -1; }
    return 0;
}

int xj_cuda_tc_selftest(const uint16_t *a, const uint16_t *b, int k, float *d, char *err, size_t errlen) {
    if (k <= 0 || k % TCS_KC) { seterr(err, errlen, "K must be a positive multiple of %d", TCS_KC); return -1; }
    __half *da = nullptr, *db = nullptr;
    float *dd = nullptr;
    int *derr = nullptr, herr = 0;
    cudaError_t e = cudaMalloc(&da, sizeof(__half) * TCS_M * (size_t)k);
    if (e == cudaSuccess) e = cudaMalloc(&db, sizeof(__half) * TCS_N * (size_t)k);
    if (e == cudaSuccess) e = cudaMalloc(&dd, sizeof(float) * TCS_M * TCS_N);
    if (e == cudaSuccess) e = cudaMalloc(&derr, sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(derr, 0, sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(dd, 0, sizeof(float) * TCS_M * TCS_N);
    if (e == cudaSuccess) e = cudaMemcpy(da, a, sizeof(__half) * TCS_M * (size_t)k, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(db, b, sizeof(__half) * TCS_N * (size_t)k, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) {
        k_tc_selftest<<<1, 128>>>(da, db, k, dd, derr);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpy(d, dd, sizeof(float) * TCS_M * TCS_N, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemcpy(&herr, derr, sizeof(int), cudaMemcpyDeviceToHost);
    cudaFree(da); cudaFree(db); cudaFree(dd); cudaFree(derr);
    if (e != cudaSuccess) { seterr(err, errlen, "CUDA error: %s", cudaGetErrorString(e)); return -1; }
    if (herr) { seterr(err, errlen, "a bounded wait on the GPU gave up (tensor-core completion)"); return -1; }
    return 0;
}

uint64_t xjc_stage_state_bytes(const xj_model *m, int l0, int l1, int n_ctx, int max_batch) {
    const xj_hparams *hp = &m->hp;
    uint64_t b = 0;
    const uint64_t kv_es = g_opt_kv_f32 ? 4 : 2;
    for (int il = l0; il < l1; il++) {
        if (il < hp->n_layer && m->layers[il].recurrent)
            b += 4ull * ((uint64_t)hp->conv_dim * (hp->conv_k - 1) + (uint64_t)hp->h_v * hp->s_v * hp->s_k);
        else
            b += 2ull * kv_es * n_ctx * hp->n_head_kv * hp->head_dim;
    }
    b += 7ull * 4 * max_batch * scratch_floats(hp);
    return b;
}


// ------------------------------------------------------------------ batch API (additive)
struct xj_cuda_batch {
    BatchImpl impl;
};

static xj_cuda_batch *batch_new(const xj_model *m, int l0, int l1, bool has_head, int n_seq, int n_ctx, int tmax, char *err,
                                size_t errlen) {
    if (!m || n_seq < 1 || n_seq > 1024 || n_ctx < 1) { seterr(err, errlen, "need 1 <= n_seq <= 1024 and n_ctx >= 1"); return nullptr; }
    if (tmax < 1 || tmax > 16 || (long long)n_seq * tmax > 4096) { seterr(err, errlen, "need 1 <= max_tokens <= 16 and n_seq * max_tokens <= 4096"); return nullptr; }
    if (l0 < 0 || l1 > m->hp.n_layer || l0 >= l1) { seterr(err, errlen, "bad layer range [%d,%d)", l0, l1); return nullptr; }
    if (tmax > 1 && m->hp.conv_k > 9) { seterr(err, errlen, "multi-token forwards need conv_k <= 9"); return nullptr; }
    // the stage holds the weights and n_seq*tmax-row activation buffers; its own single-sequence state is minimal
    xj_stage *s = xj_cuda_stage_new(m, l0, l1, 1, n_seq * tmax, has_head, err, errlen);
    if (!s) return nullptr;
    xj_cuda_batch *b = new xj_cuda_batch();
    BatchImpl *bi = &b->impl;
    bi->s = s;
    bi->B = n_seq;
    bi->n_ctx = n_ctx;
    Impl *im = I(s);
    DevGuard dg(im->dev);
    const xj_hparams *hp = &m->hp;
    auto fail = [&]() { cuda_destroy(s); delete b; return (xj_cuda_batch *)nullptr; };
    const size_t ns = (size_t)n_seq * hp->h_v * hp->s_v * hp->s_k, nc = (size_t)n_seq * hp->conv_dim * (hp->conv_k - 1);
    const size_t nkv = (size_t)n_seq * n_ctx * hp->n_head_kv * hp->head_dim, es = im->kv_f32 ? 4 : 2;
    for (int il = l0; il < l1; il++) {
        float *a = nullptr, *c = nullptr;
        uint8_t *k = nullptr, *v = nullptr;
        if (im->L[il - l0].rec) {
            if (dalloc(im, &a, ns, err, errlen) || dalloc(im, &c, nc, err, errlen)) return fail();
        } else if (dalloc(im, &k, nkv * es, err, errlen) || dalloc(im, &v, nkv * es, err, errlen)) return fail();
        bi->ssm.push_back(a); bi->conv.push_back(c); bi->kc.push_back(k); bi->vc.push_back(v);
    }
    bi->ntiles = has_head ? (im->output.N + 15) / 16 : 1;
    bi->out_cap = 1024;
    if (dalloc(im, &bi->npast, (size_t)n_seq, err, errlen) || dalloc(im, &bi->step, (size_t)n_seq, err, errlen) ||
        dalloc(im, &bi->np_scratch, (size_t)n_seq, err, errlen) || dalloc(im, &bi->cur, (size_t)n_seq, err, errlen) ||
        dalloc(im, &bi->pbest, (size_t)n_seq * bi->ntiles, err, errlen) ||
        dalloc(im, &bi->psecond, (size_t)n_seq * bi->ntiles, err, errlen) ||
        dalloc(im, &bi->pidx, (size_t)n_seq * bi->ntiles, err, errlen) ||
        dalloc(im, &bi->out_tok, (size_t)n_seq * bi->out_cap, err, errlen) ||
        dalloc(im, &bi->margin, (size_t)n_seq * bi->out_cap, err, errlen)) return fail();
    if ((l0 == 0 || has_head) && !im->tok_embd.p && upload(im, m->tok_embd, &im->tok_embd, err, errlen, true)) return fail();
    bi->tmax = tmax;
    if (dalloc(im, &bi->conv_raw, (size_t)n_seq * tmax * hp->conv_dim, err, errlen) ||
        dalloc(im, &bi->rows_tok, (size_t)n_seq * tmax, err, errlen) || dalloc(im, &bi->picks, (size_t)n_seq * tmax, err, errlen) ||
        dalloc(im, &bi->x_last, (size_t)n_seq * hp->n_embd, err, errlen))
        return fail();
    if (cudaDeviceSynchronize() != cudaSuccess) { seterr(err, errlen, "CUDA error while creating the batch"); return fail(); }
    if (batch_reset_state(bi, err, errlen)) return fail();
    return b;
}

xj_cuda_batch *xj_cuda_batch_new_range(const xj_model *m, int l0, int l1, bool has_head, int n_seq, int n_ctx, char *err,
                                       size_t errlen) {
    return batch_new(m, l0, l1, has_head, n_seq, n_ctx, 1, err, errlen);
}

xj_cuda_batch *xj_cuda_batch_new(const xj_model *m, int n_seq, int n_ctx, char *err, size_t errlen) {
    if (!m) { seterr(err, errlen, "null model"); return nullptr; }
    return batch_new(m, 0, m->hp.n_layer, true, n_seq, n_ctx, 1, err, errlen);
}

xj_cuda_batch *xj_cuda_batch_new_multi(const xj_model *m, int n_seq, int n_ctx, int max_tokens, char *err, size_t errlen) {
    if (!m) { seterr(err, errlen, "null model"); return nullptr; }
    return batch_new(m, 0, m->hp.n_layer, true, n_seq, n_ctx, max_tokens, err, errlen);
}

void xj_cuda_batch_free(xj_cuda_batch *b) {
    if (!b) return;
    BatchImpl *bi = &b->impl;
    if (bi->s) {
        DevGuard dg(I(bi->s)->dev);
        if (bi->step_graph) cudaGraphExecDestroy(bi->step_graph);
        cuda_destroy(bi->s);
    }
    delete b;
}

int xj_cuda_batch_reset(xj_cuda_batch *b, char *err, size_t errlen) {
    if (!b) { seterr(err, errlen, "null batch"); return -1; }
    DevGuard dg(I(b->impl.s)->dev);
    return batch_reset_state(&b->impl, err, errlen);
}

int xj_cuda_batch_n_past(const xj_cuda_batch *b) { return b ? b->impl.n_past : -1; }

int xj_cuda_batch_decode(xj_cuda_batch *b, const int32_t *prompts, int n_prompt, int n_gen, int32_t *out, float *margins,
                         float *gpu_ms, char *err, size_t errlen) {
    if (!b || !prompts || !out) { seterr(err, errlen, "null argument"); return -1; }
    BatchImpl *bi = &b->impl;
    xj_stage *s = bi->s;
    Impl *im = I(s);
    DevGuard dg(im->dev);
    const int B = bi->B, E = s->m->hp.n_embd;
    if (s->l0 != 0 || s->l1 != s->m->hp.n_layer || !s->has_head) { seterr(err, errlen, "decode needs a batch over all layers with the head"); return -1; }
    if (n_prompt <= 0 || n_gen <= 0) { seterr(err, errlen, "need at least one prompt token and one generated token"); return -1; }
    if (bi->n_past + n_prompt + n_gen - 1 > bi->n_ctx) { seterr(err, errlen, "context is full (%d)", bi->n_ctx); return -1; }
    if (n_gen > bi->out_cap) {
        if (bi->step_graph) { cudaGraphExecDestroy(bi->step_graph); bi->step_graph = nullptr; }
        const int cap = n_gen;
        if (dalloc(im, &bi->out_tok, (size_t)B * cap, err, errlen) || dalloc(im, &bi->margin, (size_t)B * cap, err, errlen)) return -1;
        bi->out_cap = cap;
    }
    if (n_prompt > bi->prompt_cap) {
        if (dalloc(im, &bi->prompts, (size_t)B * n_prompt, err, errlen)) return -1;
        bi->prompt_cap = n_prompt;
    }
    CK(cudaMemsetAsync(bi->step, 0, sizeof(int) * B, im->st));
    const long long nl0 = im->nlaunch;
    // a batch wider than 16 sequences takes its prompt in chunks of up to tmax tokens per sequence (its
    // matrix products run on the 64-row kernels either way, where a token's result does not depend on
    // the other rows of the launch, so the ids are those of the one-token steps); otherwise token by token
    if (bi->tmax > 1 && B > 16) {
        CK(cudaEventRecord(im->ev[0], im->st));
        const int np0 = bi->n_past;
        if (batch_prefill(bi, prompts, n_prompt, true, err, errlen)) return -1;
        bi->n_past = np0;                                                  // counted once, below
        launch(im, k_advance_batch, dim3(1), dim3(256), 0, bi->npast, B, -1);   // the last token's position
        head_batch(bi, bi->x_last, 0, B, bi->cur, im->x, bi->npast);       // out[:, 0], its embedding into x, position + 1
    } else {
        // prompts [B][n_prompt] -> device [n_prompt][B]: the tokens of step i are contiguous
        std::vector<int32_t> tp((size_t)B * n_prompt);
        for (int bq = 0; bq < B; bq++)
            for (int i = 0; i < n_prompt; i++) tp[(size_t)i * B + bq] = prompts[(size_t)bq * n_prompt + i];
        CK(cudaMemcpyAsync(bi->prompts, tp.data(), tp.size() * sizeof(int32_t), cudaMemcpyHostToDevice, im->st));
        CK(cudaEventRecord(im->ev[0], im->st));
        for (int i = 0; i < n_prompt; i++) {
            launch(im, k_embed, dim3((E / 8 + 127) / 128, B), dim3(128), 0, im->tok_embd, (const int32_t *)(bi->prompts + (size_t)i * B), B,
                   im->x, E);
            run_layers_batch(bi, im->x, 0, B);
            if (i + 1 < n_prompt) launch(im, k_advance_batch, dim3(1), dim3(256), 0, bi->npast, B, 1);
            else head_batch(bi, im->x, 0, B, bi->cur, im->x, bi->npast);   // out[:, 0], its embedding into x, position + 1
        }
        CK(cudaStreamSynchronize(im->st));   // tp is a host temporary
    }
    CK(cudaEventRecord(im->ev[1], im->st));
    bi->last_launches[0] = im->nlaunch - nl0;
    bi->last_launches[1] = 0;
    if (n_gen > 1) {
        if (!bi->step_graph) {
            cudaGraph_t g;
            CK(cudaStreamBeginCapture(im->st, cudaStreamCaptureModeThreadLocal));
            run_layers_batch(bi, im->x, 0, B);
            head_batch(bi, im->x, 0, B, bi->cur, im->x, bi->npast);
            CK(cudaStreamEndCapture(im->st, &g));
            bi->step_kernels = count_kernels(g);
            cudaError_t e = cudaGraphInstantiate(&bi->step_graph, g, 0);
            cudaGraphDestroy(g);
            if (e != cudaSuccess) { seterr(err, errlen, "graph instantiate: %s", cudaGetErrorString(e)); bi->step_graph = nullptr; return -1; }
        }
        for (int i = 1; i < n_gen; i++) CK(cudaGraphLaunch(bi->step_graph, im->st));
        bi->last_launches[1] = (long long)(n_gen - 1) * bi->step_kernels;
    }
    CK(cudaEventRecord(im->ev[2], im->st));
    CK(cudaMemcpy2DAsync(out, sizeof(int32_t) * n_gen, bi->out_tok, sizeof(int32_t) * bi->out_cap, sizeof(int32_t) * n_gen, B,
                         cudaMemcpyDeviceToHost, im->st));
    if (margins)
        CK(cudaMemcpy2DAsync(margins, sizeof(float) * n_gen, bi->margin, sizeof(float) * bi->out_cap, sizeof(float) * n_gen, B,
                             cudaMemcpyDeviceToHost, im->st));
    if (sync_check(im, err, errlen)) return -1;
    if (gpu_ms) {
        cudaEventElapsedTime(&gpu_ms[0], im->ev[0], im->ev[1]);
        cudaEventElapsedTime(&gpu_ms[1], im->ev[1], im->ev[2]);
    }
    bi->n_past += n_prompt + n_gen - 1;
    return 0;
}

// Greedy speculative decoding of a batch of sequences with a draft batch (core/xj_spec.c:131-209 for
// every sequence at once). Both batches span all layers with the head, hold the same number of sequences
// at the same position, and share the vocabulary; the target takes k + 1 tokens per sequence per forward
// (xj_cuda_batch_new_multi). Per round: the draft runs k + 1 one-token steps from each sequence's last
// emitted id (its picks d_0 .. d_k; its recurrent state is copied after each of the first k steps), the
// target verifies [last, d_0 .. d_(k-1)] of every sequence in one (k+1)-token forward with per-token
// checkpoints and greedy picks, each sequence emits its agreeing prefix plus the target's next pick, and
// both batches roll each sequence back to what it keeps.
int xj_cuda_batch_spec_decode(xj_cuda_batch *target, xj_cuda_batch *draft, const int32_t *prompts, int n_prompt, int n_gen,
                              int k, int32_t *out, long long *stats, float *gpu_ms, char *err, size_t errlen) {
    if (!target || !draft || !prompts || !out) { seterr(err, errlen, "null argument"); return -1; }
    BatchImpl *tb = &target->impl, *db = &draft->impl;
    xj_stage *ts = tb->s, *ds = db->s;
    Impl *ti = I(ts), *di = I(ds);
    DevGuard dg(ti->dev);
    const int B = tb->B, T = k + 1;
    const xj_hparams *thp = &ts->m->hp, *dhp = &ds->m->hp;
    if (ti->dev != di->dev) { seterr(err, errlen, "target and draft must be on one device"); return -1; }
    if (ts->l0 != 0 || ts->l1 != thp->n_layer || !ts->has_head || ds->l0 != 0 || ds->l1 != dhp->n_layer || !ds->has_head) {
        seterr(err, errlen, "both batches must span all layers with the head"); return -1;
    }
    if (db->B != B) { seterr(err, errlen, "target and draft hold different numbers of sequences"); return -1; }
    if (ti->output.N != di->output.N) { seterr(err, errlen, "target and draft vocabularies differ"); return -1; }
    if (k < 1 || T > tb->tmax) { seterr(err, errlen, "need 1 <= k and k + 1 <= the target's max_tokens (%d)", tb->tmax); return -1; }
    if (n_prompt < 1 || n_gen < 1) { seterr(err, errlen, "need at least one prompt token and one generated token"); return -1; }
    if (tb->n_past != db->n_past) { seterr(err, errlen, "target and draft are at different positions"); return -1; }
    const long long need = (long long)tb->n_past + n_prompt + (long long)n_gen * T + T;
    if (need > tb->n_ctx || need > db->n_ctx) { seterr(err, errlen, "contexts too short: need %lld positions", need); return -1; }
    if (db->out_cap < T) { seterr(err, errlen, "draft output buffer too small"); return -1; }
    // buffers: target checkpoints, acceptance state, output; draft state copies
    const size_t tss = (size_t)thp->h_v * thp->s_v * thp->s_k, tcs = (size_t)thp->conv_dim * (thp->conv_k - 1);
    const size_t dss = (size_t)dhp->h_v * dhp->s_v * dhp->s_k, dcs = (size_t)dhp->conv_dim * (dhp->conv_k - 1);
    if (tb->ck_ssm.empty()) {
        for (size_t li = 0; li < tb->ssm.size(); li++) {
            float *a = nullptr, *c = nullptr;
            if (tb->ssm[li] && (dalloc(ti, &a, (size_t)B * (tb->tmax - 1) * tss, err, errlen) ||
                                dalloc(ti, &c, (size_t)B * (tb->tmax - 1) * tcs, err, errlen))) return -1;
            tb->ck_ssm.push_back(a); tb->ck_conv.push_back(c);
        }
        if (dalloc(ti, &tb->keep, (size_t)B, err, errlen) || dalloc(ti, &tb->nout, (size_t)B, err, errlen) ||
            dalloc(ti, &tb->next, (size_t)B, err, errlen) ||
            dalloc(ti, (uint8_t **)&tb->spec_stats, 2 * sizeof(unsigned long long), err, errlen)) return -1;
    }
    if (n_gen > tb->spec_out_cap) {
        if (dalloc(ti, &tb->spec_out, (size_t)B * n_gen, err, errlen)) return -1;
        tb->spec_out_cap = n_gen;
    }
    if (db->snap_k < k) {
        db->snap_ssm.clear(); db->snap_conv.clear();
        for (size_t li = 0; li < db->ssm.size(); li++) {
            float *a = nullptr, *c = nullptr;
            if (db->ssm[li] && (dalloc(di, &a, (size_t)k * B * dss, err, errlen) || dalloc(di, &c, (size_t)k * B * dcs, err, errlen)))
                return -1;
            db->snap_ssm.push_back(a); db->snap_conv.push_back(c);
        }
        db->snap_k = k;
    }
    cudaStream_t st = ti->st;
    // the draft's work runs on its own stream; the two streams meet through events at each hand-over
    cudaEvent_t ev_t, ev_d;
    CK(cudaEventCreateWithFlags(&ev_t, cudaEventDisableTiming));
    CK(cudaEventCreateWithFlags(&ev_d, cudaEventDisableTiming));
    auto done = [&](int rc) { cudaEventDestroy(ev_t); cudaEventDestroy(ev_d); return rc; };
    CK(cudaEventRecord(ti->ev[0], st));
    CK(cudaMemsetAsync(tb->spec_stats, 0, 2 * sizeof(unsigned long long), st));
    // prompts: the target picks each sequence's first id after its prompt; the draft only takes the prompt
    if (batch_prefill(tb, prompts, n_prompt, true, err, errlen) || batch_prefill(db, prompts, n_prompt, false, err, errlen))
        return done(-1);
    head_pick_rows(tb, tb->x_last, B, tb->next);
    CK(cudaMemcpy2DAsync(tb->spec_out, sizeof(int32_t) * n_gen, tb->next, sizeof(int32_t), sizeof(int32_t), B,
                         cudaMemcpyDeviceToDevice, st));
    {
        std::vector<int> ones(B, 1);
        CK(cudaMemcpyAsync(tb->nout, ones.data(), sizeof(int) * B, cudaMemcpyHostToDevice, st));
        CK(cudaStreamSynchronize(st));
        CK(cudaStreamSynchronize(di->st));
    }
    std::vector<int> nout(B, 1);
    long long rounds = 0;
    const int E = dhp->n_embd, V = ti->output.N;
    (void)V;
    auto min_out = [&]() { int mn = n_gen; for (int v : nout) mn = v < mn ? v : mn; return mn; };
    while (min_out() < n_gen) {
        // ---- draft: k + 1 one-token steps from next[b], state copies after the first k
        CK(cudaEventRecord(ev_t, st));
        CK(cudaStreamWaitEvent(di->st, ev_t, 0));
        CK(cudaMemsetAsync(db->step, 0, sizeof(int) * B, di->st));
        launch(di, k_embed, dim3((E / 8 + 127) / 128, B), dim3(128), 0, di->tok_embd, (const int32_t *)tb->next, B, di->x, E);
        for (int i = 0; i <= k; i++) {
            run_layers_batch(db, di->x, 0, B);
            head_batch(db, di->x, 0, B, db->cur, di->x, db->npast);
            if (i < k)
                for (size_t li = 0; li < db->ssm.size(); li++) {
                    if (!db->ssm[li]) continue;
                    CK(cudaMemcpyAsync(db->snap_ssm[li] + (size_t)i * B * dss, db->ssm[li], sizeof(float) * B * dss,
                                       cudaMemcpyDeviceToDevice, di->st));
                    CK(cudaMemcpyAsync(db->snap_conv[li] + (size_t)i * B * dcs, db->conv[li], sizeof(float) * B * dcs,
                                       cudaMemcpyDeviceToDevice, di->st));
                }
        }
        CK(cudaEventRecord(ev_d, di->st));
        CK(cudaStreamWaitEvent(st, ev_d, 0));
        // ---- target: verify [last, d_0 .. d_(k-1)] of every sequence in one (k+1)-token forward
        launch(ti, k_spec_rows, dim3((B * T + 127) / 128), dim3(128), 0, (const int32_t *)tb->next, (const int32_t *)db->out_tok,
               db->out_cap, k, B, tb->rows_tok);
        launch(ti, k_embed, dim3((thp->n_embd / 8 + 127) / 128, B * T), dim3(128), 0, ti->tok_embd, (const int32_t *)tb->rows_tok,
               B * T, ti->x, thp->n_embd);
        run_layers_batch_multi(tb, ti->x, T, true, T);
        head_pick_rows(tb, ti->x, B * T, tb->picks);
        launch(ti, k_spec_accept_batch, dim3((B + 127) / 128), dim3(128), 0, (const int32_t *)db->out_tok, db->out_cap,
               (const int32_t *)tb->picks, k, B, tb->spec_out, (long long)n_gen, tb->nout, n_gen, tb->keep, tb->next,
               tb->spec_stats);
        // ---- both roll every sequence back to the tokens it keeps (target: checkpoints; draft: copies)
        for (size_t li = 0; li < tb->ssm.size(); li++) {
            if (!tb->ssm[li]) continue;
            launch(ti, k_batch_keep_state, dim3(64, B), dim3(256), 0, tb->ssm[li], (long long)tss, (const float *)tb->ck_ssm[li],
                   (long long)k * tss, (long long)tss, (const int *)tb->keep, T);
            launch(ti, k_batch_keep_state, dim3(8, B), dim3(256), 0, tb->conv[li], (long long)tcs, (const float *)tb->ck_conv[li],
                   (long long)k * tcs, (long long)tcs, (const int *)tb->keep, T);
        }
        launch(ti, k_batch_keep_pos, dim3(1), dim3(256), 0, tb->npast, (const int *)tb->keep, T, B);
        for (size_t li = 0; li < db->ssm.size(); li++) {
            if (!db->ssm[li]) continue;
            launch(ti, k_batch_keep_state, dim3(32, B), dim3(256), 0, db->ssm[li], (long long)dss, (const float *)db->snap_ssm[li],
                   (long long)dss, (long long)B * dss, (const int *)tb->keep, T);
            launch(ti, k_batch_keep_state, dim3(8, B), dim3(256), 0, db->conv[li], (long long)dcs, (const float *)db->snap_conv[li],
                   (long long)dcs, (long long)B * dcs, (const int *)tb->keep, T);
        }
        launch(ti, k_batch_keep_pos, dim3(1), dim3(256), 0, db->npast, (const int *)tb->keep, T, B);
        CK(cudaMemcpyAsync(nout.data(), tb->nout, sizeof(int) * B, cudaMemcpyDeviceToHost, st));
        if (sync_check(ti, err, errlen)) return done(-1);
        rounds++;
    }
    CK(cudaEventRecord(ti->ev[2], st));
    CK(cudaMemcpyAsync(out, tb->spec_out, sizeof(int32_t) * B * n_gen, cudaMemcpyDeviceToHost, st));
    unsigned long long sst[2] = {0, 0};
    CK(cudaMemcpyAsync(sst, tb->spec_stats, sizeof sst, cudaMemcpyDeviceToHost, st));
    std::vector<int> tp(B), dp(B);
    CK(cudaMemcpyAsync(tp.data(), tb->npast, sizeof(int) * B, cudaMemcpyDeviceToHost, st));
    CK(cudaMemcpyAsync(dp.data(), db->npast, sizeof(int) * B, cudaMemcpyDeviceToHost, st));
    if (sync_check(ti, err, errlen)) return done(-1);
    if (gpu_ms) cudaEventElapsedTime(gpu_ms, ti->ev[0], ti->ev[2]);
    // the sequences now sit at different positions; the host mirrors keep the furthest
    int mt = 0, md = 0;
    for (int b = 0; b < B; b++) { mt = tp[b] > mt ? tp[b] : mt; md = dp[b] > md ? dp[b] : md; }
    tb->n_past = mt; db->n_past = md;
    if (stats) { stats[0] = rounds; stats[1] = (long long)sst[0]; stats[2] = (long long)sst[1]; stats[3] = rounds * T; }
    return done(0);
}

// ---- pipeline-stage entry points: device buffers of the batch's device, rows = a micro-batch
// End of a *_rows call: wait for the stream and check errors, or in async mode only check the launches
// (errors then surface at xj_cuda_batch_sync).
static int rows_check(BatchImpl *bi, char *err, size_t errlen) {
    Impl *im = I(bi->s);
    if (!bi->async_rows) return sync_check(im, err, errlen);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { seterr(err, errlen, "GPU error: %s", cudaGetErrorString(e)); return -1; }
    return 0;
}

int xj_cuda_batch_embed_rows(xj_cuda_batch *b, const int32_t *tok_dev, float *x_dev, int nrows, char *err, size_t errlen) {
    if (!b || !tok_dev || !x_dev || nrows < 1 || nrows > b->impl.B) { seterr(err, errlen, "bad arguments"); return -1; }
    BatchImpl *bi = &b->impl;
    Impl *im = I(bi->s);
    DevGuard dg(im->dev);
    if (!im->tok_embd.p) { seterr(err, errlen, "this batch has no embedding table (layer range does not start at 0)"); return -1; }
    const int E = bi->s->m->hp.n_embd;
    launch(im, k_embed, dim3((E / 8 + 127) / 128, nrows), dim3(128), 0, im->tok_embd, tok_dev, nrows, x_dev, E);
    return rows_check(bi, err, errlen);
}

int xj_cuda_batch_forward_rows(xj_cuda_batch *b, float *x_dev, int row0, int nrows, char *err, size_t errlen) {
    if (!b || !x_dev || row0 < 0 || nrows < 1 || row0 + nrows > b->impl.B) { seterr(err, errlen, "bad row range"); return -1; }
    BatchImpl *bi = &b->impl;
    Impl *im = I(bi->s);
    DevGuard dg(im->dev);
    if (bi->n_past + 1 > bi->n_ctx) { seterr(err, errlen, "context is full (%d)", bi->n_ctx); return -1; }
    run_layers_batch(bi, x_dev, row0, nrows);
    launch(im, k_advance_batch, dim3(1), dim3(256), 0, bi->npast + row0, nrows, 1);
    if (rows_check(bi, err, errlen)) return -1;
    if (row0 + nrows == bi->B) bi->n_past++;   // the host mirror follows the last micro-batch of a step
    return 0;
}

int xj_cuda_batch_pick_rows(xj_cuda_batch *b, const float *x_dev, int row0, int nrows, int32_t *tok_dev, char *err,
                            size_t errlen) {
    if (!b || !x_dev || !tok_dev || row0 < 0 || nrows < 1 || row0 + nrows > b->impl.B) { seterr(err, errlen, "bad row range"); return -1; }
    BatchImpl *bi = &b->impl;
    Impl *im = I(bi->s);
    DevGuard dg(im->dev);
    if (!bi->s->has_head) { seterr(err, errlen, "this batch has no head"); return -1; }
    // the pick's embedding and position update go to scratch: the pipeline's first stage embeds the ids
    head_batch(bi, x_dev, row0, nrows, tok_dev, im->h, bi->np_scratch + row0);
    return rows_check(bi, err, errlen);
}

void *xj_cuda_batch_stream(xj_cuda_batch *b) { return b ? (void *)I(b->impl.s)->st : nullptr; }

int xj_cuda_batch_set_async(xj_cuda_batch *b, int on) {
    if (!b) return -1;
    b->impl.async_rows = on != 0;
    return 0;
}

int xj_cuda_batch_sync(xj_cuda_batch *b, char *err, size_t errlen) {
    if (!b) { seterr(err, errlen, "no batch"); return -1; }
    Impl *im = I(b->impl.s);
    DevGuard dg(im->dev);
    return sync_check(im, err, errlen);
}

long long xj_cuda_batch_last_launches(const xj_cuda_batch *b, long long *launches) {
    if (!b) return 0;
    if (launches) { launches[0] = b->impl.last_launches[0]; launches[1] = b->impl.last_launches[1]; }
    return b->impl.last_launches[0] + b->impl.last_launches[1];
}

}  // extern "C"
