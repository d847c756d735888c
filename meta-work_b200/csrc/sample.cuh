// Temperature sampling with top-k and top-p on the device (the sampler of the runtime's session layer,
// ios/App/XJGlue.c:251-282), for one logit row per CTA:
//
//   temperature <= 0: the greedy pick (largest logit, lowest index on ties).
//   otherwise: the k largest logits (k = top_k, 40 in the runtime), in descending order;
//              p_i = exp((v_i - v_0) / temperature) in double; the shortest prefix whose normalised
//              cumulative probability reaches top_p (0.95) is kept; r = u * (sum of the kept p_i) with u
//              uniform in [0, 1); the pick is the first kept i at which r - p_0 - ... - p_i <= 0.
//
// The top-k set is exact: a most-significant-digit radix select over order-preserving 32-bit keys of the
// logits finds the k-th largest key, then every element at or above it is gathered and sorted (key
// descending, index ascending), so equal logits at the k-th place are taken lowest index first. (The
// runtime's single-pass selection keeps the earliest of equal values too, except where its slot order
// differs; exactly equal fp32 logits at the cut are the only case where the two could differ.)
//
// u comes from a counter-based generator: SplitMix64 (Steele, Lea and Flood, "Fast splittable
// pseudorandom number generators", OOPSLA 2014) of seed + (counter + 1) * golden gamma, top 30 bits,
// times 2^-30: the same 30-bit resolution as the runtime's arc4random_uniform(1 << 30) / 2^30, but
// reproducible. The counter is the stage position at which the row's logits were computed (decode) or
// counter0 + row (the host-buffer entry point), so a seed fixes the whole sampled sequence.
#pragma once
#include "kernels.cuh"

namespace xjk {

constexpr int SAMPLE_KMAX = 64;          // largest top_k
constexpr int SAMPLE_CAND = 2048;        // gathered candidates (elements at or above the k-th largest key)
constexpr int SAMPLE_THREADS = 1024;

__host__ __device__ inline uint64_t splitmix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}
// Uniform double in [0, 1) with 30 random bits, for (seed, counter).
__host__ __device__ inline double sample_uniform(uint64_t seed, uint64_t counter) {
    const uint64_t z = splitmix64(seed + (counter + 1) * 0x9e3779b97f4a7c15ull);
    return (double)(uint32_t)(z >> 34) * (1.0 / 1073741824.0);
}
// Order-preserving key of a float: larger float -> larger unsigned key (NaN sorts above +inf).
XJ_DEV uint32_t flt_key(float v) {
    const uint32_t u = __float_as_uint(v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
XJ_DEV float key_flt(uint32_t k) { return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k); }

struct SampleSmem {
    unsigned hist[4096];
    unsigned long long cand[SAMPLE_CAND];
    unsigned ncand, need, prefix, eq;
    unsigned wcnt[32];
    float best, second;
    int pick;
};

// Picks one id from lg[0..n) with nthr threads (a multiple of 32, <= 1024, all of the CTA) and returns
// it in every thread; *margin = largest - second largest logit. S in shared memory.
template <class Bar>
XJ_DEV int sample_row_dev(const float *lg, int n, float temp, int top_k, double top_p, double u, SampleSmem &S, int tid,
                          int nthr, float *margin) {
    const int lane = tid & 31;
    if (temp <= 0.0f || top_k <= 1) {
        // greedy: largest value, lowest index
        float b = -INFINITY, b2 = -INFINITY;
        int bi = 0x7fffffff;
        for (int i = tid; i < n; i += nthr) {
            const float v = __ldcg(lg + i);
            if (v > b) { b2 = b; b = v; bi = i; } else b2 = fmaxf(b2, v);
        }
        __shared__ float sv[32], sv2[32];
        __shared__ int si[32];
        for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, b, o), ov2 = __shfl_xor_sync(0xffffffffu, b2, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > b || (ov == b && oi < bi)) { b2 = fmaxf(b, ov2); b = ov; bi = oi; } else b2 = fmaxf(b2, ov);
        }
        if (lane == 0) { sv[tid >> 5] = b; sv2[tid >> 5] = b2; si[tid >> 5] = bi; }
        Bar::sync();
        if (tid < 32) {
            const int nw = nthr >> 5;
            b = lane < nw ? sv[lane] : -INFINITY; b2 = lane < nw ? sv2[lane] : -INFINITY; bi = lane < nw ? si[lane] : 0x7fffffff;
            for (int o = 16; o; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, b, o), ov2 = __shfl_xor_sync(0xffffffffu, b2, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (ov > b || (ov == b && oi < bi)) { b2 = fmaxf(b, ov2); b = ov; bi = oi; } else b2 = fmaxf(b2, ov);
            }
            if (lane == 0) { S.pick = bi; S.best = b; S.second = b2; }
        }
        Bar::sync();
        if (margin) *margin = S.best - S.second;
        const int id = S.pick;
        Bar::sync();
        return id;
    }
    const int K = top_k < n ? top_k : n;
    // ---- radix select of the K-th largest key: digits of 12, 10 and 10 bits, most significant first
    if (tid == 0) { S.need = (unsigned)K; S.prefix = 0; }
    const int shifts[3] = {20, 10, 0}, widths[3] = {12, 10, 10};
    for (int pass = 0; pass < 3; pass++) {
        const int sh = shifts[pass], nb = 1 << widths[pass];
        for (int b = tid; b < nb; b += nthr) S.hist[b] = 0;
        Bar::sync();
        const unsigned prefix = S.prefix;
        const int hs = sh + widths[pass];            // bits above this digit must equal the prefix
        for (int i = tid; i < n; i += nthr) {
            const uint32_t k = flt_key(__ldcg(lg + i));
            if (pass == 0 || (k >> (hs & 31)) == prefix) atomicAdd(&S.hist[(k >> sh) & (nb - 1)], 1u);
        }
        Bar::sync();
        if (tid < 32) {
            // the digit b* holding the need-th largest remaining key: count from the top bin down,
            // 32 lanes scanning nb/32 consecutive bins each
            const int per = nb / 32, hi = nb - 1 - lane * per;
            unsigned cnt = 0;
            for (int b = hi; b > hi - per; b--) cnt += S.hist[b];
            unsigned incl = cnt;                     // bins above and including this lane's range
            for (int o = 1; o < 32; o <<= 1) {
                const unsigned v = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += v;
            }
            const unsigned need = S.need, excl = incl - cnt;
            const unsigned ballot = __ballot_sync(0xffffffffu, excl < need && need <= incl);
            const int owner = __ffs(ballot) - 1;     // exactly one lane's range holds it
            if (lane == owner) {
                unsigned above = excl;
                for (int b = hi; b > hi - per; b--) {
                    if (above + S.hist[b] >= need) {
                        S.need = need - above;       // elements of digit b still to take
                        S.prefix = (prefix << widths[pass]) | (unsigned)b;
                        S.eq = S.hist[b];            // after the last digit: elements equal to the K-th key
                        break;
                    }
                    above += S.hist[b];
                }
            }
        }
        Bar::sync();
    }
    // S.prefix = the K-th largest key; S.need of the S.eq elements equal to it belong to the top K
    const uint32_t kth = S.prefix;
    const unsigned need = S.need, above = (unsigned)K - need;
    // usually every element at or above the K-th key fits the candidate buffer and the sort orders
    // equal keys by index; otherwise (thousands of equal logits) the equal ones are taken in index order
    const bool all_fit = above + S.eq <= (unsigned)SAMPLE_CAND;
    if (tid == 0) S.ncand = 0;
    Bar::sync();
    for (int i = tid; i < n; i += nthr) {
        const uint32_t k = flt_key(__ldcg(lg + i));
        if (all_fit ? k >= kth : k > kth) {
            const unsigned slot = atomicAdd(&S.ncand, 1u);
            S.cand[slot] = ((unsigned long long)k << 32) | (0xffffffffu - (unsigned)i);
        }
    }
    Bar::sync();
    if (!all_fit) {
        const int warp = tid >> 5, nw = nthr >> 5;
        unsigned taken = 0;
        for (int i0 = 0; i0 < n && taken < need; i0 += nthr) {
            const int i = i0 + tid;
            const bool m = i < n && flt_key(__ldcg(lg + i)) == kth;
            const unsigned bal = __ballot_sync(0xffffffffu, m);
            if (lane == 0) S.wcnt[warp] = __popc(bal);
            Bar::sync();
            unsigned before = 0, tot = 0;
            for (int w = 0; w < nw; w++) { before += w < warp ? S.wcnt[w] : 0u; tot += S.wcnt[w]; }
            const unsigned rank = taken + before + __popc(bal & ((1u << lane) - 1u));
            if (m && rank < need) S.cand[above + rank] = ((unsigned long long)kth << 32) | (0xffffffffu - (unsigned)i);
            Bar::sync();
            taken += tot;
        }
        if (tid == 0) S.ncand = above + need;
        Bar::sync();
    }
    const int nc = (int)S.ncand;
    int P = 32;
    while (P < nc) P <<= 1;
    for (int i = nc + tid; i < P; i += nthr) S.cand[i] = 0ull;   // padding sorts last
    Bar::sync();
    // bitonic sort, descending: larger key first, then lower index (larger ~index) first
    for (int k = 2; k <= P; k <<= 1)
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = tid; i < P; i += nthr) {
                const int l = i ^ j;
                if (l > i) {
                    const unsigned long long a = S.cand[i], b = S.cand[l];
                    const bool desc = (i & k) == 0;
                    if (desc ? (a < b) : (a > b)) { S.cand[i] = b; S.cand[l] = a; }
                }
            }
            Bar::sync();
        }
    if (tid == 0) {
        // the runtime's probabilities, cut and draw (XJGlue.c:268-281), in the same order of operations
        double p[SAMPLE_KMAX], sum = 0.0;
        const float v0 = key_flt((uint32_t)(S.cand[0] >> 32));
        for (int i = 0; i < K; i++) {
            const float vi = key_flt((uint32_t)(S.cand[i] >> 32));
            p[i] = exp((double)__fdiv_rn(vi - v0, temp));   // float quotient, as the C expression computes it
            sum += p[i];
        }
        double acc = 0.0;
        int cut = K;
        for (int i = 0; i < K; i++) {
            acc += p[i] / sum;
            if (acc >= top_p) { cut = i + 1; break; }
        }
        double s2 = 0.0;
        for (int i = 0; i < cut; i++) s2 += p[i];
        double r = u * s2;
        int pick = 0;
        for (int i = 0; i < cut; i++) {
            r -= p[i];
            if (r <= 0.0) { pick = i; break; }
        }
        S.pick = (int)(0xffffffffu - (unsigned)(S.cand[pick] & 0xffffffffu));
        S.best = v0;
        S.second = K > 1 ? key_flt((uint32_t)(S.cand[1] >> 32)) : -INFINITY;
    }
    Bar::sync();
    if (margin) *margin = S.best - S.second;
    const int id = S.pick;
    Bar::sync();
    return id;
}

struct SampleArgs {
    const float *logits;          // [rows][ld]
    long long ld;
    int n;                        // vocabulary size
    float temp;
    double top_p;
    int top_k;
    unsigned long long seed, counter0;
    int32_t *out;                 // k_sample_rows: out[row]
    float *margin;                // k_sample_rows: margin[row] (may be null)
};

// One CTA per row: out[row] = the sampled id of row `row`, counter counter0 + row.
static __global__ void __launch_bounds__(SAMPLE_THREADS) k_sample_rows(SampleArgs a) {
    __shared__ SampleSmem S;
    const int row = blockIdx.x;
    float mg = 0.0f;
    const int id = sample_row_dev<BarBlock>(a.logits + (size_t)row * a.ld, a.n, a.temp, a.top_k, a.top_p,
                                            sample_uniform(a.seed, a.counter0 + (unsigned long long)row), S,
                                            threadIdx.x, blockDim.x, &mg);
    if (threadIdx.x == 0) {
        a.out[row] = id;
        if (a.margin) a.margin[row] = mg;
    }
}

// Decode-step pick from logits[0..n) (one block of SAMPLE_THREADS): the sampled id goes where the greedy
// pick of k_argmax_final goes (out_tok[*step], margin, *cur), its embedding row into x, and the position
// advances; the draw is keyed by the position the logits were computed at.
static __global__ void __launch_bounds__(SAMPLE_THREADS) k_sample_final(SampleArgs a, ArgmaxArgs g) {
    __shared__ SampleSmem S;
    griddep_wait();
    griddep_launch();   // successors may start their prologue; they wait for this grid before reading
    const int tid = threadIdx.x, nthr = blockDim.x;
    const int pos = *g.npast;
    float mg = 0.0f;
    const int id = sample_row_dev<BarBlock>(a.logits, a.n, a.temp, a.top_k, a.top_p,
                                            sample_uniform(a.seed, (unsigned long long)pos), S, tid, nthr, &mg);
    if (tid == 0) {
        const int s = *g.step;
        g.out_tok[s] = id;
        if (g.margin) g.margin[s] = mg;
        *g.cur = id;
        *g.step = s + 1;
        *g.npast = pos + 1;
    }
    const DevMat &emb = g.emb;
    for (int e0 = tid * 8; e0 < emb.K; e0 += nthr * 8) {
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

}  // namespace xjk
