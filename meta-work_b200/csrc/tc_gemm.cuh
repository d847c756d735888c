// Fifth-generation tensor cores (tcgen05) for the batched paths: accumulators in tensor memory (TMEM),
// operands in shared memory described by 64-bit matrix descriptors, one thread issuing the MMAs and a
// tcgen05.commit completing an mbarrier when they are done.
//
// Operand layout used throughout (no swizzle, K-major): a matrix of R rows x K halves is stored as
// "core matrices" of 8 rows x 8 halves (8 rows of 16 bytes, 128 contiguous bytes); core matrix (i, j)
// (rows 8i.., halves 8j..) sits at byte (i * (K / 8) + j) * 128 of the operand buffer. For one MMA
// k-step (16 halves, core columns 2s and 2s+1) the descriptor starts at byte 2s * 128 with a leading
// byte offset (next core matrix along K) of 128 and a stride byte offset (next 8 rows) of K / 8 * 128.
#pragma once
#include "gemv_mma.cuh"

namespace xjk {

// ------------------------------------------------------------------ tcgen05 primitives
XJ_DEV void tc_alloc(uint32_t *slot, uint32_t ncols) {            // one full warp
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" :: "r"(smem_u32(slot)), "r"(ncols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
XJ_DEV void tc_dealloc(uint32_t taddr, uint32_t ncols) {          // one full warp
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(taddr), "r"(ncols) : "memory");
}
XJ_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
XJ_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// Generic-proxy writes to shared memory -> visible to the tensor core (async proxy).
XJ_DEV void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// D[tmem] (+)= A . B^T for one k-step; a_desc / b_desc: shared-memory matrix descriptors.
XJ_DEV void tc_mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
                 :: "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}
// The mbarrier completes one arrival when every MMA this thread issued before has finished.
XJ_DEV void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" :: "r"(smem_u32(bar)) : "memory");
}
// 16 consecutive 32-bit columns of this warp's 32 TMEM lanes (lane i of the warp: lane base + i).
XJ_DEV void tc_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor: no swizzle, start / leading / stride byte offsets (multiples of
// 16), descriptor version 1.
XJ_DEV uint64_t tc_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
// Instruction descriptor of kind::f16: f32 accumulator, f16 A and B, both K-major, M x N.
__host__ __device__ constexpr uint32_t tc_idesc_f16(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
// Byte offset of element (r, k) in the core-matrix layout of an operand with K halves per row.
__host__ __device__ inline uint32_t tc_off(int r, int k, int K) {
    return (uint32_t)((((r >> 3) * (K >> 3) + (k >> 3)) << 7) + ((r & 7) << 4) + ((k & 7) << 1));
}

// ------------------------------------------------------------------ self-test
// D[128][64] = A[128][K] . B[64][K]^T (fp16 inputs, f32 accumulate) with K in chunks of 64 staged
// through shared memory: checks the descriptors, the MMA and the TMEM read-back against the host.
constexpr int TCS_M = 128, TCS_N = 64, TCS_KC = 64;

__global__ void __launch_bounds__(128, 1) k_tc_selftest(const __half *A, const __half *B, int K, float *D, int *err) {
    __shared__ __align__(128) uint8_t sa[TCS_M * TCS_KC * 2];
    __shared__ __align__(128) uint8_t sb[TCS_N * TCS_KC * 2];
    __shared__ __align__(8) uint64_t done;
    __shared__ uint32_t s_tmem;
    const int tid = threadIdx.x, warp = tid >> 5;
    if (tid == 0) { mbar_init(&done, 1); asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
    if (warp == 0) tc_alloc(&s_tmem, 64);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    constexpr uint32_t idesc = tc_idesc_f16(TCS_M, TCS_N);
    bool ok = true;
    int nchunk = 0;
    for (int k0 = 0; k0 < K && ok; k0 += TCS_KC, nchunk++) {
        // stage the chunk in the core-matrix layout (plain stores; the tensor core reads through the
        // async proxy, hence the proxy fence before the barrier)
        for (int e = tid; e < TCS_M * TCS_KC; e += 128) {
            const int r = e / TCS_KC, k = e % TCS_KC;
            *reinterpret_cast<__half *>(sa + tc_off(r, k, TCS_KC)) = A[(size_t)r * K + k0 + k];
        }
        for (int e = tid; e < TCS_N * TCS_KC; e += 128) {
            const int r = e / TCS_KC, k = e % TCS_KC;
            *reinterpret_cast<__half *>(sb + tc_off(r, k, TCS_KC)) = B[(size_t)r * K + k0 + k];
        }
        fence_async_smem();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
#pragma unroll
            for (int s = 0; s < TCS_KC / 16; s++) {
                const uint64_t ad = tc_desc(smem_u32(sa) + s * 256, 128, (TCS_KC / 8) * 128);
                const uint64_t bd = tc_desc(smem_u32(sb) + s * 256, 128, (TCS_KC / 8) * 128);
                tc_mma_f16(tmem, ad, bd, idesc, (k0 > 0 || s > 0) ? 1u : 0u);
            }
            tc_commit(&done);
        }
        ok = mbar_wait(&done, (uint32_t)(nchunk & 1), err);   // the MMAs finished: the buffers are free
        __syncthreads();
    }
    tc_fence_after();
    if (ok) {
        const int row = warp * 32 + (tid & 31);
#pragma unroll
        for (int c = 0; c < TCS_N; c += 16) {
            float v[16];
            tc_ld16(tmem + ((uint32_t)(warp * 32) << 16) + c, v);
#pragma unroll
            for (int i = 0; i < 16; i++) D[(size_t)row * TCS_N + c + i] = v[i];
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tc_dealloc(tmem, 64);
}

// ------------------------------------------------------------------ quantised GEMM, 17..64 tokens
// y[t][r] (epilogue)= sum_k W[r][k] x[t][k] for up to 64 tokens on the tcgen05 tensor cores. A CTA owns
// 128 rows (8 tiles of the tiled weight layout) and a contiguous range of 128-wide K chunks; when a
// matrix has fewer 128-row blocks than SMs, a block's chunks are split over a thread-block cluster
// exactly as in k_gemv_b64 (partials exchanged through distributed shared memory, summed by the owner
// in rank order, so the result does not depend on timing).
//
// The weights enter the MMA as their exact integer codes in fp16 (Q4_K q, Q6_K q - 32, Q8_0 q: a few
// logic operations per 8 weights from the tiled layout), the activations as fp16 hi / lo planes. Each
// scale block of the weights (Q4_K / Q8_0: 32 elements, Q6_K: 16) of a 64-wide half chunk accumulates
// code . (hi + lo) into its own f32 accumulator [128 rows][64 tokens] in tensor memory (exact products,
// f32 sums); when a half's MMAs are done, the compute warps read its accumulators back and add
// scale * accumulator into per-thread partial sums (one row, 16 tokens), in block order. The Q4_K
// minimum term -dmin*m * (block sum of x) is one more MMA per half into a separate accumulator: A holds
// -64 dmin*m as fp16 (hi, hi, lo) per block, B the block sums 2^-6 S as (Sh, Sl, Sh). So the result is
// fp32-level like the mma.sync path, and a token's column does not depend on the other tokens.
//
// Pipeline: a producer warp bulk-copies each chunk's 8 tiles of quantised bytes and its activation
// record into a 3-stage ring (full / empty mbarriers); per half chunk, 16 compute warps (two per tile)
// fold the half NBUF steps earlier into their partial sums, write this half's code plane, block scales
// and Q4_K minimum plane (NBUF = 3 sets for Q4_K, 2 otherwise) and arrive on the half's "ready"
// mbarrier; an MMA warp waits for it, issues the half's MMAs with precomputed descriptors and commits
// to the half's "done" mbarrier (and, after a chunk's second half, to the stage's "empty" one).
constexpr int TC_SUB = 64;                          // K of one half chunk
constexpr int TC_ROWS = 128, TC_TILES = 8, TC_WARPS = 16;   // two compute warps per tile
constexpr int TC_THREADS = TC_WARPS * 32 + 64;      // + the producer warp and the MMA warp
constexpr int TC_PLANE_A = TC_ROWS * TC_SUB * 2;    // code plane of a half chunk: 16 KB
constexpr int TC_PLANE_M = TC_ROWS * 16 * 2;        // Q4_K minimum plane of a half chunk: 4 KB
constexpr int TC_STAGES = 3;
constexpr int TC_MAXSPLIT = 16;
constexpr int TC_RS = TC_T + 4;                     // row stride (floats) of the partial sums
constexpr size_t TC_PART = (size_t)TC_ROWS * TC_RS * 4;   // this CTA's partial sums (stage area, after the K loop)
constexpr size_t TC_RECV = (size_t)(TC_ROWS + TC_MAXSPLIT) * TC_RS * 4;   // other splits' partials (stage area, after it)
constexpr int TC_DBUF = TC_ROWS * 4;                // floats of one half's block scales (<= 4 blocks)
template <int TYPE> constexpr int tc_nacc() { return TYPE == XJ_Q6_K ? 4 : 2; }   // scale blocks per half
template <int TYPE> constexpr uint32_t tc_cols() { return TYPE == XJ_Q8_0 ? 256u : 512u; }   // TMEM columns
// half chunks in flight (code planes, accumulator sets): as many as tensor memory and shared memory allow
template <int TYPE> constexpr int tc_nbuf() { return TYPE == XJ_Q4_K ? 3 : 2; }
template <int TYPE> constexpr int tc_stage() { return TC_REC + TC_TILES * b64_wbytes<TYPE>(); }
template <int TYPE> constexpr size_t tc_smem() {
    return (size_t)TC_STAGES * tc_stage<TYPE>() + tc_nbuf<TYPE>() * (TC_PLANE_A + TC_PLANE_M + 2 * TC_DBUF * 4);
}
static_assert(tc_smem<XJ_Q8_0>() <= 227 * 1024 && tc_smem<XJ_Q6_K>() <= 227 * 1024, "fits one SM");
static_assert(tc_stage<XJ_Q4_K>() % 128 == 0 && tc_stage<XJ_Q6_K>() % 128 == 0 && tc_stage<XJ_Q8_0>() % 128 == 0, "aligned stages");
static_assert(TC_PART + TC_RECV <= TC_STAGES * tc_stage<XJ_Q4_K>(), "partials fit the stage area");
static_assert(3 * 2 * 64 + 64 <= 512 && 2 * 4 * 64 <= 512 && 2 * 2 * 64 <= 256, "accumulators fit tensor memory");
static_assert(tc_smem<XJ_Q4_K>() <= 227 * 1024, "fits one SM");
XJ_DEV void tc_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(smem_u32(bar)) : "memory");
}

// Byte of (row r, element k) in a code plane ([128 rows][64 halves], core-matrix layout).
XJ_DEV uint32_t tc_aoff(int r, int k) { return (uint32_t)((((r >> 3) * (TC_SUB >> 3) + (k >> 3)) << 7) + ((r & 7) << 4) + ((k & 7) << 1)); }
// Byte of (row r, column k < 16) in a minimum plane.
XJ_DEV uint32_t tc_moff(int r, int k) { return (uint32_t)((((r >> 3) * 2 + (k >> 3)) << 7) + ((r & 7) << 4) + ((k & 7) << 1)); }

// Warp `tl` (+ 8 * part) writes the codes of k-steps (2 part, 2 part + 1) of its tile's 16 rows in half
// `h` of the staged chunk into the code plane ab. Lane (g, c) holds, per k-step, the codes of rows g,
// g+8 and elements 2c, 2c+1, 2c+8, 2c+9 (the mma.sync A-fragment order of the tiled layout): register
// r of the fragment is the pair (row g + 8 (r & 1), elements 2c + 8 (r >> 1) + {0, 1}).
template <int TYPE>
XJ_DEV void tc_codes(const uint8_t *wst, int tl, int part, int lane, int h, uint8_t *ab) {
    using BG = B64Geo<TYPE>;
    const int g = lane >> 2, c = lane & 3, r0 = tl * 16 + g;
#pragma unroll
    for (int kk = 0; kk < 2; kk++) {
        const int ks = 2 * part + kk;                      // k-step within the half
        uint32_t a[4];
        if constexpr (TYPE == XJ_Q4_K || TYPE == XJ_Q6_K) {
            const uint32_t w = *reinterpret_cast<const uint32_t *>(wst + ((h * 32 + lane) * 16) + 4 * ks);
            nib_frag(w, a);
            if constexpr (TYPE == XJ_Q6_K) {               // + 16 * high - 32: the signed code, exact
                uint32_t hw = *reinterpret_cast<const uint32_t *>(wst + BG::Q + lane * 16 + 4 * ((4 * h + ks) >> 1));
                if (ks & 1) hw >>= 8;
                uint32_t ah[4];
                hi_frag(hw, ah);
#pragma unroll
                for (int r = 0; r < 4; r++) a[r] = hadd2(a[r], ah[r]);
            }
        } else {                                           // Q8_0: unit 2h + part, k-step kk
            const uint8_t *qs = wst + ((2 * h + part) * 32 + lane) * 16 + 8 * kk;
            q8_frag(*reinterpret_cast<const uint32_t *>(qs), *reinterpret_cast<const uint32_t *>(qs + 4), a);
        }
#pragma unroll
        for (int r = 0; r < 4; r++)
            *reinterpret_cast<uint32_t *>(ab + tc_aoff(r0 + 8 * (r & 1), 16 * ks + 2 * c + 8 * (r >> 1))) = a[r];
    }
}

// The block scale of item (row, block) = (item / NB, item % NB) of half `h` (`hh`: which half of the
// K-quant super-block the chunk is) into db[row * 4 + block]; Q4_K also writes the row's minimum plane
// entries of the block (-64 dmin*m as hi, hi, lo in columns 3b .. 3b + 2; columns 6..15 stay zero).
template <int TYPE>
XJ_DEV void tc_scales(const uint8_t *wst0, int item, int nt, int hh, int h, float *db, uint8_t *mp) {
    using BG = B64Geo<TYPE>;
    constexpr int WB = b64_wbytes<TYPE>();
    constexpr int NB = tc_nacc<TYPE>();
    const int row = item / NB, b = item % NB;
    if (row >= TC_ROWS) return;
    const int tl = row >> 4, rt = row & 15;
    if (tl >= nt) {                                        // rows past the matrix: zeros (never stored)
        db[row * 4 + b] = 0.0f;
        if (TYPE == XJ_Q4_K)
            for (int k = 3 * b; k < 3 * b + 3; k++) *reinterpret_cast<__half *>(mp + tc_moff(row, k)) = __float2half_rn(0.0f);
        return;
    }
    const uint8_t *wst = wst0 + tl * WB;
    if constexpr (TYPE == XJ_Q4_K) {
        const uint8_t *hdr = wst + BG::Q + rt * 16;
        const float d = h2f(ld_u16(hdr)), dmin = h2f(ld_u16(hdr + 2));
        int s_, m_;
        k4_scale_min(4 * hh + 2 * h + b, hdr + 4, s_, m_);
        db[row * 4 + b] = __fmul_rn(d, (float)s_);
        const float mm = -64.0f * __fmul_rn(dmin, (float)m_);
        const __half mh = __float2half_rn(mm), ml = __float2half_rn(mm - __half2float(mh));
        *reinterpret_cast<__half *>(mp + tc_moff(row, 3 * b)) = mh;
        *reinterpret_cast<__half *>(mp + tc_moff(row, 3 * b + 1)) = mh;
        *reinterpret_cast<__half *>(mp + tc_moff(row, 3 * b + 2)) = ml;
    } else if constexpr (TYPE == XJ_Q6_K) {
        const float d = h2f(ld_u16(wst + BG::Q + BG::H + BG::S + rt * 2));
        const int8_t sc = reinterpret_cast<const int8_t *>(wst + BG::Q + BG::H + rt * 16)[8 * hh + 4 * h + b];
        db[row * 4 + b] = __fmul_rn(d, (float)sc);
    } else {
        db[row * 4 + b] = h2f(ld_u16(wst + BG::Q + ((2 * h + b) * 16 + rt) * 2));
    }
}

// Bounded mbarrier wait: the thread sleeps in hardware until the phase completes; gives up (setting
// *err) after about a second, or at once when *err is set (read every 8 polls, one load in flight), so
// an error anywhere ends every wait of the grid quickly. `nap` (ns) > 0 sleeps between polls: the
// producer and MMA warps share their SM sub-partitions with compute warps, whose issue slots a
// polling warp would take.
XJ_DEV bool mbar_try_wait_sleep(uint64_t *bar, uint32_t parity) {   // sleeps until the phase completes (or ~0.1 ms)
    uint32_t ok;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, 100000;\n selp.u32 %0, 1, 0, p;\n}"
                 : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}
XJ_DEV unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
XJ_DEV bool tc_wait(uint64_t *bar, uint32_t parity, int *err, int nap = 0) {
    if (mbar_try_wait_sleep(bar, parity)) return true;
    unsigned long long t0;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    int ev = *(volatile int *)err;
    for (int it = 1; it < (1 << 26); it++) {
        if (nap) __nanosleep(nap);
        if (mbar_try_wait_sleep(bar, parity)) return true;
        if ((it & 7) == 0) {
            if (ev) return false;
            ev = *(volatile int *)err;
            unsigned long long t;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
            if (t - t0 > 1000000000ull) break;
        }
    }
    atomicExch(err, 1);
    return false;
}

template <int TYPE>
__global__ void __launch_bounds__(TC_THREADS, 1) k_gemm_tc(B64Args a) {
    constexpr int WB = b64_wbytes<TYPE>(), SBY = tc_stage<TYPE>(), NB = tc_nacc<TYPE>();
    constexpr int NBUF = tc_nbuf<TYPE>(), ND = 2 * NBUF;   // plane / accumulator sets, scale buffers
    constexpr bool KQ = TYPE != XJ_Q8_0;
    constexpr uint32_t IDESC = tc_idesc_f16(TC_ROWS, TC_T), NCOL = tc_cols<TYPE>();
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t *aplane = smem + (size_t)TC_STAGES * SBY;                   // [NBUF] code planes
    uint8_t *mplane = aplane + NBUF * TC_PLANE_A;                       // [NBUF] Q4_K minimum planes
    float *dbuf = reinterpret_cast<float *>(mplane + NBUF * TC_PLANE_M);   // [ND][128][4] block scales
    // after the K loop, in the stage area: this CTA's partials, then [ns][ceil(128/ns)][TC_RS] partials
    // of its rows from the other splits (peers send only after every CTA of the cluster left its loop)
    float *recv = reinterpret_cast<float *>(smem + TC_PART);
    __shared__ __align__(8) uint64_t full[TC_STAGES], empty[TC_STAGES], mdone[3], ready[3], rbar;
    __shared__ uint32_t s_tmem;
    __shared__ float tok_inv[TC_T];                    // 1 / range scale (a power of two: exact)
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int T = a.T, K = a.K, ns = a.nsplit;
    const int blk = blockIdx.x / ns;
    const int split = ns > 1 ? (int)cluster_rank() : 0;
    int j = 0;
    while (blk >= a.blk_start[j + 1]) j++;
    const MmaJob &jb = a.job[j];
    const Tiled &W = jb.w;
    const int ntiles = (W.N + 15) / 16;
    const int t0 = (blk - a.blk_start[j]) * TC_TILES;
    const int nt = ntiles - t0 < TC_TILES ? ntiles - t0 : TC_TILES;
    const int nch = K / TC_CK;
    const int c0 = (int)((long long)split * nch / ns), c1 = (int)((long long)(split + 1) * nch / ns);
    const int nc = c1 - c0, nsub = 2 * nc;
    const int nrmax = (TC_ROWS + ns - 1) / ns;
    const int rb = split * TC_ROWS / ns, nr = (split + 1) * TC_ROWS / ns - rb;   // the rows this CTA finishes
    auto issue_w = [&](int i) {       // producer warp: weights of chunk c0 + i, one tile per lane
        const int ch = c0 + i;
        uint8_t *st = smem + (size_t)(i % TC_STAGES) * SBY + TC_REC;
        uint64_t *bar = &full[i % TC_STAGES];
        if (lane == 0) mbar_expect_tx(bar, (uint32_t)(TC_REC + nt * WB));
        __syncwarp();
        if (lane < nt) {
            uint8_t *dst = st + lane * WB;
            const size_t tile = (size_t)(t0 + lane);
            if (KQ) {
                constexpr int QB = Geo<TYPE>::QB, HB = Geo<TYPE>::HB, SB = Geo<TYPE>::SB, DB = Geo<TYPE>::DB;
                const size_t tu = tile * W.nu + (ch >> 1);
                const int hh = ch & 1;
                bulk_g2s(dst, W.q + tu * QB + hh * (QB / 2), QB / 2, bar);
                if (HB) bulk_g2s(dst + B64Geo<TYPE>::Q, W.h + tu * HB + hh * (HB / 2), HB / 2, bar);
                bulk_g2s(dst + B64Geo<TYPE>::Q + B64Geo<TYPE>::H, W.s + tu * SB, SB, bar);
                if (DB) bulk_g2s(dst + B64Geo<TYPE>::Q + B64Geo<TYPE>::H + B64Geo<TYPE>::S, W.d + tu * DB, DB, bar);
            } else {
                const size_t tu = tile * W.nu + (size_t)ch * 4;
                bulk_g2s(dst, W.q + tu * Geo<TYPE>::QB, 4 * Geo<TYPE>::QB, bar);
                bulk_g2s(dst + B64Geo<TYPE>::Q, W.d + tu * Geo<TYPE>::DB, 4 * Geo<TYPE>::DB, bar);
            }
        }
    };
    auto issue_x = [&](int i) {       // activation record of chunk c0 + i (after the predecessor finished)
        bulk_g2s(smem + (size_t)(i % TC_STAGES) * SBY, (const uint8_t *)a.xbuf + (size_t)(c0 + i) * TC_REC, TC_REC,
                 &full[i % TC_STAGES]);
    };
    if (tid == 0) {
        for (int q = 0; q < TC_STAGES; q++) { mbar_init(&full[q], 1); mbar_init(&empty[q], 1); }
        for (int q = 0; q < NBUF; q++) { mbar_init(&mdone[q], 1); mbar_init(&ready[q], TC_WARPS); }
        mbar_init(&rbar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        if (ns > 1) mbar_expect_tx(&rbar, (uint32_t)((ns - 1) * nr * TC_RS * 4));
    }
    if (warp == 0) tc_alloc(&s_tmem, NCOL);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    bool ok = true;
    float y[16];                                           // compute threads: row crow, tokens 16 tb .. 16 tb + 15
#pragma unroll
    for (int i = 0; i < 16; i++) y[i] = 0.0f;
    const int quarter = warp & 3, tb = (warp >> 2) & 3, crow = 32 * quarter + lane;
    const uint32_t tlane = (uint32_t)(32 * quarter) << 16;
    // fold half qq's accumulators (set qq % NBUF) into y, scale block by scale block
    auto fold = [&](int qq) {
        const float *db = dbuf + (qq % ND) * TC_DBUF + crow * 4;
#pragma unroll
        for (int b = 0; b < NB; b++) {
            float v[16];
            tc_ld16(tmem + tlane + (uint32_t)(((qq % NBUF) * NB + b) * 64 + 16 * tb), v);
            const float sc = db[b];
#pragma unroll
            for (int i = 0; i < 16; i++) y[i] = fmaf(sc, v[i], y[i]);
        }
    };
    if (warp == TC_WARPS) {
        // ---- producer: weights do not depend on the predecessor kernel, the activations do
        int issued = nc < TC_STAGES ? nc : TC_STAGES;
        for (int i = 0; i < issued; i++) issue_w(i);
        griddep_launch();
        griddep_wait();
        if (lane == 0)
            for (int i = 0; i < TC_STAGES && i < nc; i++) issue_x(i);
        for (int i = TC_STAGES; i < nc && ok; i++) {
            // the stage is free once the MMAs of chunk i - TC_STAGES are done
            if (lane == 0) ok = tc_wait(&empty[i % TC_STAGES], (uint32_t)(((i / TC_STAGES) - 1) & 1), a.err, 256);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            issue_w(i);
            if (lane == 0) issue_x(i);
            issued = i + 1;
        }
        // copies in flight must land before the stage area is reused (they all have, unless a wait gave up)
        if (lane == 0)
            for (int i = issued > TC_STAGES ? issued - TC_STAGES : 0; i < issued; i++) {
                const unsigned long long t0 = globaltimer_ns();
                while (!mbar_try_wait_sleep(&full[i % TC_STAGES], (uint32_t)((i / TC_STAGES) & 1)))
                    if (globaltimer_ns() - t0 > 100000000ull) break;
            }
    } else if (warp == TC_WARPS + 1) {
        // ---- MMA warp (lane 0): per half chunk, once the 16 compute warps have written its code plane
        // and scales (and folded the half two steps earlier out of the accumulators it reuses), issue its
        // MMAs with descriptors precomputed here (a descriptor's start address is its low 14 bits, in
        // 16-byte units, so an offset into the same buffer is an addition).
        griddep_launch();
        if (lane == 0) {
            const uint64_t A0 = tc_desc(smem_u32(aplane), 128, (TC_SUB / 8) * 128);
            const uint64_t M0 = tc_desc(smem_u32(mplane), 128, 256);
            const uint64_t B0 = tc_desc(smem_u32(smem), 128, (TC_CK / 8) * 128);
            const uint64_t S0 = tc_desc(smem_u32(smem) + 2 * TC_PLANE_X, 128, 256);
            for (int i = 0; i < nc && ok; i++) {
                const int s = i % TC_STAGES;
                ok = tc_wait(&full[s], (uint32_t)((i / TC_STAGES) & 1), a.err, 64);
                for (int h = 0; h < 2 && ok; h++) {
                    const int q = 2 * i + h, ab = q % NBUF;
                    ok = tc_wait(&ready[ab], (uint32_t)((q / NBUF) & 1), a.err, 64);
                    if (!ok) break;
                    tc_fence_after();
                    const uint64_t ad0 = A0 + (uint64_t)(ab * (TC_PLANE_A >> 4));
                    const uint64_t bd0 = B0 + (uint64_t)((s * SBY + 8 * h * 128) >> 4);
#pragma unroll
                    for (int ks = 0; ks < TC_SUB / 16; ks++) {
                        const int b = TYPE == XJ_Q6_K ? ks : ks >> 1;       // scale block of the k-step
                        const bool first = TYPE == XJ_Q6_K ? true : (ks & 1) == 0;
                        const uint32_t acc = tmem + (uint32_t)((ab * NB + b) * 64);
                        const uint64_t ad = ad0 + (uint64_t)(ks * 16), bh = bd0 + (uint64_t)(ks * 16);
                        tc_mma_f16(acc, ad, bh, IDESC, first ? 0u : 1u);
                        tc_mma_f16(acc, ad, bh + (uint64_t)(TC_PLANE_X >> 4), IDESC, 1u);
                    }
                    if constexpr (TYPE == XJ_Q4_K) {
                        const uint64_t md = M0 + (uint64_t)(ab * (TC_PLANE_M >> 4));
                        const uint64_t sd = S0 + (uint64_t)((s * SBY + h * TC_PLANE_S) >> 4);
                        tc_mma_f16(tmem + (uint32_t)(NBUF * NB * 64), md, sd, IDESC, q > 0 ? 1u : 0u);
                    }
                    tc_commit(&mdone[ab]);
                    if (h == 1) tc_commit(&empty[s]);
                }
            }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
    } else {
        griddep_launch();
        griddep_wait();
        if (tid < T) tok_inv[tid] = 1.0f / reinterpret_cast<const float *>((const uint8_t *)a.xbuf + (size_t)nch * TC_REC)[tid];
        // compute warps: per half chunk, fold the half NBUF steps earlier (its MMAs are done), write this
        // half's code plane and scales, and tell the MMA warp (a failed wait only skips work; `ok` is kept
        // warp-uniform for the warp-wide tensor-memory loads). A half's MMAs need every warp's arrival,
        // so warps run at most NBUF halves apart and 2 * NBUF scale buffers never collide.
        const int tl = warp & (TC_TILES - 1), part = warp >> 3;
        // the minimum planes' columns 6..15 are zero for good (the MMA multiplies them)
        if (TYPE == XJ_Q4_K)
            for (int e = tid; e < NBUF * TC_ROWS * 10; e += TC_WARPS * 32)
                *reinterpret_cast<__half *>(mplane + (e / (TC_ROWS * 10)) * TC_PLANE_M + tc_moff((e / 10) % TC_ROWS, 6 + e % 10)) =
                    __float2half_rn(0.0f);
        // scale items: NB per row; Q6_K one per thread, Q4_K / Q8_0 lanes 0..15 of every warp
        const int item = NB == 4 ? tid : (lane < 16 ? warp * 16 + lane : TC_ROWS * NB);
        for (int i = 0; i < nc; i++) {
            const int s = i % TC_STAGES;
            uint8_t *st = smem + (size_t)s * SBY;
            if (ok) ok = tc_wait(&full[s], (uint32_t)((i / TC_STAGES) & 1), a.err);
            ok = __all_sync(0xffffffffu, ok);
            const int hh = (c0 + i) & 1;
            for (int h = 0; h < 2; h++) {
                const int q = 2 * i + h, ab = q % NBUF;
                if (q >= NBUF) {
                    // half q - NBUF is done: its planes are free and its accumulators final
                    if (ok) ok = tc_wait(&mdone[ab], (uint32_t)(((q / NBUF) - 1) & 1), a.err);
                    ok = __all_sync(0xffffffffu, ok);
                    tc_fence_after();
                    if (ok) fold(q - NBUF);
                    tc_fence_before();
                }
                uint8_t *ap = aplane + (size_t)ab * TC_PLANE_A, *mp = mplane + (size_t)ab * TC_PLANE_M;
                if (ok && tl < nt) tc_codes<TYPE>(st + TC_REC + tl * WB, tl, part, lane, h, ap);
                if (ok) tc_scales<TYPE>(st + TC_REC, item, nt, hh, h, dbuf + (q % ND) * TC_DBUF, mp);
                fence_async_smem();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) tc_arrive(&ready[ab]);
            }
        }
        // the last NBUF halves
        for (int qq = nsub >= NBUF ? nsub - NBUF : 0; qq < nsub; qq++) {
            if (ok) ok = tc_wait(&mdone[qq % NBUF], (uint32_t)((qq / NBUF) & 1), a.err);
            ok = __all_sync(0xffffffffu, ok);
            tc_fence_after();
            if (ok) fold(qq);
        }
        if (TYPE == XJ_Q4_K && ok) {                       // the minimum term, unscaled
            float v[16];
            tc_ld16(tmem + tlane + (uint32_t)(NBUF * NB * 64 + 16 * tb), v);
#pragma unroll
            for (int i = 0; i < 16; i++) y[i] += v[i];
        }
    }
    const bool allok = __syncthreads_and(ok) != 0;
    if (ns == 1) {
        // one CTA per block: the epilogue straight from the partial sums in registers (row crow, tokens
        // 16 tb .. 16 tb + 15; a warp's lanes are 32 consecutive rows, so each store is coalesced), with
        // the arithmetic of the split path below
        const int ch = t0 * 16 + crow;
        if (warp < TC_WARPS && allok && ch < W.N) {
            const int epi = jb.epi, ldy = (int)jb.ldy, kc = jb.kc;
            float *yb = jb.y;
            if (epi == EPI_CONV) {
                float wc[9], wl = 0.0f;
#pragma unroll
                for (int k = 0; k < 9; k++) wc[k] = k < kc ? jb.conv_w[(size_t)ch * kc + k] : 0.0f;
#pragma unroll
                for (int k = 0; k < 9; k++)
                    if (k == kc - 1) wl = wc[k];
#pragma unroll
                for (int i = 0; i < 16; i++) {
                    const int t = 16 * tb + i;
                    if (t >= T) break;
                    float *stt = jb.conv_state + t * jb.conv_bstride + (size_t)ch * (kc - 1);
                    float cs[8];
#pragma unroll
                    for (int k = 0; k < 8; k++) cs[k] = k < kc - 1 ? stt[k] : 0.0f;
                    const float v = (0.0f + y[i]) * tok_inv[t];
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
            } else {
#pragma unroll
                for (int i = 0; i < 16; i++) {
                    const int t = 16 * tb + i;
                    if (t >= T) break;
                    const float v = (0.0f + y[i]) * tok_inv[t];
                    if (epi == EPI_ADD) yb[(size_t)t * ldy + ch] += v;
                    else yb[(size_t)t * ldy + ch] = v;
                }
            }
        }
        tc_fence_before();
        __syncthreads();
        if (warp == 0) tc_dealloc(tmem, NCOL);
        return;
    }
    // ---- partial sums [row][TC_RS] in the stage area (free: every load landed, every MMA is done)
    float *part = reinterpret_cast<float *>(smem);
    if (warp < TC_WARPS && allok) {
#pragma unroll
        for (int e = 0; e < 16; e += 4)
            *reinterpret_cast<float4 *>(part + (size_t)crow * TC_RS + 16 * tb + e) = make_float4(y[e], y[e + 1], y[e + 2], y[e + 3]);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tc_dealloc(tmem, NCOL);
    if (ns > 1) {
        // every CTA of the cluster has left its K loop (its stage area now holds partials): each owner's
        // rows to slot `split` of its receive buffer, one bulk copy per owner
        cluster_arrive();
        cluster_wait();
        if (tid < ns && tid != split) {
            const int o = tid, orb = o * TC_ROWS / ns, onr = (o + 1) * TC_ROWS / ns - orb;
            fence_async_smem();
            bulk_s2peer(peer_addr(recv + (size_t)split * nrmax * TC_RS, (uint32_t)o), part + (size_t)orb * TC_RS,
                        (uint32_t)(onr * TC_RS * 4), peer_addr(&rbar, (uint32_t)o));
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
            asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");   // the source may be reused / freed
        }
        tc_wait(&rbar, 0u, a.err);                         // every other split's partials of this CTA's rows
    }
    // ---- rows [rb, rb + nr): sum over splits in rank order, epilogue (k_gemv_b64's)
    const int epi = jb.epi, ldy = (int)jb.ldy, kc = jb.kc;
    float *yb = jb.y;
    const int tstep = TC_THREADS / nr, rl = tid % nr, tt = tid / nr;
    const int row = rb + rl, ch = t0 * 16 + row;
    if (allok && tt < tstep && ch < W.N) {
        const float *own = part + (size_t)row * TC_RS;
        const float *rcv = recv + (size_t)rl * TC_RS;
        auto total = [&](int t) {
            float sv = 0.0f;
#pragma unroll
            for (int r = 0; r < TC_MAXSPLIT; r++)
                if (r < ns) sv += r == split ? own[t] : rcv[(size_t)r * nrmax * TC_RS + t];
            return sv * tok_inv[t];
        };
        if (epi == EPI_CONV) {
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
            for (int t = tt; t < T; t += tstep) yb[(size_t)t * ldy + ch] += total(t);
        } else {
            for (int t = tt; t < T; t += tstep) yb[(size_t)t * ldy + ch] = total(t);
        }
    }
}

// Launch on activations prepared by k_prep_xt<PREP_TC> into a.xbuf: blocks of 128 rows, each block's K
// chunks split over a cluster of ns CTAs when that lowers (waves x chunks per CTA).
template <int TYPE>
inline cudaError_t launch_tc_t(B64Args a, cudaStream_t st) {
    constexpr int MAXDEV = 64;
    static int sms_dev[MAXDEV] = {0};
    static int occ[MAXDEV][TC_MAXSPLIT + 1] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= MAXDEV) dev = 0;
    constexpr size_t smem = tc_smem<TYPE>();
    if (!sms_dev[dev]) {
        cudaFuncSetAttribute(k_gemm_tc<TYPE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        cudaFuncSetAttribute(k_gemm_tc<TYPE>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        cudaDeviceGetAttribute(&sms_dev[dev], cudaDevAttrMultiProcessorCount, dev);
        occ[dev][1] = sms_dev[dev];
        for (int ns = 2; ns <= TC_MAXSPLIT; ns++) {
            cudaLaunchConfig_t q{};
            q.gridDim = dim3(ns * 64);
            q.blockDim = dim3(TC_THREADS);
            q.dynamicSmemBytes = smem;
            cudaLaunchAttribute ca[1];
            ca[0].id = cudaLaunchAttributeClusterDimension;
            ca[0].val.clusterDim.x = (unsigned)ns;
            ca[0].val.clusterDim.y = 1;
            ca[0].val.clusterDim.z = 1;
            q.attrs = ca;
            q.numAttrs = 1;
            int n = 0;
            if (cudaOccupancyMaxActiveClusters(&n, k_gemm_tc<TYPE>, &q) != cudaSuccess) { cudaGetLastError(); n = 0; }
            occ[dev][ns] = n;
        }
    }
    a.blk_start[0] = 0;
    for (int j = 0; j < a.njob; j++) a.blk_start[j + 1] = a.blk_start[j] + ((a.job[j].w.N + 15) / 16 + TC_TILES - 1) / TC_TILES;
    const int nblk = a.blk_start[a.njob], nch = a.K / TC_CK;
    constexpr int FIXED = 2;
    int best = 1;
    long long best_cost = (long long)((nblk + occ[dev][1] - 1) / occ[dev][1]) * (nch + FIXED);
    for (int ns = 2; ns <= TC_MAXSPLIT && ns <= nch; ns++) {
        if (occ[dev][ns] < 1) continue;
        const long long cost = (long long)((nblk + occ[dev][ns] - 1) / occ[dev][ns]) * ((nch + ns - 1) / ns + FIXED);
        if (cost < best_cost) { best_cost = cost; best = ns; }
    }
    const int ns = best;
    a.nsplit = ns;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(nblk * ns);
    cfg.blockDim = dim3(TC_THREADS);
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
    return cudaLaunchKernelEx(&cfg, k_gemm_tc<TYPE>, a);
}
inline cudaError_t launch_tc(const B64Args &a, int type, cudaStream_t st) {
    switch (type) {
    case XJ_Q4_K: return launch_tc_t<XJ_Q4_K>(a, st);
    case XJ_Q6_K: return launch_tc_t<XJ_Q6_K>(a, st);
    case XJ_Q8_0: return launch_tc_t<XJ_Q8_0>(a, st);
    default: return cudaErrorInvalidValue;
    }
}
// Matrices the tensor-core kernel takes: those of the 64-token kernel (b64_ok).
inline bool tc_ok(const MmaJob &j, int K) { return b64_ok(j, K) && K % TC_CK == 0; }

}  // namespace xjk
