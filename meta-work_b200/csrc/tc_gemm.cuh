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

}  // namespace xjk
