// B200 (sm_100a) CUDA backend for the xiaoju-pipe decode loop: public C ABI of libxj_cuda.so.
//
// Drop-in entry points (same signature and semantics as the runtime's other backends):
//
//   xj_cuda_stage_new      replaces xj_metal_stage_new / xj_cpu_stage_new
//                          (src/xiaoju-pipe/core/xj_stage.h:42-47; Metal: metal/xj_metal.m:554-664,
//                          CPU: core/xj_cpu.c:375-418). Returns an xj_stage whose function pointers
//                          (forward, logits, rollback, reset, destroy) follow core/xj_stage.h:28-37.
//   xj_cuda_device_name    replaces xj_metal_device_name (core/xj_stage.h:48).
//   xjc_model_load / xjc_model_free / xjc_embed / xjc_stage_state_bytes
//                          a loader and helpers with the semantics of xj_model_load
//                          (core/xj_model.c:204-210), xj_model_free (:289-294), xj_embed
//                          (core/xj_cpu.c:369-373) and xj_stage_state_bytes (core/xj_cpu.c:356-367),
//                          for hosts that do not link the runtime's own core/. Models from either
//                          loader are accepted by xj_cuda_stage_new (same struct layout, xj_abi.h).
//
// Additive extensions (no counterpart in the reference; the vtable is unchanged):
//
//   xj_cuda_decode         device-resident greedy decode on a full-model stage: token ids in, token
//                          ids out; embedding lookup, all layers, the LM head and the argmax run on
//                          the GPU and one decode step is replayed as a CUDA graph.
//   xj_cuda_set_options    backend switches (KV-cache precision, GEMV path) for tests.
//
// Error convention (as the runtime's): functions return 0 (or a pointer) on success and -1 (or
// NULL) on failure with a NUL-terminated message in err[errlen]. A stage is single-threaded; it runs
// on the CUDA device that was current when it was created.
#pragma once
#include "xj_abi.h"

#ifdef __cplusplus
extern "C" {
#endif

xj_stage *xj_cuda_stage_new(const xj_model *m, int l0, int l1, int n_ctx, int max_batch, bool has_head,
                            char *err, size_t errlen);
const char *xj_cuda_device_name(void);

xj_model *xjc_model_load(const char *path, char *err, size_t errlen);
void xjc_model_free(xj_model *m);
void xjc_embed(const xj_model *m, int32_t token, float *out);
uint64_t xjc_stage_state_bytes(const xj_model *m, int l0, int l1, int n_ctx, int max_batch);

// Options (process-wide, read when a stage is created):
//   XJC_OPT_KV_F32   1 = float32 KV cache (matches the CPU oracle's cache), 0 = float16 (default,
//                    the Metal backend's precision).
//   XJC_OPT_GEMV     0 = fastest path per type (default), 1 = generic per-element path for every type.
//   XJC_OPT_PDL      1 = kernels of a step overlap through programmatic dependent launch (default),
//                    0 = each kernel starts after its predecessor completes.
//   XJC_OPT_PERSIST  1 = xj_cuda_decode runs all decode steps after the prompt in one persistent
//                    cooperative kernel when every matrix of the stage is in the tensor-core layout
//                    (default), 0 = one CUDA-graph replay of the per-phase kernels per step.
//   XJC_OPT_TRACE    1 = the persistent kernel records when each CTA starts and ends each phase of
//                    its last step (read with xj_cuda_phase_trace), 0 = off (default).
//   XJC_OPT_GEMV_CTAS  CTAs per SM of the standalone tensor-core GEMV kernel: 2 (default) or 1.
//   XJC_OPT_TC       1 = matrix products of 17..64 tokens (batched decode, prompt chunks) on the tcgen05
//                    tensor cores (default), 0 = on the mma.sync 64-token kernel.
enum { XJC_OPT_KV_F32 = 1, XJC_OPT_GEMV = 2, XJC_OPT_PDL = 3, XJC_OPT_PERSIST = 4, XJC_OPT_TRACE = 5,
       XJC_OPT_GEMV_CTAS = 6, XJC_OPT_TC = 7 };
int xj_cuda_set_options(int which, int value);

// Greedy decode on a stage covering [0, n_layer) with the head. Feeds n_prompt ids (prefill in
// chunks of max_batch, continuing from the stage's n_past), then emits n_gen ids into out (out[0] is
// the argmax after the prompt). Each emitted id except the last is fed back, so the stage's n_past
// grows by n_prompt + n_gen - 1. margins (may be NULL) receives each step's top-2 logit gap.
// gpu_ms (may be NULL) receives [prefill ms, decode ms] measured with CUDA events on the stage stream;
// with the persistent decode kernel the prompt's last token is the kernel's first step (decode ms).
int xj_cuda_decode(xj_stage *s, const int32_t *prompt, int n_prompt, int n_gen, int32_t *out, float *margins,
                   float *gpu_ms, char *err, size_t errlen);

// Matrix-vector product on host buffers with the decode kernels: y[t][n] = W[n] . x[t] for t < T
// (1 <= T <= 64; more than 16 tokens take the 64-token kernel of batched decode), W an [n][k] matrix
// in GGUF block layout of `type`. path 0 = fastest available kernel, 1 = generic per-element kernel.
// For parity tests of the kernels that dominate decode.
int xj_cuda_gemv(int type, const void *w, int k, int n, const float *x, int T, float *y, int path, char *err,
                 size_t errlen);
// Average device time (ms) of one such launch over `iters` launches that rotate through `copies`
// distinct device copies of W, so the last-level cache cannot serve the weights (GEMV microbenchmark).
int xj_cuda_gemv_time(int type, const void *w, int k, int n, int T, int copies, int iters, int path, float *ms,
                      char *err, size_t errlen);
// Greedy speculative decoding with a separate draft model (e.g. a small Q8_0 drafter for a Q4_K_M target): both stages take the
// prompt, then each round the draft proposes k tokens (device greedy decode), the target verifies the
// last emitted token and the k drafts in one forward (k + 1 rows of logits, device greedy picks), the
// longest agreeing prefix plus the target's own next pick are emitted, the target rolls back through its
// checkpoints and the draft's recurrent state is restored and re-fed. out[0..n_gen) equals plain greedy
// decoding of the target. stats (may be NULL): target verify forwards, drafted tokens, accepted drafted
// tokens, draft re-feeds. Both stages span all layers with the head, share the vocabulary, and take
// k + 1 tokens per forward.
int xj_cuda_spec_decode(xj_stage *target, xj_stage *draft, const int32_t *prompt, int n_prompt, int n_gen, int k,
                        int32_t *out, long long *stats, char *err, size_t errlen);

// Gated DeltaNet decode microbenchmark (e.g. 16 heads x 128 x 128 state): average device time (ms) of one decode step
// of B sequences x Hv heads with an S x S fp32 state each (S in 16, 32, 64, 128), the batch kernel of
// batched decode, states rotated over >= 256 MiB of copies so the last-level cache cannot serve them.
int xj_cuda_gdn_time(int S, int Hv, int B, int iters, float *ms, char *err, size_t errlen);
// Gated DeltaNet over a prompt of T tokens (prefill): the chunked kernels that prompt
// forwards of 32 or more tokens use, against the token-by-token kernel on the same synthetic operands.
// res[4] = max relative difference of the outputs, of the final state, chunked ms, token-by-token ms.
int xj_cuda_gdn_prefill_check(int S, int Hk, int Hv, int T, float *res, char *err, size_t errlen);

// Gated DeltaNet recurrence on caller operands (host buffers), for parity against a host restatement of
// core/xj_cpu.c:194-219 (the loop inside attn_linear, after the projections and the convolution).
// path 0 = token-by-token kernel over T tokens of one sequence, 1 = chunked prefill kernels (S >= 32),
// 2 = batch decode kernel, T independent sequences of one token each. qkv [T][2*Hk*S + Hv*S] (q, k, v
// after convolution + SiLU), z [T][Hv*S] raw gate, beta / alpha [T][Hv] logits, dt / A [Hv], norm_w [S];
// state [Hv][S][S] (path 2: [T][Hv][S][S]) in and out, out [T][Hv*S] after the gated RMSNorm.
int xj_cuda_gdn_run(int path, int S, int Hk, int Hv, int T, const float *qkv, const float *z, const float *beta,
                    const float *alpha, const float *dt, const float *A, const float *norm_w, float eps, float *state,
                    float *out, char *err, size_t errlen);

// Sampling instead of the greedy pick for later xj_cuda_decode calls on this stage: the session
// layer's sampler (ios/App/XJGlue.c:251-282: top-k 40, top-p 0.95, temperature) on the device, with a
// reproducible draw. temperature <= 0 restores greedy decoding. 1 <= top_k <= 64, 0 < top_p <= 1. The
// draw for each token is uniform(seed, stage position of its logits) (SplitMix64, 30 bits), so a seed
// fixes the sampled sequence however the decode calls are split. Sampled decode runs the per-phase
// decode step (a CUDA graph), not the persistent kernel, and reports each step's top-2 logit gap.
int xj_cuda_set_sampler(xj_stage *s, float temperature, int top_k, double top_p, unsigned long long seed, char *err,
                        size_t errlen);
// The same pick on host logit rows (parity tests): out[r] = the id drawn from logits[r][0..n_vocab) with
// uniform(seed, counter0 + r); margins (may be NULL) = each row's top-2 logit gap. temperature <= 0 (or
// top_k = 1) = greedy, lowest id on ties.
int xj_cuda_sample_logits(const float *logits, int rows, int n_vocab, float temperature, int top_k, double top_p,
                          unsigned long long seed, unsigned long long counter0, int32_t *out, float *margins, char *err,
                          size_t errlen);

// Number of kernel launches in one replay of the stage's cached decode-step graph (0 before the first
// xj_cuda_decode call that generated more than one token).
int xj_cuda_graph_kernels(const xj_stage *s);

// Kernel launches made by the last xj_cuda_decode call: launches[0] for the prompt (prefill chunks and
// the first pick), launches[1] for the decode steps after it (one per 8192 steps when the persistent
// kernel ran them, else steps x xj_cuda_graph_kernels). Returns launches[0] + launches[1].
long long xj_cuda_last_decode_launches(const xj_stage *s, long long *launches);

// Phase timing of the persistent kernel's last traced step (XJC_OPT_TRACE): for each phase p < cap,
// out[13p..13p+12] = {kind (0 matrix-vector, 1 Gated DeltaNet, 2 attention, 3 token pick), longest CTA
// time in the phase (us), mean CTA time (us), first start to last end over CTAs (us), first start
// (us, device clock), mean time a CTA's consumers waited for weight chunks (us), mean lead of the
// first chunk request before the phase started (us), mean prologue time (us), mean time of the first
// tile after the prologue (us), and of that first tile (warp 0): chunk wait, tensor-core work, tile
// barrier, epilogue (us)}. Returns the number of phases, or -1.
int xj_cuda_phase_trace(const xj_stage *s, double *out, int cap);

// Dequantise n_rows rows of k elements of GGUF type `type` (host bytes in, host fp32 out) with the
// device decoder the GEMV kernels use; for checking bit-exactness against xj_dequant_row
// (core/xj_quant.h:55-122). Runs on the current device.
int xj_cuda_dequant_rows(int type, const void *src, int k, int n_rows, float *out, char *err, size_t errlen);

/* Tensor-core (tcgen05) self-test: d[128][64] = a[128][k] . b[64][k]^T with a, b fp16 (bit patterns) in
 * host memory, k a positive multiple of 64, f32 accumulation in tensor memory. Checks the shared-memory
 * descriptors, the MMA and the tensor-memory read-back used by the batched kernels. 0 or -1 + message. */
int xj_cuda_tc_selftest(const uint16_t *a, const uint16_t *b, int k, float *d, char *err, size_t errlen);

// Batch of n_seq independent sequences decoded in lockstep (no counterpart in the reference, which has
// no multi-sequence API; additive). The batch owns a stage over all layers with the head (weights,
// n_seq-row activation buffers) plus each sequence's KV caches, Gated-DeltaNet/conv states and
// position; the current device at creation is the batch's device.
typedef struct xj_cuda_batch xj_cuda_batch;
xj_cuda_batch *xj_cuda_batch_new(const xj_model *m, int n_seq, int n_ctx, char *err, size_t errlen);
void xj_cuda_batch_free(xj_cuda_batch *b);
// Forget every sequence (positions 0, states zero).
int xj_cuda_batch_reset(xj_cuda_batch *b, char *err, size_t errlen);
// Common position of the sequences (they advance in lockstep).
int xj_cuda_batch_n_past(const xj_cuda_batch *b);
// Greedy decode of every sequence: feeds prompts[b][0..n_prompt) (one token of each sequence per step,
// continuing from n_past), then emits n_gen ids per sequence into out[b][0..n_gen) (out[b][0] is the
// argmax after the prompt; every id but the last is fed back); margins[b][..] (may be NULL) receives
// the top-2 logit gaps, gpu_ms (may be NULL) [prompt ms, decode ms]. Sequence b's ids are the ones
// xj_cuda_decode gives for that sequence alone.
int xj_cuda_batch_decode(xj_cuda_batch *b, const int32_t *prompts, int n_prompt, int n_gen, int32_t *out, float *margins,
                         float *gpu_ms, char *err, size_t errlen);
// Kernel launches of the last xj_cuda_batch_decode: launches[0] for the prompt steps, launches[1] for
// the decode steps after them. Returns their sum.
long long xj_cuda_batch_last_launches(const xj_cuda_batch *b, long long *launches);

// A batch that also takes up to max_tokens (1..16) tokens of every sequence in one forward: prompts of
// batches wider than 16 sequences go through in chunks of max_tokens, and the batch can be the target of
// xj_cuda_batch_spec_decode (max_tokens >= k + 1). n_seq * max_tokens <= 4096.
xj_cuda_batch *xj_cuda_batch_new_multi(const xj_model *m, int n_seq, int n_ctx, int max_tokens, char *err, size_t errlen);
// Greedy speculative decoding of every sequence of a batch with a draft batch (core/xj_spec.c:131-209,
// for all sequences at once): both take the prompts [n_seq][n_prompt]; each round the draft proposes k
// tokens per sequence, the target verifies [last, k drafts] of all sequences in one (k+1)-token forward
// (its matrix products on the tensor cores), each sequence keeps its agreeing prefix plus the target's
// own next pick, and both batches roll each sequence back to what it keeps. out [n_seq][n_gen] equals
// plain greedy decoding of the target. stats[4] (may be NULL): verify rounds, drafted tokens, accepted
// drafted tokens, target token-rows processed. gpu_ms (may be NULL): device time of the call. Both
// batches hold the same number of sequences at the same position on one device; the contexts need
// n_past + n_prompt + n_gen * (k + 1) + k + 1 positions (a sequence can run ahead of the slowest).
int xj_cuda_batch_spec_decode(xj_cuda_batch *target, xj_cuda_batch *draft, const int32_t *prompts, int n_prompt, int n_gen,
                              int k, int32_t *out, long long *stats, float *gpu_ms, char *err, size_t errlen);

// Pipeline stages (layer pipeline across GPUs: each GPU holds a batch over its layer range [l0, l1),
// the last one with the head). Device buffers belong to the batch's device; calls return after the work
// is done. Rows [row0, row0+nrows) of the batch form a micro-batch; x_dev holds its nrows rows of
// [n_embd] fp32 activations.
xj_cuda_batch *xj_cuda_batch_new_range(const xj_model *m, int l0, int l1, bool has_head, int n_seq, int n_ctx, char *err,
                                       size_t errlen);
// x_dev[i] = embedding row of tok_dev[i] (batches whose range starts at layer 0).
int xj_cuda_batch_embed_rows(xj_cuda_batch *b, const int32_t *tok_dev, float *x_dev, int nrows, char *err, size_t errlen);
// The batch's layers on the micro-batch in place; each of its sequences advances one position.
int xj_cuda_batch_forward_rows(xj_cuda_batch *b, float *x_dev, int row0, int nrows, char *err, size_t errlen);
// Output norm, LM head and greedy pick of the micro-batch: tok_dev[i] = next id of sequence row0+i.
int xj_cuda_batch_pick_rows(xj_cuda_batch *b, const float *x_dev, int row0, int nrows, int32_t *tok_dev, char *err,
                            size_t errlen);
// The CUDA stream (cudaStream_t) the batch's kernels run on, so that a caller's transfers (e.g. NCCL
// send/recv of the activations) can be ordered with them on the device.
void *xj_cuda_batch_stream(xj_cuda_batch *b);
// on != 0: the *_rows calls return as soon as their kernels are queued (launch errors are still
// reported); xj_cuda_batch_sync waits for the stream and reports errors of queued work.
int xj_cuda_batch_set_async(xj_cuda_batch *b, int on);
int xj_cuda_batch_sync(xj_cuda_batch *b, char *err, size_t errlen);

// Layer pipeline across GPUs over NCCL (no counterpart in the reference's API: it re-expresses the
// runtime's stage split, core/xj_net.h:93-111, driven by xj_pipeline_eval, core/xj_net.c:527-605, as
// one process per GPU with activations and ids sent by NCCL instead of TCP). Each rank holds a batch of
// n_seq sequences over an even share of the layers (first rank: embedding; last rank: LM head and
// greedy pick); a decode step is one token of every sequence, split into n_micro micro-batches of rows
// so that the stages overlap. NCCL is loaded at run time (libnccl.so.2).
typedef struct xj_cuda_pipeline xj_cuda_pipeline;
// Bytes of the identifier that rank 0 creates and every rank passes to xj_cuda_pipeline_new (three
// NCCL unique ids: the two link-parity communicators and the token-id communicator).
#define XJC_PIPELINE_ID_BYTES 384
int xj_cuda_pipeline_id_new(unsigned char *id, char *err, size_t errlen);
// Collective over the world's ranks (each on its own current device); id may be NULL when world == 1.
xj_cuda_pipeline *xj_cuda_pipeline_new(const xj_model *m, int rank, int world, const unsigned char *id, int n_seq, int n_ctx,
                                       int n_micro, char *err, size_t errlen);
void xj_cuda_pipeline_free(xj_cuda_pipeline *p);
// The rank's batch (its layer range, KV caches and states).
xj_cuda_batch *xj_cuda_pipeline_batch(xj_cuda_pipeline *p);
// Greedy decode, collective: rank 0 passes prompts [n_seq][n_prompt] and receives out [n_seq][n_gen]
// (other ranks pass NULL for both); the prompt goes through in n_prompt lockstep steps, the last of which
// picks out[:, 0]; every generated id but the last is fed back; positions continue across calls.
// gpu_ms (may be NULL): device time of the call on this rank (CUDA events on its compute stream).
int xj_cuda_pipeline_decode(xj_cuda_pipeline *p, const int32_t *prompts, int n_prompt, int n_gen, int32_t *out, float *gpu_ms,
                            char *err, size_t errlen);

// Capacity, in floats, of the fixed device scratch used by xj_cuda_norm_gemv_noalloc (256 KiB).
#define XJC_NOALLOC_MAX_FLOATS 65536

// No counterpart in the reference. y[t] = W . (rmsnorm(x[t]) * norm_w) for t < T without allocating
// anything, for callers that cannot call cudaMalloc where they need it (a process whose device memory
// is a fixed pool owned by another component, or a thread on which allocation is not allowed). Every
// pointer is a DEVICE pointer on the current device: w_dev = n rows of k elements in GGUF block layout
// of `type` (F32/F16/BF16/Q8_0/Q4_K/Q5_K/Q6_K), x_dev [T][k], norm_w_dev [k] fp32, y_dev [T][n].
// 1 <= T <= 16 and T*k <= XJC_NOALLOC_MAX_FLOATS, else -1 with a message. The normalised rows live
// in a fixed device array shared by all calls on a device: calls that overlap on the GPU race. The
// first call on a device sets up that array's address; make it before any stream capture. Runs on
// the legacy default stream and returns after the GPU has finished.
int xj_cuda_norm_gemv_noalloc(int type, const void *w_dev, int k, int n, const float *x_dev, const float *norm_w_dev,
                              float eps, int T, float *y_dev, char *err, size_t errlen);

#ifdef __cplusplus
}
#endif
