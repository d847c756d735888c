// Test-only harness around the reference CPU path of xiaoju-pipe.
//
// This file is TEST INFRASTRUCTURE. It is compiled together with the reference's own, unmodified
// sources (core/gguf.c, core/xj_model.c, core/xj_cpu.c, core/xj_net.c, core/xj_spec.c, core/xj_tok.c)
// into oracle/_ref/libxjref.so by oracle/Makefile. Only tests/, __graft_entry__.smoke() and the
// cpu_baseline / --impl reference legs of bench.py load it, and only as the checker or as the timed
// CPU baseline; the CUDA product never links it.
//
// It exposes flat C entry points (plain pointers and ints) so Python can drive the reference through
// ctypes:
//   - the model loader           xj_model_load            (core/xj_model.c:204-210)
//   - the CPU stage vtable       xj_cpu_stage_new + forward/logits/rollback/reset (core/xj_cpu.c:375-418)
//   - row dequantisation         xj_dequant_row           (core/xj_quant.h:55-122)
//   - f16 conversions            xj_f16 / xj_to_f16       (core/xj_quant.h:9-43)
//   - embedding lookup           xj_embed                 (core/xj_cpu.c:369-373)
//   - the pipeline + speculative loop (core/xj_net.c:497-678, core/xj_spec.c:117-209)
// and a greedy decode loop that mirrors tools/xjpipe-run.c:24-60 (prefill in chunks of max_batch,
// then one token per step, argmax with the lowest index winning ties, core/xj_spec.c:12-16).
//
// Any xj_stage constructor with the reference signature can be plugged into the decode and
// speculative loops (xjr_*_with), which is how tests drive the CUDA stage through the reference's own
// pipeline code.
#include "xj_spec.h"
#include "xj_quant.h"

#include <stddef.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#ifdef _OPENMP
#include <omp.h>
#endif

typedef xj_stage *(*xjr_ctor)(const xj_model *m, int l0, int l1, int n_ctx, int max_batch, bool has_head,
                              char *err, size_t errlen);

static double now_s(void) { struct timespec t; clock_gettime(CLOCK_MONOTONIC, &t); return t.tv_sec + t.tv_nsec * 1e-9; }

// ---- ABI facts, so tests can check that include/xj_abi.h mirrors these structs byte for byte ----
int xjr_abi(int which) {
    switch (which) {
    case 0: return (int)sizeof(xj_w);
    case 1: return (int)sizeof(xj_layer);
    case 2: return (int)sizeof(xj_hparams);
    case 3: return (int)sizeof(xj_model);
    case 4: return (int)sizeof(xj_stage);
    case 5: return (int)offsetof(xj_model, layers);
    case 6: return (int)offsetof(xj_model, fingerprint);
    case 7: return (int)offsetof(xj_model, mtp_eh);
    case 8: return (int)offsetof(xj_stage, forward);
    case 9: return (int)offsetof(xj_stage, impl);
    case 10: return (int)offsetof(xj_stage, keep);
    case 11: return (int)offsetof(xj_layer, ssm_qkv);
    case 12: return (int)offsetof(xj_model, has_mtp);
    case 13: return (int)sizeof(gguf_file);
    case 14: return (int)offsetof(xj_stage, backend);
    default: return -1;
    }
}

int xjr_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void xjr_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

// ---- f16 / dequant ----
float xjr_f16(uint16_t h) { return xj_f16(h); }
uint16_t xjr_to_f16(float f) { return xj_to_f16(f); }
void xjr_dequant_row(uint32_t type, const void *src, float *y, int64_t n) { xj_dequant_row(type, src, y, n); }
uint64_t xjr_row_bytes(uint32_t type, int64_t n) { return xj_row_bytes(type, n); }

// ---- model ----
void *xjr_load(const char *path, char *err, int errlen) { return xj_model_load(path, err, (size_t)errlen); }
void xjr_model_free(void *m) { xj_model_free((xj_model *)m); }
const void *xjr_hparams(const void *m) { return &((const xj_model *)m)->hp; }
int xjr_n_vocab(const void *m) { return ((const xj_model *)m)->hp.n_vocab; }
int xjr_n_embd(const void *m) { return ((const xj_model *)m)->hp.n_embd; }
int xjr_n_layer(const void *m) { return ((const xj_model *)m)->hp.n_layer; }
int xjr_has_mtp(const void *m) { return ((const xj_model *)m)->has_mtp; }
uint64_t xjr_fingerprint(const void *m) { return ((const xj_model *)m)->fingerprint; }
void xjr_embed(const void *m, int32_t tok, float *out) { xj_embed((const xj_model *)m, tok, out); }
int xjr_attach_mtp(void *m, const char *path, char *err, int errlen) {
    return xj_model_attach_mtp((xj_model *)m, path, err, (size_t)errlen);
}

// ---- stages ----
void *xjr_stage_new_with(void *ctor, const void *m, int l0, int l1, int n_ctx, int max_batch, int has_head,
                         char *err, int errlen) {
    xjr_ctor f = ctor ? (xjr_ctor)ctor : xj_cpu_stage_new;
    return f((const xj_model *)m, l0, l1, n_ctx, max_batch, has_head != 0, err, (size_t)errlen);
}
void *xjr_stage_new(const void *m, int l0, int l1, int n_ctx, int max_batch, int has_head, char *err, int errlen) {
    return xjr_stage_new_with(NULL, m, l0, l1, n_ctx, max_batch, has_head, err, errlen);
}
int xjr_forward(void *s, float *x, int T, char *err, int errlen) {
    xj_stage *st = s; return st->forward(st, x, T, err, (size_t)errlen);
}
int xjr_logits(void *s, const float *x, int T, float *logits, char *err, int errlen) {
    xj_stage *st = s; return st->logits(st, x, T, logits, err, (size_t)errlen);
}
int xjr_rollback(void *s, int n_past, char *err, int errlen) {
    xj_stage *st = s; return st->rollback(st, n_past, err, (size_t)errlen);
}
void xjr_reset(void *s) { xj_stage *st = s; st->reset(st); }
void xjr_destroy(void *s) { xj_stage *st = s; if (st) st->destroy(st); }
void xjr_set_keep(void *s, int keep) { ((xj_stage *)s)->keep = keep; }
int xjr_n_past(const void *s) { return ((const xj_stage *)s)->n_past; }
int xjr_ck(const void *s, int which) { const xj_stage *st = s; return which ? st->ck_T : st->ck_start; }
const char *xjr_backend(const void *s) { return ((const xj_stage *)s)->backend; }
uint64_t xjr_state_bytes(const void *m, int l0, int l1, int n_ctx, int max_batch) {
    return xj_stage_state_bytes((const xj_model *)m, l0, l1, n_ctx, max_batch);
}

static int argmax(const float *x, int n) { int b = 0; for (int i = 1; i < n; i++) if (x[i] > x[b]) b = i; return b; }

// Top-2 margin of a logit row (for diagnosing greedy ties between backends).
static float margin(const float *x, int n) {
    int b = argmax(x, n);
    float second = -INFINITY;
    for (int i = 0; i < n; i++) if (i != b && x[i] > second) second = x[i];
    return x[b] - second;
}

// Greedy decode on one stage built by `ctor` (NULL = reference CPU stage): prefill `prompt` in chunks
// of max_batch, then n_gen steps of one token (xjpipe-run.c:24-60). Writes the generated ids to
// out_tok[n_gen], each step's top-2 margin to out_margin (may be NULL), the prefill's last-position
// logits to first_logits (may be NULL), and the prefill and decode wall times (seconds) to times[2].
int xjr_greedy_with(void *ctor, const void *mp, const int32_t *prompt, int n_prompt, int n_gen, int max_batch,
                    int n_ctx, int32_t *out_tok, float *out_margin, float *first_logits, double *times,
                    char *err, int errlen) {
    const xj_model *m = mp;
    const int E = m->hp.n_embd, V = m->hp.n_vocab, L = m->hp.n_layer;
    xjr_ctor f = ctor ? (xjr_ctor)ctor : xj_cpu_stage_new;
    xj_stage *s = f(m, 0, L, n_ctx, max_batch, true, err, (size_t)errlen);
    if (!s) return -1;
    float *x = malloc(sizeof(float) * (size_t)E * max_batch), *lg = malloc(sizeof(float) * V);
    int rc = -1;
    double t0 = now_s(), t1 = t0;
    for (int i = 0; i < n_prompt; i += max_batch) {
        int T = n_prompt - i < max_batch ? n_prompt - i : max_batch;
        for (int t = 0; t < T; t++) xj_embed(m, prompt[i + t], x + (size_t)t * E);
        if (s->forward(s, x, T, err, (size_t)errlen)) goto done;
        if (i + T == n_prompt && s->logits(s, x + (size_t)(T - 1) * E, 1, lg, err, (size_t)errlen)) goto done;
    }
    if (first_logits) memcpy(first_logits, lg, sizeof(float) * V);
    t1 = now_s();
    for (int g = 0; g < n_gen; g++) {
        int id = argmax(lg, V);
        out_tok[g] = id;
        if (out_margin) out_margin[g] = margin(lg, V);
        if (g + 1 == n_gen) break;
        xj_embed(m, id, x);
        if (s->forward(s, x, 1, err, (size_t)errlen)) goto done;
        if (s->logits(s, x, 1, lg, err, (size_t)errlen)) goto done;
    }
    rc = 0;
done:
    if (times) { times[0] = t1 - t0; times[1] = now_s() - t1; }
    free(x); free(lg);
    s->destroy(s);
    return rc;
}

int xjr_greedy(const void *m, const int32_t *prompt, int n_prompt, int n_gen, int max_batch, int n_ctx,
               int32_t *out_tok, float *out_margin, float *first_logits, double *times, char *err, int errlen) {
    return xjr_greedy_with(NULL, m, prompt, n_prompt, n_gen, max_batch, n_ctx, out_tok, out_margin, first_logits,
                           times, err, errlen);
}

// Per-layer activations: chain one-layer stages [l, l+1) and record x after every layer
// (hid[(L+1)][T][E]: row 0 is the embedding input). Feeds `steps` chunks of tokens (sizes in
// chunk[]), so multi-token prefill and single-token decode are both covered. `hid` receives the
// activations of the LAST chunk only; `logits` the logits of all T rows of the last chunk.
int xjr_layer_trace_with(void *ctor, const void *mp, const int32_t *tok, const int *chunk, int n_chunks,
                         int max_batch, int n_ctx, float *hid, float *logits, char *err, int errlen) {
    const xj_model *m = mp;
    const int E = m->hp.n_embd, L = m->hp.n_layer;
    xjr_ctor f = ctor ? (xjr_ctor)ctor : xj_cpu_stage_new;
    xj_stage **st = calloc((size_t)L, sizeof(xj_stage *));
    float *x = malloc(sizeof(float) * (size_t)E * max_batch);
    int rc = -1, pos = 0;
    for (int l = 0; l < L; l++) {
        st[l] = f(m, l, l + 1, n_ctx, max_batch, l == L - 1, err, (size_t)errlen);
        if (!st[l]) goto done;
    }
    for (int c = 0; c < n_chunks; c++) {
        const int T = chunk[c];
        const bool last = c + 1 == n_chunks;
        for (int t = 0; t < T; t++) xj_embed(m, tok[pos + t], x + (size_t)t * E);
        if (last) memcpy(hid, x, sizeof(float) * (size_t)T * E);
        for (int l = 0; l < L; l++) {
            if (st[l]->forward(st[l], x, T, err, (size_t)errlen)) goto done;
            if (last) memcpy(hid + (size_t)(l + 1) * T * E, x, sizeof(float) * (size_t)T * E);
        }
        if (last && st[L - 1]->logits(st[L - 1], x, T, logits, err, (size_t)errlen)) goto done;
        pos += T;
    }
    rc = 0;
done:
    for (int l = 0; l < L; l++) if (st[l]) st[l]->destroy(st[l]);
    free(st); free(x);
    return rc;
}

int xjr_layer_trace(const void *m, const int32_t *tok, const int *chunk, int n_chunks, int max_batch, int n_ctx,
                    float *hid, float *logits, char *err, int errlen) {
    return xjr_layer_trace_with(NULL, m, tok, chunk, n_chunks, max_batch, n_ctx, hid, logits, err, errlen);
}

// ---- pipeline + speculative decoding (reference loop, any stage backend) ----
static int greedy_cb(void *ctx, const float *x, int n) { (void)ctx; return argmax(x, n); }

// Runs the reference's xj_pipeline (local a = [0,s1), b = [s1,L) + head; s1 <= 0 means one stage) and,
// when k > 0 and the model has an MTP layer, its MTP speculative loop (xj_spec_next). Emits up to
// n_gen ids into out_tok; returns the count, or -1. stats[4] = steps, drafted, accepted, draft ms.
// `oracle` / `oracle_miss` plant known drafts as xjpipe-host --oracle does (xj_spec.c:230-234).
int xjr_spec_with(void *ctor, void *mp, const int32_t *prompt, int n_prompt, int n_gen, int max_batch, int n_ctx,
                  int s1, int k, const int32_t *oracle, int n_oracle, int oracle_miss, int32_t *out_tok,
                  double *stats, char *err, int errlen) {
    xj_model *m = mp;
    const int L = m->hp.n_layer;
    xjr_ctor f = ctor ? (xjr_ctor)ctor : xj_cpu_stage_new;
    xj_stage *a = NULL, *b = NULL, *mtp = NULL;
    int n_out = -1;
    if (s1 > 0 && s1 < L) {
        a = f(m, 0, s1, n_ctx, max_batch, false, err, (size_t)errlen);
        b = a ? f(m, s1, L, n_ctx, max_batch, true, err, (size_t)errlen) : NULL;
        if (!a || !b) goto done0;
    } else {
        a = f(m, 0, L, n_ctx, max_batch, true, err, (size_t)errlen);
        if (!a) goto done0;
    }
    if (k > 0 && m->has_mtp) {
        mtp = f(m, L, L + 1, n_ctx, max_batch, true, err, (size_t)errlen);
        if (!mtp) goto done0;
    }
    xj_pipeline p;
    xj_pipeline_init(&p, m, a, NULL, b);
    xj_spec sp;
    if (xj_spec_init(&sp, &p, mtp, k)) { snprintf(err, (size_t)errlen, "spec init failed"); goto done1; }
    sp.oracle = oracle; sp.n_oracle = n_oracle; sp.oracle_miss = oracle_miss;
    if (xj_spec_feed(&sp, prompt, n_prompt, err, (size_t)errlen)) goto done2;
    int n = 0;
    while (n < n_gen) {
        int32_t buf[XJ_SPEC_MAXK + 1];
        int room = n_gen - n;
        int got = xj_spec_next(&sp, greedy_cb, NULL, buf, room, err, (size_t)errlen);
        if (got < 0) goto done2;
        for (int i = 0; i < got && n < n_gen; i++) out_tok[n++] = buf[i];
        if (got > 0 && ((uint32_t)buf[got - 1] == m->hp.eos || (uint32_t)buf[got - 1] == m->hp.eot)) break;
    }
    n_out = n;
    if (stats) { stats[0] = (double)sp.n_steps; stats[1] = (double)sp.n_drafted; stats[2] = (double)sp.n_accepted; stats[3] = sp.t_draft_ms; }
done2:
    xj_spec_free(&sp);
done1:
    xj_pipeline_free(&p);
done0:
    if (mtp) mtp->destroy(mtp);
    if (b) b->destroy(b);
    if (a) a->destroy(a);
    return n_out;
}

int xjr_eos(const void *m, int which) { const xj_model *mm = m; return (int)(which ? mm->hp.eot : mm->hp.eos); }
