// Layer pipeline across GPUs for batched greedy decode, over NCCL: the runtime's stage split
// (core/xj_net.h:93-111, a | r | b over TCP, driven by xj_pipeline_eval, core/xj_net.c:527-605) as one
// process per GPU with activations and token ids sent between GPUs by NCCL (NVLink).
//
// Rank r holds a batch of n_seq sequences over its layer range (xj_cuda_batch_new_range), the first
// rank also embeds, the last also runs the LM head and the greedy pick. A decode step is one token of
// every sequence; its rows are split into micro-batches so that the stages work at the same time:
//
//   rank 0:     ids -> embed -> layers -> send x  -------------\      (activations, [rows][n_embd] fp32)
//   rank r:     recv x -> layers -> send x                      |
//   rank N-1:   recv x -> layers -> head + pick -> send ids ----/-> rank 0 feeds them to the next step
//
// Each rank issues everything asynchronously on four CUDA streams: the batch's compute stream, one for
// receiving activations, one for sending them, one for token ids; events order each transfer with the
// kernels that produce or consume its buffer (and a buffer's next write with its previous send). The
// link r -> r+1 uses communicator (r & 1), the ids the third one, so every rank uses each communicator
// on one stream only, and a stream never holds a receive behind a send whose peer waits for it. Token
// ids go to per-(step, row) slots on the device, so no id buffer is reused. NCCL is loaded at run time
// (libnccl.so.2), so single-GPU users of the library need none.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <type_traits>
#include <vector>

#include "../../include/xj_cuda.h"

namespace {

void seterr(char *err, size_t errlen, const char *fmt, ...) {
    if (!err || !errlen) return;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(err, errlen, fmt, ap);
    va_end(ap);
}

// The NCCL entry points used here, resolved from libnccl.so.2 on first use.
struct Nccl {
    bool tried = false, ok = false;
    ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*Send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*Recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    const char *(*GetErrorString)(ncclResult_t) = nullptr;
};
Nccl g_nccl;

bool nccl_load(char *err, size_t errlen) {
    if (g_nccl.tried) {
        if (!g_nccl.ok) seterr(err, errlen, "NCCL (libnccl.so.2) is not available");
        return g_nccl.ok;
    }
    g_nccl.tried = true;
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) { seterr(err, errlen, "cannot load libnccl.so.2: %s", dlerror()); return false; }
    bool ok = true;
    auto sym = [&](auto &fn, const char *name) {
        fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
        ok = ok && fn != nullptr;
    };
    sym(g_nccl.GetUniqueId, "ncclGetUniqueId");
    sym(g_nccl.CommInitRank, "ncclCommInitRank");
    sym(g_nccl.CommDestroy, "ncclCommDestroy");
    sym(g_nccl.Send, "ncclSend");
    sym(g_nccl.Recv, "ncclRecv");
    sym(g_nccl.GetErrorString, "ncclGetErrorString");
    if (!ok) { seterr(err, errlen, "libnccl.so.2 lacks an expected symbol"); return false; }
    g_nccl.ok = true;
    return true;
}

constexpr int N_COMMS = 3;   // link parity 0, link parity 1, token ids
static_assert(N_COMMS * sizeof(ncclUniqueId) == XJC_PIPELINE_ID_BYTES, "identifier size");

}  // namespace

struct xj_cuda_pipeline {
    int rank = 0, world = 1, n_seq = 0, n_mb = 1, dev = 0, E = 0;
    xj_cuda_batch *batch = nullptr;
    cudaStream_t cs = nullptr;                     // the batch's compute stream (owned by the batch)
    cudaStream_t s_in = nullptr, s_out = nullptr, s_ids = nullptr;
    ncclComm_t comm[N_COMMS] = {};
    std::vector<int> mb_row0, mb_rows;
    std::vector<float *> x;                        // per micro-batch activations [rows][E]
    std::vector<cudaEvent_t> ev_fwd, ev_sent, ev_recv, ev_pick, ev_ids;
    cudaEvent_t ev_t0 = nullptr, ev_t1 = nullptr;
    int32_t *ids = nullptr;                        // [slots][n_seq] token ids (prompt columns, then picks)
    int id_slots = 0;
};

namespace {

#define PCK(call)                                                                                          \
    do {                                                                                                  \
        cudaError_t e_ = (call);                                                                          \
        if (e_ != cudaSuccess) {                                                                          \
            seterr(err, errlen, "CUDA error %s at %s:%d", cudaGetErrorString(e_), __FILE__, __LINE__);    \
            return -1;                                                                                    \
        }                                                                                                 \
    } while (0)
#define NCK(call)                                                                                          \
    do {                                                                                                  \
        ncclResult_t r_ = (call);                                                                         \
        if (r_ != ncclSuccess) {                                                                          \
            seterr(err, errlen, "NCCL error %s at %s:%d", g_nccl.GetErrorString(r_), __FILE__, __LINE__); \
            return -1;                                                                                    \
        }                                                                                                 \
    } while (0)

void pipeline_release(xj_cuda_pipeline *p) {
    if (!p) return;
    cudaSetDevice(p->dev);
    for (cudaStream_t s : {p->s_in, p->s_out, p->s_ids}) if (s) cudaStreamSynchronize(s);
    if (p->cs) cudaStreamSynchronize(p->cs);
    for (auto &c : p->comm) if (c && g_nccl.ok) g_nccl.CommDestroy(c);
    for (float *b : p->x) cudaFree(b);
    if (p->ids) cudaFree(p->ids);
    for (auto *v : {&p->ev_fwd, &p->ev_sent, &p->ev_recv, &p->ev_pick, &p->ev_ids})
        for (cudaEvent_t e : *v) cudaEventDestroy(e);
    if (p->ev_t0) cudaEventDestroy(p->ev_t0);
    if (p->ev_t1) cudaEventDestroy(p->ev_t1);
    for (cudaStream_t s : {p->s_in, p->s_out, p->s_ids}) if (s) cudaStreamDestroy(s);
    if (p->batch) xj_cuda_batch_free(p->batch);
    delete p;
}

// Contiguous layer ranges, as even as possible, the first ranges one longer when uneven.
void split_range(int n_layer, int world, int rank, int *l0, int *l1) {
    const int base = n_layer / world, extra = n_layer % world;
    int a = 0;
    for (int r = 0; r < rank; r++) a += base + (r < extra ? 1 : 0);
    *l0 = a;
    *l1 = a + base + (rank < extra ? 1 : 0);
}

int ensure_id_slots(xj_cuda_pipeline *p, int slots, char *err, size_t errlen) {
    if (slots <= p->id_slots) return 0;
    PCK(cudaStreamSynchronize(p->cs));
    if (p->ids) PCK(cudaFree(p->ids));
    p->ids = nullptr;
    PCK(cudaMalloc(&p->ids, sizeof(int32_t) * (size_t)slots * p->n_seq));
    p->id_slots = slots;
    return 0;
}

}  // namespace

extern "C" {

int xj_cuda_pipeline_id_new(unsigned char *id, char *err, size_t errlen) {
    if (!id) { seterr(err, errlen, "null id buffer"); return -1; }
    if (!nccl_load(err, errlen)) return -1;
    for (int c = 0; c < N_COMMS; c++) {
        ncclUniqueId u;
        NCK(g_nccl.GetUniqueId(&u));
        memcpy(id + (size_t)c * sizeof(ncclUniqueId), &u, sizeof(ncclUniqueId));
    }
    return 0;
}

xj_cuda_pipeline *xj_cuda_pipeline_new(const xj_model *m, int rank, int world, const unsigned char *id, int n_seq, int n_ctx,
                                       int n_micro, char *err, size_t errlen) {
    if (!m || world < 1 || rank < 0 || rank >= world || n_seq < 1 || n_micro < 1 || (world > 1 && !id)) {
        seterr(err, errlen, "bad pipeline arguments");
        return nullptr;
    }
    if (world > m->hp.n_layer) { seterr(err, errlen, "more ranks (%d) than layers (%d)", world, m->hp.n_layer); return nullptr; }
    if (world > 1 && !nccl_load(err, errlen)) return nullptr;
    auto *p = new xj_cuda_pipeline();
    p->rank = rank; p->world = world; p->n_seq = n_seq; p->E = m->hp.n_embd;
    cudaGetDevice(&p->dev);
    p->n_mb = n_micro < n_seq ? n_micro : n_seq;
    for (int k = 0, r0 = 0; k < p->n_mb; k++) {
        const int n = n_seq / p->n_mb + (k < n_seq % p->n_mb ? 1 : 0);
        p->mb_row0.push_back(r0);
        p->mb_rows.push_back(n);
        r0 += n;
    }
    int l0, l1;
    split_range(m->hp.n_layer, world, rank, &l0, &l1);
    p->batch = xj_cuda_batch_new_range(m, l0, l1, rank == world - 1, n_seq, n_ctx, err, errlen);
    if (!p->batch) { pipeline_release(p); return nullptr; }
    xj_cuda_batch_set_async(p->batch, 1);
    p->cs = (cudaStream_t)xj_cuda_batch_stream(p->batch);
    bool ok = cudaStreamCreateWithFlags(&p->s_in, cudaStreamNonBlocking) == cudaSuccess &&
              cudaStreamCreateWithFlags(&p->s_out, cudaStreamNonBlocking) == cudaSuccess &&
              cudaStreamCreateWithFlags(&p->s_ids, cudaStreamNonBlocking) == cudaSuccess &&
              cudaEventCreate(&p->ev_t0) == cudaSuccess && cudaEventCreate(&p->ev_t1) == cudaSuccess;
    for (int k = 0; ok && k < p->n_mb; k++) {
        float *b = nullptr;
        ok = cudaMalloc(&b, sizeof(float) * (size_t)p->mb_rows[k] * p->E) == cudaSuccess;
        if (ok) p->x.push_back(b);
        for (auto *v : {&p->ev_fwd, &p->ev_sent, &p->ev_recv, &p->ev_pick, &p->ev_ids}) {
            cudaEvent_t e = nullptr;
            ok = ok && cudaEventCreateWithFlags(&e, cudaEventDisableTiming) == cudaSuccess;
            if (e) v->push_back(e);
        }
    }
    if (!ok) {
        seterr(err, errlen, "pipeline buffers: %s", cudaGetErrorString(cudaGetLastError()));
        pipeline_release(p);
        return nullptr;
    }
    if (world > 1) {
        // every rank creates the three communicators in the same order
        for (int c = 0; c < N_COMMS; c++) {
            ncclUniqueId u;
            memcpy(&u, id + (size_t)c * sizeof(ncclUniqueId), sizeof(ncclUniqueId));
            const ncclResult_t r = g_nccl.CommInitRank(&p->comm[c], world, u, rank);
            if (r != ncclSuccess) {
                seterr(err, errlen, "ncclCommInitRank: %s", g_nccl.GetErrorString(r));
                pipeline_release(p);
                return nullptr;
            }
        }
    }
    return p;
}

void xj_cuda_pipeline_free(xj_cuda_pipeline *p) { pipeline_release(p); }

xj_cuda_batch *xj_cuda_pipeline_batch(xj_cuda_pipeline *p) { return p ? p->batch : nullptr; }

int xj_cuda_pipeline_decode(xj_cuda_pipeline *p, const int32_t *prompts, int n_prompt, int n_gen, int32_t *out, float *gpu_ms,
                            char *err, size_t errlen) {
    if (!p || n_prompt < 1 || n_gen < 1 || (p->rank == 0 && (!prompts || !out))) {
        seterr(err, errlen, "bad decode arguments");
        return -1;
    }
    cudaSetDevice(p->dev);
    const int R = p->rank, W = p->world, N = p->n_seq, P = n_prompt, steps = n_prompt + n_gen - 1;
    const bool first = R == 0, last = R == W - 1;
    // id slots: P prompt columns, then one per generated token (the pick of step i is slot i + 1)
    if (ensure_id_slots(p, P + n_gen, err, errlen)) return -1;
    int32_t *slot = p->ids;
    auto col = [&](int s) { return slot + (size_t)s * N; };
    PCK(cudaEventRecord(p->ev_t0, p->cs));
    if (first) {
        // prompts [n_seq][P] on the host -> columns [P][n_seq] on the device
        std::vector<int32_t> t((size_t)P * N);
        for (int b = 0; b < N; b++)
            for (int i = 0; i < P; i++) t[(size_t)i * N + b] = prompts[(size_t)b * P + i];
        PCK(cudaMemcpyAsync(slot, t.data(), t.size() * sizeof(int32_t), cudaMemcpyHostToDevice, p->cs));
        PCK(cudaStreamSynchronize(p->cs));   // t lives on this host stack frame
    }
    const ncclComm_t c_prev = R > 0 ? p->comm[(R - 1) & 1] : nullptr, c_next = R < W - 1 ? p->comm[R & 1] : nullptr;
    const ncclComm_t c_ids = p->comm[2];
    for (int i = 0; i < steps; i++) {
        const bool pick = i >= P - 1;
        for (int k = 0; k < p->n_mb; k++) {
            const int r0 = p->mb_row0[k], n = p->mb_rows[k];
            float *x = p->x[k];
            const size_t xn = (size_t)n * p->E;
            if (first) {
                // step i feeds column i: a prompt column, or the pick of step i - 1 (slot i)
                if (i >= P && W > 1) {
                    NCK(g_nccl.Recv(col(i) + r0, (size_t)n, ncclInt32, W - 1, c_ids, p->s_ids));
                    PCK(cudaEventRecord(p->ev_ids[k], p->s_ids));
                    PCK(cudaStreamWaitEvent(p->cs, p->ev_ids[k], 0));
                }
                PCK(cudaStreamWaitEvent(p->cs, p->ev_sent[k], 0));    // x's previous send has left
                if (xj_cuda_batch_embed_rows(p->batch, col(i) + r0, x, n, err, errlen)) return -1;
            } else {
                // x's previous contents are consumed (sent on, or read by the head)
                PCK(cudaStreamWaitEvent(p->s_in, last ? p->ev_pick[k] : p->ev_sent[k], 0));
                NCK(g_nccl.Recv(x, xn, ncclFloat32, R - 1, c_prev, p->s_in));
                PCK(cudaEventRecord(p->ev_recv[k], p->s_in));
                PCK(cudaStreamWaitEvent(p->cs, p->ev_recv[k], 0));
            }
            if (xj_cuda_batch_forward_rows(p->batch, x, r0, n, err, errlen)) return -1;
            if (!last) {
                PCK(cudaEventRecord(p->ev_fwd[k], p->cs));
                PCK(cudaStreamWaitEvent(p->s_out, p->ev_fwd[k], 0));
                NCK(g_nccl.Send(x, xn, ncclFloat32, R + 1, c_next, p->s_out));
                PCK(cudaEventRecord(p->ev_sent[k], p->s_out));
            } else {
                if (pick && xj_cuda_batch_pick_rows(p->batch, x, r0, n, col(i + 1) + r0, err, errlen)) return -1;
                PCK(cudaEventRecord(p->ev_pick[k], p->cs));
                if (pick && W > 1) {
                    PCK(cudaStreamWaitEvent(p->s_ids, p->ev_pick[k], 0));
                    NCK(g_nccl.Send(col(i + 1) + r0, (size_t)n, ncclInt32, 0, c_ids, p->s_ids));
                }
            }
        }
    }
    if (first && W > 1) {
        // the last step's picks (slot `steps`) are not fed: receive them for the output
        for (int k = 0; k < p->n_mb; k++)
            NCK(g_nccl.Recv(col(steps) + p->mb_row0[k], (size_t)p->mb_rows[k], ncclInt32, W - 1, c_ids, p->s_ids));
    }
    // the compute stream waits for every transfer stream before the end event
    for (cudaStream_t s : {p->s_in, p->s_out, p->s_ids}) {
        cudaEvent_t e = p->ev_fwd[0];
        PCK(cudaEventRecord(e, s));
        PCK(cudaStreamWaitEvent(p->cs, e, 0));
    }
    PCK(cudaEventRecord(p->ev_t1, p->cs));
    if (xj_cuda_batch_sync(p->batch, err, errlen)) return -1;
    if (gpu_ms) PCK(cudaEventElapsedTime(gpu_ms, p->ev_t0, p->ev_t1));
    if (first) {
        // out[b][g] = slot P + g (g < n_gen): the picks of steps P - 1 .. steps - 1
        std::vector<int32_t> t((size_t)n_gen * N);
        PCK(cudaMemcpy(t.data(), col(P), t.size() * sizeof(int32_t), cudaMemcpyDeviceToHost));
        for (int b = 0; b < N; b++)
            for (int g = 0; g < n_gen; g++) out[(size_t)b * n_gen + g] = t[(size_t)g * N + b];
    }
    return 0;
}

}  // extern "C"
