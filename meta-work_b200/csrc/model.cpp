// GGUF loader producing the runtime's xj_model (include/xj_abi.h), for hosts that do not link the
// runtime's core/. Behaviour follows the runtime's loader:
//   - GGUF v2/v3 parse, 32-byte default alignment, general.alignment override   core/gguf.c:106-186
//   - whole-file read-only mmap, tensors must lie inside the file                core/gguf.c:192-215
//   - qwen35 hparams, recurrent-layer pattern, tied output, MTP layer           core/xj_model.c:129-202
//   - per-layer tensor table and dtype/shape checks                              core/xj_model.c:62-101
//   - structural fingerprint (FNV-1a over hparams + tensor table)                core/xj_model.c:37-41,188-197
// so a model loaded here has the same field values (and fingerprint) as one loaded by xj_model_load.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
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

int type_block(uint32_t type, int *bytes) {
    int n = 0, b = 0;
    switch (type) {
    case XJ_F32: n = 1; b = 4; break;
    case XJ_F16: case XJ_BF16: n = 1; b = 2; break;
    case XJ_Q4_0: n = 32; b = 18; break;
    case XJ_Q4_1: n = 32; b = 20; break;
    case XJ_Q5_0: n = 32; b = 22; break;
    case XJ_Q5_1: n = 32; b = 24; break;
    case XJ_Q8_0: n = 32; b = 34; break;
    case XJ_Q2_K: n = 256; b = 84; break;
    case XJ_Q3_K: n = 256; b = 110; break;
    case XJ_Q4_K: n = 256; b = 144; break;
    case XJ_Q5_K: n = 256; b = 176; break;
    case XJ_Q6_K: n = 256; b = 210; break;
    default: break;
    }
    if (bytes) *bytes = b;
    return n;
}

uint64_t row_bytes(uint32_t type, int64_t n) {
    int b = 0, bn = type_block(type, &b);
    return bn ? (uint64_t)(n / bn) * (uint64_t)b : 0;
}

int vsize(uint32_t t) {
    switch (t) {
    case GGUF_U8: case GGUF_I8: case GGUF_BOOL: return 1;
    case GGUF_U16: case GGUF_I16: return 2;
    case GGUF_U32: case GGUF_I32: case GGUF_F32: return 4;
    case GGUF_U64: case GGUF_I64: case GGUF_F64: return 8;
    default: return 0;
    }
}

struct Reader {
    const uint8_t *p, *end;
    bool ok = true;
    bool need(uint64_t n) { if ((uint64_t)(end - p) < n) ok = false; return ok; }
    uint32_t u32() { uint32_t v = 0; if (need(4)) { memcpy(&v, p, 4); p += 4; } return v; }
    uint64_t u64() { uint64_t v = 0; if (need(8)) { memcpy(&v, p, 8); p += 8; } return v; }
    const uint8_t *bytes(uint64_t n) { const uint8_t *s = p; if (need(n)) p += n; return ok ? s : nullptr; }
    bool skip_value(uint32_t t, uint32_t *arr_t, uint64_t *arr_n) {
        if (t == GGUF_STR) { uint64_t n = u64(); bytes(n); return ok; }
        if (t == GGUF_ARR) {
            uint32_t et = u32(); uint64_t n = u64();
            if (arr_t) *arr_t = et;
            if (arr_n) *arr_n = n;
            if (!ok) return false;
            if (et == GGUF_STR) { for (uint64_t i = 0; i < n && ok; i++) { uint64_t l = u64(); bytes(l); } return ok; }
            int es = vsize(et);
            if (!es || n > UINT64_MAX / (uint64_t)es) return false;
            bytes(n * (uint64_t)es);
            return ok;
        }
        int s = vsize(t);
        if (!s) return false;
        bytes((uint64_t)s);
        return ok;
    }
};

void gguf_free(gguf_file *f) {
    if (!f) return;
    if (f->map) munmap((void *)f->map, (size_t)f->map_len);
    if (f->fd >= 0) close(f->fd);
    free(f->hdr); free(f->kv); free(f->tensors); free(f->strpool);
    free(f);
}

gguf_file *gguf_open_file(const char *path, char *err, size_t errlen) {
    int fd = open(path, O_RDONLY);
    if (fd < 0) { seterr(err, errlen, "cannot open %s", path); return nullptr; }
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 16) { close(fd); seterr(err, errlen, "file too small"); return nullptr; }
    void *mp = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_SHARED, fd, 0);
    if (mp == MAP_FAILED) { close(fd); seterr(err, errlen, "mmap failed"); return nullptr; }
    gguf_file *f = (gguf_file *)calloc(1, sizeof(gguf_file));
    f->fd = fd; f->map = (const uint8_t *)mp; f->map_off = 0; f->map_len = (uint64_t)st.st_size;
    f->size = (uint64_t)st.st_size; f->alignment = 32;
    Reader r{f->map, f->map + f->size};
    uint32_t magic = r.u32(), version = r.u32();
    if (!r.ok || magic != 0x46554747u) { seterr(err, errlen, "not a GGUF file"); gguf_free(f); return nullptr; }
    if (version < 2 || version > 3) { seterr(err, errlen, "GGUF version %u not supported", version); gguf_free(f); return nullptr; }
    f->n_tensors = r.u64(); f->n_kv = r.u64();
    if (!r.ok || f->n_kv > (1u << 20) || f->n_tensors > (1u << 20)) { seterr(err, errlen, "bad GGUF header counts"); gguf_free(f); return nullptr; }
    f->kv = (gguf_kv *)calloc(f->n_kv ? f->n_kv : 1, sizeof(gguf_kv));
    f->tensors = (gguf_tensor *)calloc(f->n_tensors ? f->n_tensors : 1, sizeof(gguf_tensor));
    std::string pool;
    std::vector<size_t> key_at(f->n_kv), name_at(f->n_tensors);
    for (uint64_t i = 0; i < f->n_kv && r.ok; i++) {
        uint64_t n = r.u64();
        const uint8_t *s = r.bytes(n);
        if (!r.ok) break;
        key_at[i] = pool.size(); pool.append((const char *)s, n); pool.push_back('\0');
        gguf_kv *kv = &f->kv[i];
        kv->type = r.u32();
        kv->data = r.p;
        if (!r.skip_value(kv->type, &kv->arr_type, &kv->arr_n)) {
            if (r.ok) seterr(err, errlen, "unknown GGUF value type %u", kv->type);
            else seterr(err, errlen, "truncated GGUF header");
            gguf_free(f); return nullptr;
        }
        if (kv->type == GGUF_U32 && strcmp(pool.c_str() + key_at[i], "general.alignment") == 0) memcpy(&f->alignment, kv->data, 4);
    }
    if (!r.ok) { seterr(err, errlen, "truncated GGUF header"); gguf_free(f); return nullptr; }
    if (f->alignment == 0 || (f->alignment & (f->alignment - 1))) { seterr(err, errlen, "bad alignment %u", f->alignment); gguf_free(f); return nullptr; }
    for (uint64_t i = 0; i < f->n_tensors && r.ok; i++) {
        uint64_t n = r.u64();
        const uint8_t *s = r.bytes(n);
        if (!r.ok) break;
        name_at[i] = pool.size(); pool.append((const char *)s, n); pool.push_back('\0');
        gguf_tensor *t = &f->tensors[i];
        t->n_dims = r.u32();
        if (t->n_dims > 4) { seterr(err, errlen, "tensor has %u dims (max 4)", t->n_dims); gguf_free(f); return nullptr; }
        for (int k = 0; k < 4; k++) t->ne[k] = 1;
        for (uint32_t k = 0; k < t->n_dims; k++) t->ne[k] = (int64_t)r.u64();
        t->type = r.u32();
        t->offset = r.u64();
        int bb = 0, bn = type_block(t->type, &bb);
        if (!bn) { t->nbytes = 0; continue; }
        if (t->ne[0] % bn) { seterr(err, errlen, "tensor row length %lld not a multiple of the block", (long long)t->ne[0]); gguf_free(f); return nullptr; }
        t->nbytes = row_bytes(t->type, t->ne[0]) * (uint64_t)(t->ne[1] * t->ne[2] * t->ne[3]);
    }
    if (!r.ok) { seterr(err, errlen, "truncated GGUF header"); gguf_free(f); return nullptr; }
    f->strpool = (char *)malloc(pool.size() ? pool.size() : 1);
    memcpy(f->strpool, pool.data(), pool.size());
    for (uint64_t i = 0; i < f->n_kv; i++) f->kv[i].key = f->strpool + key_at[i];
    for (uint64_t i = 0; i < f->n_tensors; i++) f->tensors[i].name = f->strpool + name_at[i];
    uint64_t hdr = (uint64_t)(r.p - f->map);
    f->data_off = (hdr + f->alignment - 1) / f->alignment * f->alignment;
    for (uint64_t i = 0; i < f->n_tensors; i++) {
        const gguf_tensor *t = &f->tensors[i];
        if (f->data_off + t->offset + t->nbytes > f->size) {
            seterr(err, errlen, "tensor %s extends past the end of the file", t->name);
            gguf_free(f); return nullptr;
        }
    }
    return f;
}

const gguf_kv *find_kv(const gguf_file *f, const char *key) {
    for (uint64_t i = 0; i < f->n_kv; i++) if (strcmp(f->kv[i].key, key) == 0) return &f->kv[i];
    return nullptr;
}

const gguf_tensor *find_tensor(const gguf_file *f, const char *name) {
    for (uint64_t i = 0; i < f->n_tensors; i++) if (strcmp(f->tensors[i].name, name) == 0) return &f->tensors[i];
    return nullptr;
}

bool scalar_u32(uint32_t type, const uint8_t *p, uint32_t *out) {
    switch (type) {
    case GGUF_U8: *out = p[0]; return true;
    case GGUF_I8: *out = (uint32_t)(int8_t)p[0]; return true;
    case GGUF_U16: { uint16_t v; memcpy(&v, p, 2); *out = v; return true; }
    case GGUF_I16: { int16_t v; memcpy(&v, p, 2); *out = (uint32_t)v; return true; }
    case GGUF_U32: case GGUF_I32: memcpy(out, p, 4); return true;
    case GGUF_U64: case GGUF_I64: { uint64_t v; memcpy(&v, p, 8); *out = (uint32_t)v; return true; }
    case GGUF_BOOL: *out = p[0] != 0; return true;
    default: return false;
    }
}

bool get_u32(const gguf_file *f, const char *key, uint32_t *out) {
    const gguf_kv *kv = find_kv(f, key);
    return kv && scalar_u32(kv->type, kv->data, out);
}

bool get_f32(const gguf_file *f, const char *key, float *out) {
    const gguf_kv *kv = find_kv(f, key);
    if (!kv) return false;
    if (kv->type == GGUF_F32) { memcpy(out, kv->data, 4); return true; }
    if (kv->type == GGUF_F64) { double d; memcpy(&d, kv->data, 8); *out = (float)d; return true; }
    uint32_t u;
    if (scalar_u32(kv->type, kv->data, &u)) { *out = (float)u; return true; }
    return false;
}

bool get_arr_u32(const gguf_file *f, const char *key, uint64_t i, uint32_t *out) {
    const gguf_kv *kv = find_kv(f, key);
    if (!kv || kv->type != GGUF_ARR || i >= kv->arr_n) return false;
    int es = vsize(kv->arr_type);
    return es && scalar_u32(kv->arr_type, kv->data + 12 + i * (uint64_t)es, out);
}

bool get_w(const gguf_file *g, const char *name, xj_w *w, bool required, char *err, size_t errlen) {
    memset(w, 0, sizeof(*w));
    const gguf_tensor *t = find_tensor(g, name);
    if (!t) {
        if (required) seterr(err, errlen, "model has no tensor %s", name);
        return !required;
    }
    if (t->type != XJ_F32 && t->type != XJ_F16 && t->type != XJ_BF16 && t->type != XJ_Q8_0 && t->type != XJ_Q4_K &&
        t->type != XJ_Q5_K && t->type != XJ_Q6_K) {
        seterr(err, errlen, "tensor %s has unsupported type %u", name, t->type);
        return false;
    }
    w->data = g->map + (g->data_off + t->offset - g->map_off);
    w->file_off = g->data_off + t->offset;
    w->nbytes = t->nbytes;
    w->type = t->type;
    w->ne0 = t->ne[0];
    w->ne1 = t->ne[1] * t->ne[2] * t->ne[3];
    return true;
}

bool load_layer(const gguf_file *g, const xj_hparams *hp, int i, xj_layer *L, char *err, size_t errlen) {
    char name[96];
#define W(field, suffix, req) do { snprintf(name, sizeof name, "blk.%d.%s", i, suffix); \
        if (!get_w(g, name, &L->field, req, err, errlen)) return false; } while (0)
    W(attn_norm, "attn_norm.weight", true);
    W(post_norm, "post_attention_norm.weight", true);
    W(ffn_gate, "ffn_gate.weight", true);
    W(ffn_up, "ffn_up.weight", true);
    W(ffn_down, "ffn_down.weight", true);
    if (L->recurrent) {
        W(ssm_qkv, "attn_qkv.weight", true);
        W(ssm_gate, "attn_gate.weight", true);
        W(ssm_conv1d, "ssm_conv1d.weight", true);
        W(ssm_dt, "ssm_dt.bias", true);
        W(ssm_a, "ssm_a", true);
        W(ssm_beta, "ssm_beta.weight", true);
        W(ssm_alpha, "ssm_alpha.weight", true);
        W(ssm_norm, "ssm_norm.weight", true);
        W(ssm_out, "ssm_out.weight", true);
        if (L->ssm_qkv.ne1 != hp->conv_dim || L->ssm_conv1d.type != XJ_F32 || L->ssm_conv1d.ne0 != hp->conv_k) {
            seterr(err, errlen, "layer %d: linear-attention tensor shapes do not match", i); return false;
        }
        if (L->ssm_a.type != XJ_F32 || L->ssm_dt.type != XJ_F32 || L->ssm_norm.type != XJ_F32) {
            seterr(err, errlen, "layer %d: ssm_a / ssm_dt / ssm_norm must be F32", i); return false;
        }
    } else {
        W(wqkv, "attn_qkv.weight", false);
        if (!L->wqkv.nbytes) {
            W(wq, "attn_q.weight", true);
            W(wk, "attn_k.weight", true);
            W(wv, "attn_v.weight", true);
        }
        W(wo, "attn_output.weight", true);
        W(q_norm, "attn_q_norm.weight", true);
        W(k_norm, "attn_k_norm.weight", true);
    }
    if (L->attn_norm.type != XJ_F32 || L->post_norm.type != XJ_F32) { seterr(err, errlen, "layer %d: norms must be F32", i); return false; }
#undef W
    return true;
}

uint64_t fnv(uint64_t h, const void *p, size_t n) {
    const uint8_t *b = (const uint8_t *)p;
    for (size_t i = 0; i < n; i++) { h ^= b[i]; h *= 1099511628211ull; }
    return h;
}

}  // namespace

extern "C" {

xj_model *xjc_model_load(const char *path, char *err, size_t errlen) {
    gguf_file *g = gguf_open_file(path, err, errlen);
    if (!g) return nullptr;
    const gguf_kv *akv = find_kv(g, "general.architecture");
    uint64_t alen = 0;
    if (akv && akv->type == GGUF_STR) memcpy(&alen, akv->data, 8);
    if (!akv || akv->type != GGUF_STR || alen != 6 || memcmp(akv->data + 8, "qwen35", 6) != 0) {
        seterr(err, errlen, "not a Qwen3.5 model (general.architecture must be qwen35)");
        gguf_free(g); return nullptr;
    }
    xj_model *m = (xj_model *)calloc(1, sizeof(xj_model));
    m->gguf = g;
    xj_hparams *hp = &m->hp;
    uint32_t block_count, key_len, val_len, v;
    int nextn = 0;
    struct { const char *k; void *dst; } req[] = {
        {"qwen35.block_count", &block_count}, {"qwen35.embedding_length", &hp->n_embd},
        {"qwen35.feed_forward_length", &hp->n_ff}, {"qwen35.attention.head_count", &hp->n_head},
        {"qwen35.attention.head_count_kv", &hp->n_head_kv}, {"qwen35.attention.key_length", &key_len},
        {"qwen35.attention.value_length", &val_len}, {"qwen35.rope.dimension_count", &hp->n_rot},
        {"qwen35.ssm.conv_kernel", &hp->conv_k}, {"qwen35.ssm.inner_size", &hp->d_inner},
        {"qwen35.ssm.state_size", &hp->s_k}, {"qwen35.ssm.group_count", &hp->h_k},
        {"qwen35.ssm.time_step_rank", &hp->h_v},
    };
    for (auto &q : req) {
        if (!get_u32(g, q.k, &v)) { seterr(err, errlen, "model is missing %s", q.k); goto fail; }
        memcpy(q.dst, &v, 4);
    }
    if (get_u32(g, "qwen35.nextn_predict_layers", &v)) nextn = (int)v;
    hp->n_layer = (int)block_count - nextn;
    hp->full_attn_interval = 4;
    if (get_u32(g, "qwen35.full_attention_interval", &v)) hp->full_attn_interval = (int)v;
    hp->rope_base = 10000.0f;
    get_f32(g, "qwen35.rope.freq_base", &hp->rope_base);
    hp->eps = 1e-6f;
    get_f32(g, "qwen35.attention.layer_norm_rms_epsilon", &hp->eps);
    if (key_len != val_len) { seterr(err, errlen, "key/value head dims differ (%u/%u)", key_len, val_len); goto fail; }
    hp->head_dim = (int)key_len;
    if (hp->h_v <= 0 || hp->h_k <= 0) { seterr(err, errlen, "bad linear-attention head counts"); goto fail; }
    hp->s_v = hp->d_inner / hp->h_v;
    if (hp->s_v != hp->s_k) { seterr(err, errlen, "linear-attention key/value head dims differ"); goto fail; }
    if (hp->h_v % hp->h_k) { seterr(err, errlen, "value heads are not a multiple of key heads"); goto fail; }
    hp->key_dim = hp->s_k * hp->h_k;
    hp->conv_dim = 2 * hp->key_dim + hp->d_inner;
    if (hp->n_layer <= 0 || hp->n_layer > XJ_MAX_LAYERS) { seterr(err, errlen, "bad layer count %d", hp->n_layer); goto fail; }
    if (hp->n_rot > hp->head_dim || hp->n_rot % 2) { seterr(err, errlen, "bad rope dimension %d", hp->n_rot); goto fail; }
    {
        // special tokens by string, as the runtime does (xj_model.c:44-59)
        const gguf_kv *kv = find_kv(g, "tokenizer.ggml.tokens");
        hp->eos = hp->eot = UINT32_MAX;
        uint32_t eos;
        if (get_u32(g, "tokenizer.ggml.eos_token_id", &eos)) hp->eos = eos;
        if (kv && kv->type == GGUF_ARR && kv->arr_type == GGUF_STR) {
            const uint8_t *p = kv->data + 12;
            for (uint64_t i = 0; i < kv->arr_n; i++) {
                uint64_t n; memcpy(&n, p, 8);
                const char *s = (const char *)p + 8;
                if (n == 10 && memcmp(s, "<|im_end|>", 10) == 0) hp->eot = (uint32_t)i;
                if (n == 13 && memcmp(s, "<|endoftext|>", 13) == 0 && hp->eos == UINT32_MAX) hp->eos = (uint32_t)i;
                p += 8 + n;
            }
            hp->n_vocab = (int)kv->arr_n;
        }
    }
    for (int i = 0; i < hp->n_layer; i++) {
        uint32_t rr;
        if (get_arr_u32(g, "qwen35.attention.recurrent_layers", (uint64_t)i, &rr)) m->layers[i].recurrent = rr != 0;
        else m->layers[i].recurrent = (i + 1) % hp->full_attn_interval != 0;
    }
    if (!get_w(g, "token_embd.weight", &m->tok_embd, true, err, errlen) ||
        !get_w(g, "output_norm.weight", &m->output_norm, true, err, errlen) ||
        !get_w(g, "output.weight", &m->output, false, err, errlen)) goto fail;
    if (!m->output.nbytes) m->output = m->tok_embd;
    if (!hp->n_vocab) hp->n_vocab = (int)m->tok_embd.ne1;
    for (int i = 0; i < hp->n_layer; i++)
        if (!load_layer(g, hp, i, &m->layers[i], err, errlen)) goto fail;
    if (nextn > 0) {
        const int i = (int)block_count - 1, il = hp->n_layer;
        if (il + 1 > XJ_MAX_LAYERS) { seterr(err, errlen, "too many layers"); goto fail; }
        xj_layer *L = &m->layers[il];
        memset(L, 0, sizeof(*L));
        if (!load_layer(g, hp, i, L, err, errlen)) goto fail;
        char name[96];
        struct { xj_w *w; const char *s; } nx[] = {
            {&m->mtp_eh, "eh_proj.weight"}, {&m->mtp_enorm, "enorm.weight"},
            {&m->mtp_hnorm, "hnorm.weight"}, {&m->mtp_head_norm, "shared_head_norm.weight"}};
        for (auto &q : nx) {
            snprintf(name, sizeof name, "blk.%d.nextn.%s", i, q.s);
            if (!get_w(g, name, q.w, true, err, errlen)) goto fail;
        }
        if (m->mtp_eh.ne0 != 2 * hp->n_embd || m->mtp_eh.ne1 != hp->n_embd) { seterr(err, errlen, "MTP eh_proj has the wrong shape"); goto fail; }
        if (m->mtp_enorm.type != XJ_F32 || m->mtp_hnorm.type != XJ_F32 || m->mtp_head_norm.type != XJ_F32) {
            seterr(err, errlen, "MTP norms must be F32"); goto fail;
        }
        m->has_mtp = true;
    }
    {
        uint64_t h = 1469598103934665603ull;
        h = fnv(h, hp, sizeof(*hp));
        for (uint64_t i = 0; i < g->n_tensors; i++) {
            const gguf_tensor *t = &g->tensors[i];
            h = fnv(h, t->name, strlen(t->name));
            h = fnv(h, &t->type, sizeof t->type);
            h = fnv(h, t->ne, sizeof t->ne);
            h = fnv(h, &t->offset, sizeof t->offset);
        }
        m->fingerprint = h;
    }
    return m;
fail:
    free(m);
    gguf_free(g);
    return nullptr;
}

void xjc_model_free(xj_model *m) {
    if (!m) return;
    gguf_free(m->mtp_gguf);
    gguf_free(m->gguf);
    free(m);
}

}  // extern "C"

// ------------------------------------------------------------------ host-side embedding lookup
namespace {

float h2f_host(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1f, mnt = h & 0x3ff, bits;
    if (e == 0) {
        if (mnt == 0) bits = sign;
        else {
            e = 113;   // normalise the subnormal
            while (!(mnt & 0x400)) { mnt <<= 1; e--; }
            bits = sign | (e << 23) | ((mnt & 0x3ff) << 13);
        }
    } else if (e == 31) bits = sign | 0x7f800000u | (mnt << 13);
    else bits = sign | ((e + 112) << 23) | (mnt << 13);
    float f; memcpy(&f, &bits, 4); return f;
}

uint16_t rd16(const uint8_t *p) { uint16_t v; memcpy(&v, p, 2); return v; }

// One row of n elements to fp32, with the block formulas of core/xj_quant.h:55-122.
void dequant_row_host(uint32_t type, const uint8_t *b, float *y, int64_t n) {
    switch (type) {
    case XJ_F32: memcpy(y, b, (size_t)n * 4); return;
    case XJ_F16: for (int64_t i = 0; i < n; i++) y[i] = h2f_host(rd16(b + 2 * i)); return;
    case XJ_BF16: for (int64_t i = 0; i < n; i++) { uint32_t u = (uint32_t)rd16(b + 2 * i) << 16; memcpy(&y[i], &u, 4); } return;
    case XJ_Q8_0:
        for (int64_t i = 0; i < n / 32; i++, b += 34) {
            const float d = h2f_host(rd16(b));
            for (int l = 0; l < 32; l++) *y++ = d * (float)(int8_t)b[2 + l];
        }
        return;
    case XJ_Q4_K: case XJ_Q5_K: {
        const int bb = type == XJ_Q4_K ? 144 : 176;
        for (int64_t i = 0; i < n / 256; i++, b += bb) {
            const float d = h2f_host(rd16(b)), dmin = h2f_host(rd16(b + 2));
            const uint8_t *sc = b + 4;
            for (int j = 0; j < 8; j++) {
                int s, m;
                if (j < 4) { s = sc[j] & 63; m = sc[j + 4] & 63; }
                else { s = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4); m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4); }
                const float d1 = d * (float)s, m1 = dmin * (float)m;
                for (int l = 0; l < 32; l++) {
                    int q;
                    if (type == XJ_Q4_K) { const uint8_t v = b[16 + 32 * (j / 2) + l]; q = (j & 1) ? (v >> 4) : (v & 0xF); }
                    else {
                        const uint8_t v = b[48 + 32 * (j / 2) + l];
                        q = ((j & 1) ? (v >> 4) : (v & 0xF)) + (((b[16 + l] >> j) & 1) ? 16 : 0);
                    }
                    *y++ = d1 * (float)q - m1;   // two roundings (built with -ffp-contract=off)
                }
            }
        }
        return;
    }
    case XJ_Q6_K:
        for (int64_t i = 0; i < n / 256; i++, b += 210) {
            const float d = h2f_host(rd16(b + 208));
            for (int e = 0; e < 256; e++) {
                const int h = e / 128, r = e % 128, part = r / 32, l = r % 32;
                const uint8_t ql = b[64 * h + (part & 1) * 32 + l], qh = b[128 + 32 * h + l];
                const int q = (((ql >> ((part >> 1) * 4)) & 0xF) | (((qh >> (2 * part)) & 3) << 4)) - 32;
                *y++ = d * (float)(int8_t)b[192 + 8 * h + l / 16 + 2 * part] * (float)q;
            }
        }
        return;
    default:
        memset(y, 0, (size_t)n * 4);
    }
}

}  // namespace

extern "C" void xjc_embed(const xj_model *m, int32_t token, float *out) {
    const xj_w *w = &m->tok_embd;
    if (token < 0 || token >= w->ne1) { memset(out, 0, sizeof(float) * (size_t)w->ne0); return; }
    const uint64_t rb = row_bytes(w->type, w->ne0);
    dequant_row_host(w->type, (const uint8_t *)w->data + (uint64_t)token * rb, out, w->ne0);
}
