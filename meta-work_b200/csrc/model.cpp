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

// ------------------------------------------------------------------ the model description
// The loader is driven by tables: which metadata keys fill which hyperparameter, which tensors each kind
// of layer owns and what each must satisfy, which vocabulary strings name the special tokens, and which
// tensors the MTP head adds. One walker per table applies the rules, so the loader's behaviour can be
// read off the tables below. The rules are the runtime's (tensor names and dtype/shape requirements of
// core/xj_model.c:62-101 and :104-127, hyperparameters of :129-172); the structural fingerprint is the
// runtime's formula (:188-197), which pipeline peers compare.

// Where a tensor points into the mapped file (or a failure message).
bool bind_tensor(const gguf_file *g, const char *name, xj_w *w, bool must_exist, char *err, size_t errlen) {
    memset(w, 0, sizeof(*w));
    const gguf_tensor *t = find_tensor(g, name);
    if (!t) {
        if (must_exist) seterr(err, errlen, "model has no tensor %s", name);
        return !must_exist;
    }
    static const uint32_t kTypes[] = {XJ_F32, XJ_F16, XJ_BF16, XJ_Q8_0, XJ_Q4_K, XJ_Q5_K, XJ_Q6_K};
    bool known = false;
    for (uint32_t ty : kTypes) known = known || t->type == ty;
    if (!known) { seterr(err, errlen, "tensor %s has unsupported type %u", name, t->type); return false; }
    w->file_off = g->data_off + t->offset;
    w->data = g->map + (w->file_off - g->map_off);
    w->nbytes = t->nbytes;
    w->type = t->type;
    w->ne0 = t->ne[0];
    w->ne1 = t->ne[1] * t->ne[2] * t->ne[3];
    return true;
}

// Layer kinds a tensor rule applies to.
enum class Kind : uint8_t { Every, Linear, Full };
// When a tensor must be present.
enum class Need : uint8_t { Always, Optional, WithoutFusedQkv };
// What it must satisfy once bound.
enum class Rule : uint8_t { None, F32, RowsConvDim, F32ColsConvK };

struct LayerTensor {
    xj_w xj_layer::*field;
    const char *suffix;   // after "blk.<i>."
    Kind kind;
    Need need;
    Rule rule;
};

const LayerTensor kLayerTensors[] = {
    {&xj_layer::attn_norm, "attn_norm.weight", Kind::Every, Need::Always, Rule::F32},
    {&xj_layer::post_norm, "post_attention_norm.weight", Kind::Every, Need::Always, Rule::F32},
    {&xj_layer::ffn_gate, "ffn_gate.weight", Kind::Every, Need::Always, Rule::None},
    {&xj_layer::ffn_up, "ffn_up.weight", Kind::Every, Need::Always, Rule::None},
    {&xj_layer::ffn_down, "ffn_down.weight", Kind::Every, Need::Always, Rule::None},
    // Gated DeltaNet layers
    {&xj_layer::ssm_qkv, "attn_qkv.weight", Kind::Linear, Need::Always, Rule::RowsConvDim},
    {&xj_layer::ssm_gate, "attn_gate.weight", Kind::Linear, Need::Always, Rule::None},
    {&xj_layer::ssm_conv1d, "ssm_conv1d.weight", Kind::Linear, Need::Always, Rule::F32ColsConvK},
    {&xj_layer::ssm_dt, "ssm_dt.bias", Kind::Linear, Need::Always, Rule::F32},
    {&xj_layer::ssm_a, "ssm_a", Kind::Linear, Need::Always, Rule::F32},
    {&xj_layer::ssm_beta, "ssm_beta.weight", Kind::Linear, Need::Always, Rule::None},
    {&xj_layer::ssm_alpha, "ssm_alpha.weight", Kind::Linear, Need::Always, Rule::None},
    {&xj_layer::ssm_norm, "ssm_norm.weight", Kind::Linear, Need::Always, Rule::F32},
    {&xj_layer::ssm_out, "ssm_out.weight", Kind::Linear, Need::Always, Rule::None},
    // gated full-attention layers: a fused q|k|v matrix, or the three separate ones
    {&xj_layer::wqkv, "attn_qkv.weight", Kind::Full, Need::Optional, Rule::None},
    {&xj_layer::wq, "attn_q.weight", Kind::Full, Need::WithoutFusedQkv, Rule::None},
    {&xj_layer::wk, "attn_k.weight", Kind::Full, Need::WithoutFusedQkv, Rule::None},
    {&xj_layer::wv, "attn_v.weight", Kind::Full, Need::WithoutFusedQkv, Rule::None},
    {&xj_layer::wo, "attn_output.weight", Kind::Full, Need::Always, Rule::None},
    {&xj_layer::q_norm, "attn_q_norm.weight", Kind::Full, Need::Always, Rule::None},
    {&xj_layer::k_norm, "attn_k_norm.weight", Kind::Full, Need::Always, Rule::None},
};

bool rule_holds(Rule r, const xj_w &w, const xj_hparams *hp) {
    switch (r) {
    case Rule::None: return true;
    case Rule::F32: return w.type == XJ_F32;
    case Rule::RowsConvDim: return w.ne1 == hp->conv_dim;
    case Rule::F32ColsConvK: return w.type == XJ_F32 && w.ne0 == hp->conv_k;
    }
    return false;
}

// Binds the tensors of file block `blk` into *L (whose `recurrent` flag is already set).
bool bind_layer(const gguf_file *g, const xj_hparams *hp, int blk, xj_layer *L, char *err, size_t errlen) {
    char name[96];
    for (const LayerTensor &t : kLayerTensors) {
        if ((t.kind == Kind::Linear && !L->recurrent) || (t.kind == Kind::Full && L->recurrent)) continue;
        if (t.need == Need::WithoutFusedQkv && L->wqkv.nbytes) continue;
        snprintf(name, sizeof name, "blk.%d.%s", blk, t.suffix);
        xj_w &w = L->*t.field;
        if (!bind_tensor(g, name, &w, t.need != Need::Optional, err, errlen)) return false;
        if (w.nbytes && !rule_holds(t.rule, w, hp)) {
            seterr(err, errlen, "tensor %s: %s", name,
                   t.rule == Rule::F32 ? "must be F32" : t.rule == Rule::RowsConvDim ? "rows differ from the conv channels"
                                                                                      : "must be F32 with conv_k columns");
            return false;
        }
    }
    return true;
}

// Hyperparameters read from "qwen35.<suffix>" metadata. Keys without a default must be present.
struct Raw { uint32_t block_count, key_len, val_len, nextn; };
struct HpKey {
    const char *suffix;
    int xj_hparams::*field;   // or, when null, a slot of Raw
    uint32_t Raw::*raw;
    bool required;
    uint32_t dflt;
};
const HpKey kHpKeys[] = {
    {"block_count", nullptr, &Raw::block_count, true, 0},
    {"embedding_length", &xj_hparams::n_embd, nullptr, true, 0},
    {"feed_forward_length", &xj_hparams::n_ff, nullptr, true, 0},
    {"attention.head_count", &xj_hparams::n_head, nullptr, true, 0},
    {"attention.head_count_kv", &xj_hparams::n_head_kv, nullptr, true, 0},
    {"attention.key_length", nullptr, &Raw::key_len, true, 0},
    {"attention.value_length", nullptr, &Raw::val_len, true, 0},
    {"rope.dimension_count", &xj_hparams::n_rot, nullptr, true, 0},
    {"ssm.conv_kernel", &xj_hparams::conv_k, nullptr, true, 0},
    {"ssm.inner_size", &xj_hparams::d_inner, nullptr, true, 0},
    {"ssm.state_size", &xj_hparams::s_k, nullptr, true, 0},
    {"ssm.group_count", &xj_hparams::h_k, nullptr, true, 0},
    {"ssm.time_step_rank", &xj_hparams::h_v, nullptr, true, 0},
    {"nextn_predict_layers", nullptr, &Raw::nextn, false, 0},
    {"full_attention_interval", &xj_hparams::full_attn_interval, nullptr, false, 4},
};
// Float hyperparameters with their defaults.
const struct { const char *suffix; float xj_hparams::*field; float dflt; } kHpFloats[] = {
    {"rope.freq_base", &xj_hparams::rope_base, 10000.0f},
    {"attention.layer_norm_rms_epsilon", &xj_hparams::eps, 1e-6f},
};

bool read_hparams(const gguf_file *g, xj_hparams *hp, Raw *raw, char *err, size_t errlen) {
    char key[128];
    for (const HpKey &k : kHpKeys) {
        snprintf(key, sizeof key, "qwen35.%s", k.suffix);
        uint32_t v = k.dflt;
        if (!get_u32(g, key, &v) && k.required) { seterr(err, errlen, "model is missing %s", key); return false; }
        if (k.field) hp->*k.field = (int)v;
        else raw->*k.raw = v;
    }
    for (const auto &k : kHpFloats) {
        snprintf(key, sizeof key, "qwen35.%s", k.suffix);
        hp->*k.field = k.dflt;
        get_f32(g, key, &(hp->*k.field));
    }
    // derived sizes, then the consistency conditions the kernels rely on
    hp->n_layer = (int)raw->block_count - (int)raw->nextn;     // the MTP block is not a decoder layer
    hp->head_dim = (int)raw->key_len;
    hp->s_v = hp->h_v > 0 ? hp->d_inner / hp->h_v : 0;
    hp->key_dim = hp->s_k * hp->h_k;
    hp->conv_dim = 2 * hp->key_dim + hp->d_inner;
    const struct { bool bad; const char *why; } conds[] = {
        {raw->key_len != raw->val_len, "key and value head dims differ"},
        {hp->h_v <= 0 || hp->h_k <= 0, "bad linear-attention head counts"},
        {hp->s_v != hp->s_k, "linear-attention key and value head dims differ"},
        {hp->h_k > 0 && hp->h_v % hp->h_k != 0, "value heads are not a multiple of key heads"},
        {hp->n_layer <= 0 || hp->n_layer > XJ_MAX_LAYERS, "bad layer count"},
        {hp->n_rot > hp->head_dim || hp->n_rot % 2 != 0, "bad rope dimension"},
    };
    for (const auto &c : conds)
        if (c.bad) { seterr(err, errlen, "%s", c.why); return false; }
    return true;
}

// Special tokens: the eos id from metadata, then vocabulary strings; the chat end token takes the last
// match, the text end token fills eos only when the metadata left it unset. n_vocab = vocabulary size.
void read_specials(const gguf_file *g, xj_hparams *hp) {
    const struct { const char *text; uint32_t xj_hparams::*field; bool only_if_unset; } kSpecial[] = {
        {"<|im_end|>", &xj_hparams::eot, false},
        {"<|endoftext|>", &xj_hparams::eos, true},
    };
    hp->eos = hp->eot = UINT32_MAX;
    uint32_t id;
    if (get_u32(g, "tokenizer.ggml.eos_token_id", &id)) hp->eos = id;
    const gguf_kv *kv = find_kv(g, "tokenizer.ggml.tokens");
    if (!kv || kv->type != GGUF_ARR || kv->arr_type != GGUF_STR) return;
    const uint8_t *p = kv->data + 12;
    for (uint64_t i = 0; i < kv->arr_n; i++) {
        uint64_t n;
        memcpy(&n, p, 8);
        for (const auto &sp : kSpecial)
            if (n == strlen(sp.text) && memcmp(p + 8, sp.text, n) == 0 && (!sp.only_if_unset || hp->*sp.field == UINT32_MAX))
                hp->*sp.field = (uint32_t)i;
        p += 8 + n;
    }
    hp->n_vocab = (int)kv->arr_n;
}

// The MTP head's own tensors ("blk.<last>.nextn.<suffix>").
const struct { xj_w xj_model::*field; const char *suffix; Rule rule; } kMtpTensors[] = {
    {&xj_model::mtp_eh, "eh_proj.weight", Rule::None},
    {&xj_model::mtp_enorm, "enorm.weight", Rule::F32},
    {&xj_model::mtp_hnorm, "hnorm.weight", Rule::F32},
    {&xj_model::mtp_head_norm, "shared_head_norm.weight", Rule::F32},
};

bool bind_mtp(const gguf_file *g, xj_model *m, int blk, char *err, size_t errlen) {
    const int il = m->hp.n_layer;                 // the MTP layer sits after the decoder layers
    if (il + 1 > XJ_MAX_LAYERS) { seterr(err, errlen, "too many layers"); return false; }
    xj_layer *L = &m->layers[il];
    memset(L, 0, sizeof(*L));
    if (!bind_layer(g, &m->hp, blk, L, err, errlen)) return false;
    char name[96];
    for (const auto &t : kMtpTensors) {
        snprintf(name, sizeof name, "blk.%d.nextn.%s", blk, t.suffix);
        xj_w &w = m->*t.field;
        if (!bind_tensor(g, name, &w, true, err, errlen)) return false;
        if (!rule_holds(t.rule, w, &m->hp)) { seterr(err, errlen, "tensor %s must be F32", name); return false; }
    }
    if (m->mtp_eh.ne0 != 2 * m->hp.n_embd || m->mtp_eh.ne1 != m->hp.n_embd) {
        seterr(err, errlen, "MTP eh_proj has the wrong shape");
        return false;
    }
    m->has_mtp = true;
    return true;
}

uint64_t fnv(uint64_t h, const void *p, size_t n) {
    const uint8_t *b = (const uint8_t *)p;
    for (size_t i = 0; i < n; i++) { h ^= b[i]; h *= 1099511628211ull; }
    return h;
}

// Structural fingerprint: FNV-1a over the hyperparameters and every tensor's name, type, shape and
// offset (the runtime's formula, so that pipeline peers loaded by either loader agree).
uint64_t structure_fingerprint(const gguf_file *g, const xj_hparams *hp) {
    uint64_t h = fnv(1469598103934665603ull, hp, sizeof(*hp));
    for (uint64_t i = 0; i < g->n_tensors; i++) {
        const gguf_tensor *t = &g->tensors[i];
        h = fnv(h, t->name, strlen(t->name));
        h = fnv(h, &t->type, sizeof t->type);
        h = fnv(h, t->ne, sizeof t->ne);
        h = fnv(h, &t->offset, sizeof t->offset);
    }
    return h;
}

bool is_qwen35(const gguf_file *g) {
    const gguf_kv *kv = find_kv(g, "general.architecture");
    if (!kv || kv->type != GGUF_STR) return false;
    uint64_t n;
    memcpy(&n, kv->data, 8);
    return n == 6 && memcmp(kv->data + 8, "qwen35", 6) == 0;
}

xj_model *build_model(gguf_file *g, char *err, size_t errlen) {
    if (!is_qwen35(g)) { seterr(err, errlen, "not a Qwen3.5 model (general.architecture must be qwen35)"); return nullptr; }
    xj_model *m = (xj_model *)calloc(1, sizeof(xj_model));
    m->gguf = g;
    xj_hparams *hp = &m->hp;
    Raw raw{};
    bool ok = read_hparams(g, hp, &raw, err, errlen);
    if (ok) {
        read_specials(g, hp);
        // layer kinds: the explicit per-layer flags when present, else every full_attn_interval-th layer
        // is full attention
        for (int i = 0; i < hp->n_layer; i++) {
            uint32_t r;
            m->layers[i].recurrent = get_arr_u32(g, "qwen35.attention.recurrent_layers", (uint64_t)i, &r)
                                         ? r != 0 : (i + 1) % hp->full_attn_interval != 0;
        }
        ok = bind_tensor(g, "token_embd.weight", &m->tok_embd, true, err, errlen) &&
             bind_tensor(g, "output_norm.weight", &m->output_norm, true, err, errlen) &&
             bind_tensor(g, "output.weight", &m->output, false, err, errlen);
    }
    if (ok) {
        if (!m->output.nbytes) m->output = m->tok_embd;     // tied output
        if (!hp->n_vocab) hp->n_vocab = (int)m->tok_embd.ne1;
        for (int i = 0; ok && i < hp->n_layer; i++) ok = bind_layer(g, hp, i, &m->layers[i], err, errlen);
    }
    if (ok && raw.nextn > 0) ok = bind_mtp(g, m, (int)raw.block_count - 1, err, errlen);
    if (!ok) { free(m); return nullptr; }
    m->fingerprint = structure_fingerprint(g, hp);
    return m;
}

}  // namespace

extern "C" {

xj_model *xjc_model_load(const char *path, char *err, size_t errlen) {
    gguf_file *g = gguf_open_file(path, err, errlen);
    if (!g) return nullptr;
    xj_model *m = build_model(g, err, errlen);
    if (!m) gguf_free(g);
    return m;
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
