// Synthetic Qwen3.5-style ("qwen35") GGUF writer for tests and benchmarks.
//
// There are no real checkpoints on the test machines, so every model the tests and bench.py run is
// written here from a seed: weights N(0, w_std), norm weights 1 + 0.1 N(0,1), ssm_conv1d 0.5 N(0,1),
// ssm_dt 0.5 N(0,1), ssm_a = -exp(0.5 N(0,1)) (the same recipe as the reference fixture,
// src/xiaoju-pipe/tests/make_tiny_model.py:35-100), then quantised with the quantisers below.
//
// The quantisers are written from the block layouts that the runtime DEcodes
// (src/xiaoju-pipe/core/xj_quant.h:55-122); the reference ships no Q4_K/Q6_K quantiser, so only
// "decoding these bytes gives the same floats on CPU and GPU" is checked, never the choice of codes.
//
// Tensor names and metadata keys follow the runtime's loader (src/xiaoju-pipe/core/xj_model.c:62-101,
// 129-186). Random numbers come from a counter-based generator keyed by (seed, tensor, element), so
// the file is identical for any thread count.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "../../include/xj_abi.h"

extern "C" {

typedef struct {
    int n_layer, n_embd, n_ff, n_vocab;
    int n_head, n_head_kv, head_dim, n_rot;
    float rope_base, eps;
    int conv_k, s_k, h_k, h_v;      // d_inner = h_v * s_k, key_dim = h_k * s_k
    int full_attn_interval;         // every n-th layer is full attention (4 -> 3:1 GDN:GQA)
    int wtype;                      // 2-D weights: XJ_Q8_0, XJ_Q4_K (Q4_K_M policy), XJ_Q5_K, XJ_Q6_K, XJ_F16, XJ_BF16, XJ_F32
    int io_type;                    // token_embd / output type; -1 = policy default
    int tied;                       // no output.weight (LM head shares token_embd)
    int mtp;                        // append one MTP layer (blk.{n_layer} + nextn.*)
    int fused_qkv;                  // full-attention layers store attn_qkv instead of q/k/v
    unsigned long long seed;
    float w_std;                    // std of 2-D weights before quantisation (0.02)
} xjs_config;

}  // extern "C"

namespace {

// ---------------- half precision (IEEE binary16, round to nearest even) ----------------
uint16_t f32_to_f16(float f) {
    uint32_t x; std::memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);            // rounds to >= 65520 -> inf
    if (ax < 0x38800000u) {                                                // subnormal half or zero
        if (ax < 0x33000000u) return (uint16_t)sign;                       // < 2^-25 -> +-0
        uint32_t e = ax >> 23, man = (ax & 0x7fffffu) | 0x800000u;
        uint32_t shift = 126 - e;                                          // 14..24
        uint32_t h = man >> shift, rem = man & ((1u << shift) - 1), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (h & 1))) h++;
        return (uint16_t)(sign | h);
    }
    uint32_t h = ((ax - 0x38000000u) >> 13), rem = ax & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1))) h++;
    return (uint16_t)(sign | h);
}

float f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1f, m = h & 0x3ff, bits;
    if (e == 0) {
        if (m == 0) bits = sign;
        else { float f = std::ldexp((float)m, -24); std::memcpy(&bits, &f, 4); bits |= sign; }
    } else if (e == 31) bits = sign | 0x7f800000u | (m << 13);
    else bits = sign | ((e + 112) << 23) | (m << 13);
    float f; std::memcpy(&f, &bits, 4); return f;
}

uint16_t f32_to_bf16(float f) {
    uint32_t x; std::memcpy(&x, &f, 4);
    if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40);
    uint32_t r = x + 0x7fffu + ((x >> 16) & 1u);
    return (uint16_t)(r >> 16);
}

void put16(uint8_t *p, uint16_t v) { std::memcpy(p, &v, 2); }

// ---------------- quantisers (block layouts of xj_quant.h) ----------------
// Q8_0: 32 elements -> fp16 d, 32 x int8 (xj_quant.h:83-90).
void quant_q8_0(const float *x, uint8_t *b, int64_t n) {
    for (int64_t i = 0; i < n; i += 32, b += 34, x += 32) {
        float amax = 0;
        for (int l = 0; l < 32; l++) amax = std::max(amax, std::fabs(x[l]));
        float d = amax / 127.0f;
        uint16_t dh = f32_to_f16(d);
        float dq = f16_to_f32(dh), id = dq > 0 ? 1.0f / dq : 0.0f;
        put16(b, dh);
        for (int l = 0; l < 32; l++) {
            int q = (int)std::lrint(x[l] * id);
            b[2 + l] = (uint8_t)(int8_t)std::min(127, std::max(-127, q));
        }
    }
}

// Packs 6-bit scale/min pairs so that the runtime's xj_scale_min_k4 (xj_quant.h:49-52) reads back
// (sc[j], mn[j]) for j = 0..7.
void pack_k4_scales(const uint8_t *sc, const uint8_t *mn, uint8_t *q) {
    std::memset(q, 0, 12);
    for (int j = 0; j < 4; j++) { q[j] = sc[j] & 63; q[j + 4] = mn[j] & 63; }
    for (int j = 4; j < 8; j++) {
        q[j + 4] = (uint8_t)((sc[j] & 0xF) | ((mn[j] & 0xF) << 4));
        q[j - 4] |= (uint8_t)((sc[j] >> 4) << 6);
        q[j] |= (uint8_t)((mn[j] >> 4) << 6);
    }
}

// Q4_K / Q5_K share the super-block header: fp16 d, fp16 dmin, 12 bytes of 6-bit (scale, min) for
// eight 32-element sub-blocks; value = d*sc*q - dmin*m (xj_quant.h:91-122). nbits = 4 or 5.
void quant_k_asym(const float *x, uint8_t *b, int64_t n, int nbits) {
    const int qmax = (1 << nbits) - 1, bsize = nbits == 4 ? 144 : 176;
    for (int64_t i = 0; i < n; i += 256, b += bsize, x += 256) {
        float scale[8], mins[8];
        for (int j = 0; j < 8; j++) {
            float lo = x[32 * j], hi = x[32 * j];
            for (int l = 1; l < 32; l++) { lo = std::min(lo, x[32 * j + l]); hi = std::max(hi, x[32 * j + l]); }
            if (lo > 0) lo = 0;
            scale[j] = (hi - lo) / qmax;
            mins[j] = -lo;
        }
        float ms = 0, mm = 0;
        for (int j = 0; j < 8; j++) { ms = std::max(ms, scale[j]); mm = std::max(mm, mins[j]); }
        uint16_t dh = f32_to_f16(ms / 63.0f), mh = f32_to_f16(mm / 63.0f);
        float d = f16_to_f32(dh), dmin = f16_to_f32(mh);
        uint8_t sc[8], mn[8];
        for (int j = 0; j < 8; j++) {
            sc[j] = (uint8_t)std::min(63L, std::max(0L, d > 0 ? std::lrint(scale[j] / d) : 0L));
            mn[j] = (uint8_t)std::min(63L, std::max(0L, dmin > 0 ? std::lrint(mins[j] / dmin) : 0L));
        }
        put16(b, dh); put16(b + 2, mh);
        pack_k4_scales(sc, mn, b + 4);
        uint8_t qv[256];
        for (int j = 0; j < 8; j++) {
            const float s = d * sc[j], m = dmin * mn[j], is = s > 0 ? 1.0f / s : 0.0f;
            for (int l = 0; l < 32; l++) {
                long q = std::lrint((x[32 * j + l] + m) * is);
                qv[32 * j + l] = (uint8_t)std::min((long)qmax, std::max(0L, q));
            }
        }
        if (nbits == 4) {
            uint8_t *qs = b + 16;
            for (int g = 0; g < 4; g++)
                for (int l = 0; l < 32; l++)
                    qs[32 * g + l] = (uint8_t)((qv[64 * g + l] & 0xF) | ((qv[64 * g + 32 + l] & 0xF) << 4));
        } else {
            uint8_t *qh = b + 16, *ql = b + 48;
            std::memset(qh, 0, 32);
            for (int g = 0; g < 4; g++)
                for (int l = 0; l < 32; l++) {
                    uint8_t a = qv[64 * g + l], c = qv[64 * g + 32 + l];
                    ql[32 * g + l] = (uint8_t)((a & 0xF) | ((c & 0xF) << 4));
                    if (a & 16) qh[l] |= (uint8_t)(1u << (2 * g));
                    if (c & 16) qh[l] |= (uint8_t)(2u << (2 * g));
                }
        }
    }
}

// Q6_K: 256 elements -> ql[128], qh[64], int8 scales[16], fp16 d; value = d*sc*(q-32)
// (xj_quant.h:106-118).
void quant_q6_k(const float *x, uint8_t *b, int64_t n) {
    for (int64_t i = 0; i < n; i += 256, b += 210, x += 256) {
        float scale[16], amax = 0;
        for (int s = 0; s < 16; s++) {
            float best = 0;
            for (int l = 0; l < 16; l++) if (std::fabs(x[16 * s + l]) > std::fabs(best)) best = x[16 * s + l];
            scale[s] = best / -32.0f;   // signed so the extreme maps to -32
            amax = std::max(amax, std::fabs(scale[s]));
        }
        uint16_t dh = f32_to_f16(amax / 127.0f);
        float d = f16_to_f32(dh);
        int8_t sc[16];
        for (int s = 0; s < 16; s++) sc[s] = (int8_t)std::min(127L, std::max(-128L, d > 0 ? std::lrint(scale[s] / d) : 0L));
        uint8_t u[256];
        for (int e = 0; e < 256; e++) {
            float s = d * sc[e / 16];
            long q = s != 0 ? std::lrint(x[e] / s) : 0;
            u[e] = (uint8_t)(std::min(31L, std::max(-32L, q)) + 32);
        }
        uint8_t *ql = b, *qh = b + 128;
        std::memset(ql, 0, 128); std::memset(qh, 0, 64);
        for (int h = 0; h < 2; h++)
            for (int w = 0; w < 4; w++)
                for (int l = 0; l < 32; l++) {
                    uint8_t v = u[128 * h + 32 * w + l];
                    uint8_t *pl = &ql[64 * h + l + (w & 1) * 32];
                    *pl |= (uint8_t)((v & 0xF) << ((w >> 1) * 4));
                    qh[32 * h + l] |= (uint8_t)((v >> 4) << (2 * w));
                }
        std::memcpy(b + 192, sc, 16);
        put16(b + 208, dh);
    }
}

int type_block(int type, int *bytes) {
    switch (type) {
    case XJ_F32: *bytes = 4; return 1;
    case XJ_F16: case XJ_BF16: *bytes = 2; return 1;
    case XJ_Q8_0: *bytes = 34; return 32;
    case XJ_Q4_K: *bytes = 144; return 256;
    case XJ_Q5_K: *bytes = 176; return 256;
    case XJ_Q6_K: *bytes = 210; return 256;
    default: *bytes = 0; return 0;
    }
}

void quant_row(int type, const float *x, uint8_t *dst, int64_t n) {
    switch (type) {
    case XJ_F32: std::memcpy(dst, x, (size_t)n * 4); break;
    case XJ_F16: for (int64_t i = 0; i < n; i++) put16(dst + 2 * i, f32_to_f16(x[i])); break;
    case XJ_BF16: for (int64_t i = 0; i < n; i++) put16(dst + 2 * i, f32_to_bf16(x[i])); break;
    case XJ_Q8_0: quant_q8_0(x, dst, n); break;
    case XJ_Q4_K: quant_k_asym(x, dst, n, 4); break;
    case XJ_Q5_K: quant_k_asym(x, dst, n, 5); break;
    case XJ_Q6_K: quant_q6_k(x, dst, n); break;
    default: break;
    }
}

// ---------------- counter-based normal generator ----------------
inline uint64_t mix64(uint64_t z) {
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

// Standard normals 2p and 2p+1 of stream `key` (Box-Muller on two 24-bit uniforms from one draw).
inline void normal_pair(uint64_t key, uint64_t p, float *z0, float *z1) {
    uint64_t r = mix64(key ^ mix64(p));
    double u1 = ((double)((r >> 40) & 0xffffff) + 0.5) / 16777216.0;
    double u2 = ((double)((r >> 16) & 0xffffff) + 0.5) / 16777216.0;
    double rad = std::sqrt(-2.0 * std::log(u1)), th = 6.283185307179586 * u2;
    *z0 = (float)(rad * std::cos(th));
    *z1 = (float)(rad * std::sin(th));
}

enum Kind { K_WEIGHT, K_NORM, K_CONV, K_DT, K_A };

struct Tensor {
    std::string name;
    int64_t ne0, ne1;
    int type;
    Kind kind;
    float std;
    uint64_t key;
    uint64_t offset = 0, nbytes = 0;
};

uint64_t row_bytes(int type, int64_t n) { int b; int bn = type_block(type, &b); return (uint64_t)(n / bn) * (uint64_t)b; }

void fill_tensor(const Tensor &t, uint8_t *dst, int nthreads) {
    const uint64_t rb = row_bytes(t.type, t.ne0);
    auto work = [&](int64_t r0, int64_t r1) {
        std::vector<float> row((size_t)t.ne0);
        for (int64_t r = r0; r < r1; r++) {
            for (int64_t c = 0; c < t.ne0; c += 2) {   // every row length here is even
                uint64_t i = (uint64_t)r * (uint64_t)t.ne0 + (uint64_t)c;
                float z[2];
                normal_pair(t.key, i >> 1, &z[0], &z[1]);
                for (int h = 0; h < 2 && c + h < t.ne0; h++) {
                    float v;
                    switch (t.kind) {
                    case K_NORM: v = 1.0f + 0.1f * z[h]; break;
                    case K_CONV: v = 0.5f * z[h]; break;
                    case K_DT: v = 0.5f * z[h]; break;
                    case K_A: v = -std::exp(0.5f * z[h]); break;
                    default: v = t.std * z[h]; break;
                    }
                    row[(size_t)(c + h)] = v;
                }
            }
            quant_row(t.type, row.data(), dst + (uint64_t)r * rb, t.ne0);
        }
    };
    int nt = (int)std::min<int64_t>(nthreads, std::max<int64_t>(1, t.ne1 / 64));
    if (nt <= 1) { work(0, t.ne1); return; }
    std::vector<std::thread> th;
    for (int k = 0; k < nt; k++) {
        int64_t r0 = t.ne1 * k / nt, r1 = t.ne1 * (k + 1) / nt;
        th.emplace_back(work, r0, r1);
    }
    for (auto &x : th) x.join();
}

struct Writer {
    std::vector<uint8_t> b;
    void u32(uint32_t v) { b.insert(b.end(), (uint8_t *)&v, (uint8_t *)&v + 4); }
    void u64(uint64_t v) { b.insert(b.end(), (uint8_t *)&v, (uint8_t *)&v + 8); }
    void f32(float v) { b.insert(b.end(), (uint8_t *)&v, (uint8_t *)&v + 4); }
    void str(const std::string &s) { u64(s.size()); b.insert(b.end(), s.begin(), s.end()); }
    void kv_u32(const char *k, uint32_t v) { str(k); u32(GGUF_U32); u32(v); }
    void kv_f32(const char *k, float v) { str(k); u32(GGUF_F32); f32(v); }
    void kv_str(const char *k, const char *v) { str(k); u32(GGUF_STR); str(v); }
};

bool more_bits(int i, int n) { return i < n / 8 || i >= 7 * n / 8 || (i - n / 8) % 3 == 2; }

}  // namespace

extern "C" {

// Quantise one row of n floats (n a multiple of the block size) into dst. Exposed for tests.
int xjs_quantize_row(int type, const float *x, void *dst, long long n) {
    int b;
    int bn = type_block(type, &b);
    if (!bn || n % bn) return -1;
    quant_row(type, x, (uint8_t *)dst, n);
    return 0;
}

void xjs_default_config(xjs_config *c) {
    std::memset(c, 0, sizeof(*c));
    c->n_layer = 4; c->n_embd = 512; c->n_ff = 1408; c->n_vocab = 8192;
    c->n_head = 8; c->n_head_kv = 2; c->head_dim = 64; c->n_rot = 16;
    c->rope_base = 1e6f; c->eps = 1e-6f;
    c->conv_k = 4; c->s_k = 64; c->h_k = 4; c->h_v = 8;
    c->full_attn_interval = 4;
    c->wtype = XJ_Q8_0; c->io_type = -1; c->tied = 0; c->mtp = 0; c->fused_qkv = 0;
    c->seed = 20261201ull; c->w_std = 0.02f;
}

// Writes the model to `path`. Returns the file size in bytes, or -1 with a message in err.
long long xjs_write_gguf(const char *path, const xjs_config *c, int nthreads, char *err, int errlen) {
    const int E = c->n_embd, FF = c->n_ff, H = c->n_head, Hkv = c->n_head_kv, D = c->head_dim;
    const int S = c->s_k, Hk = c->h_k, Hv = c->h_v, DI = Hv * S, KD = Hk * S, CD = 2 * KD + DI;
    const int L = c->n_layer, V = c->n_vocab;
    if (nthreads <= 0) nthreads = (int)std::max(1u, std::thread::hardware_concurrency());
    const bool q4km = c->wtype == XJ_Q4_K;
    const int io_type = c->io_type >= 0 ? c->io_type : (q4km ? XJ_Q6_K : c->wtype);

    std::vector<Tensor> ts;
    uint64_t key = mix64(c->seed);
    auto add = [&](const std::string &name, int64_t ne0, int64_t ne1, int type, Kind kind) {
        Tensor t;
        t.name = name; t.ne0 = ne0; t.ne1 = ne1; t.type = type; t.kind = kind; t.std = c->w_std;
        t.key = mix64(key + ts.size() * 0x632be59bd9b4e019ull);
        ts.push_back(t);
    };
    auto wt = [&](int il, bool down_or_v) { return (q4km && down_or_v && more_bits(il, L)) ? (int)XJ_Q6_K : c->wtype; };

    add("token_embd.weight", E, V, io_type, K_WEIGHT);
    add("output_norm.weight", E, 1, XJ_F32, K_NORM);
    if (!c->tied) add("output.weight", E, V, io_type, K_WEIGHT);
    auto add_layer = [&](int i, bool recurrent) {
        char p[64];
        std::snprintf(p, sizeof p, "blk.%d.", i);
        std::string P(p);
        add(P + "attn_norm.weight", E, 1, XJ_F32, K_NORM);
        add(P + "post_attention_norm.weight", E, 1, XJ_F32, K_NORM);
        add(P + "ffn_gate.weight", E, FF, c->wtype, K_WEIGHT);
        add(P + "ffn_up.weight", E, FF, c->wtype, K_WEIGHT);
        add(P + "ffn_down.weight", FF, E, wt(i, true), K_WEIGHT);
        if (recurrent) {
            add(P + "attn_qkv.weight", E, CD, c->wtype, K_WEIGHT);
            add(P + "attn_gate.weight", E, DI, c->wtype, K_WEIGHT);
            add(P + "ssm_conv1d.weight", c->conv_k, CD, XJ_F32, K_CONV);
            add(P + "ssm_dt.bias", Hv, 1, XJ_F32, K_DT);
            add(P + "ssm_a", Hv, 1, XJ_F32, K_A);
            add(P + "ssm_beta.weight", E, Hv, c->wtype, K_WEIGHT);
            add(P + "ssm_alpha.weight", E, Hv, c->wtype, K_WEIGHT);
            add(P + "ssm_norm.weight", S, 1, XJ_F32, K_NORM);
            add(P + "ssm_out.weight", DI, E, c->wtype, K_WEIGHT);
        } else {
            if (c->fused_qkv) {
                add(P + "attn_qkv.weight", E, 2 * H * D + 2 * Hkv * D, c->wtype, K_WEIGHT);
            } else {
                add(P + "attn_q.weight", E, 2 * H * D, c->wtype, K_WEIGHT);
                add(P + "attn_k.weight", E, Hkv * D, c->wtype, K_WEIGHT);
                add(P + "attn_v.weight", E, Hkv * D, wt(i, true), K_WEIGHT);
            }
            add(P + "attn_output.weight", H * D, E, c->wtype, K_WEIGHT);
            add(P + "attn_q_norm.weight", D, 1, XJ_F32, K_NORM);
            add(P + "attn_k_norm.weight", D, 1, XJ_F32, K_NORM);
        }
    };
    for (int i = 0; i < L; i++) add_layer(i, (i + 1) % c->full_attn_interval != 0);
    if (c->mtp) {
        add_layer(L, false);
        char p[64];
        std::snprintf(p, sizeof p, "blk.%d.nextn.", L);
        std::string P(p);
        add(P + "eh_proj.weight", 2 * E, E, c->wtype == XJ_Q4_K ? XJ_Q8_0 : c->wtype, K_WEIGHT);
        add(P + "enorm.weight", E, 1, XJ_F32, K_NORM);
        add(P + "hnorm.weight", E, 1, XJ_F32, K_NORM);
        add(P + "shared_head_norm.weight", E, 1, XJ_F32, K_NORM);
    }
    for (auto &t : ts) {
        int b;
        int bn = type_block(t.type, &b);
        if (!bn || t.ne0 % bn) {
            std::snprintf(err, (size_t)errlen, "tensor %s: row length %lld is not a multiple of the block (%d)",
                          t.name.c_str(), (long long)t.ne0, bn);
            return -1;
        }
        t.nbytes = row_bytes(t.type, t.ne0) * (uint64_t)t.ne1;
    }

    const uint32_t ALIGN = 32;
    Writer w;
    w.u32(0x46554747u); w.u32(3);
    w.u64(ts.size());
    const int n_kv = 20 + (c->mtp ? 1 : 0);
    w.u64((uint64_t)n_kv);
    w.kv_str("general.architecture", "qwen35");
    w.kv_str("general.name", "xj-b200-synthetic");
    w.kv_u32("general.alignment", ALIGN);
    w.kv_u32("qwen35.block_count", (uint32_t)(L + (c->mtp ? 1 : 0)));
    w.kv_u32("qwen35.context_length", 32768);
    w.kv_u32("qwen35.embedding_length", (uint32_t)E);
    w.kv_u32("qwen35.feed_forward_length", (uint32_t)FF);
    w.kv_u32("qwen35.attention.head_count", (uint32_t)H);
    w.kv_u32("qwen35.attention.head_count_kv", (uint32_t)Hkv);
    w.kv_u32("qwen35.attention.key_length", (uint32_t)D);
    w.kv_u32("qwen35.attention.value_length", (uint32_t)D);
    w.kv_u32("qwen35.rope.dimension_count", (uint32_t)c->n_rot);
    w.kv_f32("qwen35.rope.freq_base", c->rope_base);
    w.kv_f32("qwen35.attention.layer_norm_rms_epsilon", c->eps);
    w.kv_u32("qwen35.ssm.conv_kernel", (uint32_t)c->conv_k);
    w.kv_u32("qwen35.ssm.inner_size", (uint32_t)DI);
    w.kv_u32("qwen35.ssm.state_size", (uint32_t)S);
    w.kv_u32("qwen35.ssm.group_count", (uint32_t)Hk);
    w.kv_u32("qwen35.ssm.time_step_rank", (uint32_t)Hv);
    w.kv_u32("qwen35.full_attention_interval", (uint32_t)c->full_attn_interval);
    if (c->mtp) w.kv_u32("qwen35.nextn_predict_layers", 1);
    uint64_t off = 0;
    for (auto &t : ts) {
        off = (off + ALIGN - 1) / ALIGN * ALIGN;
        t.offset = off;
        w.str(t.name);
        const bool one_d = t.ne1 == 1;
        w.u32(one_d ? 1 : 2);
        w.u64((uint64_t)t.ne0);
        if (!one_d) w.u64((uint64_t)t.ne1);
        w.u32((uint32_t)t.type);
        w.u64(t.offset);
        off += t.nbytes;
    }
    while (w.b.size() % ALIGN) w.b.push_back(0);
    const uint64_t data_off = w.b.size(), total = data_off + off;

    FILE *f = std::fopen(path, "wb");
    if (!f) { std::snprintf(err, (size_t)errlen, "cannot open %s for writing", path); return -1; }
    bool ok = std::fwrite(w.b.data(), 1, w.b.size(), f) == w.b.size();
    uint64_t pos = data_off;
    std::vector<uint8_t> buf;
    for (auto &t : ts) {
        if (!ok) break;
        const uint64_t at = data_off + t.offset;
        static const uint8_t zeros[64] = {0};
        while (pos < at) { ok = ok && std::fwrite(zeros, 1, (size_t)std::min<uint64_t>(64, at - pos), f) > 0; pos += std::min<uint64_t>(64, at - pos); }
        buf.assign((size_t)t.nbytes, 0);
        fill_tensor(t, buf.data(), nthreads);
        ok = ok && std::fwrite(buf.data(), 1, buf.size(), f) == buf.size();
        pos += t.nbytes;
    }
    if (std::fclose(f) != 0) ok = false;
    if (!ok) { std::snprintf(err, (size_t)errlen, "write to %s failed", path); return -1; }
    return (long long)total;
}

}  // extern "C"
