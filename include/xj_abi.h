// Binary interface shared with the xiaoju-pipe runtime.
//
// The CUDA stage is a drop-in replacement for the Metal stage, so it must read the runtime's model
// structs and fill the runtime's stage vtable with exactly the runtime's memory layout. This header
// restates those public structs field for field (same order, same C types, so the same offsets under
// the x86-64 / aarch64 SysV ABI). tests/test_abi.py checks every size and offset listed in
// oracle/ref_harness.c:xjr_abi against the reference build.
//
//   gguf_tensor / gguf_kv / gguf_file   src/xiaoju-pipe/core/gguf.h:24-53
//   enum xj_type / enum gguf_vtype      src/xiaoju-pipe/core/gguf.h:13-22
//   xj_w                                src/xiaoju-pipe/core/xj_model.h:13-19
//   xj_layer                            src/xiaoju-pipe/core/xj_model.h:21-31
//   xj_hparams                          src/xiaoju-pipe/core/xj_model.h:33-46
//   xj_model                            src/xiaoju-pipe/core/xj_model.h:48-61
//   xj_stage (vtable + state)           src/xiaoju-pipe/core/xj_stage.h:13-39
//
// Everything here is plain C (no CUDA, no C++ types), so a C host, cgo or ctypes can include it.
#pragma once
#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#ifndef XJ_MAX_LAYERS
#define XJ_MAX_LAYERS 128  // capacity of xj_model.layers (xj_model.h:10)
#endif

// ggml tensor type ids used by GGUF (the subset the runtime accepts, xj_model.c:16-17, plus the
// ids its block table knows, gguf.c:12-32).
enum xj_type {
    XJ_F32 = 0, XJ_F16 = 1, XJ_Q4_0 = 2, XJ_Q4_1 = 3, XJ_Q5_0 = 6, XJ_Q5_1 = 7,
    XJ_Q8_0 = 8, XJ_Q2_K = 10, XJ_Q3_K = 11, XJ_Q4_K = 12, XJ_Q5_K = 13, XJ_Q6_K = 14,
    XJ_BF16 = 30,
};

// GGUF metadata value types (GGUF v2/v3).
enum gguf_vtype {
    GGUF_U8 = 0, GGUF_I8, GGUF_U16, GGUF_I16, GGUF_U32, GGUF_I32, GGUF_F32, GGUF_BOOL,
    GGUF_STR, GGUF_ARR, GGUF_U64, GGUF_I64, GGUF_F64,
};

typedef struct {
    const char *name;
    uint32_t    n_dims;
    int64_t     ne[4];    // ne[0] = elements per row
    uint32_t    type;     // enum xj_type
    uint64_t    offset;   // relative to the data section
    uint64_t    nbytes;
} gguf_tensor;

typedef struct {
    const char    *key;
    uint32_t       type;      // enum gguf_vtype
    uint32_t       arr_type;  // element type when type == GGUF_ARR
    uint64_t       arr_n;
    const uint8_t *data;      // value bytes inside the header
} gguf_kv;

typedef struct {
    int            fd;
    const uint8_t *map;       // read-only mapping; covers file bytes [map_off, map_off + map_len)
    uint64_t       map_off, map_len;
    uint8_t       *hdr;       // header copy when only a range is mapped
    uint64_t       size;      // file size
    uint64_t       data_off;  // file offset of the tensor data section
    uint32_t       alignment;
    uint64_t       n_kv, n_tensors;
    gguf_kv       *kv;
    gguf_tensor   *tensors;
    char          *strpool;
} gguf_file;

// One weight: points into the mapped file. ne0 = input dim (row length), ne1 = output dim (rows).
typedef struct {
    const void *data;
    uint64_t    file_off;  // absolute file offset
    uint64_t    nbytes;
    uint32_t    type;      // enum xj_type
    int64_t     ne0, ne1;
} xj_w;

typedef struct {
    bool recurrent;        // true: Gated DeltaNet layer; false: gated full attention
    xj_w attn_norm, post_norm;
    xj_w wqkv;             // fused q|k|v (optional)
    xj_w wq, wk, wv, wo, q_norm, k_norm;
    xj_w ssm_qkv, ssm_gate, ssm_conv1d, ssm_dt, ssm_a, ssm_beta, ssm_alpha, ssm_norm, ssm_out;
    xj_w ffn_gate, ffn_up, ffn_down;
} xj_layer;

typedef struct {
    int   n_layer, n_embd, n_ff, n_vocab;
    int   n_head, n_head_kv, head_dim;
    int   n_rot;
    float rope_base, eps;
    int   conv_k;
    int   d_inner;
    int   s_k;
    int   h_k, h_v;
    int   s_v;
    int   key_dim, conv_dim;
    int   full_attn_interval;
    uint32_t eos, eot;
} xj_hparams;

typedef struct {
    gguf_file *gguf;
    xj_hparams hp;
    xj_w tok_embd, output_norm, output;   // output == tok_embd when tied
    xj_layer layers[XJ_MAX_LAYERS];       // layers[n_layer] holds the MTP layer when has_mtp
    uint64_t fingerprint;
    bool has_mtp;
    xj_w mtp_eh, mtp_enorm, mtp_hnorm, mtp_head_norm;
    gguf_file *mtp_gguf;
} xj_model;

typedef struct xj_stage xj_stage;

// A contiguous layer range [l0, l1) of one model on one device. All buffers passed to the function
// pointers are caller-owned HOST memory; x is [T][n_embd] fp32 (MTP stage: [T][2*n_embd] in,
// [T][n_embd] out), logits is [T][n_vocab] fp32. Functions return 0 or -1 with a message in err.
struct xj_stage {
    const xj_model *m;
    int l0, l1;
    int n_ctx;
    int max_batch;
    int n_past;
    bool has_head;
    bool mtp;
    const char *backend;   // "cpu" / "metal" / "cuda"
    int keep;              // one-shot: checkpoint recurrent state after each token of the next forward
    int ck_start, ck_T;
    int  (*forward)(xj_stage *s, float *x, int T, char *err, size_t errlen);
    int  (*logits)(xj_stage *s, const float *x, int T, float *logits, char *err, size_t errlen);
    int  (*rollback)(xj_stage *s, int n_past, char *err, size_t errlen);
    void (*reset)(xj_stage *s);
    void (*destroy)(xj_stage *s);
    void *impl;
};

#ifdef __cplusplus
}
#endif
