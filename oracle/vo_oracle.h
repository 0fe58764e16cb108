/*
 * vo_oracle.h - CPU restatement of voxtral.c's inference hot path.
 *
 * TEST INFRASTRUCTURE ONLY: this library is the checker the CUDA path is
 * compared against (tests/, __graft_entry__.smoke() and the cpu_baseline leg
 * of bench.py).  The product never links or calls it.
 *
 * Every function restates the reference algorithm it names (file:line in the
 * reference tree).  The restatement is pinned against the compiled reference
 * (oracle/_ref/libvoxref.so) by the golden vectors in tests/golden/.
 */
#ifndef VO_ORACLE_H
#define VO_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VO_DEC_DIM 3072
#define VO_DEC_HEADS 32
#define VO_DEC_KV_HEADS 8
#define VO_DEC_HEAD_DIM 128
#define VO_DEC_HIDDEN 9216
#define VO_DEC_WINDOW 8192
#define VO_ENC_DIM 1280
#define VO_ENC_HEADS 32
#define VO_ENC_HEAD_DIM 64
#define VO_ENC_HIDDEN 5120
#define VO_ENC_WINDOW 750
#define VO_NORM_EPS 1e-5f
#define VO_ROPE_THETA 1000000.0f

/* ---- seeded synthetic data ---- */
void vo_fill_normal_f32(float *out, size_t n, uint64_t seed, float mean, float std);
void vo_fill_normal_bf16(uint16_t *out, size_t n, uint64_t seed, float std);
uint16_t vo_f32_to_bf16(float f);

/* ---- kernels (voxtral_kernels.c) ---- */
void vo_linear_bf16(float *y, const float *x, const uint16_t *W, const float *b,
                    int M, int K, int N);
void vo_rms_norm(float *out, const float *x, const float *w, int M, int dim, float eps);
void vo_silu(float *x, size_t n);
void vo_gelu(float *x, size_t n);
void vo_rope_freqs(float *freqs, const int *pos, int seq, int dim, float theta);
void vo_apply_rope(float *x, const float *freqs, int seq, int heads, int head_dim);
void vo_causal_attention(float *out, const float *Q, const float *K, const float *V,
                         int seq_q, int seq_k, int n_heads, int n_kv_heads,
                         int head_dim, float scale, int window, int q_offset);
int vo_argmax(const float *x, int n);
int vo_fill_alts(const float *logits, int n, int best, int n_alt, float cutoff,
                 int *alt_ids);

/* ---- decoder (voxtral_decoder.c) ---- */
typedef struct {
    int n_layers;                 /* 26 for the real model */
    int vocab;                    /* 131072 for the real model */
    const uint16_t *tok_emb;      /* [vocab, 3072] bf16 */
    const float *norm;            /* [3072] */
    const float *ada_scale;       /* [n_layers*3072] or NULL */
    const uint16_t *const *lw;    /* n_layers x {wq, wk, wv, wo, w1, w2, w3} */
    const float *const *ln;       /* n_layers x {attention_norm, ffn_norm} */
} vo_dec_model_t;

typedef struct {
    float *k, *v;                 /* [n_layers, max, 1024] */
    int max;                      /* physical capacity (rows per layer) */
    int len;                      /* physical length */
    int pos_offset;               /* logical offset from compaction */
} vo_dec_kv_t;

int vo_decoder_step(const vo_dec_model_t *m, vo_dec_kv_t *kv, const float *embed,
                    float *logits);
int vo_decoder_prefill(const vo_dec_model_t *m, vo_dec_kv_t *kv,
                       const float *embeds, int seq_len);

/* ---- encoder + adapter (voxtral_encoder.c) ---- */
typedef struct {
    int n_layers;                 /* 32 for the real model */
    const uint16_t *const *lw;    /* n_layers x {wq, wk, wv, wo, w1, w2, w3} */
    const float *const *lb;       /* n_layers x {wq_bias, wv_bias, wo_bias, w2_bias} */
    const float *const *ln;       /* n_layers x {attention_norm, ffn_norm} */
    const float *norm;            /* [1280] */
} vo_enc_model_t;

typedef struct {
    float *k, *v;                 /* [n_layers, max, 2048] */
    int max, len, pos_offset;
} vo_enc_kv_t;

int vo_encoder_step(const vo_enc_model_t *m, vo_enc_kv_t *kv, float *x, int new_len);
int vo_adapter(const uint16_t *l0, const uint16_t *l1, const float *enc, int n,
               float *out);

#ifdef __cplusplus
}
#endif
#endif
