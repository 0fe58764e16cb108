/*
 * vo_oracle.c - CPU restatement of voxtral.c's inference hot path.
 *
 * TEST INFRASTRUCTURE ONLY (see vo_oracle.h).  Each function cites the
 * reference code it restates.  Parallel loops (OpenMP) only split work over
 * independent outputs (rows of a matmul, attention heads); every individual
 * reduction runs in fp32 as in the reference.
 */
#include "vo_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------
 * Seeded synthetic data: counter-based splitmix64 + Box-Muller, so any
 * element can be generated independently (and in parallel).
 * ------------------------------------------------------------------------ */

static inline uint64_t vo_mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static inline void vo_normal_pair(uint64_t seed, uint64_t j, double *a, double *b) {
    uint64_t h = vo_mix64(seed * 0xD1342543DE82EF95ull + j);
    double u1 = ((double)(h >> 40) + 1.0) / 16777217.0;          /* (0, 1] */
    double u2 = (double)((h >> 8) & 0xFFFFFFull) / 16777216.0;   /* [0, 1) */
    double r = sqrt(-2.0 * log(u1));
    *a = r * cos(6.283185307179586 * u2);
    *b = r * sin(6.283185307179586 * u2);
}

void vo_fill_normal_f32(float *out, size_t n, uint64_t seed, float mean, float std) {
    size_t pairs = (n + 1) / 2;
#pragma omp parallel for schedule(static)
    for (size_t j = 0; j < pairs; j++) {
        double a, b;
        vo_normal_pair(seed, j, &a, &b);
        out[2 * j] = (float)(mean + std * a);
        if (2 * j + 1 < n) out[2 * j + 1] = (float)(mean + std * b);
    }
}

uint16_t vo_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    u += 0x7FFFu + ((u >> 16) & 1u); /* round to nearest even */
    return (uint16_t)(u >> 16);
}

void vo_fill_normal_bf16(uint16_t *out, size_t n, uint64_t seed, float std) {
    size_t pairs = (n + 1) / 2;
#pragma omp parallel for schedule(static)
    for (size_t j = 0; j < pairs; j++) {
        double a, b;
        vo_normal_pair(seed, j, &a, &b);
        out[2 * j] = vo_f32_to_bf16((float)(std * a));
        if (2 * j + 1 < n) out[2 * j + 1] = vo_f32_to_bf16((float)(std * b));
    }
}

/* bf16 -> f32 is a 16-bit left shift (voxtral_kernels.c:124-128, 187-189). */
static inline float vo_bf16(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* ------------------------------------------------------------------------
 * Kernels (voxtral_kernels.c)
 * ------------------------------------------------------------------------ */

/* y[M,N] = x[M,K] . W[N,K]^T (+ b): the semantics of vox_linear_bf16 /
 * vox_linear_nobias_bf16 / vox_matmul_t_bf16 (voxtral_kernels.c:154-264):
 * bf16 weights widened to f32, fp32 products and sums. */
void vo_linear_bf16(float *y, const float *x, const uint16_t *W, const float *b,
                    int M, int K, int N) {
    const int RB = 16; /* output rows per block: the widened block stays in cache */
    int nblk = (N + RB - 1) / RB;
#pragma omp parallel
    {
        float *wr = (float *)malloc((size_t)RB * K * sizeof(float));
#pragma omp for schedule(static)
        for (int blk = 0; blk < nblk; blk++) {
            int o0 = blk * RB;
            int nr = N - o0 < RB ? N - o0 : RB;
            for (int r = 0; r < nr; r++) {
                const uint16_t *w = W + (size_t)(o0 + r) * K;
                for (int k = 0; k < K; k++) wr[(size_t)r * K + k] = vo_bf16(w[k]);
            }
            for (int m = 0; m < M; m++) {
                const float *xr = x + (size_t)m * K;
                for (int r = 0; r < nr; r++) {
                    const float *wrr = wr + (size_t)r * K;
                    float s = 0.0f;
#pragma omp simd reduction(+ : s)
                    for (int k = 0; k < K; k++) s += wrr[k] * xr[k];
                    y[(size_t)m * N + o0 + r] = b ? s + b[o0 + r] : s;
                }
            }
        }
        free(wr);
    }
}

/* voxtral_kernels.c:346-363 */
void vo_rms_norm(float *out, const float *x, const float *w, int M, int dim, float eps) {
    for (int m = 0; m < M; m++) {
        const float *xr = x + (size_t)m * dim;
        float *o = out + (size_t)m * dim;
        float ss = 0.0f;
        for (int i = 0; i < dim; i++) ss += xr[i] * xr[i];
        float inv = 1.0f / sqrtf(ss / (float)dim + eps);
        for (int i = 0; i < dim; i++) o[i] = xr[i] * inv * w[i];
    }
}

/* voxtral_kernels.c:369-374 */
void vo_silu(float *x, size_t n) {
    for (size_t i = 0; i < n; i++) x[i] = x[i] / (1.0f + expf(-x[i]));
}

/* tanh-approximated GELU, voxtral_kernels.c:376-384 */
void vo_gelu(float *x, size_t n) {
    for (size_t i = 0; i < n; i++) {
        float v = x[i];
        float t = 0.7978845608028654f * (v + 0.044715f * v * v * v);
        x[i] = 0.5f * v * (1.0f + tanhf(t));
    }
}

/* voxtral_kernels.c:488-500: freqs[s][d] = (cos, sin)(pos * theta^(-2d/dim)) */
void vo_rope_freqs(float *freqs, const int *pos, int seq, int dim, float theta) {
    int half = dim / 2;
    for (int s = 0; s < seq; s++) {
        float p = (float)pos[s];
        for (int d = 0; d < half; d++) {
            float f = 1.0f / powf(theta, (float)(2 * d) / (float)dim);
            float a = p * f;
            freqs[(size_t)s * dim + 2 * d] = cosf(a);
            freqs[(size_t)s * dim + 2 * d + 1] = sinf(a);
        }
    }
}

/* Interleaved-pair rotation, voxtral_kernels.c:502-526 */
void vo_apply_rope(float *x, const float *freqs, int seq, int heads, int head_dim) {
    int half = head_dim / 2;
    for (int s = 0; s < seq; s++) {
        const float *f = freqs + (size_t)s * head_dim;
        for (int h = 0; h < heads; h++) {
            float *v = x + ((size_t)s * heads + h) * head_dim;
            for (int d = 0; d < half; d++) {
                float c = f[2 * d], sn = f[2 * d + 1];
                float a = v[2 * d], b = v[2 * d + 1];
                v[2 * d] = a * c - b * sn;
                v[2 * d + 1] = a * sn + b * c;
            }
        }
    }
}

/* Online-softmax causal attention with sliding window and GQA,
 * voxtral_kernels.c:412-482.  Keys j in [max(0, g-window+1), min(g+1, seq_k))
 * for the query at global position g = q_offset + i. */
void vo_causal_attention(float *out, const float *Q, const float *K, const float *V,
                         int seq_q, int seq_k, int n_heads, int n_kv_heads,
                         int head_dim, float scale, int window, int q_offset) {
    int group = n_heads / n_kv_heads;
    size_t qh = (size_t)n_heads * head_dim, kvh = (size_t)n_kv_heads * head_dim;
#pragma omp parallel for collapse(2) schedule(static)
    for (int h = 0; h < n_heads; h++) {
        for (int i = 0; i < seq_q; i++) {
            int kvhead = h / group;
            const float *q = Q + i * qh + (size_t)h * head_dim;
            float *o = out + i * qh + (size_t)h * head_dim;
            int g = q_offset + i;
            int k0 = (window > 0 && g - window + 1 > 0) ? g - window + 1 : 0;
            int k1 = g + 1 < seq_k ? g + 1 : seq_k;
            float mx = -1e30f, den = 0.0f;
            for (int d = 0; d < head_dim; d++) o[d] = 0.0f;
            for (int j = k0; j < k1; j++) {
                const float *kr = K + j * kvh + (size_t)kvhead * head_dim;
                const float *vr = V + j * kvh + (size_t)kvhead * head_dim;
                float s = 0.0f;
                for (int d = 0; d < head_dim; d++) s += q[d] * kr[d];
                s *= scale;
                if (s > mx) {
                    float c = expf(mx - s);
                    den = den * c + 1.0f;
                    for (int d = 0; d < head_dim; d++) o[d] = o[d] * c + vr[d];
                    mx = s;
                } else {
                    float wgt = expf(s - mx);
                    den += wgt;
                    for (int d = 0; d < head_dim; d++) o[d] += wgt * vr[d];
                }
            }
            if (den > 0.0f) {
                float inv = 1.0f / den;
                for (int d = 0; d < head_dim; d++) o[d] *= inv;
            }
        }
    }
}

/* First maximum, strict '>' (voxtral_decoder.c:507-515). */
int vo_argmax(const float *x, int n) {
    int best = 0;
    float bv = x[0];
    for (int i = 1; i < n; i++)
        if (x[i] > bv) { bv = x[i]; best = i; }
    return best;
}

/* Alternatives for --alt (voxtral.c:778-833): softmax over all logits, then
 * up to n_alt-1 repeated scans over ids >= 1000 (skipping the best token and
 * ids already picked) for the highest probability; a candidate is accepted
 * while 1 - p/p_best <= cutoff.  Returns the number of ids written (>= 1). */
int vo_fill_alts(const float *logits, int n, int best, int n_alt, float cutoff,
                 int *alt_ids) {
    alt_ids[0] = best;
    if (n_alt <= 1) return 1;
    float *p = (float *)malloc((size_t)n * sizeof(float));
    float mx = logits[0];
    for (int i = 1; i < n; i++)
        if (logits[i] > mx) mx = logits[i];
    float sum = 0.0f;
    for (int i = 0; i < n; i++) {
        p[i] = expf(logits[i] - mx);
        sum += p[i];
    }
    float inv = 1.0f / sum;
    for (int i = 0; i < n; i++) p[i] *= inv;
    float pb = p[best];
    int found = 1;
    if (pb > 0.0f) {
        while (found < n_alt) {
            int bi = -1;
            float bp = -1.0f;
            for (int i = 1000; i < n; i++) {
                if (i == best) continue;
                int used = 0;
                for (int j = 1; j < found; j++)
                    if (alt_ids[j] == i) { used = 1; break; }
                if (used) continue;
                if (p[i] > bp) { bp = p[i]; bi = i; }
            }
            if (bi < 0) break;
            if (1.0f - bp / pb > cutoff) break;
            alt_ids[found++] = bi;
        }
    }
    free(p);
    return found;
}

/* ------------------------------------------------------------------------
 * Decoder (voxtral_decoder.c)
 * ------------------------------------------------------------------------ */

#define VO_Q_DIM (VO_DEC_HEADS * VO_DEC_HEAD_DIM)       /* 4096 */
#define VO_KV_DIM (VO_DEC_KV_HEADS * VO_DEC_HEAD_DIM)   /* 1024 */

static float *vo_kv_row(float *base, const vo_dec_kv_t *kv, int layer, int pos) {
    return base + ((size_t)layer * kv->max + pos) * VO_KV_DIM;
}

/* Keep the newest VO_DEC_WINDOW rows at physical 0 and advance the logical
 * offset (voxtral_decoder.c:208-227). */
static void vo_dec_compact(int n_layers, vo_dec_kv_t *kv) {
    int keep = VO_DEC_WINDOW;
    if (kv->len <= keep) return;
    int discard = kv->len - keep;
    for (int l = 0; l < n_layers; l++) {
        memmove(vo_kv_row(kv->k, kv, l, 0), vo_kv_row(kv->k, kv, l, discard),
                (size_t)keep * VO_KV_DIM * sizeof(float));
        memmove(vo_kv_row(kv->v, kv, l, 0), vo_kv_row(kv->v, kv, l, discard),
                (size_t)keep * VO_KV_DIM * sizeof(float));
    }
    kv->pos_offset += discard;
    kv->len = keep;
}

/* One decoder layer over M rows at physical start position `start`
 * (voxtral_decoder.c:281-366 for M>1, :463-500 for M=1). */
static void vo_dec_layer(const vo_dec_model_t *m, vo_dec_kv_t *kv, int layer,
                         float *x, int M, int start, const float *freqs) {
    const uint16_t *const *w = m->lw + 7 * layer;
    const float *an = m->ln[2 * layer], *fn = m->ln[2 * layer + 1];
    int dim = VO_DEC_DIM, hid = VO_DEC_HIDDEN;
    float *xn = (float *)malloc((size_t)M * dim * sizeof(float));
    float *q = (float *)malloc((size_t)M * VO_Q_DIM * sizeof(float));
    float *k = (float *)malloc((size_t)M * VO_KV_DIM * sizeof(float));
    float *v = (float *)malloc((size_t)M * VO_KV_DIM * sizeof(float));
    float *att = (float *)malloc((size_t)M * VO_Q_DIM * sizeof(float));
    float *proj = (float *)malloc((size_t)M * dim * sizeof(float));
    float *gate = (float *)malloc((size_t)M * hid * sizeof(float));
    float *up = (float *)malloc((size_t)M * hid * sizeof(float));

    vo_rms_norm(xn, x, an, M, dim, VO_NORM_EPS);
    vo_linear_bf16(q, xn, w[0], NULL, M, dim, VO_Q_DIM);
    vo_linear_bf16(k, xn, w[1], NULL, M, dim, VO_KV_DIM);
    vo_linear_bf16(v, xn, w[2], NULL, M, dim, VO_KV_DIM);
    vo_apply_rope(q, freqs, M, VO_DEC_HEADS, VO_DEC_HEAD_DIM);
    vo_apply_rope(k, freqs, M, VO_DEC_KV_HEADS, VO_DEC_HEAD_DIM);
    for (int s = 0; s < M; s++) {
        memcpy(vo_kv_row(kv->k, kv, layer, start + s), k + (size_t)s * VO_KV_DIM,
               VO_KV_DIM * sizeof(float));
        memcpy(vo_kv_row(kv->v, kv, layer, start + s), v + (size_t)s * VO_KV_DIM,
               VO_KV_DIM * sizeof(float));
    }
    vo_causal_attention(att, q, vo_kv_row(kv->k, kv, layer, 0),
                        vo_kv_row(kv->v, kv, layer, 0), M, start + M, VO_DEC_HEADS,
                        VO_DEC_KV_HEADS, VO_DEC_HEAD_DIM,
                        1.0f / sqrtf((float)VO_DEC_HEAD_DIM), VO_DEC_WINDOW, start);
    vo_linear_bf16(proj, att, w[3], NULL, M, VO_Q_DIM, dim);
    for (size_t i = 0; i < (size_t)M * dim; i++) x[i] += proj[i];

    vo_rms_norm(xn, x, fn, M, dim, VO_NORM_EPS);
    if (m->ada_scale) {
        const float *ada = m->ada_scale + (size_t)layer * dim;
        for (int s = 0; s < M; s++)
            for (int i = 0; i < dim; i++) xn[(size_t)s * dim + i] *= (1.0f + ada[i]);
    }
    vo_linear_bf16(gate, xn, w[4], NULL, M, dim, hid);
    vo_silu(gate, (size_t)M * hid);
    vo_linear_bf16(up, xn, w[6], NULL, M, dim, hid);
    for (size_t i = 0; i < (size_t)M * hid; i++) gate[i] *= up[i];
    vo_linear_bf16(proj, gate, w[5], NULL, M, hid, dim);
    for (size_t i = 0; i < (size_t)M * dim; i++) x[i] += proj[i];

    free(xn); free(q); free(k); free(v); free(att); free(proj); free(gate); free(up);
}

/* Single-token decode step, voxtral_decoder.c:401-516.  Returns the argmax
 * token, or -1 when the caller-owned cache cannot hold the next row (the
 * reference would grow its heap cache there). */
int vo_decoder_step(const vo_dec_model_t *m, vo_dec_kv_t *kv, const float *embed,
                    float *logits) {
    int dim = VO_DEC_DIM;
    int pos = kv->len;
    if (pos >= kv->max) {
        if (kv->len > VO_DEC_WINDOW) {
            vo_dec_compact(m->n_layers, kv);
            pos = kv->len;
        }
        if (pos >= kv->max) return -1;
    }
    int logical = kv->pos_offset + pos;
    float freqs[VO_DEC_HEAD_DIM];
    vo_rope_freqs(freqs, &logical, 1, VO_DEC_HEAD_DIM, VO_ROPE_THETA);

    float *x = (float *)malloc(dim * sizeof(float));
    memcpy(x, embed, dim * sizeof(float));
    for (int l = 0; l < m->n_layers; l++) vo_dec_layer(m, kv, l, x, 1, pos, freqs);
    kv->len = pos + 1;

    vo_rms_norm(x, x, m->norm, 1, dim, VO_NORM_EPS);
    vo_linear_bf16(logits, x, m->tok_emb, NULL, 1, dim, m->vocab);
    free(x);
    return vo_argmax(logits, m->vocab);
}

/* Multi-row prefill, voxtral_decoder.c:233-373.  Returns 0, or -1 when the
 * caller-owned cache is too small. */
int vo_decoder_prefill(const vo_dec_model_t *m, vo_dec_kv_t *kv,
                       const float *embeds, int seq_len) {
    int dim = VO_DEC_DIM;
    if (kv->len + seq_len > kv->max) return -1;
    int start = kv->len;
    int *pos = (int *)malloc((size_t)seq_len * sizeof(int));
    for (int i = 0; i < seq_len; i++) pos[i] = kv->pos_offset + start + i;
    float *freqs = (float *)malloc((size_t)seq_len * VO_DEC_HEAD_DIM * sizeof(float));
    vo_rope_freqs(freqs, pos, seq_len, VO_DEC_HEAD_DIM, VO_ROPE_THETA);
    float *x = (float *)malloc((size_t)seq_len * dim * sizeof(float));
    memcpy(x, embeds, (size_t)seq_len * dim * sizeof(float));
    for (int l = 0; l < m->n_layers; l++) vo_dec_layer(m, kv, l, x, seq_len, start, freqs);
    kv->len = start + seq_len;
    free(x); free(freqs); free(pos);
    return 0;
}

/* ------------------------------------------------------------------------
 * Encoder + adapter (voxtral_encoder.c)
 * ------------------------------------------------------------------------ */

#define VO_ENC_QKV (VO_ENC_HEADS * VO_ENC_HEAD_DIM) /* 2048 */

static float *vo_ekv_row(float *base, const vo_enc_kv_t *kv, int layer, int pos) {
    return base + ((size_t)layer * kv->max + pos) * VO_ENC_QKV;
}

/* voxtral_encoder.c:388-406 */
static void vo_enc_compact(int n_layers, vo_enc_kv_t *kv) {
    int keep = VO_ENC_WINDOW;
    if (kv->len <= keep) return;
    int discard = kv->len - keep;
    for (int l = 0; l < n_layers; l++) {
        memmove(vo_ekv_row(kv->k, kv, l, 0), vo_ekv_row(kv->k, kv, l, discard),
                (size_t)keep * VO_ENC_QKV * sizeof(float));
        memmove(vo_ekv_row(kv->v, kv, l, 0), vo_ekv_row(kv->v, kv, l, discard),
                (size_t)keep * VO_ENC_QKV * sizeof(float));
    }
    kv->pos_offset += discard;
    kv->len = keep;
}

/* Incremental encoder over new_len rows, in place on x [new_len, 1280]
 * (voxtral_encoder.c:452-636).  Returns new_len, or -1 when the caller-owned
 * cache is too small. */
int vo_encoder_step(const vo_enc_model_t *m, vo_enc_kv_t *kv, float *x, int new_len) {
    int dim = VO_ENC_DIM, hid = VO_ENC_HIDDEN, M = new_len;
    if (M <= 0) return 0;
    if (kv->len + M > VO_ENC_WINDOW) vo_enc_compact(m->n_layers, kv);
    if (kv->len + M > kv->max) return -1;
    int cache_len = kv->len;
    int *pos = (int *)malloc((size_t)M * sizeof(int));
    for (int i = 0; i < M; i++) pos[i] = kv->pos_offset + cache_len + i;
    float *freqs = (float *)malloc((size_t)M * VO_ENC_HEAD_DIM * sizeof(float));
    vo_rope_freqs(freqs, pos, M, VO_ENC_HEAD_DIM, VO_ROPE_THETA);

    float *xn = (float *)malloc((size_t)M * dim * sizeof(float));
    float *q = (float *)malloc((size_t)M * VO_ENC_QKV * sizeof(float));
    float *k = (float *)malloc((size_t)M * VO_ENC_QKV * sizeof(float));
    float *v = (float *)malloc((size_t)M * VO_ENC_QKV * sizeof(float));
    float *att = (float *)malloc((size_t)M * VO_ENC_QKV * sizeof(float));
    float *proj = (float *)malloc((size_t)M * dim * sizeof(float));
    float *gate = (float *)malloc((size_t)M * hid * sizeof(float));
    float *up = (float *)malloc((size_t)M * hid * sizeof(float));

    for (int l = 0; l < m->n_layers; l++) {
        const uint16_t *const *w = m->lw + 7 * l;
        const float *const *b = m->lb + 4 * l;
        vo_rms_norm(xn, x, m->ln[2 * l], M, dim, VO_NORM_EPS);
        vo_linear_bf16(q, xn, w[0], b[0], M, dim, VO_ENC_QKV);
        vo_linear_bf16(k, xn, w[1], NULL, M, dim, VO_ENC_QKV);
        vo_linear_bf16(v, xn, w[2], b[1], M, dim, VO_ENC_QKV);
        vo_apply_rope(q, freqs, M, VO_ENC_HEADS, VO_ENC_HEAD_DIM);
        vo_apply_rope(k, freqs, M, VO_ENC_HEADS, VO_ENC_HEAD_DIM);
        for (int s = 0; s < M; s++) {
            memcpy(vo_ekv_row(kv->k, kv, l, cache_len + s), k + (size_t)s * VO_ENC_QKV,
                   VO_ENC_QKV * sizeof(float));
            memcpy(vo_ekv_row(kv->v, kv, l, cache_len + s), v + (size_t)s * VO_ENC_QKV,
                   VO_ENC_QKV * sizeof(float));
        }
        vo_causal_attention(att, q, vo_ekv_row(kv->k, kv, l, 0), vo_ekv_row(kv->v, kv, l, 0),
                            M, cache_len + M, VO_ENC_HEADS, VO_ENC_HEADS, VO_ENC_HEAD_DIM,
                            1.0f / sqrtf((float)VO_ENC_HEAD_DIM), VO_ENC_WINDOW, cache_len);
        vo_linear_bf16(proj, att, w[3], b[2], M, VO_ENC_QKV, dim);
        for (size_t i = 0; i < (size_t)M * dim; i++) x[i] += proj[i];
        vo_rms_norm(xn, x, m->ln[2 * l + 1], M, dim, VO_NORM_EPS);
        vo_linear_bf16(gate, xn, w[4], NULL, M, dim, hid);
        vo_silu(gate, (size_t)M * hid);
        vo_linear_bf16(up, xn, w[6], NULL, M, dim, hid);
        for (size_t i = 0; i < (size_t)M * hid; i++) gate[i] *= up[i];
        vo_linear_bf16(proj, gate, w[5], b[3], M, hid, dim);
        for (size_t i = 0; i < (size_t)M * dim; i++) x[i] += proj[i];
    }
    vo_rms_norm(x, x, m->norm, M, dim, VO_NORM_EPS);
    kv->len = cache_len + M;
    free(xn); free(q); free(k); free(v); free(att); free(proj); free(gate); free(up);
    free(freqs); free(pos);
    return M;
}

/* 4x frame stacking + Linear(5120->3072) -> GELU -> Linear(3072->3072),
 * voxtral_encoder.c:642-674.  Stacking 4 consecutive [1280] rows is the same
 * memory as one [5120] row, so enc is used as [n/4, 5120] directly. */
int vo_adapter(const uint16_t *l0, const uint16_t *l1, const float *enc, int n,
               float *out) {
    int rows = n / 4;
    if (rows <= 0) return 0;
    float *mid = (float *)malloc((size_t)rows * VO_DEC_DIM * sizeof(float));
    vo_linear_bf16(mid, enc, l0, NULL, rows, 4 * VO_ENC_DIM, VO_DEC_DIM);
    vo_gelu(mid, (size_t)rows * VO_DEC_DIM);
    vo_linear_bf16(out, mid, l1, NULL, rows, VO_DEC_DIM, VO_DEC_DIM);
    free(mid);
    return rows;
}
