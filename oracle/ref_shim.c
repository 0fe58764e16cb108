/*
 * ref_shim.c - glue that lets tests drive the reference's own CPU path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is compiled together with the
 * unmodified reference sources (voxtral.c through the #include below, plus
 * voxtral_kernels.c, voxtral_decoder.c, voxtral_encoder.c, voxtral_audio.c,
 * voxtral_tokenizer.c and voxtral_safetensors.c, all read in place from the
 * reference tree) into oracle/_ref/libvoxref.so by oracle/Makefile.  It builds a
 * reference context (vox_ctx_t, voxtral.h:154-201) from caller-owned weight
 * arrays instead of an mmap'd safetensors file, so the reference's own
 * vox_decoder_forward / vox_decoder_prefill / vox_encoder_forward_incremental
 * / vox_adapter_forward can be run on seeded synthetic weights.  Nothing in
 * the product links this library.
 */
/* voxtral.c is compiled as part of this translation unit so that its static
 * helpers (stream_fill_alts, vox_update_time_conditioning) can be called.
 * Its calls to the tokenizer's decode are routed to a stand-in that returns
 * base + token_id, so the ids picked by stream_fill_alts can be read back
 * without a tekken.json. */
#define vox_tokenizer_decode voxref_fake_tokenizer_decode
#include "voxtral.c"
#undef vox_tokenizer_decode

#include <pthread.h>
#include <time.h>

static char voxref_fake_vocab[VOX_VOCAB_SIZE];

const char *voxref_fake_tokenizer_decode(vox_tokenizer_t *tok, int token_id) {
    (void)tok;
    if (token_id < 0 || token_id >= VOX_VOCAB_SIZE) return NULL;
    return voxref_fake_vocab + token_id;
}

/* Runs the reference's stream_fill_alts (voxtral.c:778-833) on a logits
 * buffer (softmaxed in place, as the reference does) and writes the chosen
 * ids to alt_ids[0..VOX_MAX_ALT) (-1 where none).  Returns the count. */
int voxref_fill_alts(float *logits, int best, int n_alt, float cutoff, int *alt_ids) {
    vox_stream_t s;
    memset(&s, 0, sizeof(s));
    s.logits = logits;
    s.n_alt = n_alt;
    s.alt_cutoff = cutoff;
    const char *alts[VOX_MAX_ALT];
    stream_fill_alts(&s, best, alts);
    int n = 0;
    for (int i = 0; i < VOX_MAX_ALT; i++) {
        alt_ids[i] = alts[i] ? (int)(alts[i] - voxref_fake_vocab) : -1;
        if (alts[i]) n++;
    }
    return n;
}

/* Runs vox_update_time_conditioning (voxtral.c:46-79) for delay_tokens and
 * returns ctx->ada_scale ([VOX_DEC_LAYERS*VOX_DEC_DIM], owned by ctx; freed
 * by voxref_ctx_free).  Needs the per-layer ada_norm_down/up set first. */
const float *voxref_time_conditioning(vox_ctx_t *ctx, int delay_tokens) {
    ctx->delay_tokens = delay_tokens;
    vox_update_time_conditioning(ctx);
    return ctx->ada_scale;
}

void voxref_set_ada_mlp(vox_ctx_t *ctx, int layer, const float *down, const float *up) {
    ctx->decoder.layers[layer].ada_norm_down = (float *)down;
    ctx->decoder.layers[layer].ada_norm_up = (float *)up;
}

vox_ctx_t *voxref_ctx_new(void) {
    vox_ctx_t *ctx = (vox_ctx_t *)calloc(1, sizeof(vox_ctx_t));
    if (!ctx) return NULL;
    ctx->use_bf16 = 1;
    ctx->delay_tokens = 6;
    return ctx;
}

/* lw: VOX_DEC_LAYERS x {wq, wk, wv, wo, w1, w2, w3}; ln: VOX_DEC_LAYERS x
 * {attention_norm, ffn_norm}; ada_scale: [VOX_DEC_LAYERS*VOX_DEC_DIM] or NULL
 * (the per-layer ada scale the reference precomputes at voxtral.c:46-79). */
void voxref_set_decoder(vox_ctx_t *ctx, const uint16_t *tok_emb,
                        const float *final_norm, const uint16_t *const *lw,
                        const float *const *ln, const float *ada_scale) {
    vox_decoder_t *d = &ctx->decoder;
    d->tok_embeddings_bf16 = (uint16_t *)tok_emb;
    d->norm = (float *)final_norm;
    for (int i = 0; i < VOX_DEC_LAYERS; i++) {
        vox_dec_layer_t *l = &d->layers[i];
        const uint16_t *const *w = lw + 7 * i;
        l->wq_weight_bf16 = (uint16_t *)w[0];
        l->wk_weight_bf16 = (uint16_t *)w[1];
        l->wv_weight_bf16 = (uint16_t *)w[2];
        l->wo_weight_bf16 = (uint16_t *)w[3];
        l->w1_weight_bf16 = (uint16_t *)w[4];
        l->w2_weight_bf16 = (uint16_t *)w[5];
        l->w3_weight_bf16 = (uint16_t *)w[6];
        l->attention_norm = (float *)ln[2 * i];
        l->ffn_norm = (float *)ln[2 * i + 1];
    }
    ctx->ada_scale = (float *)ada_scale;
}

/* lw: VOX_ENC_LAYERS x {wq, wk, wv, wo, w1, w2, w3}; lb: VOX_ENC_LAYERS x
 * {wq_bias, wv_bias, wo_bias, w2_bias}; ln: VOX_ENC_LAYERS x {attention_norm,
 * ffn_norm}. */
void voxref_set_encoder(vox_ctx_t *ctx, const uint16_t *const *lw,
                        const float *const *lb, const float *const *ln,
                        const float *final_norm) {
    vox_encoder_t *e = &ctx->encoder;
    for (int i = 0; i < VOX_ENC_LAYERS; i++) {
        vox_enc_layer_t *l = &e->layers[i];
        const uint16_t *const *w = lw + 7 * i;
        l->wq_weight_bf16 = (uint16_t *)w[0];
        l->wk_weight_bf16 = (uint16_t *)w[1];
        l->wv_weight_bf16 = (uint16_t *)w[2];
        l->wo_weight_bf16 = (uint16_t *)w[3];
        l->w1_weight_bf16 = (uint16_t *)w[4];
        l->w2_weight_bf16 = (uint16_t *)w[5];
        l->w3_weight_bf16 = (uint16_t *)w[6];
        l->wq_bias = (float *)lb[4 * i + 0];
        l->wv_bias = (float *)lb[4 * i + 1];
        l->wo_bias = (float *)lb[4 * i + 2];
        l->w2_bias = (float *)lb[4 * i + 3];
        l->attention_norm = (float *)ln[2 * i];
        l->ffn_norm = (float *)ln[2 * i + 1];
    }
    e->norm = (float *)final_norm;
}

void voxref_set_adapter(vox_ctx_t *ctx, const uint16_t *l0, const uint16_t *l1) {
    ctx->adapter.linear0_weight_bf16 = (uint16_t *)l0;
    ctx->adapter.linear1_weight_bf16 = (uint16_t *)l1;
}

int voxref_decoder_forward(vox_ctx_t *ctx, const float *embed, float *logits) {
    return vox_decoder_forward(ctx, embed, logits);
}

void voxref_decoder_prefill(vox_ctx_t *ctx, const float *embeds, int n) {
    vox_decoder_prefill(ctx, embeds, n);
}

int voxref_decoder_kv_preallocate(vox_ctx_t *ctx, int max_seq) {
    return vox_decoder_kv_cache_preallocate(ctx, max_seq);
}

int voxref_encoder_kv_preallocate(vox_ctx_t *ctx, int max_pos) {
    return vox_encoder_kv_cache_preallocate(ctx, max_pos);
}

/* Runs vox_encoder_forward_incremental and copies its [n, 1280] result. */
int voxref_encoder_incremental(vox_ctx_t *ctx, const float *x, int n, float *out) {
    int out_len = 0;
    float *r = vox_encoder_forward_incremental(ctx, x, n, &out_len);
    if (!r) return -1;
    memcpy(out, r, (size_t)out_len * VOX_ENC_DIM * sizeof(float));
    free(r);
    return out_len;
}

/* Runs vox_adapter_forward and copies its [n/4, 3072] result. */
int voxref_adapter(vox_ctx_t *ctx, const float *enc, int n, float *out) {
    int out_len = 0;
    float *r = vox_adapter_forward(ctx, enc, n, &out_len);
    if (!r) return -1;
    memcpy(out, r, (size_t)out_len * VOX_DEC_DIM * sizeof(float));
    free(r);
    return out_len;
}

/* state[0..5] = kv_cache_len, kv_cache_max, kv_pos_offset,
 *               enc_kv_cache_len, enc_kv_cache_max, enc_kv_pos_offset */
void voxref_get_state(const vox_ctx_t *ctx, int *state) {
    state[0] = ctx->kv_cache_len;
    state[1] = ctx->kv_cache_max;
    state[2] = ctx->kv_pos_offset;
    state[3] = ctx->enc_kv_cache_len;
    state[4] = ctx->enc_kv_cache_max;
    state[5] = ctx->enc_kv_pos_offset;
}

void voxref_set_dec_kv_state(vox_ctx_t *ctx, int len, int pos_offset) {
    ctx->kv_cache_len = len;
    ctx->kv_pos_offset = pos_offset;
}

void voxref_set_enc_kv_state(vox_ctx_t *ctx, int len, int pos_offset) {
    ctx->enc_kv_cache_len = len;
    ctx->enc_kv_pos_offset = pos_offset;
}

float *voxref_dec_kv_k(vox_ctx_t *ctx) { return ctx->kv_cache_k; }
float *voxref_dec_kv_v(vox_ctx_t *ctx) { return ctx->kv_cache_v; }
float *voxref_enc_kv_k(vox_ctx_t *ctx) { return ctx->enc_kv_cache_k; }
float *voxref_enc_kv_v(vox_ctx_t *ctx) { return ctx->enc_kv_cache_v; }

/* Frees what the reference allocated inside ctx (KV caches and the
 * persistent scratch buffers, as vox_free does at voxtral.c:288-329); the
 * weights belong to the caller.  free_ada_scale: ada_scale was allocated by
 * voxref_time_conditioning rather than passed in by the caller. */
void voxref_ctx_free(vox_ctx_t *ctx, int free_ada_scale) {
    if (!ctx) return;
    if (free_ada_scale) free(ctx->ada_scale);
    free(ctx->kv_cache_k);
    free(ctx->kv_cache_v);
    free(ctx->enc_kv_cache_k);
    free(ctx->enc_kv_cache_v);
    free(ctx->enc_inc_x_norm);
    free(ctx->enc_inc_q);
    free(ctx->enc_inc_k);
    free(ctx->enc_inc_v);
    free(ctx->enc_inc_attn_out);
    free(ctx->enc_inc_proj_out);
    free(ctx->enc_inc_gate);
    free(ctx->enc_inc_up);
    free(ctx->enc_inc_ffn_out);
    free(ctx->enc_inc_positions);
    free(ctx->enc_inc_rope_freqs);
    free(ctx->dec_x);
    free(ctx->dec_x_norm);
    free(ctx->dec_q);
    free(ctx->dec_k);
    free(ctx->dec_v);
    free(ctx->dec_attn_out);
    free(ctx->dec_proj_out);
    free(ctx->dec_gate);
    free(ctx->dec_up);
    free(ctx->dec_ffn_out);
    free(ctx->dec_rope_freqs);
    free(ctx);
}

/* ---- multi-stream CPU baseline: one host thread per stream context ---- */

typedef struct {
    vox_ctx_t *ctx;
    const float *embed;
    float *logits;
    int steps;
    int last_token;
} voxref_job_t;

static void *voxref_job_run(void *arg) {
    voxref_job_t *j = (voxref_job_t *)arg;
    for (int s = 0; s < j->steps; s++)
        j->last_token = vox_decoder_forward(j->ctx, j->embed, j->logits);
    return NULL;
}

/* Runs `steps` decode steps on each of n contexts, one pthread per context,
 * and returns the wall time in seconds.  embeds: [n, 3072]; logits:
 * [n, 131072]; tokens: [n] (last token of each stream). */
double voxref_decode_threads(vox_ctx_t **ctxs, int n, int steps,
                             const float *embeds, float *logits, int *tokens) {
    voxref_job_t *jobs = (voxref_job_t *)calloc((size_t)n, sizeof(voxref_job_t));
    pthread_t *th = (pthread_t *)calloc((size_t)n, sizeof(pthread_t));
    struct timespec t0, t1;
    clock_gettime(CLOCK_MONOTONIC, &t0);
    for (int i = 0; i < n; i++) {
        jobs[i].ctx = ctxs[i];
        jobs[i].embed = embeds + (size_t)i * VOX_DEC_DIM;
        jobs[i].logits = logits + (size_t)i * VOX_VOCAB_SIZE;
        jobs[i].steps = steps;
        pthread_create(&th[i], NULL, voxref_job_run, &jobs[i]);
    }
    for (int i = 0; i < n; i++) {
        pthread_join(th[i], NULL);
        tokens[i] = jobs[i].last_token;
    }
    clock_gettime(CLOCK_MONOTONIC, &t1);
    free(jobs);
    free(th);
    return (double)(t1.tv_sec - t0.tv_sec) + 1e-9 * (double)(t1.tv_nsec - t0.tv_nsec);
}

/* ---- conv stem (stream_conv_stem, voxtral.c:487-665) on a bare stream ---- */

/* conv0: [1280, 128, 3] + [1280]; conv1: [1280, 1280, 3] + [1280] (fp32, as
 * vox_encoder_t holds them, voxtral.h:84-88). */
void voxref_set_conv(vox_ctx_t *ctx, const float *w0, const float *b0, const float *w1, const float *b1) {
    ctx->encoder.conv0_weight = (float *)w0;
    ctx->encoder.conv0_bias = (float *)b0;
    ctx->encoder.conv1_weight = (float *)w1;
    ctx->encoder.conv1_bias = (float *)b1;
}

/* A stream with only the conv-stem state in use. */
void *voxref_stem_new(vox_ctx_t *ctx) {
    vox_stream_t *s = (vox_stream_t *)calloc(1, sizeof(vox_stream_t));
    if (s) s->ctx = ctx;
    return s;
}

/* n new mel frames [n][128] -> post-conv rows [len][1280] into out; returns len. */
int voxref_stem_step(void *st, const float *mel_new, int n, float *out) {
    int len = 0;
    float *r = stream_conv_stem((vox_stream_t *)st, mel_new, n, &len);
    if (r) {
        memcpy(out, r, (size_t)len * VOX_ENC_DIM * sizeof(float));
        free(r);
    }
    return len;
}

void voxref_stem_free(void *st) {
    vox_stream_t *s = (vox_stream_t *)st;
    if (!s) return;
    free(s->mel_tail);
    free(s->conv0_tail);
    free(s->conv0_residual);
    free(s);
}
