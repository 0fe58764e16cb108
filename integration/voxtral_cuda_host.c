/*
 * voxtral_cuda_host.c - the reference host's side of the `make cuda` build.
 *
 * Compiled with the reference's own sources (-DUSE_CUDA, voxtral.h from the
 * patched tree that integration/apply_cuda.py writes) and linked against
 * libvoxtral_cuda.so.  Every function keeps the host's cache bookkeeping as the
 * reference's CPU path leaves it, so that the logical positions it feeds RoPE
 * (voxtral_decoder.c:263-267, 437-443; voxtral_encoder.c:495-500) are the ones
 * the device rings use.  The device rings need no compaction: a position lives
 * in slot position mod capacity.
 */
#include "voxtral_cuda_host.h"

#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "voxtral_cuda.h"
#include "voxtral_kernels.h"

/* Encoder chunks longer than this are run in pieces (each row attends its own
 * 750-row window, so pieces give the same rows as one chunk); the adapter takes
 * as many rows per call.  A multiple of 4 (VOX_DOWNSAMPLE). */
#define VOX_CUDA_HOST_ENC_CHUNK 1500

static void report(const char *what) {
    fprintf(stderr, "voxtral cuda: %s: %s\n", what, vox_cuda_last_error());
}

int vox_cuda_host_attach(vox_ctx_t *ctx) {
    if (!ctx || !vox_cuda_available()) return -1;
    if (ctx->decoder.tok_embeddings_bf16 && !ctx->cuda_dec) {
        vox_cuda_dec_weights w;
        memset(&w, 0, sizeof(w));
        w.n_layers = VOX_DEC_LAYERS;
        w.vocab = VOX_VOCAB_SIZE;
        w.tok_embeddings = ctx->decoder.tok_embeddings_bf16;
        w.norm = ctx->decoder.norm;
        w.ada_scale = ctx->ada_scale;
        for (int i = 0; i < VOX_DEC_LAYERS; i++) {
            const vox_dec_layer_t *l = &ctx->decoder.layers[i];
            vox_cuda_dec_layer_weights *o = &w.layers[i];
            o->wq = l->wq_weight_bf16;
            o->wk = l->wk_weight_bf16;
            o->wv = l->wv_weight_bf16;
            o->wo = l->wo_weight_bf16;
            o->w1 = l->w1_weight_bf16;
            o->w2 = l->w2_weight_bf16;
            o->w3 = l->w3_weight_bf16;
            o->attention_norm = l->attention_norm;
            o->ffn_norm = l->ffn_norm;
        }
        vox_cuda_decoder *d = vox_cuda_decoder_create(&w);
        if (!d) {
            report("decoder upload");
            return -1;
        }
        /* the reference preallocates 8192 + 1024 positions (voxtral.c:233) */
        vox_cuda_dec_state *s = vox_cuda_dec_state_create(d, VOX_DEC_WINDOW + 1024);
        if (!s) {
            report("decoder state");
            vox_cuda_decoder_free(d);
            return -1;
        }
        ctx->cuda_dec = d;
        ctx->cuda_state = s;
    }
    if (ctx->encoder.layers[0].wq_weight_bf16 && ctx->adapter.linear0_weight_bf16 && !ctx->cuda_enc) {
        vox_cuda_enc_weights ew;
        memset(&ew, 0, sizeof(ew));
        ew.n_layers = VOX_ENC_LAYERS;
        ew.norm = ctx->encoder.norm;
        ew.adapter0 = ctx->adapter.linear0_weight_bf16;
        ew.adapter1 = ctx->adapter.linear1_weight_bf16;
        for (int i = 0; i < VOX_ENC_LAYERS; i++) {
            const vox_enc_layer_t *l = &ctx->encoder.layers[i];
            vox_cuda_enc_layer_weights *o = &ew.layers[i];
            o->wq = l->wq_weight_bf16;
            o->wk = l->wk_weight_bf16;
            o->wv = l->wv_weight_bf16;
            o->wo = l->wo_weight_bf16;
            o->w1 = l->w1_weight_bf16;
            o->w2 = l->w2_weight_bf16;
            o->w3 = l->w3_weight_bf16;
            o->wq_bias = l->wq_bias;
            o->wv_bias = l->wv_bias;
            o->wo_bias = l->wo_bias;
            o->w2_bias = l->w2_bias;
            o->attention_norm = l->attention_norm;
            o->ffn_norm = l->ffn_norm;
        }
        vox_cuda_encoder *e = vox_cuda_encoder_create(&ew);
        if (!e) {
            report("encoder upload");
            return -1;
        }
        vox_cuda_enc_state *es = vox_cuda_enc_state_create(e, VOX_CUDA_HOST_ENC_CHUNK);
        if (!es) {
            report("encoder state");
            vox_cuda_encoder_free(e);
            return -1;
        }
        ctx->cuda_enc = e;
        ctx->cuda_enc_state = es;
    }
    return 0;
}

void vox_cuda_host_detach(vox_ctx_t *ctx) {
    if (!ctx) return;
    vox_cuda_dec_state_free((vox_cuda_dec_state *)ctx->cuda_state);
    vox_cuda_decoder_free((vox_cuda_decoder *)ctx->cuda_dec);
    vox_cuda_enc_state_free((vox_cuda_enc_state *)ctx->cuda_enc_state);
    vox_cuda_encoder_free((vox_cuda_encoder *)ctx->cuda_enc);
    ctx->cuda_state = ctx->cuda_dec = NULL;
    ctx->cuda_enc_state = ctx->cuda_enc = NULL;
}

/* Bring the device state to the host's logical position.  The host moves
 * backwards only when it starts over (voxtral.c:857-858 zeroes kv_cache_len
 * and kv_pos_offset before a stream's prefill); a forward jump happens when a
 * caller set the cache length itself. */
static int sync_dec_position(vox_ctx_t *ctx, int logical) {
    vox_cuda_dec_state *s = (vox_cuda_dec_state *)ctx->cuda_state;
    if (vox_cuda_dec_state_position(s) == logical) return 0;
    return logical == 0 ? vox_cuda_dec_state_reset(s) : vox_cuda_dec_state_set_position(s, logical);
}

int vox_cuda_host_decoder_forward(vox_ctx_t *ctx, const float *input_embeds, float *logits) {
    /* the host's bookkeeping, as the CPU path leaves it: a full cache is
     * compacted to its last VOX_DEC_WINDOW positions (voxtral_decoder.c:419-428,
     * 208-227); without a host cache, the reference's preallocated size */
    const int cap = ctx->kv_cache_max > 0 ? ctx->kv_cache_max : VOX_DEC_WINDOW + 1024;
    if (ctx->kv_cache_len >= cap && ctx->kv_cache_len > VOX_DEC_WINDOW) {
        ctx->kv_pos_offset += ctx->kv_cache_len - VOX_DEC_WINDOW;
        ctx->kv_cache_len = VOX_DEC_WINDOW;
    }
    const int logical = ctx->kv_pos_offset + ctx->kv_cache_len;
    float rope[VOX_DEC_HEAD_DIM];
    int positions[1] = {logical};
    vox_compute_rope_freqs(rope, positions, 1, VOX_DEC_HEAD_DIM, VOX_ROPE_THETA);
    if (sync_dec_position(ctx, logical) != 0) {
        report("decoder position");
        return 2;
    }
    int tok = vox_cuda_decoder_full_step((vox_cuda_dec_state *)ctx->cuda_state, input_embeds, rope,
                                         logits);
    if (tok < 0) {
        report("decoder step");
        return 2;   /* EOS, as on OOM (voxtral_decoder.c:436) */
    }
    ctx->kv_cache_len += 1;
    return tok;
}

int vox_cuda_host_decoder_prefill(vox_ctx_t *ctx, const float *input_embeds, int seq_len) {
    if (seq_len <= 0) return 0;
    const int logical = ctx->kv_pos_offset + ctx->kv_cache_len;
    int *positions = (int *)malloc((size_t)seq_len * sizeof(int));
    float *rope = (float *)malloc((size_t)seq_len * VOX_DEC_HEAD_DIM * sizeof(float));
    int rc = -1;
    if (positions && rope) {
        for (int i = 0; i < seq_len; i++) positions[i] = logical + i;
        vox_compute_rope_freqs(rope, positions, seq_len, VOX_DEC_HEAD_DIM, VOX_ROPE_THETA);
        if (sync_dec_position(ctx, logical) == 0 &&
            vox_cuda_decoder_prefill_step((vox_cuda_dec_state *)ctx->cuda_state, input_embeds, seq_len,
                                          rope) == VOX_CUDA_OK) {
            ctx->kv_cache_len += seq_len;
            rc = 0;
        } else {
            report("decoder prefill");
        }
    }
    free(positions);
    free(rope);
    return rc;
}

float *vox_cuda_host_encoder_incremental(vox_ctx_t *ctx, const float *x_new, int new_len,
                                         int *out_len) {
    *out_len = 0;
    if (new_len <= 0) return NULL;
    vox_cuda_enc_state *s = (vox_cuda_enc_state *)ctx->cuda_enc_state;
    /* the host's bookkeeping, as the CPU path leaves it (compaction keeps the
     * last VOX_ENC_WINDOW positions, voxtral_encoder.c:388-406, 463-466) */
    if (ctx->enc_kv_cache_len + new_len > VOX_ENC_WINDOW && ctx->enc_kv_cache_len > VOX_ENC_WINDOW) {
        ctx->enc_kv_pos_offset += ctx->enc_kv_cache_len - VOX_ENC_WINDOW;
        ctx->enc_kv_cache_len = VOX_ENC_WINDOW;
    }
    const int logical = ctx->enc_kv_pos_offset + ctx->enc_kv_cache_len;
    if (vox_cuda_enc_state_position(s) != logical) {
        int rc = logical == 0 ? vox_cuda_enc_state_reset(s) : vox_cuda_enc_state_set_position(s, logical);
        if (rc != VOX_CUDA_OK) {
            report("encoder position");
            return NULL;
        }
    }
    float *x = (float *)malloc((size_t)new_len * VOX_ENC_DIM * sizeof(float));
    float *rope = (float *)malloc((size_t)VOX_CUDA_HOST_ENC_CHUNK * VOX_ENC_HEAD_DIM * sizeof(float));
    int *positions = (int *)malloc((size_t)VOX_CUDA_HOST_ENC_CHUNK * sizeof(int));
    if (!x || !rope || !positions) {
        free(x);
        free(rope);
        free(positions);
        return NULL;
    }
    memcpy(x, x_new, (size_t)new_len * VOX_ENC_DIM * sizeof(float));
    for (int done = 0; done < new_len;) {
        const int n = new_len - done < VOX_CUDA_HOST_ENC_CHUNK ? new_len - done : VOX_CUDA_HOST_ENC_CHUNK;
        for (int i = 0; i < n; i++) positions[i] = logical + done + i;
        vox_compute_rope_freqs(rope, positions, n, VOX_ENC_HEAD_DIM, VOX_ROPE_THETA);
        if (vox_cuda_encoder_full_step(s, x + (size_t)done * VOX_ENC_DIM, n, rope) != VOX_CUDA_OK) {
            report("encoder chunk");
            free(x);
            x = NULL;
            break;
        }
        done += n;
    }
    free(rope);
    free(positions);
    if (!x) return NULL;
    ctx->enc_kv_cache_len += new_len;
    *out_len = new_len;
    return x;
}

float *vox_cuda_host_adapter_forward(vox_ctx_t *ctx, const float *enc_out, int enc_seq_len,
                                     int *out_seq_len) {
    *out_seq_len = 0;
    const int n = enc_seq_len / VOX_DOWNSAMPLE;
    if (n <= 0) return NULL;
    float *out = (float *)malloc((size_t)n * VOX_DEC_DIM * sizeof(float));
    if (!out) return NULL;
    /* in pieces the state's workspace holds (whole groups of 4 rows) */
    for (int r0 = 0; r0 < n * VOX_DOWNSAMPLE; r0 += VOX_CUDA_HOST_ENC_CHUNK) {
        int rows = n * VOX_DOWNSAMPLE - r0;
        if (rows > VOX_CUDA_HOST_ENC_CHUNK) rows = VOX_CUDA_HOST_ENC_CHUNK;
        if (vox_cuda_adapter_forward((vox_cuda_enc_state *)ctx->cuda_enc_state,
                                     enc_out + (size_t)r0 * VOX_ENC_DIM, rows,
                                     out + (size_t)(r0 / VOX_DOWNSAMPLE) * VOX_DEC_DIM) != VOX_CUDA_OK) {
            report("adapter");
            free(out);
            return NULL;
        }
    }
    *out_seq_len = n;
    return out;
}

void vox_cuda_host_ada_changed(vox_ctx_t *ctx) {
    if (ctx && ctx->cuda_dec &&
        vox_cuda_decoder_set_ada_scale((vox_cuda_decoder *)ctx->cuda_dec, ctx->ada_scale) != VOX_CUDA_OK)
        report("ada scale");
}
