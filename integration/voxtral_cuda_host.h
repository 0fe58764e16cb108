/*
 * voxtral_cuda_host.h - the reference host's side of the `make cuda` build.
 *
 * These functions sit between voxtral.c's own types (vox_ctx_t, voxtral.h:154-201)
 * and the plain C ABI of libvoxtral_cuda.so (voxtral_cuda.h).  They are compiled
 * together with the reference's sources, under USE_CUDA, and are called from the
 * hunks integration/apply_cuda.py inserts at the sites where the `make mps` build
 * calls voxtral_metal.h.  Each keeps the host's own bookkeeping (kv_cache_len,
 * kv_pos_offset, enc_kv_cache_len, enc_kv_pos_offset) exactly as the CPU path
 * leaves it, so the rest of the host (the stream driver, vox_set_delay, the CLI)
 * runs unchanged.
 */
#ifndef VOXTRAL_CUDA_HOST_H
#define VOXTRAL_CUDA_HOST_H

#include "voxtral.h"
#include "voxtral_cuda.h"

/* Create the device decoder (weights uploaded once from the mmap'd tensors),
 * one decode state, and - when the context holds encoder weights - the device
 * encoder and an encoder state.  Called at the end of vox_load, where the Metal
 * build warms up (voxtral.c:161-242).  Returns 0, or -1 (ctx left on the CPU
 * path; vox_cuda_last_error() says why). */
int vox_cuda_host_attach(vox_ctx_t *ctx);

/* Release what attach created (vox_free, voxtral.c:253-329). */
void vox_cuda_host_detach(vox_ctx_t *ctx);

/* vox_decoder_forward (voxtral_decoder.c:401-516) on the device: the step at
 * logical position kv_pos_offset + kv_cache_len with the host's own RoPE table
 * (vox_compute_rope_freqs), then kv_cache_len += 1.  Returns the token, or 2
 * (EOS) on failure as the reference does on OOM (voxtral_decoder.c:436). */
int vox_cuda_host_decoder_forward(vox_ctx_t *ctx, const float *input_embeds, float *logits);

/* vox_decoder_prefill (voxtral_decoder.c:233-373) on the device: seq_len rows
 * from the current position; kv_cache_len += seq_len.  Returns 0 or -1. */
int vox_cuda_host_decoder_prefill(vox_ctx_t *ctx, const float *input_embeds, int seq_len);

/* vox_encoder_forward_incremental (voxtral_encoder.c:452-636) on the device:
 * a malloc'd [new_len, 1280] result (NULL on failure), the encoder position
 * advanced by new_len. */
float *vox_cuda_host_encoder_incremental(vox_ctx_t *ctx, const float *x_new, int new_len,
                                         int *out_len);

/* vox_adapter_forward (voxtral_encoder.c:642-674) on the device: a malloc'd
 * [enc_seq_len / 4, 3072] result (NULL on failure). */
float *vox_cuda_host_adapter_forward(vox_ctx_t *ctx, const float *enc_out, int enc_seq_len,
                                     int *out_seq_len);

/* After vox_update_time_conditioning recomputed ctx->ada_scale
 * (vox_set_delay, voxtral.c:1344-1350): rewrite the device's folded FFN norm. */
void vox_cuda_host_ada_changed(vox_ctx_t *ctx);

#endif /* VOXTRAL_CUDA_HOST_H */
