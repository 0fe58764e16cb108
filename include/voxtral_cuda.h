/*
 * voxtral_cuda.h - B200 (sm_100a) backend for voxtral.c's inference hot path.
 *
 * A plain C ABI (no CUDA, PyTorch or C++ types in any signature) that the
 * reference's C host calls under `#ifdef USE_CUDA`, at the same call sites
 * where the `make mps` build calls voxtral_metal.h.  Every entry point below
 * names the reference interface it replaces (file:line in voxtral.c's tree).
 *
 * Conventions
 *   - Status: functions returning int return >= 0 on success (a token id
 *     where stated) and a negative VOX_CUDA_ERR_* code on failure.  There is
 *     no CPU fallback inside this library: a failure is reported, never
 *     silently recomputed on the host.
 *   - Pointers: "host" arguments are ordinary host memory owned by the caller
 *     (e.g. the mmap'd safetensors); "_dev" entry points take device pointers
 *     and an optional cudaStream_t passed as void* (NULL = the library's
 *     stream for the calling thread's device).
 *   - Weights are bf16 row-major [out_dim, in_dim] exactly as stored in
 *     consolidated.safetensors; norms, biases and activations are fp32.
 *   - Threading: calls on one decoder/encoder state must come from one host
 *     thread at a time; different states may run concurrently.
 */
#ifndef VOXTRAL_CUDA_H
#define VOXTRAL_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VOX_CUDA_OK              0
#define VOX_CUDA_ERR_UNAVAILABLE (-1)  /* no usable sm_100 device / not initialised */
#define VOX_CUDA_ERR_ARG         (-2)  /* bad shape, NULL pointer, unsupported size */
#define VOX_CUDA_ERR_OOM         (-3)  /* device allocation failed */
#define VOX_CUDA_ERR_CUDA        (-4)  /* a CUDA runtime call or kernel failed */
#define VOX_CUDA_ERR_CAPACITY    (-5)  /* KV ring / scratch capacity exceeded */

/* ------------------------------------------------------------------------
 * Lifecycle  (voxtral_metal.h:19-26, called at main.c:162-164, 283-285)
 * ------------------------------------------------------------------------ */

/* Initialise the backend on the calling thread's device (VOX_CUDA_DEVICE env
 * var, else device 0).  Returns 1 on success, 0 if unavailable - the same
 * convention as vox_metal_init (voxtral_metal.h:20). */
int vox_cuda_init(void);

/* 1 if vox_cuda_init succeeded on this thread's device (voxtral_metal.h:23). */
int vox_cuda_available(void);

/* Release every device resource the library holds (voxtral_metal.h:26). */
void vox_cuda_shutdown(void);

/* Bind the calling host thread to a device (multi-stream / multi-GPU hosts:
 * one host thread per device).  Returns 0 or a VOX_CUDA_ERR_* code. */
int vox_cuda_set_device(int device);

/* Human-readable description of the last error on the calling thread. */
const char *vox_cuda_last_error(void);

/* Device bytes held by the library on the current device
 * (vox_metal_memory_used, voxtral_metal.h:258). */
size_t vox_cuda_memory_used(void);

/* ------------------------------------------------------------------------
 * (1) bf16-weight matmul entry points
 * ------------------------------------------------------------------------ */

/* C[M,N] = A[M,K] . B[N,K]^T (+ bias[N]) with host A, C, bias and host bf16
 * B.  B is uploaded on first use and cached on the device keyed by its host
 * pointer (the mmap'd tensor), like the Metal pointer-keyed weight cache.
 * Replaces vox_metal_sgemm_bf16 (voxtral_metal.h:38-41) at the dispatch
 * points of vox_linear_nobias_bf16 / vox_linear_bf16 / vox_matmul_t_bf16
 * (voxtral_kernels.c:197-264).  M <= 8 runs the streaming GEMV (fp32-level
 * accuracy); larger M the tcgen05 tensor-core GEMM, whose activations are
 * rounded to bf16 (<= 5e-3 relative L2 per matmul). */
int vox_cuda_sgemm_bf16(int M, int N, int K, const float *A, const uint16_t *B_bf16,
                        const float *bias, float *C);

/* Pre-upload a [N, K] weight into the pointer-keyed cache
 * (vox_metal_warmup_bf16, voxtral_metal.h:225; the shape is needed here
 * because the device copy is re-laid out into 16x16 MMA-fragment tiles). */
int vox_cuda_warmup_bf16(const uint16_t *B_bf16, int N, int K);

/* Drop every cached weight copy on the current device.  The cache assumes a
 * cached weight's memory is not rewritten (true for the mmap'd safetensors);
 * a caller that frees or rewrites weight buffers calls this first. */
void vox_cuda_weight_cache_clear(void);

/* Device-pointer form of vox_cuda_sgemm_bf16: all pointers on the device,
 * B in its row-major layout (tiled copy cached by pointer, as above). */
int vox_cuda_linear_bf16_dev(int M, int N, int K, const float *A, const uint16_t *B_bf16,
                             const float *bias, float *C, void *stream);

/* Tensor-core GEMM on device pointers: C[M,N] (fp32) = A[M,K] . W[N,K]^T
 * (+ bias) with bf16 A and W, fp32 accumulation (tcgen05 / TMEM, TMA-fed).
 * K must be a multiple of 8 and A, W 16-byte aligned.  The building block of
 * the encoder chunk and adapter (voxtral_encoder.c:542-616, 663-667). */
int vox_cuda_gemm_bf16_dev(int M, int N, int K, const uint16_t *A_bf16, const uint16_t *W_bf16,
                           const float *bias, float *C, void *stream);

/* ------------------------------------------------------------------------
 * (2) (4) (5) decoder: resident weights, KV ring, single-token step
 * ------------------------------------------------------------------------ */

#define VOX_CUDA_DEC_MAX_LAYERS 26

typedef struct {
    const uint16_t *wq, *wk, *wv, *wo;   /* [4096,3072] [1024,3072] x2 [3072,4096] */
    const uint16_t *w1, *w2, *w3;        /* [9216,3072] [3072,9216] [9216,3072] */
    const float *attention_norm;         /* [3072] */
    const float *ffn_norm;               /* [3072] */
} vox_cuda_dec_layer_weights;

/* The decoder half of vox_ctx_t (voxtral.h:101-137) plus ctx->ada_scale. */
typedef struct {
    int n_layers;                        /* VOX_DEC_LAYERS (26) */
    int vocab;                           /* VOX_VOCAB_SIZE (131072) */
    int weights_on_device;               /* 0: host pointers (uploaded), 1: device */
    const uint16_t *tok_embeddings;      /* [vocab, 3072]; also the LM head */
    const float *norm;                   /* [3072] final norm */
    const float *ada_scale;              /* [n_layers, 3072] or NULL */
    vox_cuda_dec_layer_weights layers[VOX_CUDA_DEC_MAX_LAYERS];
} vox_cuda_dec_weights;

typedef struct vox_cuda_decoder vox_cuda_decoder;   /* resident weights (per device) */
typedef struct vox_cuda_dec_state vox_cuda_dec_state; /* one stream: KV ring + scratch */

/* Upload (or adopt, when weights_on_device) the decoder weights into the
 * fused device layout: wq|wk|wv concatenated, w1/w3 row-interleaved.  The
 * counterpart of the Metal warm-up (voxtral.c:161-242).  NULL on failure. */
vox_cuda_decoder *vox_cuda_decoder_create(const vox_cuda_dec_weights *w);
void vox_cuda_decoder_free(vox_cuda_decoder *d);

/* Replace the per-layer ada scale (host [n_layers][3072], or NULL for none)
 * after vox_set_delay recomputed it (voxtral.c:1344-1350, 46-79).  The scale
 * is folded into the FFN norm weights on the device (ffn_norm * (1 + ada),
 * voxtral_decoder.c:488-492), so only those 26 x 3072 floats are rewritten:
 * no weight re-upload.  The decoder's states share the new scale from their
 * next step on; steps already queued finish with the old one. */
int vox_cuda_decoder_set_ada_scale(vox_cuda_decoder *d, const float *ada_scale);

/* Per-stream state: device KV ring of kv_cap positions per layer (>= 8192 to
 * hold the full sliding window; the reference preallocates 8192+1024,
 * voxtral.c:233).  Replaces kv_cache_init / vox_decoder_kv_cache_preallocate
 * (voxtral_decoder.c:114-139). */
vox_cuda_dec_state *vox_cuda_dec_state_create(vox_cuda_decoder *d, int kv_cap);
void vox_cuda_dec_state_free(vox_cuda_dec_state *s);

/* Forget the cached positions (voxtral.c:857-858 sets kv_cache_len = 0 and
 * kv_pos_offset = 0 before a new prefill). */
int vox_cuda_dec_state_reset(vox_cuda_dec_state *s);

/* Number of logical positions consumed so far (kv_pos_offset + kv_cache_len
 * in the reference's bookkeeping). */
int vox_cuda_dec_state_position(const vox_cuda_dec_state *s);

/* Set the logical position of the next row without computing anything: the
 * ring then holds whatever was loaded with vox_cuda_dec_state_load_kv.  Used
 * to resume from a cache the caller filled (and by tests). */
int vox_cuda_dec_state_set_position(vox_cuda_dec_state *s, int logical_pos);

/* Copy rows of K and V ([n_rows, 1024] fp32 host arrays) for one layer into
 * the ring at logical positions first_pos..first_pos+n_rows-1 (slot =
 * position mod kv_cap).  Lets a caller migrate an existing CPU cache. */
int vox_cuda_dec_state_load_kv(vox_cuda_dec_state *s, int layer, int first_pos, int n_rows,
                               const float *k_rows, const float *v_rows);

/* Read back rows of the ring (same layout as load_kv). */
int vox_cuda_dec_state_read_kv(vox_cuda_dec_state *s, int layer, int first_pos, int n_rows,
                               float *k_rows, float *v_rows);

/* One decode step for one token: all layers, the final norm, the LM head and
 * the argmax (first maximum, voxtral_decoder.c:507-515), with RoPE, the KV
 * ring write and the windowed attention in-kernel.  embed: host [3072].
 * rope_freqs: host [64][2] (cos, sin) as vox_compute_rope_freqs produces for
 * the step's logical position, or NULL to derive them on the device.  logits:
 * host [vocab] or NULL.  Returns the token id.  Replaces the CPU layer loop of
 * vox_decoder_forward (voxtral_decoder.c:401-516) the way
 * vox_metal_decoder_full_step does (voxtral_metal.h:219). */
int vox_cuda_decoder_full_step(vox_cuda_dec_state *s, const float *embed,
                               const float *rope_freqs, float *logits);

/* Alternatives for the last step's logits, computed on the device with the
 * semantics of stream_fill_alts (voxtral.c:778-833): ids >= 1000 other than
 * the best, by probability, accepted while 1 - p/p_best <= cutoff.  Writes
 * alt_ids[0] = best and returns the number of ids written (1..n_alt). */
int vox_cuda_decoder_fill_alts(vox_cuda_dec_state *s, int n_alt, float cutoff, int *alt_ids);

/* Prefill seq_len rows (host x [seq_len, 3072]) at the current position
 * (voxtral_decoder.c:233-373; vox_metal_decoder_prefill_step,
 * voxtral_metal.h:254).  rope_freqs: host [seq_len][64][2] or NULL. */
int vox_cuda_decoder_prefill_step(vox_cuda_dec_state *s, const float *x, int seq_len,
                                  const float *rope_freqs);

/* Prefill of several streams in shared launches: state i takes the next
 * seq_lens[i] rows of x (host [sum seq_lens, 3072]; rope_freqs host
 * [sum seq_lens][64][2] or NULL) from its current position.  Up to 128 rows
 * (e.g. three streams' 38-row prompts) share each tensor-core GEMM, whose
 * weight reads dominate at these sizes.  The prefill runs on the tcgen05
 * tensor cores with bf16 weights and activations split into bf16 hi + lo
 * (fp32-level products); VOX_CUDA_DEC_TC_PREFILL=0 at decoder creation keeps
 * no row-major weight copies (-6 GB at 4B) and prefills through the decode
 * kernels instead.  Additive: the reference prefills one context at a time
 * (voxtral.c:843-891). */
int vox_cuda_decoder_prefill_batch(vox_cuda_dec_state *const *states, int n, const float *x,
                                   const int *seq_lens, const float *rope_freqs);

/* Batched decode step over n independent streams that share one decoder:
 * the weights are read once for all n tokens (n <= 8).  embeds: host
 * [n, 3072]; tokens: host [n].  An additive entry with no single-stream
 * counterpart in the reference (each stream is its own vox_ctx_t there). */
int vox_cuda_decoder_step_batch(vox_cuda_dec_state *const *states, int n, const float *embeds,
                                int *tokens);

/* The batched step with the per-stream inputs and outputs of
 * vox_cuda_decoder_full_step (voxtral_metal.h:219): rope_freqs host
 * [n][64][2] (each stream's table as vox_compute_rope_freqs produces it for
 * that stream's position, voxtral_decoder.c:441-443) or NULL to derive them,
 * and logits host [n][vocab] (voxtral_decoder.c:504-506, the buffer
 * stream_fill_alts and teacher-forced checks read) or NULL. */
int vox_cuda_decoder_step_batch_ex(vox_cuda_dec_state *const *states, int n, const float *embeds,
                                   const float *rope_freqs, int *tokens, float *logits);

/* Device-resident form of the batched step for callers that keep the
 * embeddings on the device: embeds_dev [n, 3072], tokens_dev [n] (int32),
 * enqueued on `stream` (NULL: the library's stream) without waiting for it,
 * so the host prepares step k + 1 while step k runs; tokens_dev is valid once
 * `stream` reaches this call's work.  Only the slot and RoPE tables (a few
 * hundred bytes) cross from the host.  A device-side wait that timed out is
 * reported by a later call.  Every synchronous entry point of the decoder and
 * its states is ordered after the pending asynchronous steps. */
int vox_cuda_decoder_step_batch_dev(vox_cuda_dec_state *const *states, int n,
                                    const float *embeds_dev, int *tokens_dev, void *stream);

/* The stream loop's decode step on the device (stream_run_decoder,
 * voxtral.c:893-921: step_embed = adapter[gen_pos] + tok_embed(prev_token)):
 * stream i's input row is rows_dev[i] (a device pointer to its [3072] adapter
 * row; rows_dev itself is a host array of n pointers) plus the bf16 token
 * embedding of prev_tokens_dev[i] (device int32, e.g. the tokens_dev of the
 * previous call), added on the device.  Tokens land in tokens_dev [n]; no
 * token or embedding crosses to the host, so a serving loop can enqueue its
 * steps back to back.  Asynchronous as vox_cuda_decoder_step_batch_dev.  An id
 * outside [0, vocab) adds no embedding and is reported as an error by a later
 * call. */
int vox_cuda_decoder_step_batch_tokens_dev(vox_cuda_dec_state *const *states, int n,
                                           const float *const *rows_dev,
                                           const int *prev_tokens_dev, int *tokens_dev,
                                           void *stream);

/* out_dev[i] = rows_dev[i] + tok_embed(tokens_dev[i]) for i < n ([n][3072]
 * fp32, device pointers; rows_dev may be NULL for the plain lookup): the
 * prompt rows of a stream start (voxtral.c:846-851, BOS / STREAMING_PAD
 * embeddings added to the adapter rows) without the bf16 table on the host.
 * Enqueued on `stream` (NULL: the library's stream). */
int vox_cuda_decoder_embed_dev(vox_cuda_decoder *d, int n, const float *rows_dev, const int *tokens_dev,
                               float *out_dev, void *stream);

/* Per-phase device time of the batched step, for profiling (the CUDA-event
 * phase timers the reference keeps with gettimeofday, voxtral.c:679-680,
 * 895-919).  Runs `iters` steps kernel by kernel (no graph, no overlap) with
 * an event pair around every launch and writes the mean milliseconds per
 * step of each phase to ms[VOX_CUDA_PROF_PHASES].  The states' positions do
 * not advance. */
#define VOX_CUDA_PROF_QKV      0   /* norm + wq|wk|wv GEMV + RoPE + ring write */
#define VOX_CUDA_PROF_ATTN     1   /* split-K decode attention */
#define VOX_CUDA_PROF_WO       2   /* wo GEMV + residual */
#define VOX_CUDA_PROF_W13      3   /* norm + w1|w3 GEMV + SwiGLU */
#define VOX_CUDA_PROF_W2       4   /* w2 GEMV + residual */
#define VOX_CUDA_PROF_LM_HEAD  5   /* final norm + LM head + argmax */
#define VOX_CUDA_PROF_PHASES   6
int vox_cuda_decoder_profile_batch(vox_cuda_dec_state *const *states, int n,
                                   const float *embeds_dev, int iters, float *ms);

/* Steady-state device time of one phase's kernel: after one whole step, the
 * phase's launches of all layers (the LM head: its one launch) are captured
 * back to back in a CUDA graph with programmatic dependent launch, as in the
 * step, and replayed `iters` times between two events; *ms_per_launch =
 * elapsed / (iters x launches).  Each layer streams its own weights, so
 * successive launches do not hit in L2.  Profiling only: the states'
 * activations are left as garbage (positions do not advance). */
int vox_cuda_decoder_profile_sequence(vox_cuda_dec_state *const *states, int n,
                                      const float *embeds_dev, int phase, int iters,
                                      float *ms_per_launch);

/* ------------------------------------------------------------------------
 * (3) (5) encoder chunk + adapter: tcgen05 GEMMs, windowed attention, ring
 * ------------------------------------------------------------------------ */

#define VOX_CUDA_ENC_MAX_LAYERS 32

typedef struct {
    const uint16_t *wq, *wk, *wv;        /* bf16 [2048,1280] each */
    const uint16_t *wo;                  /* bf16 [1280,2048] */
    const uint16_t *w1, *w2, *w3;        /* bf16 [5120,1280] [1280,5120] [5120,1280] */
    const float *wq_bias, *wv_bias;      /* [2048] (wk has no bias) */
    const float *wo_bias, *w2_bias;      /* [1280] */
    const float *attention_norm;         /* [1280] */
    const float *ffn_norm;               /* [1280] */
} vox_cuda_enc_layer_weights;

/* The encoder and adapter halves of vox_ctx_t (voxtral.h:56-95, 143-148). */
typedef struct {
    int n_layers;                        /* VOX_ENC_LAYERS (32) */
    int weights_on_device;               /* 0: host pointers (uploaded), 1: device */
    const float *norm;                   /* [1280] final encoder norm */
    const uint16_t *adapter0;            /* bf16 [3072, 5120] */
    const uint16_t *adapter1;            /* bf16 [3072, 3072] */
    vox_cuda_enc_layer_weights layers[VOX_CUDA_ENC_MAX_LAYERS];
} vox_cuda_enc_weights;

typedef struct vox_cuda_encoder vox_cuda_encoder;     /* resident encoder + adapter weights */
typedef struct vox_cuda_enc_state vox_cuda_enc_state; /* one stream: encoder KV ring + workspace */

/* Upload the encoder and adapter weights (wq|wk|wv concatenated, w1/w3
 * row-interleaved, bf16 row-major for the TMA-fed tensor-core GEMM).  The
 * counterpart of the Metal encoder warm-up (voxtral.c:169-192). */
vox_cuda_encoder *vox_cuda_encoder_create(const vox_cuda_enc_weights *w);
void vox_cuda_encoder_free(vox_cuda_encoder *e);

/* Per-stream encoder state for chunks of up to max_chunk rows: an fp16 KV
 * ring of 750 + max_chunk positions per layer (the 750-row window plus a
 * chunk; the Metal build preallocates 750+256, voxtral.c:236) and the chunk
 * workspace.  Replaces vox_encoder_kv_cache_preallocate and the enc_inc_*
 * buffers (voxtral_encoder.c:328-446). */
vox_cuda_enc_state *vox_cuda_enc_state_create(vox_cuda_encoder *e, int max_chunk);
void vox_cuda_enc_state_free(vox_cuda_enc_state *s);
int vox_cuda_enc_state_reset(vox_cuda_enc_state *s);      /* voxtral.c:959-961 */
int vox_cuda_enc_state_position(const vox_cuda_enc_state *s);

/* Incremental encoder over new_len post-conv-stem rows, in place on host x
 * [new_len, 1280]: 32 layers of RMSNorm, QKV (+bias, RoPE, ring write),
 * causal window-750 attention, wo (+bias) + residual, RMSNorm, w1|w3 SwiGLU,
 * w2 (+bias) + residual, then the final norm (vox_encoder_forward_incremental,
 * voxtral_encoder.c:452-636; vox_metal_encoder_full_step, voxtral_metal.h:245).
 * rope_freqs: host [new_len][32][2] or NULL.  GEMM activations are rounded to
 * fp16 and attention runs in fp16 with fp32 accumulation. */
int vox_cuda_encoder_full_step(vox_cuda_enc_state *s, float *x, int new_len, const float *rope_freqs);

/* Device-resident form: x_dev [new_len, 1280] on the device, in place,
 * enqueued on `stream` (NULL: the library's stream) without waiting for it,
 * so several states (streams of audio) can run concurrently on their own
 * CUDA streams.  A device-side wait that timed out is reported by the next
 * call on the same state.  No counterpart in the reference (its encoder is
 * synchronous on the host). */
int vox_cuda_encoder_step_dev(vox_cuda_enc_state *s, float *x_dev, int new_len, void *stream);

/* Several streams' chunks as one launch: state i takes new_lens[i] rows at
 * x_dev[i] (device, in place), n <= 8 states of one encoder.  The norms and
 * the tensor-core GEMMs run once over all rows (8 x 100 rows -> M = 800,
 * tensor-bound instead of SM-count-bound); each state's windowed attention
 * runs over its own ring, concurrently.  Enqueued on `stream` without
 * waiting, like vox_cuda_encoder_step_dev; each state's position advances.
 * Additive: the reference runs one encoder context at a time. */
int vox_cuda_encoder_step_batch_dev(vox_cuda_enc_state *const *states, int n, float *const *x_dev,
                                    const int *new_lens, void *stream);

/* Set the logical position of the next chunk's first row (resume, tests). */
int vox_cuda_enc_state_set_position(vox_cuda_enc_state *s, int logical_pos);

/* Per-phase device time of an encoder chunk (kernel by kernel, an event pair
 * around every launch; the stream position does not advance): mean ms per
 * chunk written to ms[VOX_CUDA_EPROF_PHASES]. */
#define VOX_CUDA_EPROF_NORM   0   /* RMSNorm -> bf16 activations (both norms, final norm) */
#define VOX_CUDA_EPROF_QKV    1   /* wq|wk|wv GEMM + bias + RoPE + ring write */
#define VOX_CUDA_EPROF_ATTN   2   /* window-750 flash attention */
#define VOX_CUDA_EPROF_WO     3   /* wo GEMM + bias + residual */
#define VOX_CUDA_EPROF_W13    4   /* w1|w3 GEMM + SwiGLU */
#define VOX_CUDA_EPROF_W2     5   /* w2 GEMM + bias + residual */
#define VOX_CUDA_EPROF_PHASES 6
int vox_cuda_encoder_profile(vox_cuda_enc_state *s, const float *x_dev, int new_len, int iters, float *ms);

/* Adapter over n encoder rows (n a multiple of 4, at most 4 * max_chunk / 4 of
 * the state's workspace): 4x frame stacking, Linear(5120->3072), GELU,
 * Linear(3072->3072); host enc [n, 1280] -> out [n/4, 3072]
 * (vox_adapter_forward, voxtral_encoder.c:642-674). */
int vox_cuda_adapter_forward(vox_cuda_enc_state *s, const float *enc, int n, float *out);

/* Device-resident form: enc_dev [n, 1280] -> out_dev [n/4, 3072] (device
 * pointers), enqueued on `stream` (NULL: the library's stream) without a host
 * wait, ordered after the state's earlier asynchronous work (it shares the
 * state's workspace).  A device-side wait that timed out is reported by a later
 * call on the state. */
int vox_cuda_adapter_forward_dev(vox_cuda_enc_state *s, const float *enc_dev, int n, float *out_dev,
                                 void *stream);

/* The encoder path keeps its GEMM operands, its K / V ring and its attention
 * operands in fp16 (where the reference keeps fp32, voxtral_encoder.c:452-636).
 * Conversions to fp16 saturate: a value beyond fp16's range (|v| > 65504)
 * becomes +-65504 rather than infinite.  This returns, for the current device
 * (every encoder and adapter on it), since the library was loaded or the last
 * reset (reset != 0), the number of range events: SwiGLU output chunks (32
 * values of a row) holding a clamped value - the product silu(g) * u is where
 * the encoder's magnitudes peak - and residual rows that reached a norm with
 * a non-finite value.  It waits for the device's queued work first.  Non-zero
 * means the results may deviate from the fp32 reference: a caller with
 * unusual weights checks it. */
int vox_cuda_fp16_saturations(unsigned long long *count, int reset);

/* Conv stem: the encoder's two causal convolutions over the mel stream,
 * conv0 (128 -> 1280, kernel 3, stride 1) and conv1 (1280 -> 1280, kernel 3,
 * stride 2), each followed by GELU, with the streaming state of
 * stream_conv_stem (voxtral.c:487-665; vox_causal_conv1d,
 * voxtral_kernels.c:293-340).  Weights as vox_encoder_t holds them
 * (voxtral.h:84-88): conv0 [1280, 128, 3], conv1 [1280, 1280, 3] fp32, biases
 * [1280]; they are copied (as fp16) at creation.  max_mel bounds the mel
 * frames of one step. */
typedef struct vox_cuda_conv_stem vox_cuda_conv_stem;
vox_cuda_conv_stem *vox_cuda_conv_stem_create(const float *conv0_weight, const float *conv0_bias,
                                              const float *conv1_weight, const float *conv1_bias, int max_mel);
void vox_cuda_conv_stem_free(vox_cuda_conv_stem *s);
/* Start a new stream (the reference's conv_stem_initialized = 0). */
int vox_cuda_conv_stem_reset(vox_cuda_conv_stem *s);
/* n_new >= 1 mel frames, host [n_new, 128] row-major as the mel context
 * yields them -> host out [rows, 1280] post-conv positions, the encoder's
 * input; returns rows = floor((T + n_new) / 2) - floor(T / 2) for T frames
 * consumed before (0 is possible), or a negative error.  out must hold
 * n_new / 2 + 1 rows. */
int vox_cuda_conv_stem_step(vox_cuda_conv_stem *s, const float *mel_new, int n_new, float *out);
/* Device-resident form: mel_dev [n_new, 128] and out_dev [rows, 1280] on the
 * device, enqueued on `stream` without waiting (the mel context's _dev rows
 * feed it directly, and its rows the encoder's step_dev).  Returns rows; a
 * GEMM wait that timed out is reported by a later call.  Synchronous entry
 * points on the state are ordered after the pending steps. */
int vox_cuda_conv_stem_step_dev(vox_cuda_conv_stem *s, const float *mel_dev, int n_new, float *out_dev,
                                void *stream);

/* ------------------------------------------------------------------------
 * (6) log-mel front end: 16 kHz mono fp32 samples -> [frames, 128] log-mel
 * rows (hop 160, window 400, direct 201-bin DFT, Slaney filters, log10).
 * ------------------------------------------------------------------------ */

/* Incremental context: vox_mel_ctx_init (voxtral_audio.h:46; called at
 * voxtral.c:936 with 32 tokens of silence, 40960 samples).  The stream starts
 * with 200 + left_pad_samples zeros.  max_feed_samples sizes the device
 * sample ring; longer feeds are processed in pieces. */
typedef struct vox_cuda_mel vox_cuda_mel;
vox_cuda_mel *vox_cuda_mel_create(int left_pad_samples, int max_feed_samples);
void vox_cuda_mel_free(vox_cuda_mel *m);                 /* vox_mel_free (voxtral_audio.h:63) */

/* Frames computed so far (the count vox_mel_data reports, voxtral_audio.h:60). */
int vox_cuda_mel_frames(const vox_cuda_mel *m);

/* Frames that feeding n_samples more will produce (for sizing mel_out). */
int vox_cuda_mel_frames_for(const vox_cuda_mel *m, int n_samples);

/* vox_mel_feed (voxtral_audio.h:50; called at voxtral.c:972, 998): append host
 * samples and compute every frame whose window now fits.  The new rows go to
 * host mel_out [max_frames, 128]; returns their count, VOX_CUDA_ERR_CAPACITY
 * (nothing consumed) if more than max_frames, VOX_CUDA_ERR_ARG after finish
 * (the reference would keep appending past its reflection padding). */
int vox_cuda_mel_feed(vox_cuda_mel *m, const float *samples, int n_samples, float *mel_out,
                      int max_frames);

/* Device-resident form: samples_dev and mel_dev on the device, enqueued on
 * `stream` without waiting. */
int vox_cuda_mel_feed_dev(vox_cuda_mel *m, const float *samples_dev, int n_samples, float *mel_dev,
                          int max_frames, void *stream);

/* vox_mel_finish (voxtral_audio.h:56; called at voxtral.c:1003): append
 * right_pad_samples zeros, then the 200-sample reflection of the signal that
 * preceded them, compute the remaining frames and drop the last one.  The
 * rows kept go to mel_out; returns their count (0 when already finished). */
int vox_cuda_mel_finish(vox_cuda_mel *m, int right_pad_samples, float *mel_out, int max_frames);
int vox_cuda_mel_finish_dev(vox_cuda_mel *m, int right_pad_samples, float *mel_dev, int max_frames,
                            void *stream);

/* One-shot log-mel of a whole clip: vox_mel_spectrogram (voxtral_audio.h:33):
 * reflection padding of 200 on both sides, the last frame dropped.  Returns
 * the frame count (n_samples / 160) or VOX_CUDA_ERR_ARG when it is 0 (the
 * reference's "audio too short"). */
int vox_cuda_mel_spectrogram(const float *samples, int n_samples, float *mel_out, int max_frames);

/* ------------------------------------------------------------------------
 * Kernel-level entry points (device pointers) - the decode attention and the
 * LM-head argmax on their own, for callers that compose their own step.
 * ------------------------------------------------------------------------ */

/* Decode attention for one token over a KV ring: q [32*128] (RoPE already
 * applied), k_ring/v_ring [kv_cap, 1024], keys at logical positions
 * max(0, pos-8191)..pos stored at slot = position mod kv_cap; out [32*128].
 * vox_causal_attention with seq_q = 1 (voxtral_kernels.c:412-482, called at
 * voxtral_decoder.c:481-483).  Scratch for the split-K partials comes from
 * the library's per-device pool.  Enqueued on `stream` without a host wait;
 * calls on different streams are ordered on the device (they share the
 * scratch). */
int vox_cuda_attention_decode_dev(const float *q, const float *k_ring, const float *v_ring,
                                  int kv_cap, int pos, float *out, void *stream);

/* The same decode attention for callers that cannot allocate device memory
 * (hosts that forbid cudaMalloc after start-up, e.g. a real-time audio
 * pipeline that must not stall in the allocator, or code handed a fixed
 * device arena).  No counterpart in the reference: the reference has no GPU
 * path with allocation constraints.  Arguments and result are those of
 * vox_cuda_attention_decode_dev, except that `stream` may be NULL (the legacy
 * default stream) and vox_cuda_init is not required; the CUDA device that is
 * current on the calling thread is used.  The split scratch is a fixed
 * ~2.1 MB array in device memory that every GPU loading the library holds
 * until the process exits; it bounds the attended keys to 8192 (128 splits
 * of 64 keys), the decoder's full window, and larger requests are rejected
 * with VOX_CUDA_ERR_CAPACITY.  The first call on a device looks up the
 * array's device address and should come before any stream capture.  All
 * calls on a device share the array, which keeps the last call's contents:
 * calls that overlap on the GPU (other threads or streams) race, so callers
 * serialise them.  Every call blocks the calling thread until its work on
 * `stream` has finished (it synchronises `stream`), and returns 0 or a
 * VOX_CUDA_ERR_* code with the result in `out`.  The array's address is looked
 * up once per device ordinal, in the device's primary context: a caller that
 * resets the device (cudaDeviceReset) or runs in another driver context does
 * not use this entry point afterwards. */
int vox_cuda_attention_decode_noalloc(const float *q, const float *k_ring, const float *v_ring,
                                      int kv_cap, int pos, float *out, void *stream);

/* Interleaved-pair RoPE of x [n_heads*head_dim] at logical position pos,
 * cos/sin from rope_freqs ([head_dim/2][2], device) or, when NULL, derived on
 * the device (vox_apply_rope, voxtral_kernels.c:502-526). */
int vox_cuda_rope_dev(float *x, int n_heads, int head_dim, int pos, const float *rope_freqs,
                      void *stream);

/* Diagnostics: runs a kernel whose bounded wait (the mbarrier wait with a
 * %globaltimer deadline that every tensor-core kernel uses) can never
 * complete, with a deadline of wait_ms.  The kernel raises its error word at
 * the deadline and returns; the call reports it exactly as a step reports a
 * timed-out wait: VOX_CUDA_ERR_CUDA with a "timed out" message.  The GPU does
 * not fault and the context stays usable.  No counterpart in the reference
 * (it has no device-side waits). */
int vox_cuda_selftest_wait_timeout(int wait_ms);

/* ------------------------------------------------------------------------
 * Synthetic weights (benchmarks and tests): fill a device bf16 buffer with
 * seeded N(0, std) values, rounded to nearest even.
 * ------------------------------------------------------------------------ */
int vox_cuda_fill_normal_bf16_dev(uint16_t *dst, size_t n, uint64_t seed, float std,
                                  void *stream);

#ifdef __cplusplus
}
#endif
#endif /* VOXTRAL_CUDA_H */
