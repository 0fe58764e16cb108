// vc_internal.h - internal (C++) interfaces between the runtime and kernels.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace vc {

// One stream's view of its KV ring for one decode step.  Device memory; the
// runtime fills it before every step.
struct StreamSlot {
    float *k_ring;    // K ring, layer 0 base: [n_layers][cap][1024] fp32
    float *v_ring;    // V ring, same layout
    int cap;          // positions per layer
    int pos;          // logical position of this step's row
    int slot;         // pos % cap
    int n_keys;       // keys attended: min(pos + 1, window)
    int fresh;        // the lowest position this launch writes into this ring (the
                      //   launch's first row of this sequence): older keys predate it
};

enum GemvEpi : int {
    EPI_STORE = 0,    // y = acc (+ bias)
    EPI_ADD = 1,      // y += acc (+ bias)        (residual add)
    EPI_QKV = 2,      // q (RoPE) / k (RoPE, ring write) / v (ring write)
    EPI_SWIGLU = 3,   // rows (2i, 2i+1) = (gate_i, up_i) -> h_i = silu(g) * u
    EPI_LOGITS = 4,   // y = acc, plus argmax across the whole launch
};

struct alignas(8) ArgmaxPartial {   // read back as one 8-byte load
    float v;
    int i;
};
static_assert(sizeof(ArgmaxPartial) == 8, "(value, index) pairs are 8 bytes");

struct GemvParams {
    const uint16_t *W;      // fragment-tiled weights (launch_tile_weights), [Np, Kp]
    int N, K;               // logical shape
    int Kp;                 // K rounded up to 16 (the tiled row length)
    const uint32_t *xfrag;  // activations as B fragments (xfrag_put*), [Kp/16][32][4]
    const float *ss_in;     // RMSNorm: per-row-block sums of x^2, [M][ss_parts], or NULL
    int ss_parts;
    float *ss_out;          // EPI_ADD: per-row-block sums of the new y^2, [M][row blocks], or NULL
    uint32_t *xfrag_out;    // EPI_ADD: y * g_next as B fragments; EPI_SWIGLU: h as B fragments
    const float *g_next;    // EPI_ADD: the next RMSNorm's weights (* (1 + ada)), [N], or NULL
    unsigned *err;          // raised when a bounded wait expires
    float *y;               // output [M, ldy]
    int ldy;
    const float *bias;      // [N] or NULL
    // EPI_QKV
    const StreamSlot *slots;  // [M]
    const float *rope;        // [M][128]: (cos, sin) pairs for the step's position
    int layer;
    // EPI_LOGITS
    ArgmaxPartial *partials;  // [gridDim.x * M]
    unsigned *counter;        // 1 counter, zero between launches
    int *tokens;              // [M]
    int *const *tokens_to;    // EPI_LOGITS: a device word holding a second destination of the tokens
                              //   (read when the argmax finishes; NULL pointer or word: none)
    // weights of a later kernel to start pulling into L2 (or NULL)
    const void *pf;
    unsigned long long pf_bytes;   // a multiple of 16
};

// Launch the fused streaming GEMV (M = 1..8 activation rows).
cudaError_t launch_gemv(int M, int epi, const GemvParams &p, cudaStream_t st, bool pdl);
// x [M, K] (row stride ldx) -> B fragments of x * g (g may be NULL), and, when
// ss_out is given, per-64-block sums of x^2 ([M][ceil(K/64)]).
cudaError_t launch_prep_xfrag(const float *x, int M, int K, int ldx, const float *g, uint32_t *xfrag,
                              float *ss_out, cudaStream_t st, bool pdl);
size_t xfrag_bytes(int K);
int gemv_grid(int M, int epi, int N);      // row blocks (64 rows) of a launch
int gemv_row_blocks(int N);
constexpr int kGemvRowAlign = 64;           // tiled weights are padded to this many rows
// Row-major [N, K] bf16 -> the GEMV's fragment-tiled layout [Np, Kp]
// (Np = N rounded up to kGemvRowAlign, Kp = K rounded up to 16).
cudaError_t launch_tile_weights(uint16_t *dst, const uint16_t *src, int N, int K, int Np, int Kp,
                                cudaStream_t st);
// x[m][k] = rows_m[k] + E[tokens[m]][k] for m < n, k < K, with E [vocab, K]
// bf16 in the fragment-tiled layout above.  Row m of the addend is
// row_ptrs[m] (a device array of n pointers) when row_ptrs is given, else
// rows + m * row_stride, else nothing (a plain lookup).  A token outside
// [0, vocab) adds no embedding and sets bit 1 of *err.
cudaError_t launch_embed_tokens(float *x, const float *const *row_ptrs, const float *rows, size_t row_stride,
                                const int *tokens, int n, const uint16_t *E, int vocab, int K,
                                unsigned *err, cudaStream_t st);

struct AttnParams {
    const float *q;           // [M][4096], RoPE applied
    const StreamSlot *slots;  // [M]
    int layer;
    float *out;               // [M][4096] or NULL
    uint32_t *xfrag_out;      // the output as the wo GEMV's B fragments, or NULL
    uint16_t *out_hilo;       // the output as bf16 hi / lo rows (hilo_row layout), or NULL
    float *part_o;            // [M][32][S][128]
    float *part_ml;           // [M][32][S][2]
    unsigned *counters;       // [M][8], zero between launches
    int S;                    // key splits per KV head
    const void *pf;           // weights of a later kernel to start pulling into L2 (or NULL)
    unsigned long long pf_bytes;   // a multiple of 16
    int deep_hint;            // keys the caller expects per row (0: unknown); selects v5 for long contexts
    int min_keys;             // v5: fewest keys per CTA (set by launch_attn_decode)
    StreamSlot slot1;         // with slot_inline (M = 1): the row's slot by value, slots unused
    int slot_inline;
    int variant;              // 0: chosen by launch_attn_decode; 4: the v4 kernel
};
constexpr int kAttnSplits = 128;   // >= 8192 / 64 keys per split
constexpr int kAttnDeepKeys = 2048;  // keys from which one or two rows take the v5 attention kernel

// fp16 range events of the encoder path since the last reset, on the
// current device (vc_gemm_tc.cu: clamped SwiGLU output chunks and
// non-finite rows reaching a norm pass).
unsigned long long f16_saturations_gemm(bool reset);

// ---- the persistent decode step (vc_step_persist.cu) ----
struct PersistLayer {             // device array, one entry per decoder layer
    const uint16_t *qkv, *wo, *w13, *w2;   // fragment-tiled weights
    const float *g_attn, *g_ffn;           // the folded norm weights
};
struct PersistParams {
    const PersistLayer *layers;   // [n_layers]
    int n_layers;
    int M;                        // streams (1..8)
    int with_head;                // LM head + argmax after the layers
    int vocab;
    const uint16_t *lm;           // tiled LM head / token table
    const float *final_norm;
    const StreamSlot *slots;      // [M]
    const float *rope;            // [M][128]
    float *x;                     // [M][3072] residual stream
    float *q;                     // [M][4096]
    uint32_t *xf_attn, *xf_ffn, *xf_att, *xf_h;   // activation fragments
    float *ss_attn, *ss_ffn;      // [M][48] sums of x^2 per row block
    float *logits;                // [M][vocab]
    ArgmaxPartial *amax;          // [vocab / 64][M]
    int *tokens;                  // [M]
    float *part_o, *part_ml;      // attention split partials ([M][32][kAttnSplits] x 128 / x 2)
    float *gpart;                 // split-K partials: [items][64][8]
    unsigned *sync;               // persist_sync_words() words, zero at launch
    unsigned *err;
    int ks[5];                    // K slices of q|k|v, wo, w1|w3, w2, LM head
    int l2_ahead;                 // weight stages the L2 prefetch runs ahead of the ring
};
// Whether this slicing's activation slices fit one CTA's shared area (host check).
bool persist_slicing_fits(const int *ks, int vocab, int grid);
size_t persist_sync_words();
size_t persist_gpart_floats(const PersistParams &p);
// One cooperative launch of gridDim = the SM count.
cudaError_t launch_step_persist(const PersistParams &p, cudaStream_t st, int *grid_out);

cudaError_t launch_attn_decode(int M, const AttnParams &p, cudaStream_t st, bool pdl);

// Alternatives from device logits (stream_fill_alts semantics).
cudaError_t launch_fill_alts(const float *logits, int vocab, const int *best, int n_alt,
                             float cutoff, int *out_ids, cudaStream_t st);

// ---- tcgen05 tensor-core GEMM (vc_gemm_tc.cu) ----
enum TcEpi : int {
    TC_STORE = 0,     // out = acc (+ bias) (GELU if act == 1); fp32, or bf16 when out_bf16
    TC_RESID = 1,     // out += acc (+ bias)   (fp32 residual stream)
    TC_SWIGLU = 2,    // cols (2i, 2i+1) = (gate_i, up_i) -> out_bf16[i] = silu(g) * u
    TC_QKV_ENC = 3,   // encoder q|k|v: bias, RoPE, q (fp16) out, k / v (fp16) to the ring
    TC_QKV_DEC = 4,   // decoder q|k|v: RoPE, q (fp32) out, k / v (fp32) to each row's ring slot
};

// One stream's rows in a batched encoder launch: rows [row0, next row0) of
// the launch sit at logical positions *pos0_dev + (row - row0) of this
// state's ring (layer `TcGemmParams::layer` at k_ring + layer * cap * 2048).
struct EncSeg {
    uint16_t *k_ring, *v_ring;   // layer 0 base, fp16 [layers][cap][2048]
    const int *pos0_dev;
    int cap;
    int row0;
};
constexpr int kEncMaxSegs = 8;

struct TcGemmParams {
    int M, N, K;
    float *out;              // fp32 [M, ldo]
    int ldo;
    const float *bias;       // [N] (TC_QKV_ENC: the q bias) or NULL
    const float *bias2;      // TC_QKV_ENC: the v bias, or NULL
    int act;                 // TC_STORE: 0 none, 1 tanh-GELU
    uint16_t *out_bf16;      // bf16 output [M, ldo_bf16] or NULL
    int ldo_bf16;
    // TC_QKV_ENC
    const float *rope;       // cos plane [32][rope_ld] then sin plane [32][rope_ld], indexed
    int rope_ld;             //   [pair d][row]; or NULL: cos/sin(pos * inv_freq[d]) on the device
    const float *inv_freq;   // [32]
    const int *pos0_dev;     // if non-NULL, the logical position of row 0 (overrides pos0)
    uint16_t *q_out;         // fp16 [M][2048]
    uint16_t *k_ring;        // fp16 [cap][2048] (this layer)
    uint16_t *v_ring;
    int cap, pos0;           // row r sits at logical position pos0 + r, slot (pos0 + r) % cap
    unsigned *err;           // raised when a bounded wait expires
    // split-K (few tiles, long K): the caller's fp32 workspace and zeroed
    // counters; launch_tc_gemm picks the split count ksplit (1: none)
    float *ws;               // ws_floats; launch_tc_gemm fits ksplit x tiles x 128 x BN floats
    size_t ws_floats;
    unsigned *ws_cnt;        // kTcSplitCounters counters, zero between launches
    int ksplit;
    int f16;                 // A and W are fp16 (kind::f16 with fp16 operands) and so are the
                             //   16-bit outputs (out_bf16, SwiGLU h); else bf16
    // split activations (decoder prefill): A is in the hi / lo layout of
    // hilo_row() (per 64 output rows, their bf16 hi rows then their bf16
    // lo = x - hi rows); one 128-row MMA tile covers both and the epilogue
    // adds accumulator rows r and r + 64: fp32-level products from bf16 MMAs
    int hilo;
    int out_hilo;            // TC_SWIGLU: h written as bf16 hi / lo rows in that layout
    // TC_QKV_DEC
    float *q32;              // fp32 [M][4096]
    const StreamSlot *slots; // [M]: each row's ring and slot
    int layer;
    const float *rope_rows;  // [M][128]: (cos, sin) of pair d at [2d], [2d + 1]
    // TC_QKV_ENC over several streams' rows (batched encoder), or NULL
    const EncSeg *segs;      // device [n_segs], row0 ascending
    int n_segs;
    // RMSNorm folded into the GEMMs around it (encoder): TC_RESID also writes
    // the next GEMM's operand fp16(x * xn_gain) (x the updated residual, not
    // yet normalised) and, per row, the sum of squares of x over each
    // 32-column chunk; TC_QKV_ENC / TC_SWIGLU scale accumulator row r by
    // 1 / sqrt(sum / K + eps) from those sums (ss_in) before their epilogue
    uint16_t *xn_out;        // TC_RESID: [M][ldo] fp16, or NULL
    const float *xn_gain;    // TC_RESID: [N], the next norm's weights
    float *ss_out;           // TC_RESID: [N / 32][ss_ld]
    const float *ss_in;      // TC_QKV_ENC / TC_SWIGLU: [K / 32][ss_ld], or NULL
    int ss_ld;               // rows per chunk plane (>= M)
    int vec;                 // set by launch_tc_gemm: all destinations allow 16-byte stores
    int tma_out;             // set by launch_tc_gemm: the epilogue stores through TMA
    int cluster;             // set by launch_tc_gemm: the ksplit slices of a tile are one cluster,
                             //   reduced through distributed shared memory (one row tile)
    int fold_tma;            // set by launch_tc_gemm: the folded norm's producer (TC_RESID with xn_out)
                             //   moves the residual tiles through TMA (a CTA's last tile)
};

constexpr int kTcSplitCounters = 4096;   // split-K tickets a caller provides (8 per tile)
constexpr size_t kEncSplitFloats = (size_t)4 << 20;   // the encoder state's split-K workspace (16 MB)

// C = A . W^T with bf16 A [M, K] and W [N, K] (row-major, 16-byte aligned,
// K % 8 == 0).  bn = 0 picks the tile width.  With pdl the kernel starts
// loading W before the preceding kernel has finished: W must not be written
// by that kernel (resident weights only).
cudaError_t launch_tc_gemm(int epi, const TcGemmParams &p, const void *A, const void *W, cudaStream_t st,
                           bool pdl, int bn = 0);
int tc_gemm_bn(int M, int N);
// fp32 rows -> bf16 (or fp16, f16) rows, optionally RMS-normalised with weights w.
cudaError_t launch_rows_to_bf16(const float *x, int M, int K, int ld, const float *w, uint16_t *out,
                                cudaStream_t st, bool pdl, bool f16 = false);
// fp32 rows -> fp16(x * w) rows (not normalised) and, per row, the sum of
// squares of x over each 32-column chunk, ss[K / 32][ss_ld]: the operand and
// the row scales of a consumer GEMM with ss_in (K % 128 == 0, K <= 2048)
cudaError_t launch_rows_prenorm(const float *x, int M, int K, const float *w, uint16_t *out, float *ss, int ss_ld,
                                cudaStream_t st, bool pdl);
// the same as bf16 hi / lo rows in the hilo_row layout (split activations)
cudaError_t launch_rows_prenorm_hilo(const float *x, int M, int K, const float *w, uint16_t *out, float *ss,
                                     int ss_ld, cudaStream_t st, bool pdl);
// In place: bf16 -> fp16 (round to nearest even; the values of bf16 weights
// are inside fp16's range).
// fp32 rows -> bf16 hi / lo rows in the hilo_row layout, v = x
// (RMS-normalised with weights w when w).
cudaError_t launch_rows_hilo(const float *x, int M, int K, int ld, const float *w, uint16_t *out,
                             cudaStream_t st, bool pdl);
cudaError_t launch_bf16_to_f16(uint16_t *p, size_t n, cudaStream_t st);

// ---- encoder (vc_encoder.cu) ----
struct EncAttnParams {
    const uint16_t *q;        // fp16 [M][2048], RoPE applied
    const uint16_t *k_ring;   // fp16 [cap][2048], this layer
    const uint16_t *v_ring;
    int cap;                  // ring positions (>= M + 749)
    int pos0;                 // logical position of query row 0
    const int *pos0_dev;      // if non-NULL, overrides pos0
    int M;
    uint16_t *out;            // [M][2048], bf16 or (f16) fp16: the wo GEMM's A operand
    int f16;
    unsigned *err;            // raised when a bounded wait expires (tensor-core kernel)
    // key split (tensor-core kernel, chunks with few row tiles): ksplit CTAs
    // per (row tile, head) take consecutive key blocks and leave unnormalised
    // partials; the last to finish merges them (ticket in cnt)
    int ksplit;               // 1 (or 0): no split
    float *part;              // [ksplit][M][32 heads] x (64 o + max + sum) floats
    unsigned *cnt;            // [row tiles][32], zero between launches
    // 1: with ksplit <= 1, the launcher may split the key blocks over a
    // thread-block cluster instead (partials merged through distributed
    // shared memory; no workspace); set by the launcher to the cluster size
    int kcluster;
    // 1: launched beside other attention launches (one per stream of a
    // batched encoder step): three CTAs per SM unless VOX_CUDA_ENC_ATTN_SPREAD
    // asks otherwise (spreading one CTA per SM would queue the streams)
    int shared_sms;
};
// key splits of the tensor-core encoder attention for an M-row chunk whose
// partials may take ws_floats floats
int enc_attn_ksplit(int M, size_t ws_floats);
// Windowed encoder attention: the tcgen05 kernel when enc_attn_tc_supported
// (ring capacity a multiple of 128, err set) unless VOX_CUDA_ENC_ATTN=mma,
// else the mma.sync kernel.
cudaError_t launch_enc_attn(const EncAttnParams &p, cudaStream_t st, bool pdl);
bool enc_attn_tc_supported(const EncAttnParams &p);
cudaError_t launch_enc_attn_tc(const EncAttnParams &p, cudaStream_t st, bool pdl);
constexpr int kEncRingAlign = 128;   // encoder ring capacities are multiples of this
cudaError_t launch_rows_rmsnorm(float *x, int M, int K, const float *w, cudaStream_t st, bool pdl);
// RoPE planes of a batched encoder launch: each row's position from its segment
cudaError_t launch_enc_rope_table_segs(float *tab, int ld, int M, const EncSeg *segs, int n_segs,
                                       const float *inv_freq, cudaStream_t st, bool pdl);
// A kernel whose bounded wait cannot complete: raises *err after wait_ns.
cudaError_t launch_stuck_wait(unsigned *err, unsigned long long wait_ns, cudaStream_t st);
// *dst = v in stream order (the value travels as a kernel argument)
cudaError_t launch_set_int(int *dst, int v, cudaStream_t st);
// RoPE planes of a chunk for the q|k epilogue: tab[d][row] = cos and
// tab[32 + d][row] = sin (row stride ld) of the angle of logical position
// *pos0_dev + row, taken from the host table src[row][32] (cos, sin) pairs
// when src is non-NULL, else computed on the device from inv_freq.
cudaError_t launch_enc_rope_table(float *tab, int ld, int M, const float *src, const int *pos0_dev,
                                  const float *inv_freq, cudaStream_t st, bool pdl);

// ---- conv stem (vc_stem.cu) ----
cudaError_t launch_stem_im2col0(const float *mel_new, const float *mel_hist, int n, uint16_t *a0, cudaStream_t st);
cudaError_t launch_stem_im2col1(const uint16_t *c0_new, const uint16_t *c0_hist, long long f0, long long u0,
                                int n_out, uint16_t *a1, cudaStream_t st);
cudaError_t launch_stem_state(const float *mel_new, int n, float *mel_hist, const uint16_t *c0_new,
                              uint16_t *c0_hist, cudaStream_t st);
cudaError_t launch_f32_to_f16(const float *src, uint16_t *dst, size_t n, cudaStream_t st);

// log-mel front end (vc_mel.cu; voxtral_audio.c:31-37 constants)
constexpr int kMelRate = 16000;
constexpr int kMelBins = 128;
constexpr int kMelHop = 160;
constexpr int kMelWin = 400;                  // window = DFT length
constexpr int kMelFreq = kMelWin / 2 + 1;     // 201 bins
constexpr int kMelCenterPad = kMelWin / 2;    // center=True padding
constexpr float kMelLogMax = 1.5f;
constexpr int kMelFrames = 4;                 // frames per CTA

struct MelTables {          // device copies of mel_host_tables' output
    const float *win;       // [400] periodic Hann
    const float *cos_t;     // [400][201] cos(2 pi k n / 400), bin fastest
    const float *sin_t;     // [400][201]
    const float *filt_t;    // [201][128] mel filters, mel fastest
};
void mel_host_tables(float *win, float *cos_t, float *sin_t, float *filt_t);
cudaError_t launch_mel_frames(const float *ring, long long mask, long long pad, long long t0, int n_frames,
                              const MelTables &t, float *out, cudaStream_t st);
cudaError_t launch_mel_reflect(const float *ring, long long mask, long long pad, long long src0, int n,
                               float *dst, cudaStream_t st);

// Set the message vox_cuda_last_error() returns on the calling thread.
void set_last_error(const char *fmt, ...);

cudaError_t launch_rope(float *x, int n_heads, int head_dim, const float *cs, cudaStream_t st);
cudaError_t launch_fill_normal_bf16(uint16_t *dst, size_t n, uint64_t seed, float std,
                                    cudaStream_t st);

}  // namespace vc
