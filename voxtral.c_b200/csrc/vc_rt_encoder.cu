// vc_rt_encoder.cu - the C ABI of voxtral_cuda.h, part 3: the resident
// encoder and adapter (fp16 tensor-core operands), per-stream encoder rings,
// the synchronous / asynchronous / batched chunk steps and the profile entry.
#include "vc_runtime.h"

#include <map>

using namespace vc;
using namespace vc::rt;

// ---------------------------------------------------------------------------
// encoder chunk + adapter
// ---------------------------------------------------------------------------

namespace {

constexpr int kEncSsChunks = kEncDim / 32;   // folded RMSNorm: 32-column chunks of a residual row

// The RMSNorms fold into the GEMMs around them (the residual epilogues write
// the next operand and sums of squares, the consumers scale their rows):
// five launches per layer instead of seven, for chunks of any size (or of
// up to VOX_CUDA_ENC_FOLD_MAX_ROWS rows).  Measured per 32-layer chunk: 100
// rows 2.36 -> 2.12 ms, 500 rows 3.62 -> 3.49 ms; 1500 rows 4.62 -> 4.74 ms
// while the residual epilogue read and wrote its rows with per-row direct
// loads and stores (one tile per CTA leaves that epilogue exposed), and
// 4.63 -> 4.53 ms since the drained stage ring takes the residual tiles in
// and out by TMA.  VOX_CUDA_ENC_FOLD_NORM = 0 turns folding off (read when a
// graph is captured).
bool enc_fold_norm(int M) {
    const char *e = getenv("VOX_CUDA_ENC_FOLD_NORM");
    if (e && e[0] == '0') return false;
    const char *r = getenv("VOX_CUDA_ENC_FOLD_MAX_ROWS");
    const int max_rows = (r && atoi(r) > 0) ? atoi(r) : 1 << 30;
    return M <= max_rows;
}

struct EncLayer {
    const uint16_t *qkv = nullptr;   // [6144, 1280] wq|wk|wv
    const uint16_t *wo = nullptr;    // [1280, 2048]
    const uint16_t *w13 = nullptr;   // [10240, 1280] w1/w3 row-interleaved
    const uint16_t *w2 = nullptr;    // [1280, 5120]
    const float *bq = nullptr, *bv = nullptr, *bo = nullptr, *b2 = nullptr;
    const float *attn_norm = nullptr, *ffn_norm = nullptr;
};

}  // namespace

namespace {

// Workspace of batched encoder launches (several states' chunks as one row
// block, vox_cuda_encoder_step_batch_dev): the row-wise kernels and GEMMs run
// once over all rows; each state's attention runs on its own side stream,
// forked and joined inside the captured graph.
struct EncBatch {
    int cap = 0;                  // rows
    char *ws = nullptr;
    size_t ws_bytes = 0;
    float *x = nullptr;           // [cap][1280]
    uint16_t *xn16 = nullptr;     // [cap][1280] fp16
    uint16_t *att16 = nullptr;    // [cap][2048]
    uint16_t *h16 = nullptr;      // [cap][5120]
    uint16_t *q16 = nullptr;      // [cap][2048]
    float *rope = nullptr;        // planes [64][cap]
    float *ss = nullptr;          // folded RMSNorm: sums of squares [1280 / 32][cap]
    float *split = nullptr;       // split-K partials [kEncSplitFloats]
    unsigned *split_cnt = nullptr;
    unsigned *err = nullptr;
    unsigned *h_err = nullptr;    // pinned
    cudaEvent_t err_ev = nullptr;
    bool err_pending = false;
    cudaStream_t side[kEncMaxSegs] = {};
    cudaEvent_t fork = nullptr, join[kEncMaxSegs] = {};
    struct Graph {
        cudaGraphExec_t exec = nullptr;
        EncSeg *segs = nullptr;   // device [n]: this key's segments
    };
    // (states, rows) of a launch -> its graph
    std::map<std::vector<std::pair<const void *, int>>, Graph> graphs;
};
void free_enc_batch(DevCtx *c, EncBatch *b);
// Destroy the batched graphs that name `state` (all of them when NULL): a
// graph holds its states' ring and position pointers.
void drop_batch_graphs(EncBatch *b, const void *state);

}  // namespace

struct vox_cuda_encoder {
    int device = 0;
    int n_layers = 0;
    EncLayer L[kEncLayers];
    const float *norm = nullptr;
    const uint16_t *adapter0 = nullptr, *adapter1 = nullptr;
    const float *inv_freq = nullptr;   // [32] RoPE inverse frequencies (head_dim 64)
    std::vector<std::pair<void *, size_t>> owned;
    bool pdl = true;
    EncBatch *batch = nullptr;
    std::mutex mu;   // serialises batched launches (they share `batch`)
};

struct vox_cuda_enc_state {
    vox_cuda_encoder *enc = nullptr;
    int max_chunk = 0, cap = 0, pos = 0;
    uint16_t *k_ring = nullptr, *v_ring = nullptr;   // fp16 [layers][cap][2048]
    size_t ring_bytes = 0;
    char *ws = nullptr;                              // workspace block
    size_t ws_bytes = 0;
    float *x = nullptr;          // [Mx][1280] residual stream (fp32)
    uint16_t *xn16 = nullptr;    // [Mx][1280] fp16 activations of the next GEMM: normalised, or
                                 //   (folded RMSNorm) x * norm weights, rows scaled by the consumer
    float *ss = nullptr;         // folded RMSNorm: sums of squares per 32-column chunk [40][Mx]
    uint16_t *att16 = nullptr;   // [Mx][2048] bf16 attention output
    uint16_t *h16 = nullptr;     // [Mx][5120] bf16 SwiGLU output
    uint16_t *q16 = nullptr;     // [Mx][2048] fp16 queries
    float *rope = nullptr;       // RoPE planes [64][Mx]: cos of pair d at [d][row], sin at [32 + d][row]
    float *rope_src = nullptr;   // the host's table [Mx][64] (cos, sin pairs), when given
    float *aout = nullptr;       // adapter: [Mx/4][3072] fp32 out (Mx/4 x 5120 fp32 in shares x)
    uint16_t *a16 = nullptr;     // adapter: [Mx/4][5120] bf16 in
    uint16_t *mid16 = nullptr;   // adapter: [Mx/4][3072] bf16 mid
    unsigned *err = nullptr;
    int *pos_dev = nullptr;      // logical position of the chunk's first row
    float *split = nullptr;      // split-K partials of small-M GEMMs [kEncSplitFloats]
    unsigned *split_cnt = nullptr;
    float *h_rope = nullptr;     // pinned [Mx][64]
    int *h_pos = nullptr;        // pinned
    unsigned *h_err = nullptr;   // pinned: the error flag as of the last asynchronous step
    cudaEvent_t err_ev = nullptr;
    bool err_pending = false;
    cudaEvent_t tail = nullptr;  // the end of the last asynchronous step
    bool tail_set = false;
    std::map<std::pair<int, int>, cudaGraphExec_t> graphs;   // (rows, rope table?) -> step graph
};

extern "C" vox_cuda_encoder *vox_cuda_encoder_create(const vox_cuda_enc_weights *w) {
    DevCtx *c = cur_ctx();
    if (!c) return nullptr;
    if (!w || w->n_layers <= 0 || w->n_layers > kEncLayers || !w->norm || !w->adapter0 || !w->adapter1) {
        set_error("encoder_create: bad weight descriptor");
        return nullptr;
    }
    for (int l = 0; l < w->n_layers; l++) {
        const vox_cuda_enc_layer_weights &L = w->layers[l];
        if (!L.wq || !L.wk || !L.wv || !L.wo || !L.w1 || !L.w2 || !L.w3 || !L.wq_bias || !L.wv_bias ||
            !L.wo_bias || !L.w2_bias || !L.attention_norm || !L.ffn_norm) {
            set_error("encoder_create: layer %d has a NULL tensor", l);
            return nullptr;
        }
    }
    vox_cuda_encoder *e = new vox_cuda_encoder();
    e->device = c->device;
    e->n_layers = w->n_layers;
    const char *pdl_env = getenv("VOX_CUDA_PDL");
    e->pdl = !(pdl_env && pdl_env[0] == '0');
    const cudaMemcpyKind kind = w->weights_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    bool ok = true;
    Uploader up(c->stream, !w->weights_on_device, c);   // host weights: pinned, pipelined
    auto alloc = [&](size_t bytes) -> void * {
        void *p = nullptr;
        if (dev_alloc(c, &p, bytes) != cudaSuccess) return nullptr;
        e->owned.push_back({p, bytes});
        return p;
    };
    auto copy_f32 = [&](const float *src, size_t n) -> const float * {
        float *d = (float *)alloc(n * 4);
        if (!d || cudaMemcpy(d, src, n * 4, kind) != cudaSuccess) {
            ok = false;
            return nullptr;
        }
        return d;
    };
    const size_t D = kEncDim, Q = kEncQkv, H = kEncHidden;
    for (int l = 0; l < w->n_layers && ok; l++) {
        const vox_cuda_enc_layer_weights &L = w->layers[l];
        EncLayer &o = e->L[l];
        for (int j = 0; j < l; j++) {   // aliased layers share device copies
            const vox_cuda_enc_layer_weights &J = w->layers[j];
            if (J.wq == L.wq && J.wk == L.wk && J.wv == L.wv && J.wo == L.wo && J.w1 == L.w1 && J.w2 == L.w2 &&
                J.w3 == L.w3) {
                o.qkv = e->L[j].qkv;
                o.wo = e->L[j].wo;
                o.w13 = e->L[j].w13;
                o.w2 = e->L[j].w2;
                break;
            }
        }
        if (!o.qkv) {
            uint16_t *qkv = (uint16_t *)alloc(3 * Q * D * 2);
            uint16_t *wo = (uint16_t *)alloc(D * Q * 2);
            uint16_t *w13 = (uint16_t *)alloc(2 * H * D * 2);
            uint16_t *w2 = (uint16_t *)alloc(D * H * 2);
            ok = qkv && wo && w13 && w2;
            if (!ok) break;
            ok &= up.copy(qkv, L.wq, Q * D * 2) == cudaSuccess;
            ok &= up.copy(qkv + Q * D, L.wk, Q * D * 2) == cudaSuccess;
            ok &= up.copy(qkv + 2 * Q * D, L.wv, Q * D * 2) == cudaSuccess;
            ok &= up.copy(wo, L.wo, D * Q * 2) == cudaSuccess;
            ok &= up.copy2d(w13, 2 * D * 2, L.w1, D * 2, D * 2, H) == cudaSuccess;
            ok &= up.copy2d(w13 + D, 2 * D * 2, L.w3, D * 2, D * 2, H) == cudaSuccess;
            ok &= up.copy(w2, L.w2, D * H * 2) == cudaSuccess;
            // the tensor-core GEMMs take fp16 operands: activations keep 11
            // mantissa bits instead of bf16's 8 (weights convert exactly
            // except below fp16's normal range, ~6e-5); on the upload stream
            ok &= launch_bf16_to_f16(qkv, 3 * Q * D, c->stream) == cudaSuccess;
            ok &= launch_bf16_to_f16(wo, D * Q, c->stream) == cudaSuccess;
            ok &= launch_bf16_to_f16(w13, 2 * H * D, c->stream) == cudaSuccess;
            ok &= launch_bf16_to_f16(w2, D * H, c->stream) == cudaSuccess;
            o.qkv = qkv;
            o.wo = wo;
            o.w13 = w13;
            o.w2 = w2;
        }
        o.bq = copy_f32(L.wq_bias, Q);
        o.bv = copy_f32(L.wv_bias, Q);
        o.bo = copy_f32(L.wo_bias, D);
        o.b2 = copy_f32(L.w2_bias, D);
        o.attn_norm = copy_f32(L.attention_norm, D);
        o.ffn_norm = copy_f32(L.ffn_norm, D);
    }
    if (ok) {
        // RoPE inverse frequencies with the host formula of vox_compute_rope_freqs
        // (voxtral_kernels.c:494); the device forms pos * inv_freq and its cos/sin
        float invf[kEncHeadDim / 2];
        for (int d = 0; d < kEncHeadDim / 2; d++)
            invf[d] = 1.0f / powf(kRopeTheta, (float)(2 * d) / (float)kEncHeadDim);
        float *dinv = (float *)alloc(sizeof(invf));
        ok = dinv && cudaMemcpy(dinv, invf, sizeof(invf), cudaMemcpyHostToDevice) == cudaSuccess;
        e->inv_freq = dinv;
    }
    if (ok) {
        e->norm = copy_f32(w->norm, D);
        uint16_t *a0 = (uint16_t *)alloc((size_t)kDecDim * 4 * D * 2);
        uint16_t *a1 = (uint16_t *)alloc((size_t)kDecDim * kDecDim * 2);
        ok = ok && a0 && a1;
        if (ok) {
            ok &= up.copy(a0, w->adapter0, (size_t)kDecDim * 4 * D * 2) == cudaSuccess;
            ok &= up.copy(a1, w->adapter1, (size_t)kDecDim * kDecDim * 2) == cudaSuccess;
            ok &= launch_bf16_to_f16(a0, (size_t)kDecDim * 4 * D, c->stream) == cudaSuccess;
            ok &= launch_bf16_to_f16(a1, (size_t)kDecDim * kDecDim, c->stream) == cudaSuccess;
            ok &= cudaStreamSynchronize(c->stream) == cudaSuccess;
            e->adapter0 = a0;
            e->adapter1 = a1;
        }
    }
    if (!ok) {
        set_error("encoder_create: weight upload failed (%s)", cudaGetErrorString(cudaGetLastError()));
        vox_cuda_encoder_free(e);
        return nullptr;
    }
    return e;
}

extern "C" void vox_cuda_encoder_free(vox_cuda_encoder *e) {
    if (!e) return;
    DevCtx *c = ctx_for(e->device);
    cudaSetDevice(e->device);
    if (c) cudaStreamSynchronize(c->stream);
    free_enc_batch(c, e->batch);
    for (auto &pr : e->owned)
        if (c) dev_free(c, pr.first, pr.second);
        else cudaFree(pr.first);
    delete e;
}

extern "C" vox_cuda_enc_state *vox_cuda_enc_state_create(vox_cuda_encoder *e, int max_chunk) {
    if (!e || max_chunk <= 0 || max_chunk > 8192) {
        set_error("enc_state_create: max_chunk must be 1..8192");
        return nullptr;
    }
    DevCtx *c = ctx_for(e->device);
    if (!c) {
        set_error("enc_state_create: device not initialised");
        return nullptr;
    }
    cudaSetDevice(e->device);
    vox_cuda_enc_state *s = new vox_cuda_enc_state();
    s->enc = e;
    s->max_chunk = (max_chunk + 3) / 4 * 4;
    s->cap = (kEncWindow + s->max_chunk + kEncRingAlign - 1) / kEncRingAlign * kEncRingAlign;
    s->ring_bytes = (size_t)e->n_layers * s->cap * kEncQkv * 2;
    const size_t Mx = s->max_chunk;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        size_t o = off;
        off = align_up(off + bytes, 256);
        return o;
    };
    const size_t o_x = take(Mx * kEncDim * 4);
    const size_t o_xn = take(Mx * kEncDim * 2);
    const size_t o_att = take(Mx * kEncQkv * 2);
    const size_t o_h = take(Mx * kEncHidden * 2);
    const size_t o_q = take(Mx * kEncQkv * 2);
    const size_t o_rope = take(Mx * kEncHeadDim * 4);
    const size_t o_rope_src = take(Mx * kEncHeadDim * 4);
    const size_t o_ss = take(Mx * kEncSsChunks * 4);
    const size_t o_aout = take(Mx / 4 * kDecDim * 4);
    const size_t o_a16 = take(Mx / 4 * 4 * kEncDim * 2);
    const size_t o_mid = take(Mx / 4 * kDecDim * 2);
    const size_t o_err = take(sizeof(unsigned));
    const size_t o_pos = take(sizeof(int));
    const size_t o_split = take(kEncSplitFloats * 4);            // split-K partials
    const size_t o_split_cnt = take(kTcSplitCounters * 4);       // split-K tickets
    s->ws_bytes = off;
    if (dev_alloc(c, (void **)&s->k_ring, s->ring_bytes) != cudaSuccess ||
        dev_alloc(c, (void **)&s->v_ring, s->ring_bytes) != cudaSuccess ||
        dev_alloc(c, (void **)&s->ws, s->ws_bytes) != cudaSuccess ||
        cudaHostAlloc((void **)&s->h_rope, Mx * kEncHeadDim * 4, cudaHostAllocDefault) != cudaSuccess ||
        cudaHostAlloc((void **)&s->h_pos, sizeof(int), cudaHostAllocDefault) != cudaSuccess ||
        cudaHostAlloc((void **)&s->h_err, sizeof(unsigned), cudaHostAllocDefault) != cudaSuccess ||
        cudaEventCreateWithFlags(&s->err_ev, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&s->tail, cudaEventDisableTiming) != cudaSuccess) {
        set_error("enc_state_create: allocation failed");
        vox_cuda_enc_state_free(s);
        return nullptr;
    }
    *s->h_err = 0;
    s->x = (float *)(s->ws + o_x);
    s->xn16 = (uint16_t *)(s->ws + o_xn);
    s->att16 = (uint16_t *)(s->ws + o_att);
    s->h16 = (uint16_t *)(s->ws + o_h);
    s->q16 = (uint16_t *)(s->ws + o_q);
    s->rope = (float *)(s->ws + o_rope);
    s->rope_src = (float *)(s->ws + o_rope_src);
    s->ss = (float *)(s->ws + o_ss);
    s->aout = (float *)(s->ws + o_aout);
    s->a16 = (uint16_t *)(s->ws + o_a16);
    s->mid16 = (uint16_t *)(s->ws + o_mid);
    s->err = (unsigned *)(s->ws + o_err);
    s->pos_dev = (int *)(s->ws + o_pos);
    s->split = (float *)(s->ws + o_split);
    s->split_cnt = (unsigned *)(s->ws + o_split_cnt);
    if (cudaMemset(s->k_ring, 0, s->ring_bytes) != cudaSuccess ||
        cudaMemset(s->v_ring, 0, s->ring_bytes) != cudaSuccess ||
        cudaMemset(s->ws, 0, s->ws_bytes) != cudaSuccess) {
        set_error("enc_state_create: clear failed");
        vox_cuda_enc_state_free(s);
        return nullptr;
    }
    return s;
}

extern "C" void vox_cuda_enc_state_free(vox_cuda_enc_state *s) {
    if (!s) return;
    DevCtx *c = ctx_for(s->enc->device);
    cudaSetDevice(s->enc->device);
    if (c) cudaStreamSynchronize(c->stream);   // also waits for asynchronous steps (see step_dev)
    if (c) {
        dev_free(c, s->k_ring, s->k_ring ? s->ring_bytes : 0);
        dev_free(c, s->v_ring, s->v_ring ? s->ring_bytes : 0);
        dev_free(c, s->ws, s->ws ? s->ws_bytes : 0);
    }
    if (s->h_rope) cudaFreeHost(s->h_rope);
    if (s->h_pos) cudaFreeHost(s->h_pos);
    if (s->h_err) cudaFreeHost(s->h_err);
    if (s->err_ev) cudaEventDestroy(s->err_ev);
    if (s->tail) cudaEventDestroy(s->tail);
    for (auto &kv : s->graphs) cudaGraphExecDestroy(kv.second);
    {   // batched launches captured with this state must not outlive it
        std::lock_guard<std::mutex> lk(s->enc->mu);
        if (s->enc->batch) drop_batch_graphs(s->enc->batch, s);
    }
    delete s;
}

extern "C" int vox_cuda_enc_state_reset(vox_cuda_enc_state *s) {
    if (!s) return VOX_CUDA_ERR_ARG;
    s->pos = 0;
    return VOX_CUDA_OK;
}

extern "C" int vox_cuda_enc_state_position(const vox_cuda_enc_state *s) { return s ? s->pos : -1; }

namespace {

// The 32 layers + final norm over s->x: M rows at the logical positions
// *s->pos_dev.. (read on the device, so the sequence can be replayed as a
// graph); RoPE from the uploaded table (table) or from a table computed on
// the device for this chunk.  evs (profiling only): 2 events per launch,
// recorded around it.
int enqueue_encoder(vox_cuda_enc_state *s, int M, bool table, cudaStream_t st, cudaEvent_t *evs = nullptr,
                    int *ev_phase = nullptr) {
    vox_cuda_encoder *e = s->enc;
    const bool pdl = e->pdl && evs == nullptr;
    const bool fold = enc_fold_norm(M);
    int ei = 0;
#define VC_EV_BEGIN(ph) do { if (evs) { ev_phase[ei / 2] = (ph); VC_TRY(cudaEventRecord(evs[ei++], st)); } } while (0)
#define VC_EV_END() do { if (evs) VC_TRY(cudaEventRecord(evs[ei++], st)); } while (0)
    const size_t ring_layer = (size_t)s->cap * kEncQkv;
    VC_TRY(launch_enc_rope_table(s->rope, s->max_chunk, M, table ? s->rope_src : nullptr, s->pos_dev, e->inv_freq,
                                 st, false));
    if (fold) {   // the first layer's operand and row sums; later ones come from the w2 epilogues
        VC_EV_BEGIN(VOX_CUDA_EPROF_NORM);
        VC_TRY(launch_rows_prenorm(s->x, M, kEncDim, e->L[0].attn_norm, s->xn16, s->ss, s->max_chunk, st, pdl));
        VC_EV_END();
    }
    for (int l = 0; l < e->n_layers; l++) {
        const EncLayer &L = e->L[l];
        if (!fold) {
            VC_EV_BEGIN(VOX_CUDA_EPROF_NORM);
            VC_TRY(launch_rows_to_bf16(s->x, M, kEncDim, kEncDim, L.attn_norm, s->xn16, st, pdl, true));
            VC_EV_END();
        }
        TcGemmParams p = {};
        p.M = M;
        p.N = 3 * kEncQkv;
        p.K = kEncDim;
        p.bias = L.bq;
        p.bias2 = L.bv;
        p.rope = s->rope;
        p.rope_ld = s->max_chunk;
        p.inv_freq = e->inv_freq;
        p.pos0_dev = s->pos_dev;
        p.q_out = s->q16;
        p.k_ring = s->k_ring + l * ring_layer;
        p.v_ring = s->v_ring + l * ring_layer;
        p.cap = s->cap;
        p.err = s->err;
        p.f16 = 1;
        p.ws = s->split;
        p.ws_floats = kEncSplitFloats;
        p.ws_cnt = s->split_cnt;
        if (fold) {
            p.ss_in = s->ss;
            p.ss_ld = s->max_chunk;
        }
        VC_EV_BEGIN(VOX_CUDA_EPROF_QKV);
        VC_TRY(launch_tc_gemm(TC_QKV_ENC, p, s->xn16, L.qkv, st, pdl));
        VC_EV_END();
        EncAttnParams a = {};
        a.q = s->q16;
        a.k_ring = s->k_ring + l * ring_layer;
        a.v_ring = s->v_ring + l * ring_layer;
        a.cap = s->cap;
        a.pos0_dev = s->pos_dev;
        a.M = M;
        a.out = s->att16;
        a.f16 = 1;
        a.err = s->err;
        // few row tiles: split the key blocks (partials in the split-K
        // workspace, which no GEMM uses while the attention runs)
        a.ksplit = enc_attn_ksplit(M, kEncSplitFloats);
        a.part = s->split;
        a.cnt = s->split_cnt;
        a.kcluster = 1;   // (unless split above: the launcher may split over a cluster)
        VC_EV_BEGIN(VOX_CUDA_EPROF_ATTN);
        VC_TRY(launch_enc_attn(a, st, pdl));
        VC_EV_END();
        p = TcGemmParams{};
        p.M = M;
        p.N = kEncDim;
        p.K = kEncQkv;
        p.out = s->x;
        p.ldo = kEncDim;
        p.bias = L.bo;
        p.err = s->err;
        p.f16 = 1;
        p.ws = s->split;
        p.ws_floats = kEncSplitFloats;
        p.ws_cnt = s->split_cnt;
        if (fold) {
            p.xn_out = s->xn16;
            p.xn_gain = L.ffn_norm;
            p.ss_out = s->ss;
            p.ss_ld = s->max_chunk;
        }
        VC_EV_BEGIN(VOX_CUDA_EPROF_WO);
        VC_TRY(launch_tc_gemm(TC_RESID, p, s->att16, L.wo, st, pdl));
        VC_EV_END();
        if (!fold) {
            VC_EV_BEGIN(VOX_CUDA_EPROF_NORM);
            VC_TRY(launch_rows_to_bf16(s->x, M, kEncDim, kEncDim, L.ffn_norm, s->xn16, st, pdl, true));
            VC_EV_END();
        }
        p = TcGemmParams{};
        p.M = M;
        p.N = 2 * kEncHidden;
        p.K = kEncDim;
        p.out_bf16 = s->h16;
        p.ldo_bf16 = kEncHidden;
        p.err = s->err;
        p.f16 = 1;
        p.ws = s->split;
        p.ws_floats = kEncSplitFloats;
        p.ws_cnt = s->split_cnt;
        if (fold) {
            p.ss_in = s->ss;
            p.ss_ld = s->max_chunk;
        }
        VC_EV_BEGIN(VOX_CUDA_EPROF_W13);
        VC_TRY(launch_tc_gemm(TC_SWIGLU, p, s->xn16, L.w13, st, pdl));
        VC_EV_END();
        p = TcGemmParams{};
        p.M = M;
        p.N = kEncDim;
        p.K = kEncHidden;
        p.out = s->x;
        p.ldo = kEncDim;
        p.bias = L.b2;
        p.err = s->err;
        p.f16 = 1;
        p.ws = s->split;
        p.ws_floats = kEncSplitFloats;
        p.ws_cnt = s->split_cnt;
        if (fold && l + 1 < e->n_layers) {   // the next layer's operand and row sums
            p.xn_out = s->xn16;
            p.xn_gain = e->L[l + 1].attn_norm;
            p.ss_out = s->ss;
            p.ss_ld = s->max_chunk;
        }
        VC_EV_BEGIN(VOX_CUDA_EPROF_W2);
        VC_TRY(launch_tc_gemm(TC_RESID, p, s->h16, L.w2, st, pdl));
        VC_EV_END();
    }
    VC_EV_BEGIN(VOX_CUDA_EPROF_NORM);
    VC_TRY(launch_rows_rmsnorm(s->x, M, kEncDim, e->norm, st, pdl));
    VC_EV_END();
#undef VC_EV_BEGIN
#undef VC_EV_END
    return VOX_CUDA_OK;
}

// Upload the chunk position, then replay (capturing on first use) the
// encoder graph for this chunk shape.
int run_encoder(vox_cuda_enc_state *s, int M, bool table, cudaStream_t st) {
    // the position by value: back-to-back asynchronous calls cannot race on it
    VC_TRY(launch_set_int(s->pos_dev, s->pos, st));
    cudaGraphExec_t &g = s->graphs[std::make_pair(M, table ? 1 : 0)];
    if (!g) {
        cudaGraph_t graph = nullptr;
        VC_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
        int rc = enqueue_encoder(s, M, table, st);
        cudaError_t e = cudaStreamEndCapture(st, &graph);
        if (rc) {
            if (graph) cudaGraphDestroy(graph);
            return rc;
        }
        VC_TRY(e);
        e = cudaGraphInstantiate(&g, graph, 0);
        cudaGraphDestroy(graph);
        VC_TRY(e);
    }
    VC_TRY(cudaGraphLaunch(g, st));
    return VOX_CUDA_OK;
}

int enc_check(vox_cuda_enc_state *s, int new_len) {
    if (!s || new_len <= 0) {
        set_error("encoder step: bad arguments");
        return VOX_CUDA_ERR_ARG;
    }
    if (new_len > s->max_chunk) {
        set_error("encoder step: %d rows exceed the state's max_chunk %d", new_len, s->max_chunk);
        return VOX_CUDA_ERR_CAPACITY;
    }
    if (!ctx_for(s->enc->device)) return VOX_CUDA_ERR_UNAVAILABLE;
    cudaSetDevice(s->enc->device);
    return VOX_CUDA_OK;
}

int enc_err_check(vox_cuda_enc_state *s, cudaStream_t st) {
    unsigned err = 0;
    VC_TRY(cudaMemcpyAsync(&err, s->err, sizeof(err), cudaMemcpyDeviceToHost, st));
    VC_TRY(cudaStreamSynchronize(st));
    s->err_pending = false;   // this check covered the asynchronous steps before it
    if (err) {
        cudaMemset(s->err, 0, sizeof(unsigned));
        set_error("encoder: a device-side wait timed out (results discarded)");
        return VOX_CUDA_ERR_CUDA;
    }
    return VOX_CUDA_OK;
}

}  // namespace

extern "C" int vox_cuda_encoder_full_step(vox_cuda_enc_state *s, float *x, int new_len,
                                          const float *rope_freqs) {
    int rc = enc_check(s, new_len);
    if (rc) return rc;
    if (!x) return VOX_CUDA_ERR_ARG;
    DevCtx *c = ctx_for(s->enc->device);
    cudaStream_t st = c->stream;
    if (rope_freqs) {
        memcpy(s->h_rope, rope_freqs, (size_t)new_len * kEncHeadDim * 4);
        VC_TRY(cudaMemcpyAsync(s->rope_src, s->h_rope, (size_t)new_len * kEncHeadDim * 4, cudaMemcpyHostToDevice,
                               st));
    }
    VC_TRY(cudaMemcpyAsync(s->x, x, (size_t)new_len * kEncDim * 4, cudaMemcpyHostToDevice, st));
    if ((rc = run_encoder(s, new_len, rope_freqs != nullptr, st))) return rc;
    VC_TRY(cudaMemcpyAsync(x, s->x, (size_t)new_len * kEncDim * 4, cudaMemcpyDeviceToHost, st));
    if ((rc = enc_err_check(s, st))) return rc;
    s->pos += new_len;
    return VOX_CUDA_OK;
}

extern "C" int vox_cuda_encoder_step_dev(vox_cuda_enc_state *s, float *x_dev, int new_len, void *stream) {
    int rc = enc_check(s, new_len);
    if (rc) return rc;
    if (!x_dev) return VOX_CUDA_ERR_ARG;
    DevCtx *c = ctx_for(s->enc->device);
    cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
    // a timeout raised by an earlier chunk on this state (its flag was copied
    // back behind err_ev) is reported now
    if (s->err_pending && cudaEventQuery(s->err_ev) == cudaSuccess) {
        s->err_pending = false;
        if (*s->h_err) {
            *s->h_err = 0;
            VC_TRY(cudaMemsetAsync(s->err, 0, sizeof(unsigned), st));
            set_error("encoder: a device-side wait of an earlier chunk timed out (its results are invalid)");
            return VOX_CUDA_ERR_CUDA;
        }
    }
    // the previous asynchronous chunk may have run on another stream
    if (s->tail_set && st != c->stream) VC_TRY(cudaStreamWaitEvent(st, s->tail, 0));
    VC_TRY(cudaMemcpyAsync(s->x, x_dev, (size_t)new_len * kEncDim * 4, cudaMemcpyDeviceToDevice, st));
    if ((rc = run_encoder(s, new_len, false, st))) return rc;
    VC_TRY(cudaMemcpyAsync(x_dev, s->x, (size_t)new_len * kEncDim * 4, cudaMemcpyDeviceToDevice, st));
    if (!s->err_pending) {   // one flag copy in flight at a time
        VC_TRY(cudaMemcpyAsync(s->h_err, s->err, sizeof(unsigned), cudaMemcpyDeviceToHost, st));
        VC_TRY(cudaEventRecord(s->err_ev, st));
        s->err_pending = true;
    }
    // order the library stream (every synchronous entry point, the frees)
    // after this chunk, without a host wait
    VC_TRY(cudaEventRecord(s->tail, st));
    if (st != c->stream) VC_TRY(cudaStreamWaitEvent(c->stream, s->tail, 0));
    s->tail_set = true;
    s->pos += new_len;
    return VOX_CUDA_OK;
}

namespace {

void drop_batch_graphs(EncBatch *b, const void *state) {
    for (auto it = b->graphs.begin(); it != b->graphs.end();) {
        bool hit = state == nullptr;
        for (const auto &kv : it->first) hit = hit || kv.first == state;
        if (!hit) {
            ++it;
            continue;
        }
        if (it->second.exec) cudaGraphExecDestroy(it->second.exec);
        if (it->second.segs) cudaFree(it->second.segs);
        it = b->graphs.erase(it);
    }
}

void free_enc_batch(DevCtx *c, EncBatch *b) {
    if (!b) return;
    drop_batch_graphs(b, nullptr);
    if (c) dev_free(c, b->ws, b->ws ? b->ws_bytes : 0);
    if (b->h_err) cudaFreeHost(b->h_err);
    if (b->err_ev) cudaEventDestroy(b->err_ev);
    if (b->fork) cudaEventDestroy(b->fork);
    for (int i = 0; i < kEncMaxSegs; i++) {
        if (b->side[i]) cudaStreamDestroy(b->side[i]);
        if (b->join[i]) cudaEventDestroy(b->join[i]);
    }
    delete b;
}

EncBatch *make_enc_batch(DevCtx *c, int rows) {
    EncBatch *b = new EncBatch();
    b->cap = (int)align_up((size_t)rows, 128);
    const size_t R = (size_t)b->cap;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        size_t o = off;
        off = align_up(off + bytes, 256);
        return o;
    };
    const size_t o_x = take(R * kEncDim * 4), o_xn = take(R * kEncDim * 2), o_att = take(R * kEncQkv * 2);
    const size_t o_h = take(R * kEncHidden * 2), o_q = take(R * kEncQkv * 2), o_rope = take(R * kEncHeadDim * 4);
    const size_t o_ss = take(R * kEncSsChunks * 4);
    const size_t o_split = take(kEncSplitFloats * 4), o_cnt = take(kTcSplitCounters * 4), o_err = take(4);
    b->ws_bytes = off;
    bool ok = dev_alloc(c, (void **)&b->ws, b->ws_bytes) == cudaSuccess &&
              cudaMemset(b->ws, 0, b->ws_bytes) == cudaSuccess &&
              cudaHostAlloc((void **)&b->h_err, sizeof(unsigned), cudaHostAllocDefault) == cudaSuccess &&
              cudaEventCreateWithFlags(&b->err_ev, cudaEventDisableTiming) == cudaSuccess &&
              cudaEventCreateWithFlags(&b->fork, cudaEventDisableTiming) == cudaSuccess;
    for (int i = 0; i < kEncMaxSegs && ok; i++)
        ok = cudaStreamCreateWithFlags(&b->side[i], cudaStreamNonBlocking) == cudaSuccess &&
             cudaEventCreateWithFlags(&b->join[i], cudaEventDisableTiming) == cudaSuccess;
    if (!ok) {
        set_error("encoder batch workspace: allocation of %zu bytes failed", b->ws_bytes);
        free_enc_batch(c, b);
        return nullptr;
    }
    *b->h_err = 0;
    char *w = b->ws;
    b->x = (float *)(w + o_x);
    b->xn16 = (uint16_t *)(w + o_xn);
    b->att16 = (uint16_t *)(w + o_att);
    b->h16 = (uint16_t *)(w + o_h);
    b->q16 = (uint16_t *)(w + o_q);
    b->rope = (float *)(w + o_rope);
    b->ss = (float *)(w + o_ss);
    b->split = (float *)(w + o_split);
    b->split_cnt = (unsigned *)(w + o_cnt);
    b->err = (unsigned *)(w + o_err);
    return b;
}

// The layers of one batched launch over M rows of n states (segments `segs`,
// rows[i] rows of state i from row0[i]): the encoder chunk of
// vox_encoder_forward_incremental (voxtral_encoder.c:452-636) for all of them,
// the row-wise work once, the attention per state on forked side streams.
int enqueue_encoder_batch(vox_cuda_encoder *e, EncBatch *b, vox_cuda_enc_state *const *states, const int *rows,
                          const int *row0, int n, int M, const EncSeg *segs, cudaStream_t st) {
    const bool pdl = e->pdl;
    const bool fold = enc_fold_norm(M);
    VC_TRY(launch_enc_rope_table_segs(b->rope, b->cap, M, segs, n, e->inv_freq, st, false));
    if (fold) VC_TRY(launch_rows_prenorm(b->x, M, kEncDim, e->L[0].attn_norm, b->xn16, b->ss, b->cap, st, pdl));
    auto gemm = [&](int N, int K) {
        TcGemmParams p = {};
        p.M = M;
        p.N = N;
        p.K = K;
        p.err = b->err;
        p.f16 = 1;
        p.ws = b->split;
        p.ws_floats = kEncSplitFloats;
        p.ws_cnt = b->split_cnt;
        return p;
    };
    for (int l = 0; l < e->n_layers; l++) {
        const EncLayer &L = e->L[l];
        if (!fold) VC_TRY(launch_rows_to_bf16(b->x, M, kEncDim, kEncDim, L.attn_norm, b->xn16, st, pdl, true));
        TcGemmParams p = gemm(3 * kEncQkv, kEncDim);
        if (fold) {
            p.ss_in = b->ss;
            p.ss_ld = b->cap;
        }
        p.bias = L.bq;
        p.bias2 = L.bv;
        p.rope = b->rope;
        p.rope_ld = b->cap;
        p.inv_freq = e->inv_freq;
        p.q_out = b->q16;
        p.segs = segs;
        p.n_segs = n;
        p.layer = l;
        p.cap = 1 << 30;   // (the rings are the segments')
        VC_TRY(launch_tc_gemm(TC_QKV_ENC, p, b->xn16, L.qkv, st, pdl));
        // each state's windowed attention over its own ring, concurrently
        VC_TRY(cudaEventRecord(b->fork, st));
        for (int i = 0; i < n; i++) {
            vox_cuda_enc_state *s = states[i];
            const size_t ring_layer = (size_t)s->cap * kEncQkv;
            VC_TRY(cudaStreamWaitEvent(b->side[i], b->fork, 0));
            EncAttnParams a = {};
            a.q = b->q16 + (size_t)row0[i] * kEncQkv;
            a.k_ring = s->k_ring + l * ring_layer;
            a.v_ring = s->v_ring + l * ring_layer;
            a.cap = s->cap;
            a.pos0_dev = s->pos_dev;
            a.M = rows[i];
            a.out = b->att16 + (size_t)row0[i] * kEncQkv;
            a.f16 = 1;
            a.err = b->err;
            a.shared_sms = 1;   // the other states' attention runs beside it
            VC_TRY(launch_enc_attn(a, b->side[i], false));
            VC_TRY(cudaEventRecord(b->join[i], b->side[i]));
            VC_TRY(cudaStreamWaitEvent(st, b->join[i], 0));
        }
        p = gemm(kEncDim, kEncQkv);
        p.out = b->x;
        p.ldo = kEncDim;
        p.bias = L.bo;
        if (fold) {
            p.xn_out = b->xn16;
            p.xn_gain = L.ffn_norm;
            p.ss_out = b->ss;
            p.ss_ld = b->cap;
        }
        VC_TRY(launch_tc_gemm(TC_RESID, p, b->att16, L.wo, st, false));
        if (!fold) VC_TRY(launch_rows_to_bf16(b->x, M, kEncDim, kEncDim, L.ffn_norm, b->xn16, st, pdl, true));
        p = gemm(2 * kEncHidden, kEncDim);
        p.out_bf16 = b->h16;
        p.ldo_bf16 = kEncHidden;
        if (fold) {
            p.ss_in = b->ss;
            p.ss_ld = b->cap;
        }
        VC_TRY(launch_tc_gemm(TC_SWIGLU, p, b->xn16, L.w13, st, pdl));
        p = gemm(kEncDim, kEncHidden);
        p.out = b->x;
        p.ldo = kEncDim;
        p.bias = L.b2;
        if (fold && l + 1 < e->n_layers) {
            p.xn_out = b->xn16;
            p.xn_gain = e->L[l + 1].attn_norm;
            p.ss_out = b->ss;
            p.ss_ld = b->cap;
        }
        VC_TRY(launch_tc_gemm(TC_RESID, p, b->h16, L.w2, st, pdl));
    }
    VC_TRY(launch_rows_rmsnorm(b->x, M, kEncDim, e->norm, st, pdl));
    return VOX_CUDA_OK;
}

}  // namespace

extern "C" int vox_cuda_encoder_step_batch_dev(vox_cuda_enc_state *const *states, int n, float *const *x_dev,
                                               const int *new_lens, void *stream) {
    if (!states || n <= 0 || n > kEncMaxSegs || !x_dev || !new_lens || !states[0]) {
        set_error("encoder_step_batch_dev: 1..%d states with their rows", kEncMaxSegs);
        return VOX_CUDA_ERR_ARG;
    }
    vox_cuda_encoder *e = states[0]->enc;
    int M = 0, row0[kEncMaxSegs];
    for (int i = 0; i < n; i++) {
        int rc = enc_check(states[i], new_lens[i]);
        if (rc) return rc;
        if (!x_dev[i] || states[i]->enc != e) {
            set_error("encoder_step_batch_dev: states must share one encoder, x_dev non-NULL");
            return VOX_CUDA_ERR_ARG;
        }
        for (int j = 0; j < i; j++)
            if (states[j] == states[i]) {
                set_error("encoder_step_batch_dev: a state appears twice");
                return VOX_CUDA_ERR_ARG;
            }
        row0[i] = M;
        M += new_lens[i];
    }
    DevCtx *c = ctx_for(e->device);
    cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
    std::lock_guard<std::mutex> lk(e->mu);
    EncBatch *b = e->batch;
    if (b && b->cap < M) {   // grow: the graphs hold the old pointers
        VC_TRY(cudaDeviceSynchronize());
        free_enc_batch(c, b);
        b = e->batch = nullptr;
    }
    if (!b && !(b = e->batch = make_enc_batch(c, std::max(M, 1024)))) return VOX_CUDA_ERR_OOM;
    // a timeout raised by an earlier batched launch is reported now
    if (b->err_pending && cudaEventQuery(b->err_ev) == cudaSuccess) {
        b->err_pending = false;
        if (*b->h_err) {
            *b->h_err = 0;
            VC_TRY(cudaMemsetAsync(b->err, 0, sizeof(unsigned), st));
            set_error("encoder batch: a device-side wait of an earlier launch timed out (its results are invalid)");
            return VOX_CUDA_ERR_CUDA;
        }
    }
    std::vector<std::pair<const void *, int>> key;
    for (int i = 0; i < n; i++) key.push_back({states[i], new_lens[i]});
    if (b->graphs.size() >= 64 && !b->graphs.count(key)) {   // bound the cache (ragged chunk sizes)
        VC_TRY(cudaStreamSynchronize(st));
        drop_batch_graphs(b, nullptr);
    }
    EncBatch::Graph &g = b->graphs[key];
    if (!g.exec) {
        EncSeg h[kEncMaxSegs];
        for (int i = 0; i < n; i++) h[i] = EncSeg{states[i]->k_ring, states[i]->v_ring, states[i]->pos_dev,
                                                  states[i]->cap, row0[i]};
        if (cudaMalloc((void **)&g.segs, sizeof(EncSeg) * n) != cudaSuccess ||
            cudaMemcpy(g.segs, h, sizeof(EncSeg) * n, cudaMemcpyHostToDevice) != cudaSuccess) {
            set_error("encoder_step_batch_dev: segment table allocation failed");
            b->graphs.erase(key);
            return VOX_CUDA_ERR_CUDA;
        }
        cudaGraph_t graph = nullptr;
        VC_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
        int rc = enqueue_encoder_batch(e, b, states, new_lens, row0, n, M, g.segs, st);
        cudaError_t ce = cudaStreamEndCapture(st, &graph);
        if (rc == VOX_CUDA_OK && ce == cudaSuccess) ce = cudaGraphInstantiate(&g.exec, graph, 0);
        if (graph) cudaGraphDestroy(graph);
        if (rc || ce != cudaSuccess) {
            cudaFree(g.segs);
            b->graphs.erase(key);
            if (!rc) set_error("encoder_step_batch_dev: graph capture failed: %s", cudaGetErrorString(ce));
            return rc ? rc : VOX_CUDA_ERR_CUDA;
        }
    }
    for (int i = 0; i < n; i++) {
        vox_cuda_enc_state *s = states[i];
        // the previous asynchronous step of this state may have run on another stream
        if (s->tail_set && st != c->stream) VC_TRY(cudaStreamWaitEvent(st, s->tail, 0));
        VC_TRY(launch_set_int(s->pos_dev, s->pos, st));
        VC_TRY(cudaMemcpyAsync(b->x + (size_t)row0[i] * kEncDim, x_dev[i], (size_t)new_lens[i] * kEncDim * 4,
                               cudaMemcpyDeviceToDevice, st));
    }
    VC_TRY(cudaGraphLaunch(g.exec, st));
    for (int i = 0; i < n; i++)
        VC_TRY(cudaMemcpyAsync(x_dev[i], b->x + (size_t)row0[i] * kEncDim, (size_t)new_lens[i] * kEncDim * 4,
                               cudaMemcpyDeviceToDevice, st));
    if (!b->err_pending) {   // one flag copy in flight at a time
        VC_TRY(cudaMemcpyAsync(b->h_err, b->err, sizeof(unsigned), cudaMemcpyDeviceToHost, st));
        VC_TRY(cudaEventRecord(b->err_ev, st));
        b->err_pending = true;
    }
    // order the library stream after this launch for every state (as step_dev)
    for (int i = 0; i < n; i++) {
        vox_cuda_enc_state *s = states[i];
        VC_TRY(cudaEventRecord(s->tail, st));
        if (st != c->stream) VC_TRY(cudaStreamWaitEvent(c->stream, s->tail, 0));
        s->tail_set = true;
        s->pos += new_lens[i];
    }
    return VOX_CUDA_OK;
}

namespace {

// Adapter over n encoder rows already on the device (enc_dev [n][1280]) into
// out_dev [n/4][3072] fp32, on stream st: 4x stacking (4 consecutive [1280]
// rows are one [5120] row: the same memory), Linear + GELU, Linear.
int enqueue_adapter(vox_cuda_enc_state *s, const float *enc_dev, int n, float *out_dev, cudaStream_t st) {
    vox_cuda_encoder *e = s->enc;
    const int rows = n / 4, K0 = 4 * kEncDim;
    VC_TRY(launch_rows_to_bf16(enc_dev, rows, K0, K0, nullptr, s->a16, st, false, true));
    TcGemmParams p = {};
    p.M = rows;
    p.N = kDecDim;
    p.K = K0;
    p.act = 1;                  // GELU (voxtral_encoder.c:664)
    p.out_bf16 = s->mid16;      // fp16, the next GEMM's A
    p.ldo_bf16 = kDecDim;
    p.err = s->err;
    p.f16 = 1;
    p.ws = s->split;
    p.ws_floats = kEncSplitFloats;
    p.ws_cnt = s->split_cnt;
    VC_TRY(launch_tc_gemm(TC_STORE, p, s->a16, e->adapter0, st, false));
    p = TcGemmParams{};
    p.M = rows;
    p.N = kDecDim;
    p.K = kDecDim;
    p.out = out_dev;
    p.ldo = kDecDim;
    p.err = s->err;
    p.f16 = 1;
    p.ws = s->split;
    p.ws_floats = kEncSplitFloats;
    p.ws_cnt = s->split_cnt;
    VC_TRY(launch_tc_gemm(TC_STORE, p, s->mid16, e->adapter1, st, false));
    return VOX_CUDA_OK;
}

int adapter_check(vox_cuda_enc_state *s, const void *enc, int n, const void *out) {
    int rc = enc_check(s, n);
    if (rc) return rc;
    if (!enc || !out || n % 4 != 0) {
        set_error("adapter_forward: n must be a positive multiple of 4");
        return VOX_CUDA_ERR_ARG;
    }
    return VOX_CUDA_OK;
}

}  // namespace

extern "C" int vox_cuda_adapter_forward(vox_cuda_enc_state *s, const float *enc, int n, float *out) {
    int rc = adapter_check(s, enc, n, out);
    if (rc) return rc;
    DevCtx *c = ctx_for(s->enc->device);
    cudaStream_t st = c->stream;
    VC_TRY(cudaMemcpyAsync(s->x, enc, (size_t)n * kEncDim * 4, cudaMemcpyHostToDevice, st));
    if ((rc = enqueue_adapter(s, s->x, n, s->aout, st))) return rc;
    VC_TRY(cudaMemcpyAsync(out, s->aout, (size_t)(n / 4) * kDecDim * 4, cudaMemcpyDeviceToHost, st));
    return enc_err_check(s, st);
}

extern "C" int vox_cuda_adapter_forward_dev(vox_cuda_enc_state *s, const float *enc_dev, int n, float *out_dev,
                                            void *stream) {
    int rc = adapter_check(s, enc_dev, n, out_dev);
    if (rc) return rc;
    DevCtx *c = ctx_for(s->enc->device);
    cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
    // the state's workspace may still be in use by its asynchronous chunk
    if (s->tail_set && st != c->stream) VC_TRY(cudaStreamWaitEvent(st, s->tail, 0));
    if ((rc = enqueue_adapter(s, enc_dev, n, out_dev, st))) return rc;
    if (!s->err_pending) {   // one flag copy in flight at a time
        VC_TRY(cudaMemcpyAsync(s->h_err, s->err, sizeof(unsigned), cudaMemcpyDeviceToHost, st));
        VC_TRY(cudaEventRecord(s->err_ev, st));
        s->err_pending = true;
    }
    VC_TRY(cudaEventRecord(s->tail, st));
    if (st != c->stream) VC_TRY(cudaStreamWaitEvent(c->stream, s->tail, 0));
    s->tail_set = true;
    return VOX_CUDA_OK;
}

extern "C" int vox_cuda_enc_state_set_position(vox_cuda_enc_state *s, int logical_pos) {
    if (!s || logical_pos < 0) {
        set_error("enc_state_set_position: bad arguments");
        return VOX_CUDA_ERR_ARG;
    }
    s->pos = logical_pos;
    return VOX_CUDA_OK;
}

extern "C" int vox_cuda_encoder_profile(vox_cuda_enc_state *s, const float *x_dev, int new_len, int iters,
                                        float *ms) {
    int rc = enc_check(s, new_len);
    if (rc) return rc;
    if (!x_dev || !ms || iters <= 0) return VOX_CUDA_ERR_ARG;
    DevCtx *c = ctx_for(s->enc->device);
    cudaStream_t st = c->stream;
    const int max_launch = 7 * s->enc->n_layers + 2;   // the unfolded sequence, with room to spare
    std::vector<cudaEvent_t> evs(2 * max_launch);
    std::vector<int> phase(max_launch, -1);
    for (auto &e : evs)
        if (cudaEventCreate(&e) != cudaSuccess) return VOX_CUDA_ERR_CUDA;
    double acc[VOX_CUDA_EPROF_PHASES] = {0};
    for (int it = 0; it < iters && rc == VOX_CUDA_OK; it++) {
        *s->h_pos = s->pos;
        if (cudaMemcpyAsync(s->pos_dev, s->h_pos, sizeof(int), cudaMemcpyHostToDevice, st) != cudaSuccess ||
            cudaMemcpyAsync(s->x, x_dev, (size_t)new_len * kEncDim * 4, cudaMemcpyDeviceToDevice, st) !=
                cudaSuccess) {
            rc = VOX_CUDA_ERR_CUDA;
            break;
        }
        std::fill(phase.begin(), phase.end(), -1);
        rc = enqueue_encoder(s, new_len, false, st, evs.data(), phase.data());
        if (rc) break;
        if (cudaStreamSynchronize(st) != cudaSuccess) {
            rc = VOX_CUDA_ERR_CUDA;
            break;
        }
        for (int i = 0; i < max_launch && phase[i] >= 0; i++) {
            float t = 0.f;
            cudaEventElapsedTime(&t, evs[2 * i], evs[2 * i + 1]);
            acc[phase[i]] += t;
        }
    }
    for (auto &e : evs) cudaEventDestroy(e);
    if (rc) return rc;
    for (int i = 0; i < VOX_CUDA_EPROF_PHASES; i++) ms[i] = (float)(acc[i] / iters);
    return VOX_CUDA_OK;
}

