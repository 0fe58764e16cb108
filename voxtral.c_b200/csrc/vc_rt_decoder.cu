// vc_rt_decoder.cu - the C ABI of voxtral_cuda.h, part 2: the resident
// decoder (fused weight layouts), per-stream KV rings, the single / batched /
// asynchronous decode steps (one CUDA graph of programmatic-dependent launches
// per step shape), the tensor-core prefill and the profiling entries.
#include "vc_runtime.h"

#include <map>

using namespace vc;
using namespace vc::rt;

// ---------------------------------------------------------------------------
// decoder
// ---------------------------------------------------------------------------

namespace {

struct DecLayer {
    // fused, fragment-tiled device copies: wq|wk|wv [6144, 3072],
    // wo [3072, 4096], w1/w3 row-interleaved [18432, 3072], w2 [3072, 9216]
    const uint16_t *qkv = nullptr, *wo = nullptr, *w13 = nullptr, *w2 = nullptr;
    // the same fused matrices row-major (bf16, as stored), the tcgen05
    // prefill's TMA-fed W operands; NULL when the tensor-core prefill is off
    const uint16_t *qkv_rm = nullptr, *wo_rm = nullptr, *w13_rm = nullptr, *w2_rm = nullptr;
    // RMSNorm weights as folded into the activation fragments:
    // g_attn = attention_norm, g_ffn = ffn_norm * (1 + ada_scale)
    const float *g_attn = nullptr, *g_ffn = nullptr;
};

// Device workspace for one step shape (n rows).  The host staging block is
// pinned; its layout mirrors the device block it is copied to.
struct StepWork {
    int n = 0;
    int vocab = 0;
    // device
    char *dblock = nullptr;            // [slots | rope | embeds] uploaded per step
    size_t dblock_bytes = 0;
    StreamSlot *slots = nullptr;
    float *rope = nullptr;             // [n][128]
    const float **rows = nullptr;      // [n] addend rows of the token-embedding steps
    int **tokens_to = nullptr;         // [1] the caller's token buffer of an asynchronous step (or NULL)
    float *x = nullptr;                // [n][3072] residual stream
    float *q = nullptr, *att = nullptr;  // [n][4096]
    float *h = nullptr;                // [n][9216]
    float *logits = nullptr;           // [n][vocab]
    float *part_o = nullptr, *part_ml = nullptr;
    unsigned *counters = nullptr;      // attention [n][8] + argmax [1]
    ArgmaxPartial *amax = nullptr;
    int *tokens = nullptr;             // [n]
    int *alt_ids = nullptr;            // [4]
    float *ss_attn = nullptr;          // [n][48] sums of x^2 per row block, after w2 (next QKV norm)
    float *ss_ffn = nullptr;           // [n][48] after wo (the FFN norm)
    uint32_t *xf_attn = nullptr;       // B fragments of x * g_attn (QKV / LM head input)
    uint32_t *xf_ffn = nullptr;        // B fragments of x * g_ffn (w1|w3 input)
    uint32_t *xf_att = nullptr;        // B fragments of the attention output (wo input)
    uint32_t *xf_h = nullptr;          // B fragments of silu(g) * u (w2 input)
    unsigned *err = nullptr;           // follows tokens: bounded-wait error word
    float *gpart = nullptr;            // persistent step: split-K partials
    unsigned *psync = nullptr;         // persistent step: counters, zeroed per step
    size_t psync_bytes = 0;
    size_t bytes = 0;
    // host (pinned)
    char *hblock = nullptr;
    int *h_tokens = nullptr;
    // asynchronous steps (step_batch_dev): the host block's upload and the
    // error word's copy back, each behind an event
    cudaEvent_t staged = nullptr;
    cudaEvent_t err_ev = nullptr;
    bool staged_pending = false;
    bool err_pending = false;
    unsigned err_tick = 0;             // asynchronous steps since the last error-word copy
    bool graph_persist = false;        // graph[1] holds the persistent step (its tokens are copied out)
    // graphs: [0] layers only (prefill), [1] layers + LM head
    cudaGraphExec_t graph[2] = {nullptr, nullptr};
};

// Device workspace of the tensor-core prefill (shared by the decoder's
// states, serialised by the decoder's mutex): up to `cap` rows per launch
// sequence.  Split activations (xn, att16, h16) are in the hilo_row layout:
// per 64 rows their bf16 hi rows, then their bf16 lo rows (2 x cap rows).
struct PrefillTc {
    int cap = 0;                 // rows
    int splits = 0;              // attention key splits the partial buffers hold
    char *block = nullptr;
    size_t bytes = 0;
    float *part = nullptr;       // attention partials (grown with `splits`)
    size_t part_bytes = 0;
    // the head, uploaded per call: slots, RoPE tables, input rows
    StreamSlot *slots = nullptr; // [cap]
    float *rope = nullptr;       // [cap][128]
    float *x = nullptr;          // [cap][3072] fp32 residual stream
    size_t head_bytes = 0;       // bytes before x
    float *q = nullptr;          // [cap][4096] fp32 (RoPE applied)
    uint16_t *xn = nullptr;      // [2 cap][3072] bf16 hi / lo
    uint16_t *att16 = nullptr;   // [2 cap][4096]
    uint16_t *h16 = nullptr;     // [2 cap][9216]
    unsigned *counters = nullptr;  // [cap][8]
    float *ss = nullptr;         // folded RMSNorm: sums of squares per 32-column chunk [96][cap]
    float *split = nullptr;      // split-K partials [kEncSplitFloats]
    unsigned *split_cnt = nullptr;
    unsigned *err = nullptr;
    char *hblock = nullptr;      // pinned mirror of the head
    unsigned *h_err = nullptr;   // pinned
    std::map<std::pair<int, int>, cudaGraphExec_t> graphs;   // (rows, splits) -> layers
};

}  // namespace

struct vox_cuda_decoder {
    int device = 0;
    int n_layers = 0;
    int vocab = 0;
    DecLayer L[kDecLayersMax];
    const uint16_t *tok_emb = nullptr;
    const float *norm = nullptr;
    std::vector<std::pair<void *, size_t>> owned;
    StepWork *batch_work[kMaxBatch + 1] = {};
    std::mutex mu;   // serialises batched steps (they share batch_work)
    bool pdl = true;
    cudaEvent_t tail = nullptr;   // the end of the last asynchronous step
    bool tail_set = false;
    bool tc_prefill = false;      // row-major weights kept: prefill on the tensor cores
    PrefillTc *pf = nullptr;
    std::vector<float> ffn_norm;  // [n_layers][3072] host copy: g_ffn is recomputed when ada changes
    PersistLayer *players = nullptr;   // device [n_layers]: the persistent step's weight table
};

struct vox_cuda_dec_state {
    vox_cuda_decoder *dec = nullptr;
    int cap = 0;
    int pos = 0;                       // logical position of the next row
    float *k_ring = nullptr, *v_ring = nullptr;
    size_t ring_bytes = 0;
    StepWork *work = nullptr;          // single-stream workspace (n = 1)
    StepWork *prefill_work = nullptr;  // n = 8 workspace for prefill chunks
    int last_token = -1;
    bool have_logits = false;
};

namespace {

void free_work(DevCtx *c, StepWork *w) {
    if (!w) return;
    for (auto &g : w->graph)
        if (g) cudaGraphExecDestroy(g);
    if (w->staged) cudaEventDestroy(w->staged);
    if (w->err_ev) cudaEventDestroy(w->err_ev);
    if (w->dblock) cudaFree(w->dblock);
    if (w->hblock) cudaFreeHost(w->hblock);
    if (c) {
        std::lock_guard<std::mutex> lk(c->mu);
        c->bytes -= w->bytes;
    }
    delete w;
}

// K slices of the persistent step's GEMV phases (q|k|v, wo, w1|w3, w2, LM
// head): the fewest items that still give most SMs work (96, 48 x 3, 288,
// 48 x 3, 2048); per-item reduction and epilogue latency made finer slicing
// slower.  VOX_CUDA_PERSIST_KS="a,b,c,d,e" overrides.
void persist_ks(int *ks) {
    static int v[5] = {0, 0, 0, 0, 0};
    if (v[0] == 0) {
        int t[5] = {1, 3, 1, 3, 1};
        const char *e = getenv("VOX_CUDA_PERSIST_KS");
        if (e && *e) {
            int r[5];
            if (sscanf(e, "%d,%d,%d,%d,%d", &r[0], &r[1], &r[2], &r[3], &r[4]) == 5) {
                bool good = true;
                for (int i = 0; i < 5; i++) good &= r[i] >= 1 && r[i] <= 16;
                if (good) memcpy(t, r, sizeof(t));
            }
        }
        memcpy(v, t, sizeof(v));
    }
    memcpy(ks, v, sizeof(v));
}

// The decode steps launch the per-phase kernels (the GEMVs of vc_gemv.cu and
// the attention of vc_decode.cu) with programmatic dependent launch.
// VOX_CUDA_PERSIST=1 runs each step with the LM head as one persistent kernel
// instead (vc_step_persist.cu): correct, but measured slower at 8 streams
// (3.0 ms against 1.73 ms per step), so it is not the default.
bool persist_on() {   // read when a step's graph is captured (once per workspace)
    const char *e = getenv("VOX_CUDA_PERSIST");
    return e && e[0] == '1';
}

StepWork *make_work(DevCtx *c, int n, int vocab) {
    StepWork *w = new StepWork();
    w->n = n;
    w->vocab = vocab;
    const size_t S = kAttnSplits;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        size_t o = off;
        off = align_up(off + bytes, 256);
        return o;
    };
    const size_t o_slots = take(sizeof(StreamSlot) * n);
    const size_t o_rope = take(sizeof(float) * n * kHeadDim);
    const size_t o_rows = take(sizeof(float *) * n);
    const size_t o_tto = take(sizeof(int *));
    const size_t o_x = take(sizeof(float) * n * kDecDim);
    w->dblock_bytes = o_x + sizeof(float) * n * kDecDim;   // the uploaded prefix
    const size_t o_q = take(sizeof(float) * n * kQDim);
    const size_t o_att = take(sizeof(float) * n * kQDim);
    const size_t o_h = take(sizeof(float) * n * kDecHidden);
    const size_t o_logits = take(sizeof(float) * n * (size_t)vocab);
    const size_t o_po = take(sizeof(float) * n * kDecHeads * S * kHeadDim);
    const size_t o_pml = take(sizeof(float) * n * kDecHeads * S * 2);
    const size_t o_cnt = take(sizeof(unsigned) * (n * kDecKvHeads + 1));
    const size_t grid = (size_t)gemv_grid(n, EPI_LOGITS, vocab);
    const size_t o_amax = take(sizeof(ArgmaxPartial) * grid * n);
    const size_t o_tok = take(sizeof(int) * (n + 1));   // tokens then the error word
    const size_t o_alt = take(sizeof(int) * 4);
    const size_t n_ss = (size_t)n * gemv_row_blocks(kDecDim);
    const size_t o_ssa = take(sizeof(float) * n_ss);
    const size_t o_ssf = take(sizeof(float) * n_ss);
    const size_t o_frag0 = off;
    const size_t o_xfa = take(xfrag_bytes(kDecDim));
    const size_t o_xff = take(xfrag_bytes(kDecDim));
    const size_t o_xft = take(xfrag_bytes(kQDim));
    const size_t o_xfh = take(xfrag_bytes(kDecHidden));
    const size_t frag_bytes = off - o_frag0;
    PersistParams pk = {};
    persist_ks(pk.ks);
    pk.vocab = vocab;
    const size_t o_gpart = take(sizeof(float) * std::max<size_t>(persist_gpart_floats(pk), 1));
    const size_t o_psync = take(sizeof(unsigned) * persist_sync_words());
    if (dev_alloc(c, (void **)&w->dblock, off) != cudaSuccess) {
        set_error("decoder workspace: cudaMalloc(%zu) failed", off);
        delete w;
        return nullptr;
    }
    w->bytes = off;
    char *b = w->dblock;
    w->slots = (StreamSlot *)(b + o_slots);
    w->rope = (float *)(b + o_rope);
    w->rows = (const float **)(b + o_rows);
    w->tokens_to = (int **)(b + o_tto);
    w->x = (float *)(b + o_x);
    w->q = (float *)(b + o_q);
    w->att = (float *)(b + o_att);
    w->h = (float *)(b + o_h);
    w->logits = (float *)(b + o_logits);
    w->part_o = (float *)(b + o_po);
    w->part_ml = (float *)(b + o_pml);
    w->counters = (unsigned *)(b + o_cnt);
    w->amax = (ArgmaxPartial *)(b + o_amax);
    w->tokens = (int *)(b + o_tok);
    w->alt_ids = (int *)(b + o_alt);
    w->ss_attn = (float *)(b + o_ssa);
    w->ss_ffn = (float *)(b + o_ssf);
    w->xf_attn = (uint32_t *)(b + o_xfa);
    w->xf_ffn = (uint32_t *)(b + o_xff);
    w->xf_att = (uint32_t *)(b + o_xft);
    w->xf_h = (uint32_t *)(b + o_xfh);
    w->err = (unsigned *)(w->tokens + n);
    w->gpart = (float *)(b + o_gpart);
    w->psync = (unsigned *)(b + o_psync);
    w->psync_bytes = sizeof(unsigned) * persist_sync_words();
    // fragments of streams >= n are never written and must read as zeros
    if (cudaMemset(b + o_frag0, 0, frag_bytes) != cudaSuccess ||
        cudaMemset(w->tokens, 0, sizeof(int) * (n + 1)) != cudaSuccess ||
        cudaMemset(w->counters, 0, sizeof(unsigned) * (n * kDecKvHeads + 1)) != cudaSuccess ||
        cudaHostAlloc((void **)&w->hblock, align_up(w->dblock_bytes, 16) + sizeof(int) * (n + 1), cudaHostAllocDefault) != cudaSuccess ||
        cudaEventCreateWithFlags(&w->staged, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&w->err_ev, cudaEventDisableTiming) != cudaSuccess) {
        set_error("decoder workspace: staging allocation failed");
        free_work(c, w);
        return nullptr;
    }
    memset(w->hblock, 0, align_up(w->dblock_bytes, 16) + sizeof(int) * (n + 1));   // (tokens_to: none)
    w->h_tokens = (int *)(w->hblock + align_up(w->dblock_bytes, 16));
    return w;
}

// host-side views of the staging block
StreamSlot *h_slots(StepWork *w) { return (StreamSlot *)w->hblock; }
float *h_rope(StepWork *w) { return (float *)(w->hblock + ((char *)w->rope - w->dblock)); }
float *h_x(StepWork *w) { return (float *)(w->hblock + ((char *)w->x - w->dblock)); }
const float **h_rows(StepWork *w) { return (const float **)(w->hblock + ((char *)w->rows - w->dblock)); }
int **h_tokens_to(StepWork *w) { return (int **)(w->hblock + ((char *)w->tokens_to - w->dblock)); }

// Bytes of a decode weight matrix [N, K] in the tiled layout.
size_t tiled_bytes(int N, int K) { return (size_t)round_up(N, kGemvRowAlign) * round_up(K, 16) * 2; }

// L2 prefetch budgets per launch: each GEMV of a step starts pulling the
// first 16 MB of the next GEMV's weights into L2, so that HBM stays busy
// through the launch ramps and reduction tails between the kernels, and the
// attention kernel (which leaves HBM mostly idle) all 25 MB of wo.  Measured
// at 8 streams: 1.81 -> 1.765 ms per step; 32 MB or more per GEMV is slower
// than none (the prefetch then competes with the running GEMV's own stream).
// VOX_CUDA_L2PF_MB / VOX_CUDA_L2PF_ATTN_MB override them (0: off).
unsigned long long env_mb(const char *name, long long dflt) {
    const char *e = getenv(name);
    const long long mb = e && *e ? atoll(e) : dflt;
    return (unsigned long long)(mb > 0 ? mb : 0) << 20;
}
unsigned long long l2pf_budget() { return env_mb("VOX_CUDA_L2PF_MB", 16); }
unsigned long long l2pf_attn_budget() { return env_mb("VOX_CUDA_L2PF_ATTN_MB", 32); }

// The kernel sequence of one step over w->n rows: the embeddings' norm
// statistics and fragments, the decoder layers, then the LM head + argmax
// when with_head.  Each producer writes its consumer's activation fragments.
// evs (profiling only): 2 events per launch, recorded around it.
// only (profiling only): >= 0 enqueues that phase's launches alone
// (VOX_CUDA_PROF_*), one per layer, back to back.
int enqueue_persist(vox_cuda_decoder *d, StepWork *w, cudaStream_t st) {
    PersistParams p = {};
    p.layers = d->players;
    p.n_layers = d->n_layers;
    p.M = w->n;
    p.with_head = 1;
    p.vocab = d->vocab;
    p.lm = d->tok_emb;
    p.final_norm = d->norm;
    p.slots = w->slots;
    p.rope = w->rope;
    p.x = w->x;
    p.q = w->q;
    p.xf_attn = w->xf_attn;
    p.xf_ffn = w->xf_ffn;
    p.xf_att = w->xf_att;
    p.xf_h = w->xf_h;
    p.ss_attn = w->ss_attn;
    p.ss_ffn = w->ss_ffn;
    p.logits = w->logits;
    p.amax = w->amax;
    p.tokens = w->tokens;
    p.part_o = w->part_o;
    p.part_ml = w->part_ml;
    p.gpart = w->gpart;
    p.sync = w->psync;
    p.err = w->err;
    persist_ks(p.ks);
    // weight stages (16 KB) the L2 prefetch runs ahead of the shared ring;
    // VOX_CUDA_PERSIST_L2 overrides
    const char *e = getenv("VOX_CUDA_PERSIST_L2");
    p.l2_ahead = (e && *e) ? std::max(0, atoi(e)) : 16;
    VC_TRY(cudaMemsetAsync(w->psync, 0, w->psync_bytes, st));
    VC_TRY(launch_prep_xfrag(w->x, w->n, kDecDim, kDecDim, d->L[0].g_attn, w->xf_attn, w->ss_attn, st, false));
    VC_TRY(launch_step_persist(p, st, nullptr));
    return VOX_CUDA_OK;
}

int enqueue_layers(vox_cuda_decoder *d, StepWork *w, bool with_head, cudaStream_t st,
                   cudaEvent_t *evs = nullptr, int only = -1) {
    if (with_head && evs == nullptr && only < 0 && d->players && persist_on()) return enqueue_persist(d, w, st);
    const int n = w->n;
    const bool pdl = d->pdl && evs == nullptr;
    const int ss_parts = gemv_row_blocks(kDecDim);
    // prefetch of the next launch's weights (not while profiling launches alone)
    const bool pf_on = evs == nullptr && only < 0;
    auto pf_gemv = [&](GemvParams &p, const void *next, size_t bytes) {
        const unsigned long long cap = pf_on ? l2pf_budget() : 0ull;
        p.pf = cap ? next : nullptr;
        p.pf_bytes = std::min<unsigned long long>(cap, bytes) & ~15ull;
    };
    int ei = 0;
#define VC_EV_BEGIN() do { if (evs) VC_TRY(cudaEventRecord(evs[ei++], st)); } while (0)
#define VC_EV_END() do { if (evs) VC_TRY(cudaEventRecord(evs[ei++], st)); } while (0)
#define VC_PHASE(ph) if (only < 0 || only == (ph))
    if (only < 0) {
        VC_EV_BEGIN();
        VC_TRY(launch_prep_xfrag(w->x, n, kDecDim, kDecDim, d->L[0].g_attn, w->xf_attn, w->ss_attn, st, pdl));
        VC_EV_END();
    }
    for (int l = 0; l < d->n_layers && only != VOX_CUDA_PROF_LM_HEAD; l++) {
        const DecLayer &L = d->L[l];
        GemvParams p = {};
        // q|k|v = rms_norm(x) Wqkv^T, RoPE, ring write
        p.W = L.qkv;
        p.N = kQkvRows;
        p.K = p.Kp = kDecDim;
        p.xfrag = w->xf_attn;
        p.ss_in = w->ss_attn;
        p.ss_parts = ss_parts;
        p.y = w->q;
        p.ldy = kQDim;
        p.slots = w->slots;
        p.rope = w->rope;
        p.layer = l;
        p.err = w->err;
        VC_PHASE(VOX_CUDA_PROF_QKV) {
            VC_EV_BEGIN();
            VC_TRY(launch_gemv(n, EPI_QKV, p, st, pdl));
            VC_EV_END();
        }
        // attention over the ring -> wo's fragments
        AttnParams a = {};
        a.q = w->q;
        a.slots = w->slots;
        a.layer = l;
        a.out = nullptr;
        a.xfrag_out = w->xf_att;
        a.part_o = w->part_o;
        a.part_ml = w->part_ml;
        a.counters = w->counters;
        a.S = kAttnSplits;
        {
            const unsigned long long cap = pf_on ? l2pf_attn_budget() : 0ull;
            a.pf = cap ? L.wo : nullptr;
            a.pf_bytes = std::min<unsigned long long>(cap, tiled_bytes(kDecDim, kQDim)) & ~15ull;
        }
        VC_PHASE(VOX_CUDA_PROF_ATTN) {
            VC_EV_BEGIN();
            VC_TRY(launch_attn_decode(n, a, st, pdl));
            VC_EV_END();
        }
        // x += att Wo^T; fragments of x * g_ffn and sums of x^2 for the FFN norm
        p = GemvParams{};
        p.W = L.wo;
        p.N = kDecDim;
        p.K = p.Kp = kQDim;
        p.xfrag = w->xf_att;
        p.y = w->x;
        p.ldy = kDecDim;
        p.ss_out = w->ss_ffn;
        p.xfrag_out = w->xf_ffn;
        p.g_next = L.g_ffn;
        p.err = w->err;
        pf_gemv(p, L.w13, tiled_bytes(2 * kDecHidden, kDecDim));
        VC_PHASE(VOX_CUDA_PROF_WO) {
            VC_EV_BEGIN();
            VC_TRY(launch_gemv(n, EPI_ADD, p, st, pdl));
            VC_EV_END();
        }
        // h = silu(xn W1^T) * (xn W3^T), xn = rms_norm(x) * (1 + ada)
        p = GemvParams{};
        p.W = L.w13;
        p.N = 2 * kDecHidden;
        p.K = p.Kp = kDecDim;
        p.xfrag = w->xf_ffn;
        p.ss_in = w->ss_ffn;
        p.ss_parts = ss_parts;
        p.xfrag_out = w->xf_h;
        p.err = w->err;
        pf_gemv(p, L.w2, tiled_bytes(kDecDim, kDecHidden));
        VC_PHASE(VOX_CUDA_PROF_W13) {
            VC_EV_BEGIN();
            VC_TRY(launch_gemv(n, EPI_SWIGLU, p, st, pdl));
            VC_EV_END();
        }
        // x += h W2^T; fragments for the next norm (next layer's, or the final)
        p = GemvParams{};
        p.W = L.w2;
        p.N = kDecDim;
        p.K = p.Kp = kDecHidden;
        p.xfrag = w->xf_h;
        p.y = w->x;
        p.ldy = kDecDim;
        p.ss_out = w->ss_attn;
        p.xfrag_out = w->xf_attn;
        p.g_next = (l + 1 < d->n_layers) ? d->L[l + 1].g_attn : d->norm;
        p.err = w->err;
        if (l + 1 < d->n_layers) pf_gemv(p, d->L[l + 1].qkv, tiled_bytes(kQkvRows, kDecDim));
        else if (with_head) pf_gemv(p, d->tok_emb, tiled_bytes(d->vocab, kDecDim));
        VC_PHASE(VOX_CUDA_PROF_W2) {
            VC_EV_BEGIN();
            VC_TRY(launch_gemv(n, EPI_ADD, p, st, pdl));
            VC_EV_END();
        }
    }
    if (with_head && (only < 0 || only == VOX_CUDA_PROF_LM_HEAD)) {
        GemvParams p = {};
        p.W = d->tok_emb;
        p.N = d->vocab;
        p.K = p.Kp = kDecDim;
        p.xfrag = w->xf_attn;
        p.ss_in = w->ss_attn;
        p.ss_parts = ss_parts;
        p.y = w->logits;
        p.ldy = d->vocab;
        p.partials = w->amax;
        p.counter = w->counters + n * kDecKvHeads;
        p.tokens = w->tokens;
        p.tokens_to = w->tokens_to;
        p.err = w->err;
        VC_EV_BEGIN();
        VC_TRY(launch_gemv(n, EPI_LOGITS, p, st, pdl));
        VC_EV_END();
    }
#undef VC_EV_BEGIN
#undef VC_EV_END
#undef VC_PHASE
    return VOX_CUDA_OK;
}

// The error word copied back after the tokens: a device-side bounded wait
// expired during the step.
int check_step_error(StepWork *w, cudaStream_t st) {
    const unsigned e = (unsigned)w->h_tokens[w->n];
    if (e == 0) return VOX_CUDA_OK;
    w->h_tokens[w->n] = 0;
    cudaMemsetAsync(w->err, 0, sizeof(unsigned), st);
    if (e == 2u) {   // launch_embed_tokens: an id outside the vocabulary
        set_error("decoder step: a previous token id was outside [0, vocab) (its embedding was skipped)");
        return VOX_CUDA_ERR_ARG;
    }
    set_error("decoder step: a device-side wait timed out (results discarded)");
    return VOX_CUDA_ERR_CUDA;
}

// Upload the staged step inputs, run the (captured) kernel sequence, fetch
// the tokens.
int run_step(vox_cuda_decoder *d, DevCtx *c, StepWork *w, bool with_head, cudaStream_t st,
             bool sync) {
    *h_tokens_to(w) = nullptr;   // the tokens come back through h_tokens
    VC_TRY(cudaMemcpyAsync(w->dblock, w->hblock, w->dblock_bytes, cudaMemcpyHostToDevice, st));
    cudaGraphExec_t &g = w->graph[with_head ? 1 : 0];
    if (!g) {
        cudaGraph_t graph = nullptr;
        if (with_head) w->graph_persist = d->players && persist_on();   // (as enqueue_layers decides)
        VC_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
        int rc = enqueue_layers(d, w, with_head, st);
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
    // tokens and the error word in one copy
    VC_TRY(cudaMemcpyAsync(w->h_tokens, w->tokens, sizeof(int) * (w->n + 1), cudaMemcpyDeviceToHost, st));
    if (sync) {
        VC_TRY(cudaStreamSynchronize(st));
        int rc = check_step_error(w, st);
        if (rc) return rc;
    }
    (void)c;
    return VOX_CUDA_OK;
}

void fill_slot(vox_cuda_dec_state *s, int pos, StreamSlot *slot) {
    slot->k_ring = s->k_ring;
    slot->v_ring = s->v_ring;
    slot->cap = s->cap;
    slot->pos = pos;
    slot->slot = pos % s->cap;
    slot->n_keys = (pos + 1 < kDecWindow) ? pos + 1 : kDecWindow;
    slot->fresh = pos;   // a launch with more rows of this sequence lowers it
}

// Rows first..last are written in one launch: the ring must hold, at once,
// the window of the first row and every later row of the launch.
int check_capacity(const vox_cuda_dec_state *s, int first, int last) {
    const int oldest = (first - kDecWindow + 1 > 0) ? first - kDecWindow + 1 : 0;
    const int span = last - oldest + 1;
    if (span > s->cap) {
        set_error("KV ring of %d positions cannot hold %d positions (%d..%d)", s->cap, span,
                  oldest, last);
        return VOX_CUDA_ERR_CAPACITY;
    }
    return VOX_CUDA_OK;
}

// ---- tensor-core prefill -------------------------------------------------

constexpr int kPrefillRows = 128;   // rows per launch sequence (one M tile)

void free_prefill(DevCtx *c, PrefillTc *f) {
    if (!f) return;
    for (auto &kv : f->graphs) cudaGraphExecDestroy(kv.second);
    if (c) {
        dev_free(c, f->block, f->block ? f->bytes : 0);
        dev_free(c, f->part, f->part ? f->part_bytes : 0);
    }
    if (f->hblock) cudaFreeHost(f->hblock);
    if (f->h_err) cudaFreeHost(f->h_err);
    delete f;
}

PrefillTc *make_prefill(DevCtx *c, int cap) {
    PrefillTc *f = new PrefillTc();
    f->cap = cap;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        size_t o = off;
        off = align_up(off + bytes, 256);
        return o;
    };
    const size_t C = (size_t)cap;
    const size_t o_slots = take(sizeof(StreamSlot) * C), o_rope = take(4 * C * kHeadDim);
    const size_t o_x = take(4 * C * kDecDim);
    f->head_bytes = o_x;   // + the rows of x actually used
    const size_t o_q = take(4 * C * kQDim);
    const size_t o_xn = take(2 * 2 * C * kDecDim), o_att16 = take(2 * 2 * C * kQDim);
    const size_t o_h16 = take(2 * 2 * C * kDecHidden), o_cnt = take(4 * C * kDecKvHeads);
    const size_t o_ss = take(4 * C * (kDecDim / 32));
    const size_t o_split = take(4 * kEncSplitFloats), o_scnt = take(4 * kTcSplitCounters), o_err = take(4);
    f->bytes = off;
    if (dev_alloc(c, (void **)&f->block, f->bytes) != cudaSuccess ||
        cudaMemset(f->block, 0, f->bytes) != cudaSuccess ||
        cudaHostAlloc((void **)&f->hblock, o_x + 4 * C * kDecDim, cudaHostAllocDefault) != cudaSuccess ||
        cudaHostAlloc((void **)&f->h_err, sizeof(unsigned), cudaHostAllocDefault) != cudaSuccess) {
        set_error("prefill workspace: allocation of %zu bytes failed", f->bytes);
        free_prefill(c, f);
        return nullptr;
    }
    char *b = f->block;
    f->slots = (StreamSlot *)(b + o_slots);
    f->rope = (float *)(b + o_rope);
    f->x = (float *)(b + o_x);
    f->q = (float *)(b + o_q);
    f->xn = (uint16_t *)(b + o_xn);
    f->att16 = (uint16_t *)(b + o_att16);
    f->h16 = (uint16_t *)(b + o_h16);
    f->counters = (unsigned *)(b + o_cnt);
    f->ss = (float *)(b + o_ss);
    f->split = (float *)(b + o_split);
    f->split_cnt = (unsigned *)(b + o_scnt);
    f->err = (unsigned *)(b + o_err);
    *f->h_err = 0;
    return f;
}

// Grow the attention partials to `splits` key splits per (row, head).
int prefill_reserve_splits(DevCtx *c, PrefillTc *f, int splits) {
    if (splits <= f->splits) return VOX_CUDA_OK;
    const size_t bytes = (size_t)f->cap * kDecHeads * splits * (kHeadDim + 2) * 4;
    float *np = nullptr;
    if (dev_alloc(c, (void **)&np, bytes) != cudaSuccess) {
        set_error("prefill workspace: attention partials (%zu bytes) failed", bytes);
        return VOX_CUDA_ERR_OOM;
    }
    VC_TRY(cudaStreamSynchronize(c->stream));
    dev_free(c, f->part, f->part ? f->part_bytes : 0);
    for (auto &kv : f->graphs) cudaGraphExecDestroy(kv.second);   // they hold the old pointers
    f->graphs.clear();
    f->part = np;
    f->part_bytes = bytes;
    f->splits = splits;
    return VOX_CUDA_OK;
}

// The layers of one prefill launch sequence over M rows (their slots, RoPE
// tables and inputs already in f): per layer RMSNorm -> hi / lo rows,
// q|k|v GEMM (RoPE, ring writes), attention over each row's ring, wo GEMM +
// residual, FFN RMSNorm * (1 + ada), w1|w3 GEMM + SwiGLU, w2 GEMM + residual
// (vox_decoder_prefill, voxtral_decoder.c:233-373).  bf16 tensor-core
// operands: the weights as stored, the activations as hi + lo pairs.
int enqueue_prefill(vox_cuda_decoder *d, PrefillTc *f, int M, int S, cudaStream_t st) {
    const bool pdl = d->pdl;
    float *part_o = f->part;
    float *part_ml = f->part + (size_t)f->cap * kDecHeads * S * kHeadDim;
    auto gemm = [&](int M_, int N, int K) {
        TcGemmParams p = {};
        p.M = M_;
        p.N = N;
        p.K = K;
        p.hilo = 1;
        p.err = f->err;
        p.ws = f->split;
        p.ws_floats = kEncSplitFloats;
        p.ws_cnt = f->split_cnt;
        return p;
    };
    // VOX_CUDA_DEC_FOLD_NORM = 1 folds the RMSNorms into the GEMMs around
    // them (the residual epilogues write the next operand's hi / lo rows of
    // x * g and the row sums of squares, the consumers scale their rows by
    // 1 / rms), as the encoder does.  Off by default: measured 2.68 -> 2.72 ms
    // for 38 rows and 3.82 -> 3.80 ms for 114 (the consumers' 96-chunk row
    // sums and the wider residual epilogue cost what the two norm launches
    // per layer saved).
    const char *fe = getenv("VOX_CUDA_DEC_FOLD_NORM");
    const bool fold = fe && fe[0] == '1';
    if (fold) VC_TRY(launch_rows_prenorm_hilo(f->x, M, kDecDim, d->L[0].g_attn, f->xn, f->ss, f->cap, st, pdl));
    for (int l = 0; l < d->n_layers; l++) {
        const DecLayer &L = d->L[l];
        if (!fold) VC_TRY(launch_rows_hilo(f->x, M, kDecDim, kDecDim, L.g_attn, f->xn, st, pdl));
        TcGemmParams p = gemm(M, kQkvRows, kDecDim);
        if (fold) {
            p.ss_in = f->ss;
            p.ss_ld = f->cap;
        }
        p.q32 = f->q;
        p.slots = f->slots;
        p.layer = l;
        p.rope_rows = f->rope;
        VC_TRY(launch_tc_gemm(TC_QKV_DEC, p, f->xn, L.qkv_rm, st, pdl));
        AttnParams a = {};
        a.q = f->q;
        a.slots = f->slots;
        a.layer = l;
        a.out_hilo = f->att16;   // straight into the wo GEMM's split operand
        a.part_o = part_o;
        a.part_ml = part_ml;
        a.counters = f->counters;
        a.S = S;
        VC_TRY(launch_attn_decode(M, a, st, pdl));
        p = gemm(M, kDecDim, kQDim);
        p.out = f->x;
        p.ldo = kDecDim;
        if (fold) {
            p.xn_out = f->xn;
            p.xn_gain = L.g_ffn;
            p.ss_out = f->ss;
            p.ss_ld = f->cap;
        }
        VC_TRY(launch_tc_gemm(TC_RESID, p, f->att16, L.wo_rm, st, pdl));
        if (!fold) VC_TRY(launch_rows_hilo(f->x, M, kDecDim, kDecDim, L.g_ffn, f->xn, st, pdl));
        p = gemm(M, 2 * kDecHidden, kDecDim);
        p.out_bf16 = f->h16;
        p.ldo_bf16 = kDecHidden;
        p.out_hilo = 1;
        if (fold) {
            p.ss_in = f->ss;
            p.ss_ld = f->cap;
        }
        VC_TRY(launch_tc_gemm(TC_SWIGLU, p, f->xn, L.w13_rm, st, pdl));
        p = gemm(M, kDecDim, kDecHidden);
        p.out = f->x;
        p.ldo = kDecDim;
        if (fold && l + 1 < d->n_layers) {   // the next layer's operand and row sums
            p.xn_out = f->xn;
            p.xn_gain = d->L[l + 1].g_attn;
            p.ss_out = f->ss;
            p.ss_ld = f->cap;
        }
        VC_TRY(launch_tc_gemm(TC_RESID, p, f->h16, L.w2_rm, st, pdl));
    }
    return VOX_CUDA_OK;
}

// Rows of one or more states (state i contributes n_rows[i] consecutive
// rows from its current position), in launch sequences of <= kPrefillRows
// rows; x: host [sum n_rows][3072]; rope: host [sum n_rows][64][2] or NULL.
// Caller holds d->mu.
int prefill_tc_rows(vox_cuda_decoder *d, DevCtx *c, vox_cuda_dec_state *const *states, const int *n_rows,
                    int n_states, const float *x, const float *rope) {
    if (!d->pf && !(d->pf = make_prefill(c, kPrefillRows))) return VOX_CUDA_ERR_OOM;
    PrefillTc *f = d->pf;
    cudaStream_t st = c->stream;
    StreamSlot *h_slots = (StreamSlot *)f->hblock;
    float *h_rope = (float *)(f->hblock + ((char *)f->rope - f->block));
    float *h_x = (float *)(f->hblock + ((char *)f->x - f->block));
    int si = 0, done_in_state = 0;   // next row: state si, its row done_in_state
    size_t row_in = 0;               // next row of x / rope
    while (si < n_states) {
        // gather up to kPrefillRows rows
        int M = 0, max_keys = 1;
        while (si < n_states && M < f->cap) {
            const int take = std::min(n_rows[si] - done_in_state, f->cap - M);
            vox_cuda_dec_state *s = states[si];
            for (int r = 0; r < take; r++) {
                const int pos = s->pos + done_in_state + r;
                fill_slot(s, pos, h_slots + M + r);
                h_slots[M + r].fresh = s->pos + done_in_state;   // this launch's first row of the state
                max_keys = std::max(max_keys, h_slots[M + r].n_keys);
                if (rope) memcpy(h_rope + (size_t)(M + r) * kHeadDim, rope + (row_in + r) * kHeadDim, kHeadDim * 4);
                else host_rope_table(pos, kHeadDim, h_rope + (size_t)(M + r) * kHeadDim);
            }
            memcpy(h_x + (size_t)M * kDecDim, x + row_in * kDecDim, (size_t)take * kDecDim * 4);
            M += take;
            row_in += take;
            done_in_state += take;
            if (done_in_state == n_rows[si]) {
                si++;
                done_in_state = 0;
            }
        }
        const int S = (max_keys + 63) / 64;
        int rc = prefill_reserve_splits(c, f, S);
        if (rc) return rc;
        VC_TRY(cudaMemcpyAsync(f->block, f->hblock, f->head_bytes + (size_t)M * kDecDim * 4, cudaMemcpyHostToDevice,
                               st));
        cudaGraphExec_t &g = f->graphs[std::make_pair(M, S)];
        if (!g) {
            cudaGraph_t graph = nullptr;
            VC_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
            rc = enqueue_prefill(d, f, M, S, st);
            cudaError_t e = cudaStreamEndCapture(st, &graph);
            if (rc) {
                if (graph) cudaGraphDestroy(graph);
                f->graphs.erase(std::make_pair(M, S));
                return rc;
            }
            VC_TRY(e);
            e = cudaGraphInstantiate(&g, graph, 0);
            cudaGraphDestroy(graph);
            VC_TRY(e);
        }
        VC_TRY(cudaGraphLaunch(g, st));
        VC_TRY(cudaMemcpyAsync(f->h_err, f->err, sizeof(unsigned), cudaMemcpyDeviceToHost, st));
        VC_TRY(cudaStreamSynchronize(st));   // the host block is reused by the next sequence
        if (*f->h_err) {
            *f->h_err = 0;
            cudaMemset(f->err, 0, sizeof(unsigned));
            set_error("decoder prefill: a device-side wait timed out (results discarded)");
            return VOX_CUDA_ERR_CUDA;
        }
    }
    return VOX_CUDA_OK;
}

}  // namespace

extern "C" vox_cuda_decoder *vox_cuda_decoder_create(const vox_cuda_dec_weights *w) {
    DevCtx *c = cur_ctx();
    if (!c) return nullptr;
    if (!w || w->n_layers <= 0 || w->n_layers > kDecLayersMax || w->vocab <= 0 ||
        !w->tok_embeddings || !w->norm) {
        set_error("decoder_create: bad weight descriptor");
        return nullptr;
    }
    for (int l = 0; l < w->n_layers; l++) {
        const vox_cuda_dec_layer_weights &L = w->layers[l];
        if (!L.wq || !L.wk || !L.wv || !L.wo || !L.w1 || !L.w2 || !L.w3 || !L.attention_norm ||
            !L.ffn_norm) {
            set_error("decoder_create: layer %d has a NULL weight", l);
            return nullptr;
        }
    }
    vox_cuda_decoder *d = new vox_cuda_decoder();
    d->device = c->device;
    d->n_layers = w->n_layers;
    d->vocab = w->vocab;
    const char *pdl_env = getenv("VOX_CUDA_PDL");
    d->pdl = !(pdl_env && pdl_env[0] == '0');
    const cudaMemcpyKind kind = w->weights_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    cudaStream_t st = c->stream;
    auto alloc = [&](size_t bytes) -> void * {
        void *p = nullptr;
        if (dev_alloc(c, &p, bytes) != cudaSuccess) return nullptr;
        d->owned.push_back({p, bytes});
        return p;
    };
    const size_t D = kDecDim;
    Uploader up(st, !w->weights_on_device, c);   // host weights: pinned, pipelined
    // row-major staging for one fused matrix (the largest is the LM head)
    const size_t stage_elems = std::max((size_t)w->vocab, (size_t)2 * kDecHidden) * D;
    uint16_t *stage = nullptr;
    if (cudaMalloc(&stage, stage_elems * 2) != cudaSuccess) {
        set_error("decoder_create: staging allocation (%zu bytes) failed", stage_elems * 2);
        delete d;
        return nullptr;
    }
    bool ok = true;
    bool reported = false;   // the first failure's message is kept
    auto chk = [&](cudaError_t e, const char *what) {
        if (e == cudaSuccess) return;
        if (!reported) set_error("decoder_create: %s: %s", what, cudaGetErrorString(e));
        reported = true;
        ok = false;
    };
    // Fused matrix from row-major pieces: [rows_i x K] blocks stacked (or
    // row-interleaved when interleave), then tiled for the GEMV.
    // VOX_CUDA_DEC_TC_PREFILL = 0 drops the row-major copies (6 GB at 4B):
    // the prefill then runs through the decode-step kernels
    const char *tcp_env = getenv("VOX_CUDA_DEC_TC_PREFILL");
    d->tc_prefill = !(tcp_env && tcp_env[0] == '0');
    auto fuse = [&](const uint16_t *const *parts, const int *rows, int n_parts, int K, bool interleave,
                    const uint16_t **rm = nullptr) -> uint16_t * {
        int N = 0;
        for (int i = 0; i < n_parts; i++) N += rows[i];
        uint16_t *dst = (uint16_t *)alloc((size_t)round_up(N, kGemvRowAlign) * round_up(K, 16) * 2);
        if (!dst) return nullptr;
        if (interleave) {  // row 2i = parts[0][i], row 2i+1 = parts[1][i]
            for (int i = 0; i < n_parts && ok; i++)
                chk(up.copy2d(stage + (size_t)i * K, (size_t)n_parts * K * 2, parts[i], (size_t)K * 2,
                              (size_t)K * 2, rows[i]),
                    "interleaved weight copy");
        } else {
            size_t off = 0;
            for (int i = 0; i < n_parts && ok; i++) {
                chk(up.copy(stage + off, parts[i], (size_t)rows[i] * K * 2), "weight copy");
                off += (size_t)rows[i] * K;
            }
        }
        chk(launch_tile_weights(dst, stage, N, K, round_up(N, kGemvRowAlign), round_up(K, 16), st), "tiling");
        if (rm && ok) {   // the row-major fused matrix as staged
            uint16_t *r = (uint16_t *)alloc((size_t)N * K * 2);
            if (!r) chk(cudaErrorMemoryAllocation, "row-major copy allocation");
            else chk(cudaMemcpyAsync(r, stage, (size_t)N * K * 2, cudaMemcpyDeviceToDevice, st), "row-major copy");
            *rm = r;
        }
        chk(cudaStreamSynchronize(st), "upload");   // the stage is reused next
        return ok ? dst : nullptr;
    };
    for (int l = 0; l < w->n_layers && ok; l++) {
        const vox_cuda_dec_layer_weights &L = w->layers[l];
        DecLayer &o = d->L[l];
        // layers that alias an earlier layer's tensors share its device copies
        for (int j = 0; j < l; j++) {
            const vox_cuda_dec_layer_weights &J = w->layers[j];
            if (J.wq == L.wq && J.wk == L.wk && J.wv == L.wv && J.wo == L.wo && J.w1 == L.w1 &&
                J.w2 == L.w2 && J.w3 == L.w3) {
                o.qkv = d->L[j].qkv;
                o.wo = d->L[j].wo;
                o.w13 = d->L[j].w13;
                o.w2 = d->L[j].w2;
                o.qkv_rm = d->L[j].qkv_rm;
                o.wo_rm = d->L[j].wo_rm;
                o.w13_rm = d->L[j].w13_rm;
                o.w2_rm = d->L[j].w2_rm;
                break;
            }
        }
        if (!o.qkv) {
            const uint16_t *qkv_parts[3] = {L.wq, L.wk, L.wv};
            const int qkv_rows[3] = {kQDim, kKvDim, kKvDim};
            const uint16_t *wo_parts[1] = {L.wo};
            const int wo_rows[1] = {kDecDim};
            const uint16_t *w13_parts[2] = {L.w1, L.w3};
            const int w13_rows[2] = {kDecHidden, kDecHidden};
            const uint16_t *w2_parts[1] = {L.w2};
            const int w2_rows[1] = {kDecDim};
            const bool rm = d->tc_prefill;
            o.qkv = fuse(qkv_parts, qkv_rows, 3, kDecDim, false, rm ? &o.qkv_rm : nullptr);
            o.wo = ok ? fuse(wo_parts, wo_rows, 1, kQDim, false, rm ? &o.wo_rm : nullptr) : nullptr;
            o.w13 = ok ? fuse(w13_parts, w13_rows, 2, kDecDim, true, rm ? &o.w13_rm : nullptr) : nullptr;
            o.w2 = ok ? fuse(w2_parts, w2_rows, 1, kDecHidden, false, rm ? &o.w2_rm : nullptr) : nullptr;
            ok &= o.qkv && o.wo && o.w13 && o.w2;
            if (!ok) break;
        }
        // g_attn = attention_norm; g_ffn = ffn_norm * (1 + ada_scale[l])
        // (voxtral_decoder.c:466, 488-492), folded into the activation fragments
        std::vector<float> ha(D), hf(D), hada(D, 0.0f);
        // host vectors are read on the host (a host-to-host cudaMemcpy may take
        // a DMA path when the source page is registered)
        auto fetch = [&](float *dst, const float *src) {
            if (w->weights_on_device) chk(cudaMemcpy(dst, src, D * 4, cudaMemcpyDeviceToHost), "norm fetch");
            else memcpy(dst, src, D * 4);
        };
        fetch(ha.data(), L.attention_norm);
        fetch(hf.data(), L.ffn_norm);
        d->ffn_norm.insert(d->ffn_norm.end(), hf.begin(), hf.end());
        if (w->ada_scale) fetch(hada.data(), w->ada_scale + (size_t)l * D);
        for (size_t i = 0; i < D; i++) hf[i] = hf[i] * (1.0f + hada[i]);
        float *g = (float *)alloc(2 * D * 4);
        if (!g || !ok) {
            ok = false;
            break;
        }
        ok &= cudaMemcpy(g, ha.data(), D * 4, cudaMemcpyHostToDevice) == cudaSuccess;
        ok &= cudaMemcpy(g + D, hf.data(), D * 4, cudaMemcpyHostToDevice) == cudaSuccess;
        o.g_attn = g;
        o.g_ffn = g + D;
    }
    if (ok) {
        const uint16_t *emb_parts[1] = {w->tok_embeddings};
        const int emb_rows[1] = {w->vocab};
        d->tok_emb = fuse(emb_parts, emb_rows, 1, kDecDim, false);
        float *nrm = (float *)alloc(D * 4);
        ok = d->tok_emb && nrm;
        if (ok) {
            ok &= cudaMemcpy(nrm, w->norm, D * 4, kind) == cudaSuccess;
            d->norm = nrm;
        }
    }
    cudaFree(stage);
    if (ok) {   // the persistent step's table of per-layer weights
        std::vector<PersistLayer> pl(d->n_layers);
        for (int l = 0; l < d->n_layers; l++)
            pl[l] = PersistLayer{d->L[l].qkv, d->L[l].wo, d->L[l].w13, d->L[l].w2, d->L[l].g_attn, d->L[l].g_ffn};
        d->players = (PersistLayer *)alloc(sizeof(PersistLayer) * pl.size());
        ok = d->players && cudaMemcpy(d->players, pl.data(), sizeof(PersistLayer) * pl.size(),
                                      cudaMemcpyHostToDevice) == cudaSuccess;
    }
    if (!ok) {
        if (!reported) set_error("decoder_create: weight upload failed (out of device memory?)");
        vox_cuda_decoder_free(d);
        return nullptr;
    }
    return d;
}

extern "C" int vox_cuda_decoder_set_ada_scale(vox_cuda_decoder *d, const float *ada_scale) {
    if (!d || d->ffn_norm.size() != (size_t)d->n_layers * kDecDim) {
        set_error("decoder_set_ada_scale: bad arguments");
        return VOX_CUDA_ERR_ARG;
    }
    DevCtx *c = ctx_for(d->device);
    if (!c) return VOX_CUDA_ERR_UNAVAILABLE;
    cudaSetDevice(d->device);
    // the g_ffn vectors are read by every step and prefill: the update is
    // ordered after the pending ones on the library stream (which the
    // asynchronous steps join) and completes before this call returns
    std::lock_guard<std::mutex> lk(d->mu);
    std::vector<float> g((size_t)d->n_layers * kDecDim);
    for (int l = 0; l < d->n_layers; l++)
        for (int i = 0; i < kDecDim; i++) {
            const size_t j = (size_t)l * kDecDim + i;
            g[j] = d->ffn_norm[j] * (1.0f + (ada_scale ? ada_scale[j] : 0.0f));
        }
    VC_TRY(cudaStreamSynchronize(c->stream));
    for (int l = 0; l < d->n_layers; l++)
        VC_TRY(cudaMemcpy((void *)d->L[l].g_ffn, g.data() + (size_t)l * kDecDim, kDecDim * sizeof(float),
                          cudaMemcpyHostToDevice));
    return VOX_CUDA_OK;
}

extern "C" void vox_cuda_decoder_free(vox_cuda_decoder *d) {
    if (!d) return;
    DevCtx *c = ctx_for(d->device);
    cudaSetDevice(d->device);
    if (c) cudaStreamSynchronize(c->stream);   // also waits for asynchronous steps (see step_batch_dev)
    for (int i = 0; i <= kMaxBatch; i++) free_work(c, d->batch_work[i]);
    free_prefill(c, d->pf);
    if (d->tail) cudaEventDestroy(d->tail);
    for (auto &pr : d->owned)
        if (c) dev_free(c, pr.first, pr.second);
        else cudaFree(pr.first);
    delete d;
}

extern "C" vox_cuda_dec_state *vox_cuda_dec_state_create(vox_cuda_decoder *d, int kv_cap) {
    if (!d || kv_cap <= 0) {
        set_error("dec_state_create: bad arguments");
        return nullptr;
    }
    DevCtx *c = ctx_for(d->device);
    if (!c) {
        set_error("dec_state_create: device not initialised");
        return nullptr;
    }
    vox_cuda_dec_state *s = new vox_cuda_dec_state();
    s->dec = d;
    s->cap = kv_cap;
    s->ring_bytes = (size_t)d->n_layers * kv_cap * kKvDim * sizeof(float);
    if (dev_alloc(c, (void **)&s->k_ring, s->ring_bytes) != cudaSuccess ||
        dev_alloc(c, (void **)&s->v_ring, s->ring_bytes) != cudaSuccess) {
        set_error("dec_state_create: KV ring allocation (%zu bytes x 2) failed", s->ring_bytes);
        vox_cuda_dec_state_free(s);
        return nullptr;
    }
    if (cudaMemset(s->k_ring, 0, s->ring_bytes) != cudaSuccess ||
        cudaMemset(s->v_ring, 0, s->ring_bytes) != cudaSuccess) {
        set_error("dec_state_create: ring clear failed");
        vox_cuda_dec_state_free(s);
        return nullptr;
    }
    s->work = make_work(c, 1, d->vocab);
    if (!s->work) {
        vox_cuda_dec_state_free(s);
        return nullptr;
    }
    return s;
}

extern "C" void vox_cuda_dec_state_free(vox_cuda_dec_state *s) {
    if (!s) return;
    DevCtx *c = ctx_for(s->dec->device);
    cudaSetDevice(s->dec->device);
    if (c) cudaStreamSynchronize(c->stream);
    free_work(c, s->work);
    free_work(c, s->prefill_work);
    if (c) {
        dev_free(c, s->k_ring, s->k_ring ? s->ring_bytes : 0);
        dev_free(c, s->v_ring, s->v_ring ? s->ring_bytes : 0);
    }
    delete s;
}

extern "C" int vox_cuda_dec_state_reset(vox_cuda_dec_state *s) {
    if (!s) return VOX_CUDA_ERR_ARG;
    s->pos = 0;
    s->have_logits = false;
    s->last_token = -1;
    return VOX_CUDA_OK;
}

extern "C" int vox_cuda_dec_state_position(const vox_cuda_dec_state *s) { return s ? s->pos : -1; }

extern "C" int vox_cuda_dec_state_set_position(vox_cuda_dec_state *s, int logical_pos) {
    if (!s || logical_pos < 0) {
        set_error("dec_state_set_position: bad arguments");
        return VOX_CUDA_ERR_ARG;
    }
    s->pos = logical_pos;
    s->have_logits = false;
    return VOX_CUDA_OK;
}

static int kv_rows_check(vox_cuda_dec_state *s, int layer, int first_pos, int n_rows) {
    if (!s || layer < 0 || layer >= s->dec->n_layers || first_pos < 0 || n_rows <= 0 ||
        n_rows > s->cap) {
        set_error("dec_state kv copy: bad arguments");
        return VOX_CUDA_ERR_ARG;
    }
    return VOX_CUDA_OK;
}

static int ring_copy(vox_cuda_dec_state *s, int layer, int first_pos, int n_rows, float *host_k,
                     float *host_v, bool to_device) {
    int rc = kv_rows_check(s, layer, first_pos, n_rows);
    if (rc) return rc;
    cudaSetDevice(s->dec->device);
    // the library stream is ordered after pending asynchronous steps, which write the ring
    if (DevCtx *c = ctx_for(s->dec->device)) VC_TRY(cudaStreamSynchronize(c->stream));
    const size_t row = (size_t)kKvDim * sizeof(float);
    int done = 0;
    while (done < n_rows) {
        const int slot = (first_pos + done) % s->cap;
        int run = s->cap - slot;
        if (run > n_rows - done) run = n_rows - done;
        float *dk = s->k_ring + ((size_t)layer * s->cap + slot) * kKvDim;
        float *dv = s->v_ring + ((size_t)layer * s->cap + slot) * kKvDim;
        if (to_device) {
            VC_TRY(cudaMemcpy(dk, host_k + (size_t)done * kKvDim, run * row, cudaMemcpyHostToDevice));
            VC_TRY(cudaMemcpy(dv, host_v + (size_t)done * kKvDim, run * row, cudaMemcpyHostToDevice));
        } else {
            VC_TRY(cudaMemcpy(host_k + (size_t)done * kKvDim, dk, run * row, cudaMemcpyDeviceToHost));
            VC_TRY(cudaMemcpy(host_v + (size_t)done * kKvDim, dv, run * row, cudaMemcpyDeviceToHost));
        }
        done += run;
    }
    return VOX_CUDA_OK;
}

extern "C" int vox_cuda_dec_state_load_kv(vox_cuda_dec_state *s, int layer, int first_pos,
                                          int n_rows, const float *k_rows, const float *v_rows) {
    if (!k_rows || !v_rows) return VOX_CUDA_ERR_ARG;
    return ring_copy(s, layer, first_pos, n_rows, const_cast<float *>(k_rows),
                     const_cast<float *>(v_rows), true);
}

extern "C" int vox_cuda_dec_state_read_kv(vox_cuda_dec_state *s, int layer, int first_pos,
                                          int n_rows, float *k_rows, float *v_rows) {
    if (!k_rows || !v_rows) return VOX_CUDA_ERR_ARG;
    return ring_copy(s, layer, first_pos, n_rows, k_rows, v_rows, false);
}

extern "C" int vox_cuda_decoder_full_step(vox_cuda_dec_state *s, const float *embed,
                                          const float *rope_freqs, float *logits) {
    if (!s || !embed) {
        set_error("decoder_full_step: bad arguments");
        return VOX_CUDA_ERR_ARG;
    }
    vox_cuda_decoder *d = s->dec;
    DevCtx *c = ctx_for(d->device);
    if (!c) return VOX_CUDA_ERR_UNAVAILABLE;
    cudaSetDevice(d->device);
    int rc = check_capacity(s, s->pos, s->pos);
    if (rc) return rc;
    StepWork *w = s->work;
    fill_slot(s, s->pos, h_slots(w));
    if (rope_freqs) memcpy(h_rope(w), rope_freqs, kHeadDim * sizeof(float));
    else host_rope_table(s->pos, kHeadDim, h_rope(w));
    memcpy(h_x(w), embed, kDecDim * sizeof(float));
    rc = run_step(d, c, w, true, c->stream, logits == nullptr);
    if (rc) return rc;
    if (logits) {
        VC_TRY(cudaMemcpyAsync(logits, w->logits, (size_t)d->vocab * 4, cudaMemcpyDeviceToHost, c->stream));
        VC_TRY(cudaStreamSynchronize(c->stream));
        if ((rc = check_step_error(w, c->stream))) return rc;
    }
    s->pos += 1;
    s->last_token = w->h_tokens[0];
    s->have_logits = true;
    return s->last_token;
}

extern "C" int vox_cuda_decoder_fill_alts(vox_cuda_dec_state *s, int n_alt, float cutoff,
                                          int *alt_ids) {
    if (!s || !alt_ids || n_alt < 1 || n_alt > 4) {
        set_error("decoder_fill_alts: bad arguments");
        return VOX_CUDA_ERR_ARG;
    }
    if (!s->have_logits) {
        set_error("decoder_fill_alts: no decode step since the last reset");
        return VOX_CUDA_ERR_ARG;
    }
    DevCtx *c = ctx_for(s->dec->device);
    if (!c) return VOX_CUDA_ERR_UNAVAILABLE;
    cudaSetDevice(s->dec->device);
    StepWork *w = s->work;
    VC_TRY(launch_fill_alts(w->logits, s->dec->vocab, w->tokens, n_alt, cutoff, w->alt_ids, c->stream));
    int ids[4];
    VC_TRY(cudaMemcpyAsync(ids, w->alt_ids, sizeof(ids), cudaMemcpyDeviceToHost, c->stream));
    VC_TRY(cudaStreamSynchronize(c->stream));
    int n = 0;
    for (int i = 0; i < n_alt; i++) {
        if (ids[i] < 0) break;
        alt_ids[n++] = ids[i];
    }
    return n;
}

extern "C" int vox_cuda_decoder_prefill_step(vox_cuda_dec_state *s, const float *x, int seq_len,
                                             const float *rope_freqs) {
    if (!s || !x || seq_len <= 0) {
        set_error("decoder_prefill_step: bad arguments");
        return VOX_CUDA_ERR_ARG;
    }
    vox_cuda_decoder *d = s->dec;
    DevCtx *c = ctx_for(d->device);
    if (!c) return VOX_CUDA_ERR_UNAVAILABLE;
    cudaSetDevice(d->device);
    int rc = VOX_CUDA_OK;
    if (d->tc_prefill) {
        // rows in launch sequences of kPrefillRows on the tensor cores
        for (int r0 = 0; r0 < seq_len; r0 += kPrefillRows) {
            const int last = s->pos + std::min(seq_len, r0 + kPrefillRows) - 1;
            if ((rc = check_capacity(s, s->pos + r0, last))) return rc;
        }
        std::lock_guard<std::mutex> lk(d->mu);
        rc = prefill_tc_rows(d, c, &s, &seq_len, 1, x, rope_freqs);
        if (rc) return rc;
        s->pos += seq_len;
        s->have_logits = false;
        return VOX_CUDA_OK;
    }
    // a row must not overwrite a ring slot still inside the window of an
    // earlier row of the same chunk: positions pos..pos+seq_len-1 all fit
    for (int r0 = 0; r0 < seq_len; r0 += kMaxBatch) {
        const int last = s->pos + ((seq_len - r0 < kMaxBatch) ? seq_len : r0 + kMaxBatch) - 1;
        if ((rc = check_capacity(s, s->pos + r0, last))) return rc;
    }
    // Rows are processed kMaxBatch at a time as parallel "streams" sharing one
    // ring: each row's attention covers positions <= its own, so the causal
    // mask of the prefill (voxtral_decoder.c:321-323) is preserved.
    for (int r0 = 0; r0 < seq_len; r0 += kMaxBatch) {
        const int n = (seq_len - r0 < kMaxBatch) ? seq_len - r0 : kMaxBatch;
        StepWork *&w = (n == kMaxBatch) ? s->prefill_work : d->batch_work[n];
        std::unique_lock<std::mutex> lk(d->mu, std::defer_lock);
        if (n != kMaxBatch) lk.lock();
        if (!w) w = make_work(c, n, d->vocab);
        if (!w) return VOX_CUDA_ERR_OOM;
        if (w->staged_pending) {   // an asynchronous step's upload of the host block
            VC_TRY(cudaEventSynchronize(w->staged));
            w->staged_pending = false;
        }
        for (int i = 0; i < n; i++) {
            const int pos = s->pos + r0 + i;
            fill_slot(s, pos, h_slots(w) + i);
            h_slots(w)[i].fresh = s->pos + r0;   // the chunk's first row
            if (rope_freqs) memcpy(h_rope(w) + i * kHeadDim, rope_freqs + (size_t)(r0 + i) * kHeadDim, kHeadDim * 4);
            else host_rope_table(pos, kHeadDim, h_rope(w) + i * kHeadDim);
        }
        memcpy(h_x(w), x + (size_t)r0 * kDecDim, (size_t)n * kDecDim * sizeof(float));
        rc = run_step(d, c, w, false, c->stream, true);
        if (rc) return rc;
    }
    s->pos += seq_len;
    s->have_logits = false;
    return VOX_CUDA_OK;
}

extern "C" int vox_cuda_decoder_prefill_batch(vox_cuda_dec_state *const *states, int n, const float *x,
                                              const int *seq_lens, const float *rope_freqs) {
    if (!states || n <= 0 || !x || !seq_lens || !states[0]) {
        set_error("decoder_prefill_batch: bad arguments");
        return VOX_CUDA_ERR_ARG;
    }
    vox_cuda_decoder *d = states[0]->dec;
    for (int i = 0; i < n; i++) {
        if (!states[i] || states[i]->dec != d || seq_lens[i] < 0) {
            set_error("decoder_prefill_batch: states must share one decoder, lengths >= 0");
            return VOX_CUDA_ERR_ARG;
        }
        for (int j = 0; j < i; j++)
            if (states[j] == states[i]) {
                set_error("decoder_prefill_batch: a state appears twice");
                return VOX_CUDA_ERR_ARG;
            }
    }
    if (!d->tc_prefill) {   // one state after the other through the decode-step kernels
        size_t off = 0;
        for (int i = 0; i < n; i++) {
            if (seq_lens[i] == 0) continue;
            int rc = vox_cuda_decoder_prefill_step(states[i], x + off * kDecDim,
                                                   seq_lens[i], rope_freqs ? rope_freqs + off * kHeadDim : nullptr);
            if (rc) return rc;
            off += seq_lens[i];
        }
        return VOX_CUDA_OK;
    }
    // a launch sequence holds at most kPrefillRows rows: each state's rows in
    // any one of them fit its ring together with the window before them
    for (int i = 0; i < n; i++)
        for (int r0 = 0; r0 < seq_lens[i]; r0 += kPrefillRows) {
            const int last = states[i]->pos + std::min(seq_lens[i], r0 + kPrefillRows) - 1;
            int rc = check_capacity(states[i], states[i]->pos + r0, last);
            if (rc) return rc;
        }
    DevCtx *c = ctx_for(d->device);
    if (!c) return VOX_CUDA_ERR_UNAVAILABLE;
    cudaSetDevice(d->device);
    std::lock_guard<std::mutex> lk(d->mu);
    int rc = prefill_tc_rows(d, c, states, seq_lens, n, x, rope_freqs);
    if (rc) return rc;
    for (int i = 0; i < n; i++) {
        states[i]->pos += seq_lens[i];
        if (seq_lens[i]) states[i]->have_logits = false;
    }
    return VOX_CUDA_OK;
}

static int batch_prepare(vox_cuda_dec_state *const *states, int n, vox_cuda_decoder **pd,
                         DevCtx **pc) {
    if (!states || n <= 0 || n > kMaxBatch) {
        set_error("decoder_step_batch: n must be 1..%d", kMaxBatch);
        return VOX_CUDA_ERR_ARG;
    }
    vox_cuda_decoder *d = states[0] ? states[0]->dec : nullptr;
    for (int i = 0; i < n; i++) {
        if (!states[i] || states[i]->dec != d) {
            set_error("decoder_step_batch: states must share one decoder");
            return VOX_CUDA_ERR_ARG;
        }
        for (int j = 0; j < i; j++)
            if (states[j] == states[i]) {
                set_error("decoder_step_batch: a state appears twice");
                return VOX_CUDA_ERR_ARG;
            }
        int rc = check_capacity(states[i], states[i]->pos, states[i]->pos);
        if (rc) return rc;
    }
    DevCtx *c = ctx_for(d->device);
    if (!c) return VOX_CUDA_ERR_UNAVAILABLE;
    cudaSetDevice(d->device);
    if (!d->batch_work[n]) d->batch_work[n] = make_work(c, n, d->vocab);
    if (!d->batch_work[n]) return VOX_CUDA_ERR_OOM;
    StepWork *w = d->batch_work[n];
    // an asynchronous step's upload of the host block may still be queued
    if (w->staged_pending) {
        VC_TRY(cudaEventSynchronize(w->staged));
        w->staged_pending = false;
    }
    for (int i = 0; i < n; i++) {
        fill_slot(states[i], states[i]->pos, h_slots(w) + i);
        host_rope_table(states[i]->pos, kHeadDim, h_rope(w) + i * kHeadDim);
    }
    // no caller token buffer unless the asynchronous step sets one (a
    // profile or synchronous launch must not write an earlier call's buffer)
    *h_tokens_to(w) = nullptr;
    *pd = d;
    *pc = c;
    return VOX_CUDA_OK;
}

extern "C" int vox_cuda_decoder_step_batch_ex(vox_cuda_dec_state *const *states, int n,
                                              const float *embeds, const float *rope_freqs,
                                              int *tokens, float *logits) {
    if (!embeds || !tokens) {
        set_error("decoder_step_batch: bad arguments");
        return VOX_CUDA_ERR_ARG;
    }
    vox_cuda_decoder *d = nullptr;
    DevCtx *c = nullptr;
    if (!states || n <= 0 || n > kMaxBatch || !states[0]) return batch_prepare(states, n, &d, &c);
    std::lock_guard<std::mutex> lk(states[0]->dec->mu);
    int rc = batch_prepare(states, n, &d, &c);
    if (rc) return rc;
    StepWork *w = d->batch_work[n];
    memcpy(h_x(w), embeds, (size_t)n * kDecDim * sizeof(float));
    if (rope_freqs) memcpy(h_rope(w), rope_freqs, (size_t)n * kHeadDim * sizeof(float));
    rc = run_step(d, c, w, true, c->stream, true);
    w->err_pending = false;   // this step's error check covered the earlier ones
    if (rc) return rc;
    if (logits) {   // the step has completed: [n][vocab] in one copy
        VC_TRY(cudaMemcpy(logits, w->logits, (size_t)n * d->vocab * sizeof(float),
                          cudaMemcpyDeviceToHost));
    }
    for (int i = 0; i < n; i++) {
        tokens[i] = w->h_tokens[i];
        states[i]->pos += 1;
        states[i]->have_logits = false;
    }
    return VOX_CUDA_OK;
}

extern "C" int vox_cuda_decoder_step_batch(vox_cuda_dec_state *const *states, int n,
                                           const float *embeds, int *tokens) {
    return vox_cuda_decoder_step_batch_ex(states, n, embeds, nullptr, tokens, nullptr);
}

// The asynchronous batched step.  The step's input rows x come either from
// embeds_dev ([n][3072], copied), or - token-embedding steps - from
// rows[i] + E[prev_tokens_dev[i]] (E the tiled LM head / token table), built
// on the device by one kernel ahead of the step's graph.
static int step_batch_async(vox_cuda_dec_state *const *states, int n, const float *embeds_dev,
                            const float *const *rows, const int *prev_tokens_dev, int *tokens_dev,
                            void *stream, const char *what) {
    vox_cuda_decoder *d = nullptr;
    DevCtx *c = nullptr;
    if (!states || n <= 0 || n > kMaxBatch || !states[0]) return batch_prepare(states, n, &d, &c);
    std::lock_guard<std::mutex> lk(states[0]->dec->mu);
    int rc = batch_prepare(states, n, &d, &c);
    if (rc) return rc;
    StepWork *w = d->batch_work[n];
    cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
    // a timeout raised by an earlier asynchronous step (its error word was
    // copied back behind err_ev) is reported now
    if (w->err_pending && cudaEventQuery(w->err_ev) == cudaSuccess) {
        w->err_pending = false;
        if ((rc = check_step_error(w, st))) return rc;
    }
    if (!d->tail && cudaEventCreateWithFlags(&d->tail, cudaEventDisableTiming) != cudaSuccess) {
        set_error("%s: event creation failed", what);
        return VOX_CUDA_ERR_CUDA;
    }
    // the previous asynchronous step may have run on another stream
    if (d->tail_set && st != c->stream) VC_TRY(cudaStreamWaitEvent(st, d->tail, 0));
    // slots, rope tables and row addresses from the host block; the step's
    // input rows from the device
    if (rows)
        for (int i = 0; i < n; i++) h_rows(w)[i] = rows[i];
    // the LM head's argmax writes the caller's tokens itself (per-phase
    // kernels; the persistent step writes its own buffer, copied below)
    const bool persist = w->graph[1] ? w->graph_persist : (d->players && persist_on());
    *h_tokens_to(w) = persist ? nullptr : tokens_dev;
    const size_t head = (char *)w->x - w->dblock;
    VC_TRY(cudaMemcpyAsync(w->dblock, w->hblock, head, cudaMemcpyHostToDevice, st));
    VC_TRY(cudaEventRecord(w->staged, st));
    w->staged_pending = true;
    if (prev_tokens_dev)
        VC_TRY(launch_embed_tokens(w->x, w->rows, nullptr, 0, prev_tokens_dev, n, d->tok_emb, d->vocab, kDecDim,
                                   w->err, st));
    else
        VC_TRY(cudaMemcpyAsync(w->x, embeds_dev, (size_t)n * kDecDim * 4, cudaMemcpyDeviceToDevice, st));
    cudaGraphExec_t &g = w->graph[1];
    if (!g) {
        cudaGraph_t graph = nullptr;
        w->graph_persist = persist;
        VC_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
        rc = enqueue_layers(d, w, true, st);
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
    if (w->graph_persist) VC_TRY(cudaMemcpyAsync(tokens_dev, w->tokens, sizeof(int) * n, cudaMemcpyDeviceToDevice, st));
    // the sticky error word comes back every 8th asynchronous step (and with
    // every synchronous one), one copy in flight at a time
    if (!w->err_pending && (++w->err_tick & 7u) == 0u) {
        VC_TRY(cudaMemcpyAsync(w->h_tokens + n, w->err, sizeof(unsigned), cudaMemcpyDeviceToHost, st));
        VC_TRY(cudaEventRecord(w->err_ev, st));
        w->err_pending = true;
    }
    // order the library stream (every synchronous entry point, the frees)
    // after this step, without a host wait
    VC_TRY(cudaEventRecord(d->tail, st));
    if (st != c->stream) VC_TRY(cudaStreamWaitEvent(c->stream, d->tail, 0));
    d->tail_set = true;
    for (int i = 0; i < n; i++) {
        states[i]->pos += 1;
        states[i]->have_logits = false;
    }
    return VOX_CUDA_OK;
}

extern "C" int vox_cuda_decoder_step_batch_dev(vox_cuda_dec_state *const *states, int n,
                                               const float *embeds_dev, int *tokens_dev,
                                               void *stream) {
    if (!embeds_dev || !tokens_dev) {
        set_error("decoder_step_batch_dev: bad arguments");
        return VOX_CUDA_ERR_ARG;
    }
    if (((uintptr_t)embeds_dev & 3u) || ((uintptr_t)tokens_dev & 3u)) {
        set_error("decoder_step_batch_dev: misaligned device pointers");
        return VOX_CUDA_ERR_ARG;
    }
    return step_batch_async(states, n, embeds_dev, nullptr, nullptr, tokens_dev, stream,
                            "decoder_step_batch_dev");
}

extern "C" int vox_cuda_decoder_step_batch_tokens_dev(vox_cuda_dec_state *const *states, int n,
                                                      const float *const *rows_dev,
                                                      const int *prev_tokens_dev, int *tokens_dev,
                                                      void *stream) {
    if (!rows_dev || !prev_tokens_dev || !tokens_dev) {
        set_error("decoder_step_batch_tokens_dev: bad arguments");
        return VOX_CUDA_ERR_ARG;
    }
    if (((uintptr_t)prev_tokens_dev & 3u) || ((uintptr_t)tokens_dev & 3u)) {
        set_error("decoder_step_batch_tokens_dev: misaligned device pointers");
        return VOX_CUDA_ERR_ARG;
    }
    for (int i = 0; i < n && i < kMaxBatch; i++)
        if (!rows_dev[i] || ((uintptr_t)rows_dev[i] & 7u)) {
            set_error("decoder_step_batch_tokens_dev: row %d is NULL or misaligned", i);
            return VOX_CUDA_ERR_ARG;
        }
    return step_batch_async(states, n, nullptr, rows_dev, prev_tokens_dev, tokens_dev, stream,
                            "decoder_step_batch_tokens_dev");
}

extern "C" int vox_cuda_decoder_embed_dev(vox_cuda_decoder *d, int n, const float *rows_dev,
                                          const int *tokens_dev, float *out_dev, void *stream) {
    if (!d || n <= 0 || !tokens_dev || !out_dev || ((uintptr_t)tokens_dev & 3u) ||
        ((uintptr_t)out_dev & 7u) || ((uintptr_t)rows_dev & 7u)) {
        set_error("decoder_embed_dev: bad arguments");
        return VOX_CUDA_ERR_ARG;
    }
    DevCtx *c = ctx_for(d->device);
    if (!c) return VOX_CUDA_ERR_UNAVAILABLE;
    cudaSetDevice(d->device);
    cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
    VC_TRY(launch_embed_tokens(out_dev, nullptr, rows_dev, kDecDim, tokens_dev, n, d->tok_emb, d->vocab,
                               kDecDim, nullptr, st));
    return VOX_CUDA_OK;
}

extern "C" int vox_cuda_decoder_profile_batch(vox_cuda_dec_state *const *states, int n,
                                              const float *embeds_dev, int iters, float *ms) {
    if (!embeds_dev || !ms || iters <= 0) {
        set_error("decoder_profile_batch: bad arguments");
        return VOX_CUDA_ERR_ARG;
    }
    vox_cuda_decoder *d = nullptr;
    DevCtx *c = nullptr;
    if (!states || n <= 0 || n > kMaxBatch || !states[0]) return batch_prepare(states, n, &d, &c);
    std::lock_guard<std::mutex> lk(states[0]->dec->mu);
    int rc = batch_prepare(states, n, &d, &c);
    if (rc) return rc;
    StepWork *w = d->batch_work[n];
    cudaStream_t st = c->stream;
    const int n_launch = 5 * d->n_layers + 2;   // prep, 5 per layer, LM head
    std::vector<cudaEvent_t> evs(2 * n_launch);
    for (auto &e : evs)
        if (cudaEventCreate(&e) != cudaSuccess) {
            set_error("profile: event creation failed");
            return VOX_CUDA_ERR_CUDA;
        }
    double acc[VOX_CUDA_PROF_PHASES] = {0};
    const size_t head = (char *)w->x - w->dblock;
    for (int it = 0; it < iters && rc == VOX_CUDA_OK; it++) {
        if (cudaMemcpyAsync(w->dblock, w->hblock, head, cudaMemcpyHostToDevice, st) != cudaSuccess ||
            cudaMemcpyAsync(w->x, embeds_dev, (size_t)n * kDecDim * 4, cudaMemcpyDeviceToDevice, st) !=
                cudaSuccess) {
            set_error("profile: staging copy failed");
            rc = VOX_CUDA_ERR_CUDA;
            break;
        }
        rc = enqueue_layers(d, w, true, st, evs.data());
        if (rc) break;
        if (cudaStreamSynchronize(st) != cudaSuccess) {
            set_error("profile: step failed");
            rc = VOX_CUDA_ERR_CUDA;
            break;
        }
        for (int i = 0; i < n_launch; i++) {
            float t = 0.f;
            cudaEventElapsedTime(&t, evs[2 * i], evs[2 * i + 1]);
            const int phase = (i == n_launch - 1) ? VOX_CUDA_PROF_LM_HEAD
                              : (i == 0)           ? VOX_CUDA_PROF_QKV
                                                   : ((i - 1) % 5);
            acc[phase] += t;
        }
    }
    for (auto &e : evs) cudaEventDestroy(e);
    if (rc) return rc;
    for (int i = 0; i < VOX_CUDA_PROF_PHASES; i++) ms[i] = (float)(acc[i] / iters);
    return VOX_CUDA_OK;
}

extern "C" int vox_cuda_decoder_profile_sequence(vox_cuda_dec_state *const *states, int n,
                                                 const float *embeds_dev, int phase, int iters,
                                                 float *ms_per_launch) {
    if (!embeds_dev || !ms_per_launch || iters <= 0 || phase < 0 || phase >= VOX_CUDA_PROF_PHASES) {
        set_error("decoder_profile_sequence: bad arguments");
        return VOX_CUDA_ERR_ARG;
    }
    vox_cuda_decoder *d = nullptr;
    DevCtx *c = nullptr;
    if (!states || n <= 0 || n > kMaxBatch || !states[0]) return batch_prepare(states, n, &d, &c);
    std::lock_guard<std::mutex> lk(states[0]->dec->mu);
    int rc = batch_prepare(states, n, &d, &c);
    if (rc) return rc;
    StepWork *w = d->batch_work[n];
    cudaStream_t st = c->stream;
    const size_t head = (char *)w->x - w->dblock;
    // one whole step first: every phase's inputs then hold real activations
    VC_TRY(cudaMemcpyAsync(w->dblock, w->hblock, head, cudaMemcpyHostToDevice, st));
    VC_TRY(cudaMemcpyAsync(w->x, embeds_dev, (size_t)n * kDecDim * 4, cudaMemcpyDeviceToDevice, st));
    if ((rc = enqueue_layers(d, w, true, st))) return rc;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    VC_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    rc = enqueue_layers(d, w, true, st, nullptr, phase);
    cudaError_t e = cudaStreamEndCapture(st, &graph);
    if (rc) {
        if (graph) cudaGraphDestroy(graph);
        return rc;
    }
    VC_TRY(e);
    e = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    VC_TRY(e);
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    float t = 0.f;
    bool ok = cudaEventCreate(&e0) == cudaSuccess && cudaEventCreate(&e1) == cudaSuccess;
    for (int i = 0; ok && i < 2; i++) ok = cudaGraphLaunch(exec, st) == cudaSuccess;   // warm-up
    ok = ok && cudaEventRecord(e0, st) == cudaSuccess;
    for (int i = 0; ok && i < iters; i++) ok = cudaGraphLaunch(exec, st) == cudaSuccess;
    ok = ok && cudaEventRecord(e1, st) == cudaSuccess && cudaEventSynchronize(e1) == cudaSuccess &&
         cudaEventElapsedTime(&t, e0, e1) == cudaSuccess;
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    cudaGraphExecDestroy(exec);
    if (!ok) {
        set_error("decoder_profile_sequence: timing failed");
        return VOX_CUDA_ERR_CUDA;
    }
    VC_TRY(cudaMemcpyAsync(w->h_tokens + n, w->err, sizeof(unsigned), cudaMemcpyDeviceToHost, st));
    VC_TRY(cudaStreamSynchronize(st));
    w->err_pending = false;
    if ((rc = check_step_error(w, st))) return rc;
    const int launches = phase == VOX_CUDA_PROF_LM_HEAD ? 1 : d->n_layers;
    *ms_per_launch = t / ((float)iters * launches);
    return VOX_CUDA_OK;
}

