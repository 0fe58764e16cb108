// vc_step_persist.cu - the whole decode step (26 layers + LM head + argmax)
// as one persistent kernel: one CTA per SM, a weight stream that never waits
// on activations, and fine-grained device-side dependencies between phases.
//
// Why: the step is a chain of ~130 HBM-bound GEMVs and attentions.  As
// separate launches, each pays a ramp and a reduction tail (4-8 us) during
// which HBM idles.  Here the weights - which depend on nothing the step
// computes - are streamed by a producer warp into a shared-memory ring as far
// ahead as the ring allows, across phase and layer boundaries.  The consumer
// warps wait only for the activations they multiply, so HBM keeps streaming
// while they wait (for the attention, for the last row block of the previous
// phase, for a split-K partner).
//
// Layout of the work (identical on every CTA, computed from the parameters):
//   * GEMV phases (q|k|v, wo, w1|w3, w2, LM head): items (row block rb of 64
//     rows, K slice ks); item i of a phase belongs to CTA i mod gridDim.x and
//     is processed in increasing i.  An item's weights are a contiguous run
//     of the fragment-tiled matrix (vc_gemv.cu), moved by one bulk copy per
//     8 k-blocks (16 KB stage).  The 8 consumer warps take one k-block of a
//     stage each (4 tiles x (x_hi, x_lo) = 8 mma.sync).  The producer also
//     runs a second cursor a few hundred KB ahead of the ring that pulls the
//     coming stages into L2 (cp.async.bulk.prefetch.L2), so the ring's copies
//     are served at L2 latency and 112 KB in flight per SM keeps HBM busy.
//   * A phase's activation fragments (the K slices of this CTA's items, at
//     most 96 KB) are bulk-copied into shared memory once, right after the
//     phase's dependency is met, in 4 KB chunks that complete on their own
//     mbarriers: the first stage starts when its chunk lands.
//   * K slices of a row block are summed in slice order by the last CTA to
//     finish one (atomic ticket): deterministic, no cluster needed, no CTA
//     waits for another inside a phase.  That CTA runs the epilogue of the
//     row block (the same epilogues as vc_gemv.cu) and counts the row block
//     done for the phase.
//   * Attention phase: items (stream, KV head, 64-key split); the last split
//     of a (stream, KV head) to finish merges them and writes the wo
//     fragments.
//   * A consumer CTA starts a phase once the phase it depends on has counted
//     all its row blocks (q|k|v after the previous w2, attention after q|k|v,
//     wo after every merge, w1|w3 after wo, w2 after w1|w3, the LM head after
//     the last w2): a bounded spin on a device counter.  The producer never
//     waits on these counters, so it runs ahead into the next phases.
//   * Every wait (ring barriers, dependency counters) is bounded (2 s of
//     %globaltimer).  On expiry the CTA raises the step's error word, stops
//     issuing copies, lets the ones in flight land, and exits; the other
//     CTAs' waits then expire the same way.  The launch is cooperative, so
//     all CTAs are resident together and the counters they wait on are
//     written by running CTAs.
#include "vc_common.cuh"
#include "vc_internal.h"

#include <math.h>

#include <algorithm>

namespace vc {

namespace {

constexpr int kPConsWarps = 8;
constexpr int kPConsumers = kPConsWarps * 32;            // 256
constexpr int kPThreads = kPConsumers + 32;              // + the producer warp
constexpr int kPStages = 7;
constexpr int kPStageKB = 8;                             // k-blocks per stage
constexpr int kPKbBytes = 4 * 512;                       // one k-block of a 64-row block
constexpr int kPStageBytes = kPStageKB * kPKbBytes;      // 16 KB
constexpr int kPActKB = 192;                             // activation k-blocks held (96 KB)
constexpr int kPActChunks = kPActKB / kPStageKB;         // 24 chunks of 4 KB
constexpr unsigned long long kPWaitNs = 2000000000ull;
constexpr int kPKeys = 64;                               // keys per attention split

__device__ __forceinline__ uint32_t psmem(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint64_t ptimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void pbar_init(uint64_t *b, uint32_t c) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(psmem(b)), "r"(c) : "memory");
}
__device__ __forceinline__ void pbar_expect_tx(uint64_t *b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(psmem(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void pbar_arrive(uint64_t *b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(psmem(b)) : "memory");
}
__device__ __forceinline__ bool pbar_try(uint64_t *b, uint32_t par) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(psmem(b)), "r"(par)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool pbar_wait(uint64_t *b, uint32_t par, uint64_t deadline) {
    while (!pbar_try(b, par))
        if (ptimer() > deadline) return false;
    return true;
}
__device__ __forceinline__ void pbulk(void *dst, const void *src, uint32_t bytes, uint64_t *bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1], %2, [%3], %4;" ::"r"(psmem(dst)),
        "l"(src), "r"(bytes), "r"(psmem(bar)), "l"(pol)
        : "memory");
}
__device__ __forceinline__ void pl2_prefetch(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void pcp16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(psmem(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void pcp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// arrive on *b once all of this thread's earlier cp.async have landed (the
// barrier counts this arrival among its expected ones: .noinc)
__device__ __forceinline__ void pcp_arrive_noinc(uint64_t *b) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(psmem(b)) : "memory");
}
__device__ __forceinline__ void pcp_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void pmma(float (&c)[4], const uint4 &a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1));
}

// consumer-only barrier (the producer warp never takes part)
__device__ __forceinline__ void cons_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kPConsumers) : "memory"); }

__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// ticket / counter atomics at gpu scope: release of this CTA's writes (which
// the preceding barrier ordered before this thread) and acquire of the
// writes released by the other arrivals
__device__ __forceinline__ unsigned atom_add_acq_rel(unsigned *p, unsigned v) {
    unsigned old;
    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
__device__ __forceinline__ void red_add_release(unsigned *p, unsigned v) {
    asm volatile("red.add.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ bool p_better(float v, int i, float bv, int bi) {
    return v > bv || (v == bv && i < bi);
}

// The GEMV phases of a layer, in order, and the LM head.
enum : int { G_QKV = 0, G_WO = 1, G_W13 = 2, G_W2 = 3, G_LM = 4, G_N = 5 };

struct PhaseShape {
    const uint16_t *W;   // tiled weights
    int N, KB, KS, per;  // rows, k-blocks, K slices, k-blocks per slice
    int RB, items;
};

__device__ __forceinline__ PhaseShape phase_shape(const PersistParams &p, int layer, int g) {
    PhaseShape s;
    const PersistLayer &L = p.layers[layer < p.n_layers ? layer : 0];
    switch (g) {
        case G_QKV: s.W = L.qkv; s.N = kQkvRows; s.KB = kDecDim / 16; s.KS = p.ks[G_QKV]; break;
        case G_WO: s.W = L.wo; s.N = kDecDim; s.KB = kQDim / 16; s.KS = p.ks[G_WO]; break;
        case G_W13: s.W = L.w13; s.N = 2 * kDecHidden; s.KB = kDecDim / 16; s.KS = p.ks[G_W13]; break;
        case G_W2: s.W = L.w2; s.N = kDecDim; s.KB = kDecHidden / 16; s.KS = p.ks[G_W2]; break;
        default: s.W = p.lm; s.N = p.vocab; s.KB = kDecDim / 16; s.KS = p.ks[G_LM]; break;
    }
    s.per = (s.KB + s.KS - 1) / s.KS;
    s.RB = (s.N + 63) / 64;
    s.items = s.RB * s.KS;
    return s;
}

// item i of a phase -> (row block, first k-block, k-blocks)
struct Item {
    int rb, ks, kb0, nkb, nst;
};
__device__ __forceinline__ Item item_of(const PhaseShape &s, int i) {
    Item it;
    it.rb = i / s.KS;
    it.ks = i - it.rb * s.KS;
    it.kb0 = it.ks * s.per;
    it.nkb = max(0, min(s.per, s.KB - it.kb0));
    it.nst = (it.nkb + kPStageKB - 1) / kPStageKB;
    return it;
}

// The producer's walk over this CTA's weight stages, in consumption order:
// layers, their GEMV phases, the CTA's items of each phase, their stages.
struct Cursor {
    int layer, g, i, st;
    bool valid;
    PhaseShape s;
    Item itm;
};
__device__ __forceinline__ void cur_settle(Cursor &c, const PersistParams &p, int cta, int G) {
    while (true) {
        const int last_layer = p.with_head ? p.n_layers : p.n_layers - 1;
        if (c.layer > last_layer) {
            c.valid = false;
            return;
        }
        if (c.i < c.s.items) {
            if (c.st < c.itm.nst) {
                c.valid = true;
                return;
            }
            c.i += G;
            c.st = 0;
            if (c.i < c.s.items) c.itm = item_of(c.s, c.i);
            continue;
        }
        // next phase
        const bool head = c.layer == p.n_layers;
        if (head || c.g == G_W2) {
            c.layer++;
            c.g = (c.layer == p.n_layers) ? G_LM : G_QKV;
        } else {
            c.g++;
        }
        if (c.layer > last_layer) {
            c.valid = false;
            return;
        }
        c.s = phase_shape(p, c.layer, c.g);
        c.i = cta;
        c.st = 0;
        if (c.i < c.s.items) c.itm = item_of(c.s, c.i);
    }
}
__device__ __forceinline__ void cur_begin(Cursor &c, const PersistParams &p, int cta, int G) {
    c.layer = 0;
    c.g = (p.n_layers == 0) ? G_LM : G_QKV;
    c.s = phase_shape(p, 0, c.g);
    c.i = cta;
    c.st = 0;
    if (c.i < c.s.items) c.itm = item_of(c.s, c.i);
    cur_settle(c, p, cta, G);
}
__device__ __forceinline__ void cur_next(Cursor &c, const PersistParams &p, int cta, int G) {
    c.st++;
    cur_settle(c, p, cta, G);
}
__device__ __forceinline__ const char *cur_src(const Cursor &c) {
    return reinterpret_cast<const char *>(c.s.W) + ((size_t)c.itm.rb * c.s.KB + c.itm.kb0) * kPKbBytes +
           (size_t)c.st * kPStageBytes;
}
__device__ __forceinline__ uint32_t cur_bytes(const Cursor &c) {
    return (uint32_t)min(kPStageKB, c.itm.nkb - c.st * kPStageKB) * kPKbBytes;
}

struct PAtt {
    float k[kPKeys][kHeadDim];   // 32 KB; the merge's weights reuse it
    float v[kPKeys][kHeadDim];   // 32 KB
    float q[4][kHeadDim];
    float p[4][kPKeys];
    float mx[4][2], sum[4][2];
};

struct PShared {
    uint64_t full[kPStages], empty[kPStages], actb[kPActChunks];
    alignas(128) unsigned char ring[kPStages][kPStageBytes];          // 112 KB of weights
    union alignas(128) {
        unsigned char act[kPActKB][512];                              // 96 KB: a phase's activations
        PAtt att;                                                     // the attention's staging
    } u;
    alignas(16) float red[4][4 * 32 * 4];                             // 8 KB: warp partials
    float part[64][8];
    float s_inv[8];
    float red_v[kPConsWarps][8];
    int red_i[kPConsWarps][8];
    int act_base[16];     // K slice -> its first k-block in u.act (-1: not held)
    int slot_ks[16];      // slot -> K slice
    int nslot;
    int flag;             // last-arriver decisions
    int abort;            // a bounded wait of this CTA expired
};
static_assert(sizeof(float) * kPKeys * kHeadDim >= sizeof(float) * 4 * kAttnSplits, "merge weights fit");
static_assert(sizeof(PAtt) <= (size_t)kPActKB * 512, "attention staging fits the activation area");

// Sync region (unsigned words, zeroed before every launch):
//   done counters: 8 per layer slot (the 4 GEMV phases, [5] the attention
//     merges), the LM head's row-block ticket in the slot after the layers;
//   split-K tickets: one per row block of every split GEMV phase of every layer
//     (q|k|v 96, wo 48, w1|w3 288, w2 48), then the LM head's 2048 (its vocab
//     is at most kVocab);
//   attention tickets: one per (layer, stream, KV head).
constexpr int kPDoneWords = (kDecLayersMax + 1) * 8;
constexpr int kPTicketsPerLayer = kQkvRows / 64 + kDecDim / 64 + 2 * kDecHidden / 64 + kDecDim / 64;   // 480
constexpr int kPTicketWords = kDecLayersMax * kPTicketsPerLayer + kVocab / 64;
constexpr int kPAttWords = kDecLayersMax * kMaxBatch * kDecKvHeads;

__device__ __forceinline__ unsigned *done_ctr(const PersistParams &p, int layer, int ph) {
    return p.sync + layer * 8 + ph;
}
__device__ __forceinline__ unsigned *ticket_ctr(const PersistParams &p, int layer, int g, int rb) {
    constexpr int off[4] = {0, kQkvRows / 64, kQkvRows / 64 + kDecDim / 64,
                            kQkvRows / 64 + kDecDim / 64 + 2 * kDecHidden / 64};
    if (g == G_LM) return p.sync + kPDoneWords + kDecLayersMax * kPTicketsPerLayer + rb;
    return p.sync + kPDoneWords + layer * kPTicketsPerLayer + off[g] + rb;
}
__device__ __forceinline__ unsigned *att_ctr(const PersistParams &p, int layer, int m, int kvh) {
    return p.sync + kPDoneWords + kPTicketWords + (layer * kMaxBatch + m) * kDecKvHeads + kvh;
}

// attention splits of stream m: 64-key splits of its window
__device__ __forceinline__ int att_splits(const StreamSlot &sl) {
    return max(1, min(kAttnSplits, (sl.n_keys + kPKeys - 1) / kPKeys));
}

// attention item a -> (stream, KV head, split, splits)
__device__ __forceinline__ void att_item(const PersistParams &p, int a, int &m, int &kvh, int &s, int &S) {
    int rem = a;
    for (m = 0; m < p.M; m++) {
        S = att_splits(p.slots[m]);
        if (rem < kDecKvHeads * S) break;
        rem -= kDecKvHeads * S;
    }
    kvh = rem / S;
    s = rem - kvh * S;
}

}  // namespace

// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(kPThreads, 1)
step_persist_kernel(const PersistParams p) {
    extern __shared__ __align__(128) unsigned char psm[];
    PShared &sh = *reinterpret_cast<PShared *>(psm);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, cta = blockIdx.x;
    const int M = p.M;
    const uint64_t deadline = ptimer() + kPWaitNs;

    if (tid == 0) {
        for (int s = 0; s < kPStages; s++) {
            pbar_init(&sh.full[s], 1);
            pbar_init(&sh.empty[s], kPConsWarps);
        }
        for (int c = 0; c < kPActChunks; c++) pbar_init(&sh.actb[c], kPConsumers);
        sh.abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    // ======================= producer warp =======================
    if (warp == kPConsWarps) {
        if (lane == 0) {
            const uint64_t pol = make_evict_first_policy();
            Cursor a, b;
            cur_begin(a, p, cta, G);
            cur_begin(b, p, cta, G);
            for (int k = 0; k < p.l2_ahead && b.valid; k++) {   // the L2 cursor starts ahead
                pl2_prefetch(cur_src(b), cur_bytes(b));
                cur_next(b, p, cta, G);
            }
            uint32_t it = 0;
            bool ok = true;
            while (a.valid) {
                const int slot = it % kPStages;
                if (it >= (uint32_t)kPStages && !pbar_wait(&sh.empty[slot], ((it / kPStages) + 1) & 1u, deadline)) {
                    ok = false;
                    break;
                }
                if (*(volatile int *)&sh.abort) {
                    ok = false;
                    break;
                }
                const uint32_t bytes = cur_bytes(a);
                pbar_expect_tx(&sh.full[slot], bytes);
                pbulk(sh.ring[slot], cur_src(a), bytes, &sh.full[slot], pol);
                if (b.valid) {
                    pl2_prefetch(cur_src(b), cur_bytes(b));
                    cur_next(b, p, cta, G);
                }
                cur_next(a, p, cta, G);
                it++;
            }
            if (!ok) {
                atomicExch(p.err, 1u);
                *(volatile int *)&sh.abort = 1;
                // copies already issued land before the CTA's shared memory goes away
                const uint64_t grace = ptimer() + 10000000ull;
                while (ptimer() < grace) {
                }
            }
        }
        return;
    }

    // ======================= consumer warps =======================
    uint32_t it = 0;          // ring stage counter (the producer's sequence)
    uint32_t gen = 0;         // GEMV phases started: the activation barriers' parity
    bool ok = true;
    auto fail = [&]() {
        ok = false;
        atomicExch(p.err, 1u);
        *(volatile int *)&sh.abort = 1;
    };
    // thread 0 waits for a counter to reach `target`; CTA-uniform after the barrier
    auto wait_done = [&](const unsigned *ctr, unsigned target) {
        if (tid == 0 && ok) {
            while (ld_acquire(ctr) < target) {
                if (ptimer() > deadline) {
                    fail();
                    break;
                }
                __nanosleep(64);
            }
        }
        cons_sync();
        if (*(volatile int *)&sh.abort) ok = false;
    };
    const int ss_parts = kDecDim / 64;   // row blocks of x: the norm's partial sums

    for (int layer = 0; layer <= p.n_layers && ok; layer++) {
        const bool head = layer == p.n_layers;
        if (head && !p.with_head) break;
        for (int g = head ? G_LM : G_QKV; g <= (head ? G_LM : G_W2) && ok; g++) {
            // ---------------- attention (between q|k|v and wo) ----------------
            if (g == G_WO) {
                int total = 0;
                for (int m = 0; m < M; m++) total += kDecKvHeads * att_splits(p.slots[m]);
                if (cta < total) wait_done(done_ctr(p, layer, G_QKV), (unsigned)((kQkvRows + 63) / 64));
                PAtt &at = sh.u.att;
                for (int a = cta; a < total && ok; a += G) {
                    int m, kvh, s, S;
                    att_item(p, a, m, kvh, s, S);
                    const StreamSlot slt = p.slots[m];
                    const int n_keys = slt.n_keys;
                    const int chunk = (n_keys + S - 1) / S;
                    const int kb = s * chunk, nk = max(0, min(kb + chunk, n_keys) - kb);
                    const int first = slt.pos - n_keys + 1;
                    const size_t loff = (size_t)layer * slt.cap * kKvDim + kvh * kHeadDim;
                    const float *kbase = slt.k_ring + loff, *vbase = slt.v_ring + loff;
                    cons_sync();   // the previous item's staging is consumed
                    for (int c = tid; c < nk * (kHeadDim / 4); c += kPConsumers) {
                        const int j = c / (kHeadDim / 4), piece = c % (kHeadDim / 4);
                        const size_t row = (size_t)((first + kb + j) % slt.cap) * kKvDim + 4 * piece;
                        pcp16(&at.k[j][4 * piece], kbase + row);
                        pcp16(&at.v[j][4 * piece], vbase + row);
                    }
                    pcp_commit();
                    if (tid < 128) {   // 4 query heads x 128
                        const int h = tid >> 5;
                        const float4 v = __ldcg(reinterpret_cast<const float4 *>(
                            p.q + (size_t)m * kQDim + (kvh * 4 + h) * kHeadDim + 4 * lane));
                        *reinterpret_cast<float4 *>(&at.q[h][4 * lane]) = v;
                    }
                    pcp_wait_all();
                    cons_sync();
                    // scores: warp -> head (warp & 3), keys 32 * (warp >> 2) + lane
                    const float scale = 1.0f / sqrtf((float)kHeadDim);
                    {
                        const int h = warp & 3, half = warp >> 2, j = 32 * half + lane;
                        const float4 *q4 = reinterpret_cast<const float4 *>(at.q[h]);
                        const float4 *k4 = reinterpret_cast<const float4 *>(at.k[j]);
                        float acc = 0.f;
#pragma unroll 8
                        for (int i = 0; i < kHeadDim / 4; i++) {
                            const int f = (i + lane) & (kHeadDim / 4 - 1);
                            const float4 kk = k4[f], qq = q4[f];
                            acc = fmaf(qq.x, kk.x, acc);
                            acc = fmaf(qq.y, kk.y, acc);
                            acc = fmaf(qq.z, kk.z, acc);
                            acc = fmaf(qq.w, kk.w, acc);
                        }
                        const float sc = (j < nk) ? acc * scale : -INFINITY;
                        float mx = sc;
#pragma unroll
                        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
                        if (lane == 0) at.mx[h][half] = mx;
                        cons_sync();
                        const float gm = fmaxf(at.mx[h][0], at.mx[h][1]);
                        const float pv = (j < nk) ? expf(sc - gm) : 0.f;
                        at.p[h][j] = pv;
                        const float sum = warp_sum(pv);
                        if (lane == 0) at.sum[h][half] = sum;
                    }
                    cons_sync();
                    // P.V: thread -> dimension (tid & 127), heads 2 * (tid >> 7) + {0, 1}
                    {
                        const int d = tid & 127, h0 = 2 * (tid >> 7);
                        float a0 = 0.f, a1 = 0.f;
                        for (int j = 0; j < nk; j++) {
                            const float vj = at.v[j][d];
                            a0 = fmaf(at.p[h0][j], vj, a0);
                            a1 = fmaf(at.p[h0 + 1][j], vj, a1);
                        }
                        const size_t p0 = ((size_t)m * kDecHeads + kvh * 4 + h0) * kAttnSplits + s;
                        const size_t p1 = p0 + kAttnSplits;
                        p.part_o[p0 * kHeadDim + d] = a0;
                        p.part_o[p1 * kHeadDim + d] = a1;
                        if (tid < 4) {
                            const size_t pi = ((size_t)m * kDecHeads + kvh * 4 + tid) * kAttnSplits + s;
                            p.part_ml[pi * 2] = fmaxf(at.mx[tid][0], at.mx[tid][1]);
                            p.part_ml[pi * 2 + 1] = at.sum[tid][0] + at.sum[tid][1];
                        }
                    }
                    // release the partials, take a ticket; the last one acquires them
                    cons_sync();
                    if (tid == 0) sh.flag = atom_add_acq_rel(att_ctr(p, layer, m, kvh), 1u) + 1u == (unsigned)S;
                    cons_sync();
                    if (!sh.flag) continue;
                    // merge the S splits: warps 0..3 -> heads, lane -> 4 dimensions
                    if (warp < 4) {
                        float(*smw)[kAttnSplits] = reinterpret_cast<float(*)[kAttnSplits]>(&at.k[0][0]);
                        const int hh = warp, d4 = 4 * lane, h = kvh * 4 + hh;
                        const size_t pbase = ((size_t)m * kDecHeads + h) * kAttnSplits;
                        float gm = -INFINITY;
                        for (int t = lane; t < S; t += 32) {
                            const float mt = __ldcg(p.part_ml + (pbase + t) * 2);
                            const float dt = __ldcg(p.part_ml + (pbase + t) * 2 + 1);
                            if (dt > 0.f) gm = fmaxf(gm, mt);
                        }
#pragma unroll
                        for (int o = 16; o > 0; o >>= 1) gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, o));
                        float gd = 0.f;
                        for (int t = lane; t < S; t += 32) {
                            const float mt = __ldcg(p.part_ml + (pbase + t) * 2);
                            const float dt = __ldcg(p.part_ml + (pbase + t) * 2 + 1);
                            const float c = (dt > 0.f) ? expf(mt - gm) : 0.f;
                            gd += dt * c;
                            smw[hh][t] = c;
                        }
                        gd = warp_sum(gd);
                        __syncwarp();
                        float go[4] = {0.f, 0.f, 0.f, 0.f};
                        for (int t = 0; t < S; t++) {
                            const float4 ov =
                                __ldcg(reinterpret_cast<const float4 *>(p.part_o + (pbase + t) * kHeadDim + d4));
                            const float c = smw[hh][t];
                            go[0] += ov.x * c;
                            go[1] += ov.y * c;
                            go[2] += ov.z * c;
                            go[3] += ov.w * c;
                        }
                        const float inv = (gd > 0.f) ? 1.0f / gd : 0.f;
                        const int idx = h * kHeadDim + d4;
                        xfrag_put2(p.xf_att, m, idx, go[0] * inv, go[1] * inv);
                        xfrag_put2(p.xf_att, m, idx + 2, go[2] * inv, go[3] * inv);
                    }
                    cons_sync();
                    if (tid == 0) red_add_release(done_ctr(p, layer, 5), 1u);
                }
                if (!ok) break;
                cons_sync();   // the staging area becomes the activation area
            }

            // ---------------- a GEMV phase ----------------
            const PhaseShape s = phase_shape(p, layer, g);
            if (cta >= s.items) continue;
            // the activations this phase multiplies, and the counter to wait for
            const uint32_t *xf;
            const unsigned *dep = nullptr;
            unsigned dep_n = 0;
            switch (g) {
                case G_QKV:
                    xf = p.xf_attn;
                    if (layer > 0) { dep = done_ctr(p, layer - 1, G_W2); dep_n = kDecDim / 64; }
                    break;
                case G_WO: xf = p.xf_att; dep = done_ctr(p, layer, 5); dep_n = (unsigned)(M * kDecKvHeads); break;
                case G_W13: xf = p.xf_ffn; dep = done_ctr(p, layer, G_WO); dep_n = kDecDim / 64; break;
                case G_W2: xf = p.xf_h; dep = done_ctr(p, layer, G_W13); dep_n = (2 * kDecHidden) / 64; break;
                default: xf = p.xf_attn; dep = done_ctr(p, p.n_layers - 1, G_W2); dep_n = kDecDim / 64; break;
            }
            if (dep) wait_done(dep, dep_n);
            else cons_sync();   // (the previous phase's activation area is consumed)
            if (!ok) break;

            // ---- this CTA's K slices of the activations, into u.act in 4 KB chunks ----
            // (cp.async on the load path, not the bulk-copy engine, whose queue
            // holds the weight stream: chunk c completes on actb[c] once all
            // 256 threads' copies up to it have landed)
            const int r8 = (s.per + kPStageKB - 1) / kPStageKB * kPStageKB;
            if (tid == 0) {
                int nslot = 0;
                for (int k = 0; k < 16; k++) sh.act_base[k] = -1;
                for (int i = cta; i < s.items; i += G) {
                    const int ks = i % s.KS;
                    if (sh.act_base[ks] < 0 && nslot < 16) {
                        sh.act_base[ks] = nslot * r8;
                        sh.slot_ks[nslot++] = ks;
                    }
                }
                sh.nslot = nslot;
                if (nslot * r8 > kPActKB) fail();   // the host checks the slicing fits
            }
            cons_sync();
            {
                const int nslot = (*(volatile int *)&sh.abort) ? 0 : sh.nslot;
                for (int c = 0; c < kPActChunks; c++) {
                    const int q = (c * kPStageKB) / r8, local = c * kPStageKB - q * r8;
                    if (q < nslot) {
                        const int ks = sh.slot_ks[q];
                        const int nkb = max(0, min(s.per, s.KB - ks * s.per));
                        const int n = max(0, min(kPStageKB, nkb - local));
                        if (tid < n * 32) {   // one 16-byte piece per thread
                            const int kbl = tid >> 5, off = (tid & 31) * 16;
                            pcp16(&sh.u.act[c * kPStageKB + kbl][off],
                                  reinterpret_cast<const char *>(xf) + (size_t)(ks * s.per + local + kbl) * 512 + off);
                        }
                    }
                    pcp_arrive_noinc(&sh.actb[c]);
                }
            }
            if (*(volatile int *)&sh.abort) ok = false;
            if (!ok) break;
            const uint32_t apar = gen & 1u;
            gen++;

            for (int i = cta; i < s.items && ok; i += G) {
                const Item itm = item_of(s, i);
                const int abase = sh.act_base[itm.ks];
                float acc[4][4];
#pragma unroll
                for (int t = 0; t < 4; t++)
#pragma unroll
                    for (int j = 0; j < 4; j++) acc[t][j] = 0.f;
                for (int st = 0; st < itm.nst; st++, it++) {
                    const int slot = it % kPStages;
                    const bool got = __all_sync(0xffffffffu,
                                                pbar_wait(&sh.actb[(abase + st * kPStageKB) / kPStageKB], apar,
                                                          deadline) &&
                                                    pbar_wait(&sh.full[slot], (it / kPStages) & 1u, deadline));
                    if (!got) {
                        if (lane == 0) fail();
                        ok = false;
                    } else if (st * kPStageKB + warp < itm.nkb) {
                        const uint4 b = *reinterpret_cast<const uint4 *>(
                            &sh.u.act[abase + st * kPStageKB + warp][lane * 16]);
                        const unsigned char *base = sh.ring[slot] + warp * kPKbBytes;
#pragma unroll
                        for (int t = 0; t < 4; t++) {
                            const uint4 a = *reinterpret_cast<const uint4 *>(base + t * 512 + lane * 16);
                            pmma(acc[t], a, b.x, b.y);
                            pmma(acc[t], a, b.z, b.w);
                        }
                    }
                    __syncwarp();
                    if (lane == 0) pbar_arrive(&sh.empty[slot]);
                }
                // ---- sum the 8 warps into part[64][8]: (w, w + 4) pairs, then the 4 pairs ----
                if (warp >= 4)
#pragma unroll
                    for (int t = 0; t < 4; t++)
#pragma unroll
                        for (int j = 0; j < 4; j++) sh.red[warp - 4][(t * 32 + lane) * 4 + j] = acc[t][j];
                cons_sync();
                if (*(volatile int *)&sh.abort) ok = false;
                if (!ok) break;
                if (warp < 4)
#pragma unroll
                    for (int t = 0; t < 4; t++)
#pragma unroll
                        for (int j = 0; j < 4; j++) {
                            float &r = sh.red[warp][(t * 32 + lane) * 4 + j];
                            r = acc[t][j] + r;
                        }
                cons_sync();
                for (int e = tid; e < 4 * 32 * 4; e += kPConsumers) {
                    const float v = (sh.red[0][e] + sh.red[1][e]) + (sh.red[2][e] + sh.red[3][e]);
                    const int t = e >> 7, ln = (e >> 2) & 31, j = e & 3;
                    sh.part[t * 16 + (ln >> 2) + ((j >> 1) << 3)][2 * (ln & 3) + (j & 1)] = v;
                }
                cons_sync();
                // ---- K slices: the last of a row block sums them in slice order ----
                if (s.KS > 1) {
                    float *gp = p.gpart + (size_t)i * 512;
                    for (int e = tid; e < 512; e += kPConsumers) gp[e] = (&sh.part[0][0])[e];
                    cons_sync();
                    if (tid == 0) sh.flag = atom_add_acq_rel(ticket_ctr(p, layer, g, itm.rb), 1u) + 1u == (unsigned)s.KS;
                    cons_sync();
                    if (!sh.flag) continue;
                    for (int e = tid; e < 512; e += kPConsumers) {
                        const float *b0 = p.gpart + (size_t)itm.rb * s.KS * 512 + e;
                        float v = __ldcg(b0);
                        for (int k = 1; k < s.KS; k++) v += __ldcg(b0 + (size_t)k * 512);
                        (&sh.part[0][0])[e] = v;
                    }
                }
                // ---- 1 / rms of the RMSNorm consumers ----
                if (tid < 8) {
                    float inv = 1.0f;
                    const float *ss = (g == G_QKV || g == G_LM) ? p.ss_attn : (g == G_W13 ? p.ss_ffn : nullptr);
                    if (ss != nullptr && tid < M) {
                        float a = 0.f;
                        for (int j = 0; j < ss_parts; j++) a += __ldcg(ss + tid * ss_parts + j);
                        inv = 1.0f / sqrtf(a / (float)kDecDim + kNormEps);
                    }
                    sh.s_inv[tid] = inv;
                }
                cons_sync();

                // ---- epilogue: thread -> stream m = tid & 7, rows (2pp, 2pp + 1) ----
                const int m = tid & 7, pp = tid >> 3;
                const int r0 = itm.rb * 64 + 2 * pp;
                const bool active = (m < M) && (r0 < s.N);
                const bool has1 = r0 + 1 < s.N;
                float v0 = sh.part[2 * pp][m] * sh.s_inv[m];
                float v1 = sh.part[2 * pp + 1][m] * sh.s_inv[m];
                if (g == G_QKV) {
                    // q / k with RoPE (vox_apply_rope, voxtral_kernels.c:502-526), k / v to the ring
                    if (active) {
                        const StreamSlot sl = p.slots[m];
                        const size_t ring_row = ((size_t)layer * sl.cap + sl.slot) * kKvDim;
                        if (r0 < kQDim + kKvDim) {
                            const int d = (r0 & (kHeadDim - 1)) >> 1;
                            const float cs = p.rope[m * kHeadDim + 2 * d];
                            const float sn = p.rope[m * kHeadDim + 2 * d + 1];
                            const float oa = __fsub_rn(__fmul_rn(v0, cs), __fmul_rn(v1, sn));
                            const float ob = __fadd_rn(__fmul_rn(v0, sn), __fmul_rn(v1, cs));
                            float *dst = (r0 < kQDim) ? p.q + (size_t)m * kQDim + r0
                                                      : sl.k_ring + ring_row + (r0 - kQDim);
                            dst[0] = oa;
                            dst[1] = ob;
                        } else {
                            float *dst = sl.v_ring + ring_row + (r0 - kQDim - kKvDim);
                            dst[0] = v0;
                            dst[1] = v1;
                        }
                    }
                } else if (g == G_W13) {
                    // rows (2i, 2i + 1) = (gate_i, up_i): h_i = silu(g) * u as w2's fragments
                    if (active) {
                        const float sg = v0 / (1.0f + expf(-v0));
                        xfrag_put1(p.xf_h, m, r0 >> 1, sg * v1);
                    }
                } else if (g == G_WO || g == G_W2) {
                    // x += acc; the next norm's fragments (x * g) and per-row-block sums of x^2
                    const float *gn = (g == G_WO) ? p.layers[layer].g_ffn
                                                  : (layer + 1 < p.n_layers ? p.layers[layer + 1].g_attn
                                                                             : p.final_norm);
                    uint32_t *xfo = (g == G_WO) ? p.xf_ffn : p.xf_attn;
                    float *sso = (g == G_WO) ? p.ss_ffn : p.ss_attn;
                    float ssq = 0.f;
                    if (active) {
                        float *dst = p.x + (size_t)m * kDecDim + r0;
                        v0 += __ldcg(dst);            // written by other CTAs: read through L2
                        if (has1) v1 += __ldcg(dst + 1);
                        dst[0] = v0;
                        if (has1) dst[1] = v1;
                        if (!has1) v1 = 0.f;
                        ssq = v0 * v0 + v1 * v1;
                        const float g0 = gn[r0], g1 = has1 ? gn[r0 + 1] : 1.0f;
                        xfrag_put2(xfo, m, r0, v0 * g0, v1 * g1);
                    }
                    ssq += __shfl_xor_sync(0xffffffffu, ssq, 8);
                    ssq += __shfl_xor_sync(0xffffffffu, ssq, 16);
                    if (lane < 8) sh.red_v[warp][lane] = ssq;
                    cons_sync();
                    if (tid < M) {
                        float t = 0.f;
                        for (int w = 0; w < kPConsWarps; w++) t += sh.red_v[w][tid];
                        sso[tid * ss_parts + itm.rb] = t;
                    }
                } else {   // G_LM: logits and the first maximum (voxtral_decoder.c:504-515)
                    float bv = -INFINITY;
                    int bi = 0x7fffffff;
                    if (active) {
                        float *dst = p.logits + (size_t)m * p.vocab + r0;
                        dst[0] = v0;
                        if (has1) dst[1] = v1;
                        bv = v0;
                        bi = r0;
                        if (has1 && v1 > bv) { bv = v1; bi = r0 + 1; }
                    }
#pragma unroll
                    for (int o = 8; o <= 16; o <<= 1) {
                        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                        if (p_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
                    }
                    if (lane < 8) {
                        sh.red_v[warp][lane] = bv;
                        sh.red_i[warp][lane] = bi;
                    }
                    cons_sync();
                    if (tid < M) {
                        float b = -INFINITY;
                        int ib = 0x7fffffff;
                        for (int w = 0; w < kPConsWarps; w++)
                            if (p_better(sh.red_v[w][tid], sh.red_i[w][tid], b, ib)) {
                                b = sh.red_v[w][tid];
                                ib = sh.red_i[w][tid];
                            }
                        p.amax[(size_t)itm.rb * M + tid] = {b, ib};
                    }
                }
                cons_sync();
                if (g == G_LM) {
                    if (tid == 0) sh.flag = atom_add_acq_rel(done_ctr(p, p.n_layers, 0), 1u) + 1u == (unsigned)s.RB;
                    cons_sync();
                    if (sh.flag) {   // the last row block: the argmax over all partials
                        if (warp < M) {
                            float b = -INFINITY;
                            int ib = 0x7fffffff;
                            const int2 *ap = reinterpret_cast<const int2 *>(p.amax);
                            for (int j0 = lane; j0 < s.RB; j0 += 32 * 8) {
                                int2 tv[8];
#pragma unroll
                                for (int u = 0; u < 8; u++) {
                                    const int j = j0 + 32 * u;
                                    tv[u] = j < s.RB ? __ldcg(ap + (size_t)j * M + warp)
                                                     : make_int2(__float_as_int(-INFINITY), 0x7fffffff);
                                }
#pragma unroll
                                for (int u = 0; u < 8; u++) {
                                    const float v = __int_as_float(tv[u].x);
                                    if (p_better(v, tv[u].y, b, ib)) { b = v; ib = tv[u].y; }
                                }
                            }
#pragma unroll
                            for (int o = 16; o > 0; o >>= 1) {
                                const float ov = __shfl_xor_sync(0xffffffffu, b, o);
                                const int oi = __shfl_xor_sync(0xffffffffu, ib, o);
                                if (p_better(ov, oi, b, ib)) { b = ov; ib = oi; }
                            }
                            if (lane == 0) p.tokens[warp] = ib;
                        }
                    }
                } else if (tid == 0) {
                    red_add_release(done_ctr(p, layer, g), 1u);
                }
            }
        }
    }
    if (!ok) {
        // the producer stops at the abort flag; its copies in flight land first
        const uint64_t grace = ptimer() + 10000000ull;
        while (ptimer() < grace) {
        }
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

size_t persist_sync_words() { return (size_t)kPDoneWords + kPTicketWords + kPAttWords; }

size_t persist_gpart_floats(const PersistParams &p) {
    // the largest phase's items x 64 rows x 8 streams
    const int rbs[5] = {kQkvRows / 64, kDecDim / 64, 2 * kDecHidden / 64, kDecDim / 64, (p.vocab + 63) / 64};
    size_t mx = 0;
    for (int g = 0; g < 5; g++)
        if (p.ks[g] > 1) mx = std::max(mx, (size_t)rbs[g] * p.ks[g]);
    return mx * 512;
}

bool persist_slicing_fits(const int *ks, int vocab, int grid) {
    const int KB[5] = {kDecDim / 16, kQDim / 16, kDecDim / 16, kDecHidden / 16, kDecDim / 16};
    const int RB[5] = {kQkvRows / 64, kDecDim / 64, 2 * kDecHidden / 64, kDecDim / 64, (vocab + 63) / 64};
    for (int g = 0; g < 5; g++) {
        const int KS = ks[g], per = (KB[g] + KS - 1) / KS, r8 = (per + 7) / 8 * 8, items = RB[g] * KS;
        for (int c = 0; c < grid && c < items; c++) {
            unsigned seen = 0;
            int n = 0;
            for (int i = c; i < items; i += grid)
                if (!(seen & (1u << (i % KS)))) {
                    seen |= 1u << (i % KS);
                    n++;
                }
            if (n * r8 > kPActKB) return false;
        }
    }
    return true;
}

cudaError_t launch_step_persist(const PersistParams &p, cudaStream_t st, int *grid_out) {
    // per device: the shared-memory opt-in and the SM count (the grid)
    constexpr int kMaxDev = 64;
    static int sms[kMaxDev] = {0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDev) return cudaErrorInvalidDevice;
    if (sms[dev] == 0) {
        int n = 0;
        e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(step_persist_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)sizeof(PShared));
        if (e != cudaSuccess) return e;
        int per_sm = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, step_persist_kernel, kPThreads,
                                                          sizeof(PShared));
        if (e != cudaSuccess) return e;
        if (per_sm < 1) return cudaErrorInvalidConfiguration;
        sms[dev] = n;
    }
    if (p.M < 1 || p.M > kMaxBatch || p.n_layers < 1 || p.n_layers > kDecLayersMax) return cudaErrorInvalidValue;
    if (p.ks[G_LM] > 1 && p.vocab > kVocab) return cudaErrorInvalidValue;   // the LM head's tickets
    if (p.l2_ahead < 0 || !persist_slicing_fits(p.ks, p.vocab, sms[dev])) return cudaErrorInvalidValue;
    for (int g = 0; g < 5; g++)
        if (p.ks[g] < 1 || p.ks[g] > 16) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sms[dev]);
    cfg.blockDim = dim3(kPThreads);
    cfg.dynamicSmemBytes = sizeof(PShared);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (grid_out) *grid_out = sms[dev];
    return cudaLaunchKernelEx(&cfg, step_persist_kernel, p);
}

}  // namespace vc
