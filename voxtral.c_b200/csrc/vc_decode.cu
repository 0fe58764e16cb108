// vc_decode.cu - decode-step kernels besides the GEMV (vc_gemv.cu): split-K
// GQA decode attention over the KV ring, the --alt selection, stand-alone
// RoPE and the seeded bf16 fill used by benchmarks.
#include "vc_common.cuh"
#include "vc_internal.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <atomic>

namespace vc {

__device__ __forceinline__ bool arg_better(float v, int i, float bv, int bi) {
    return v > bv || (v == bv && i < bi);
}

// ---------------------------------------------------------------------------
// Split-K GQA decode attention over the KV ring (vox_causal_attention with
// seq_q = 1, voxtral_kernels.c:412-482, as called at voxtral_decoder.c:481-483).
//
// grid (G, 8 KV heads, M streams), 128 threads.  A CTA takes one KV head and
// splits of up to 64 consecutive keys (s = blockIdx.x, + G, ...); its 4 query
// heads share every K/V row.  The split's K and V rows (512 bytes each per
// key) are staged in shared memory with cp.async, so registers do not bound
// the bytes in flight.  Keys older than the step's own position are not
// written by the preceding kernel (the q|k|v GEMV writes only this step's
// slot), so their copies are issued before griddepcontrol.wait and overlap
// that kernel's tail; the newest key and q are read after it.
// (Within one launch, streams that share a ring are consecutive rows of one
// sequence, the decoder prefill: keys from the lowest such position on,
// which the host passes as the slot's `fresh`, are all fresh.)
// Instead of the reference's per-key online softmax (a serial chain), each
// split runs three parallel passes: scores (warp = query head, lane = key,
// rotated float4 reads), the softmax of the split (per warp), then P.V
// (thread = dimension).  Splits are merged with the usual max rescaling by the
// last CTA of each (stream, KV head) to finish (atomic ticket; no spinning).
// ---------------------------------------------------------------------------

constexpr int kKeysPerSplit = 64;

struct AttnShared {
    float k[kKeysPerSplit][kHeadDim];   // 32 KB; the merge reuses it for its weights
    float v[kKeysPerSplit][kHeadDim];   // 32 KB
    float q[4][kHeadDim];
    float p[4][kKeysPerSplit];          // exp(score - split max)
    float ml[4][2];                     // per head: (split max, sum of exp)
    int last;
};
static_assert(sizeof(float) * kKeysPerSplit * kHeadDim >= sizeof(float) * 4 * kAttnSplits, "merge weights fit");

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// The merged output of 4 dimensions (idx .. idx + 3 of row m's 4096) in every
// form the launch asks for: fp32 rows, the wo GEMV's B fragments, the split
// bf16 hi / lo rows of a tensor-core consumer.
__device__ __forceinline__ void attn_store_out(const AttnParams &p, int m, int idx, float o0, float o1, float o2,
                                               float o3) {
    if (p.out != nullptr)
        *reinterpret_cast<float4 *>(p.out + (size_t)m * kQDim + idx) = make_float4(o0, o1, o2, o3);
    if (p.xfrag_out != nullptr) {
        xfrag_put2(p.xfrag_out, m, idx, o0, o1);
        xfrag_put2(p.xfrag_out, m, idx + 2, o2, o3);
    }
    if (p.out_hilo != nullptr) {
        uint32_t h0, l0, h1, l1, h2, l2, h3, l3;
        split_bf16(o0, h0, l0);
        split_bf16(o1, h1, l1);
        split_bf16(o2, h2, l2);
        split_bf16(o3, h3, l3);
        const size_t e = (size_t)hilo_row(m) * kQDim + idx;
        *reinterpret_cast<uint2 *>(p.out_hilo + e) = make_uint2(h0 | (h1 << 16), h2 | (h3 << 16));
        *reinterpret_cast<uint2 *>(p.out_hilo + e + (size_t)64 * kQDim) = make_uint2(l0 | (l1 << 16), l2 | (l3 << 16));
    }
}

// cp.async of the K and V rows of keys [j0, j1) of a split (key j of the
// split at ring slot (first + kb + j) % cap), 16 bytes per copy.
__device__ __forceinline__ void attn_stage_keys(AttnShared &sh, const float *kbase, const float *vbase, int first,
                                                int kb, int cap, int j0, int j1, int tid) {
    const int n = (j1 - j0) * (kHeadDim / 4);   // 16-byte pieces per matrix
    for (int c = tid; c < n; c += 128) {
        const int j = j0 + c / (kHeadDim / 4), piece = c % (kHeadDim / 4);
        const size_t row = (size_t)((first + kb + j) % cap) * kKvDim + 4 * piece;
        cp_async16(&sh.k[j][4 * piece], kbase + row);
        cp_async16(&sh.v[j][4 * piece], vbase + row);
    }
}

__global__ void __launch_bounds__(128)
attn_decode_kernel(const AttnParams p) {
    extern __shared__ __align__(16) unsigned char attn_smem[];
    AttnShared &sh = *reinterpret_cast<AttnShared *>(attn_smem);
    const int kvh = blockIdx.y, m = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) l2_prefetch_share(p.pf, p.pf_bytes);   // the wo GEMV's weights (this kernel leaves HBM idle)

    // The slots were written before this step's first kernel; ring rows of
    // positions below slt.pos were written by earlier steps.
    const StreamSlot slt = p.slots[m];
    const int n_keys = slt.n_keys;
    const int S = max(1, min(p.S, (n_keys + kKeysPerSplit - 1) / kKeysPerSplit));
    if ((int)blockIdx.x >= S) return;   // CTA-uniform, before any barrier
    const int chunk = (n_keys + S - 1) / S;               // <= kKeysPerSplit
    const int first = slt.pos - n_keys + 1;              // logical position of key 0
    const int cap = slt.cap;
    const float scale = 1.0f / sqrtf((float)kHeadDim);
    const size_t layer_off = (size_t)p.layer * cap * kKvDim + kvh * kHeadDim;
    const float *kbase = slt.k_ring + layer_off;
    const float *vbase = slt.v_ring + layer_off;

    // keys [0, n_old) predate this launch
    const int n_old = max(0, min(slt.fresh, slt.pos) - first);
    {   // the first split's old keys, before the wait
        const int kb = blockIdx.x * chunk;
        const int nk = max(0, min(kb + chunk, n_keys) - kb);
        attn_stage_keys(sh, kbase, vbase, first, kb, cap, 0, max(0, min(nk, n_old - kb)), tid);
        cp_async_commit();
    }
    grid_dep_wait();
    grid_dep_launch();
    {   // queries (warp = head, lane = 4 dims)
        const float4 v = *reinterpret_cast<const float4 *>(p.q + (size_t)m * kQDim +
                                                           (kvh * 4 + warp) * kHeadDim + 4 * lane);
        *reinterpret_cast<float4 *>(&sh.q[warp][4 * lane]) = v;
    }

    int n_done = 0;
    for (int s = blockIdx.x; s < S; s += gridDim.x) {
        const int kb = s * chunk;
        const int nk = max(0, min(kb + chunk, n_keys) - kb);
        if (s == (int)blockIdx.x) {
            // the fresh keys of the first split (written by the preceding kernel)
            attn_stage_keys(sh, kbase, vbase, first, kb, cap, max(0, min(nk, n_old - kb)), nk, tid);
        } else {
            __syncthreads();   // the previous split's K / V / p consumed
            attn_stage_keys(sh, kbase, vbase, first, kb, cap, 0, nk, tid);
        }
        cp_async_commit();
        cp_async_wait_all();
        __syncthreads();

        // ---- scores and softmax: warp = query head, lane = keys lane, lane + 32 ----
        {
            const int h = warp;
            const float4 *q4 = reinterpret_cast<const float4 *>(sh.q[h]);
            float sc[2];
#pragma unroll
            for (int u = 0; u < 2; u++) {
                const int j = lane + 32 * u;
                const float4 *k4 = reinterpret_cast<const float4 *>(sh.k[j]);
                float a = 0.f;
#pragma unroll 8
                for (int i = 0; i < kHeadDim / 4; i++) {
                    const int f = (i + lane) & (kHeadDim / 4 - 1);   // rotation: no bank conflicts
                    const float4 kk = k4[f], qq = q4[f];
                    a = fmaf(qq.x, kk.x, a);
                    a = fmaf(qq.y, kk.y, a);
                    a = fmaf(qq.z, kk.z, a);
                    a = fmaf(qq.w, kk.w, a);
                }
                sc[u] = (j < nk) ? a * scale : -INFINITY;
            }
            float mx = fmaxf(sc[0], sc[1]);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            const float pa = (lane < nk) ? expf(sc[0] - mx) : 0.f;
            const float pb = (lane + 32 < nk) ? expf(sc[1] - mx) : 0.f;
            sh.p[h][lane] = pa;
            sh.p[h][lane + 32] = pb;
            const float sum = warp_sum(pa + pb);
            if (lane == 0) {
                sh.ml[h][0] = mx;
                sh.ml[h][1] = sum;
            }
        }
        __syncthreads();

        // ---- P.V: thread = dimension, 4 heads ----
        {
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            for (int j = 0; j < nk; j++) {
                const float vj = sh.v[j][tid];
#pragma unroll
                for (int h = 0; h < 4; h++) acc[h] = fmaf(sh.p[h][j], vj, acc[h]);
            }
#pragma unroll
            for (int h = 0; h < 4; h++) {
                const size_t pidx = ((size_t)m * kDecHeads + kvh * 4 + h) * p.S + s;
                p.part_o[pidx * kHeadDim + tid] = acc[h];
            }
            if (tid < 4) {
                const size_t pidx = ((size_t)m * kDecHeads + kvh * 4 + tid) * p.S + s;
                p.part_ml[pidx * 2] = sh.ml[tid][0];
                p.part_ml[pidx * 2 + 1] = sh.ml[tid][1];
            }
        }
        n_done++;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0)
        sh.last = (atomicAdd(&p.counters[m * kDecKvHeads + kvh], (unsigned)n_done) + n_done == (unsigned)S);
    __syncthreads();
    if (!sh.last) return;
    __threadfence();

    // ---- merge the S splits (last CTA of this stream / KV head): warp = head ----
    {
        float(*smw)[kAttnSplits] = reinterpret_cast<float(*)[kAttnSplits]>(&sh.k[0][0]);
        const int hh = warp, d4 = 4 * lane;
        const int h = kvh * 4 + hh;
        const size_t pbase = ((size_t)m * kDecHeads + h) * p.S;
        float mloc[kAttnSplits / 32], dloc[kAttnSplits / 32];
        float gm = -INFINITY;
#pragma unroll
        for (int i = 0; i < kAttnSplits / 32; i++) {
            const int t = lane + 32 * i;
            mloc[i] = (t < S) ? __ldcg(p.part_ml + (pbase + t) * 2) : -INFINITY;
            dloc[i] = (t < S) ? __ldcg(p.part_ml + (pbase + t) * 2 + 1) : 0.f;
        }
#pragma unroll
        for (int i = 0; i < kAttnSplits / 32; i++)
            if (dloc[i] > 0.f) gm = fmaxf(gm, mloc[i]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, o));
        float gd = 0.f;
#pragma unroll
        for (int i = 0; i < kAttnSplits / 32; i++) {
            const int t = lane + 32 * i;
            const float c = (dloc[i] > 0.f) ? expf(mloc[i] - gm) : 0.f;
            gd += dloc[i] * c;
            smw[hh][t] = c;
        }
        gd = warp_sum(gd);
        __syncwarp();
        float go[4] = {0.f, 0.f, 0.f, 0.f};
        int t = 0;
        for (; t + 4 <= S; t += 4) {   // 4 independent loads in flight
            float4 ov[4];
#pragma unroll
            for (int u = 0; u < 4; u++)
                ov[u] = __ldcg(reinterpret_cast<const float4 *>(p.part_o + (pbase + t + u) * kHeadDim + d4));
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const float c = smw[hh][t + u];
                go[0] += ov[u].x * c;
                go[1] += ov[u].y * c;
                go[2] += ov[u].z * c;
                go[3] += ov[u].w * c;
            }
        }
        for (; t < S; t++) {
            const float4 ov = __ldcg(reinterpret_cast<const float4 *>(p.part_o + (pbase + t) * kHeadDim + d4));
            const float c = smw[hh][t];
            go[0] += ov.x * c;
            go[1] += ov.y * c;
            go[2] += ov.z * c;
            go[3] += ov.w * c;
        }
        const float inv = (gd > 0.f) ? 1.0f / gd : 0.f;
        attn_store_out(p, m, h * kHeadDim + d4, go[0] * inv, go[1] * inv, go[2] * inv, go[3] * inv);
        if (tid == 0) p.counters[m * kDecKvHeads + kvh] = 0u;
    }
}

// ---------------------------------------------------------------------------
// v4: the same attention with 32-key tiles pipelined inside each CTA.
//
// A CTA takes a contiguous range of 32-key tiles of one (row, KV head) and
// runs an online softmax over them: while tile t is computed, tile t + 1 is
// in flight (cp.async double buffer), so one CTA keeps loading as it
// computes and a row's keys need fewer CTAs (fewer partials to merge).  K
// rows are staged chunk-swizzled (16-byte chunk c of key j at c ^ j), so
// lane j reading its key's chunk c is conflict-free while the query chunk is
// one broadcast read per warp; each K element is read once per query head.
// P.V: thread = dimension, V rows coalesced, probabilities broadcast.
// ---------------------------------------------------------------------------

constexpr int kTileKeys = 32;

template <int NS>
struct Attn4SharedT {
    float k[NS][kTileKeys][kHeadDim];   // NS x 16 KB, chunk-swizzled
    float v[NS][kTileKeys][kHeadDim];   // NS x 16 KB
    float q[4][kHeadDim];
    float p[4][kTileKeys];             // this tile's exp(s - m)
    float alpha[4];                    // this tile's rescale of the running sums
    int last;
};
using Attn4Shared = Attn4SharedT<2>;
static_assert(sizeof(float) * 2 * kTileKeys * kHeadDim >= sizeof(float) * 4 * kAttnSplits, "merge weights fit");

// cp.async of keys [j0, j1) of the tile starting at key kb (logical index
// from `first`) into buffer b: K swizzled, V as is.
template <int NS>
__device__ __forceinline__ void attn4_stage(Attn4SharedT<NS> &sh, int b, const float *kbase, const float *vbase,
                                            int first, int kb, int cap, int j0, int j1, int tid) {
    const int n = (j1 - j0) * (kHeadDim / 4);
    for (int c = tid; c < n; c += 128) {
        const int j = j0 + c / (kHeadDim / 4), ch = c % (kHeadDim / 4);
        const size_t row = (size_t)((first + kb + j) % cap) * kKvDim + 4 * ch;
        cp_async16(&sh.k[b][j][4 * (ch ^ j)], kbase + row);
        cp_async16(&sh.v[b][j][4 * ch], vbase + row);
    }
}

// NS tile buffers: NS - 1 tiles in flight while one is computed.  NS = 2 with
// three CTAs per SM (v4), or NS = 6 with one CTA per SM (the deep variant
// for long contexts: 160 KB of keys in flight per SM).
template <int NS>
__global__ void __launch_bounds__(128)
attn_decode_v4_kernel(const AttnParams p) {
    extern __shared__ __align__(16) unsigned char attn_smem[];
    Attn4SharedT<NS> &sh = *reinterpret_cast<Attn4SharedT<NS> *>(attn_smem);
    const int kvh = blockIdx.y, m = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) l2_prefetch_share(p.pf, p.pf_bytes);   // the wo GEMV's weights (this kernel leaves HBM idle)

    const StreamSlot slt = p.slots[m];
    const int n_keys = slt.n_keys;
    const int tiles = (n_keys + kTileKeys - 1) / kTileKeys;
    const int P = min((int)gridDim.x, tiles);           // CTAs with keys = partials
    if ((int)blockIdx.x >= P) return;                   // CTA-uniform, before any barrier
    const int t0 = (int)((long long)blockIdx.x * tiles / P), t1 = (int)((long long)(blockIdx.x + 1) * tiles / P);
    const int first = slt.pos - n_keys + 1;
    const int cap = slt.cap;
    const float scale = 1.0f / sqrtf((float)kHeadDim);
    const size_t layer_off = (size_t)p.layer * cap * kKvDim + kvh * kHeadDim;
    const float *kbase = slt.k_ring + layer_off;
    const float *vbase = slt.v_ring + layer_off;
    const int n_old = max(0, min(slt.fresh, slt.pos) - first);   // keys [0, n_old) predate this launch
    auto tile_keys = [&](int t) { return min(kTileKeys, n_keys - t * kTileKeys); };

    // the old keys of the first NS - 1 tiles, before the wait (they overlap
    // the producer kernel's tail): one commit group
    for (int t = t0; t < min(t1, t0 + NS - 1); t++) {
        const int kb = t * kTileKeys;
        attn4_stage(sh, t % NS, kbase, vbase, first, kb, cap, 0, max(0, min(tile_keys(t), n_old - kb)), tid);
    }
    cp_async_commit();
    grid_dep_wait();
    grid_dep_launch();
    {   // queries (warp = head, lane = 4 dims)
        const float4 v = *reinterpret_cast<const float4 *>(p.q + (size_t)m * kQDim +
                                                           (kvh * 4 + warp) * kHeadDim + 4 * lane);
        *reinterpret_cast<float4 *>(&sh.q[warp][4 * lane]) = v;
    }
    for (int t = t0; t < t0 + NS - 1; t++) {   // their fresh keys: one group per tile (empty past t1)
        if (t < t1) {
            const int kb = t * kTileKeys;
            attn4_stage(sh, t % NS, kbase, vbase, first, kb, cap, max(0, min(tile_keys(t), n_old - kb)),
                        tile_keys(t), tid);
        }
        cp_async_commit();
    }

    float m_run = -INFINITY, l_run = 0.f;    // warp h: head h's running max / sum
    float o[4] = {0.f, 0.f, 0.f, 0.f};       // thread = dimension, 4 heads
    for (int t = t0; t < t1; t++) {
        const int b = t % NS, nk = tile_keys(t);
        // tile t + NS - 1 into the buffer freed by tile t - 1; then tile t has landed
        if (t + NS - 1 < t1)
            attn4_stage(sh, (t + NS - 1) % NS, kbase, vbase, first, (t + NS - 1) * kTileKeys, cap, 0,
                        tile_keys(t + NS - 1), tid);
        cp_async_commit();
        cp_async_wait_group<NS - 1>();
        __syncthreads();
        {   // scores (warp = head, lane = key): swizzled K chunks, broadcast q
            const int h = warp;
            const float4 *q4 = reinterpret_cast<const float4 *>(sh.q[h]);
            const float *kr = sh.k[b][lane];
            float a0 = 0.f, a1 = 0.f;
#pragma unroll 8
            for (int c = 0; c < kHeadDim / 4; c += 2) {
                const float4 k0 = *reinterpret_cast<const float4 *>(kr + 4 * (c ^ lane));
                const float4 k1 = *reinterpret_cast<const float4 *>(kr + 4 * ((c + 1) ^ lane));
                const float4 x0 = q4[c], x1 = q4[c + 1];
                a0 = fmaf(x0.x, k0.x, a0);
                a0 = fmaf(x0.y, k0.y, a0);
                a0 = fmaf(x0.z, k0.z, a0);
                a0 = fmaf(x0.w, k0.w, a0);
                a1 = fmaf(x1.x, k1.x, a1);
                a1 = fmaf(x1.y, k1.y, a1);
                a1 = fmaf(x1.z, k1.z, a1);
                a1 = fmaf(x1.w, k1.w, a1);
            }
            const bool valid = lane < nk;
            const float sc = valid ? (a0 + a1) * scale : -INFINITY;
            float tm = sc;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, off));
            const float nm = fmaxf(m_run, tm);                       // finite: the tile has a valid key
            const float alpha = (m_run == -INFINITY) ? 0.f : expf(m_run - nm);
            const float pj = valid ? expf(sc - nm) : 0.f;
            l_run = l_run * alpha + warp_sum(pj);
            m_run = nm;
            sh.p[h][lane] = pj;
            if (lane == 0) sh.alpha[h] = alpha;
        }
        __syncthreads();
        {   // P.V: thread = dimension
#pragma unroll
            for (int h = 0; h < 4; h++) o[h] *= sh.alpha[h];
            for (int j = 0; j < nk; j++) {
                const float vj = sh.v[b][j][tid];
#pragma unroll
                for (int h = 0; h < 4; h++) o[h] = fmaf(sh.p[h][j], vj, o[h]);
            }
        }
        __syncthreads();   // buffer b consumed
    }
    cp_async_wait_group<0>();   // (only empty groups remain)
    // this CTA's partial: unnormalised o, running (max, sum) per head
    const int s = blockIdx.x;
#pragma unroll
    for (int h = 0; h < 4; h++) {
        const size_t pidx = ((size_t)m * kDecHeads + kvh * 4 + h) * p.S + s;
        p.part_o[pidx * kHeadDim + tid] = o[h];
    }
    if (lane == 0) {
        const size_t pidx = ((size_t)m * kDecHeads + kvh * 4 + warp) * p.S + s;
        p.part_ml[pidx * 2] = m_run;
        p.part_ml[pidx * 2 + 1] = l_run;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) sh.last = (atomicAdd(&p.counters[m * kDecKvHeads + kvh], 1u) + 1u == (unsigned)P);
    __syncthreads();
    if (!sh.last) return;
    __threadfence();

    // ---- merge the P partials (last CTA of this row / KV head): warp = head ----
    {
        float(*smw)[kAttnSplits] = reinterpret_cast<float(*)[kAttnSplits]>(&sh.k[0][0][0]);
        const int hh = warp, d4 = 4 * lane;
        const int h = kvh * 4 + hh;
        const size_t pbase = ((size_t)m * kDecHeads + h) * p.S;
        float mloc[kAttnSplits / 32], dloc[kAttnSplits / 32];
        float gm = -INFINITY;
#pragma unroll
        for (int i = 0; i < kAttnSplits / 32; i++) {
            const int t = lane + 32 * i;
            mloc[i] = (t < P) ? __ldcg(p.part_ml + (pbase + t) * 2) : -INFINITY;
            dloc[i] = (t < P) ? __ldcg(p.part_ml + (pbase + t) * 2 + 1) : 0.f;
        }
#pragma unroll
        for (int i = 0; i < kAttnSplits / 32; i++)
            if (dloc[i] > 0.f) gm = fmaxf(gm, mloc[i]);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, off));
        float gd = 0.f;
#pragma unroll
        for (int i = 0; i < kAttnSplits / 32; i++) {
            const int t = lane + 32 * i;
            const float c = (dloc[i] > 0.f) ? expf(mloc[i] - gm) : 0.f;
            gd += dloc[i] * c;
            smw[hh][t] = c;
        }
        gd = warp_sum(gd);
        __syncwarp();
        float go[4] = {0.f, 0.f, 0.f, 0.f};
        int t = 0;
        for (; t + 4 <= P; t += 4) {   // 4 independent loads in flight
            float4 ov[4];
#pragma unroll
            for (int u = 0; u < 4; u++)
                ov[u] = __ldcg(reinterpret_cast<const float4 *>(p.part_o + (pbase + t + u) * kHeadDim + d4));
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const float c = smw[hh][t + u];
                go[0] += ov[u].x * c;
                go[1] += ov[u].y * c;
                go[2] += ov[u].z * c;
                go[3] += ov[u].w * c;
            }
        }
        for (; t < P; t++) {
            const float4 ov = __ldcg(reinterpret_cast<const float4 *>(p.part_o + (pbase + t) * kHeadDim + d4));
            const float c = smw[hh][t];
            go[0] += ov.x * c;
            go[1] += ov.y * c;
            go[2] += ov.z * c;
            go[3] += ov.w * c;
        }
        const float inv = (gd > 0.f) ? 1.0f / gd : 0.f;
        attn_store_out(p, m, h * kHeadDim + d4, go[0] * inv, go[1] * inv, go[2] * inv, go[3] * inv);
        if (tid == 0) p.counters[m * kDecKvHeads + kvh] = 0u;
    }
}

// CTAs per (stream, KV head): each loops over splits blockIdx.x + G*i.
// v4: CTAs per (row, KV head).  A long context (8192 keys = 256 tiles) at
// M = 1 gets 48 CTAs of ~5 pipelined tiles (3 CTAs/SM x 148 SMs over the 8 KV
// heads); several rows share the SMs, 16 CTAs each at M >= 3.
int attn4_ctas_per_head(int M) {
    static int fixed = -1;
    if (fixed < 0) {   // tuning knob: VOX_CUDA_ATTN_CTAS fixes the CTAs per (stream, KV head)
        const char *e = getenv("VOX_CUDA_ATTN_CTAS");
        fixed = (e && atoi(e) >= 1 && atoi(e) <= kAttnSplits) ? atoi(e) : 0;
    }
    if (fixed > 0) return fixed;
    const int g = 48 / (M > 0 ? M : 1);
    return g < 16 ? 16 : g;
}

// The deep variant: two CTAs of 3 tile buffers (96 KB) per SM, the SMs
// shared by the launch's (row, KV head) pairs.
constexpr int kDeepStages = 3;
int attn_deep_ctas_per_head(int M) {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int g = 2 * sms / (kDecKvHeads * (M > 0 ? M : 1));
    return g < 1 ? 1 : g;
}

// Long contexts take the deep variant: 2 tiles in flight per CTA keep
// ~128 KB of keys moving per SM, where v4's 3 CTAs x 1 tile do ~96 KB.  The
// caller passes a hint of the keys it expects (0: unknown, v4).
// VOX_CUDA_ATTN = deep forces it.
bool attn_use_deep(int M, int keys_hint) {
    static int forced = -1;
    if (forced < 0) {
        const char *e = getenv("VOX_CUDA_ATTN");
        forced = (e && strcmp(e, "deep") == 0) ? 1 : (e && strcmp(e, "v4") == 0) ? 0 : -2;
    }
    if (forced >= 0) return forced == 1;
    return M <= 2 && keys_hint >= kAttnDeepKeys;
}

int attn_ctas_per_head(int M) {
    static int fixed = -1;
    if (fixed < 0) {   // tuning knob: VOX_CUDA_ATTN_CTAS fixes the CTAs per (stream, KV head)
        const char *e = getenv("VOX_CUDA_ATTN_CTAS");
        fixed = (e && atoi(e) >= 1 && atoi(e) <= kAttnSplits) ? atoi(e) : 0;
    }
    if (fixed > 0) return fixed;
    const int g = kAttnSplits / (M > 0 ? M : 1);
    return g < 16 ? 16 : g;
}

__global__ void set_slot_kernel(StreamSlot *dst, StreamSlot v) { *dst = v; }

cudaError_t launch_set_slot(StreamSlot *dst, const StreamSlot &v, cudaStream_t st) {
    set_slot_kernel<<<1, 1, 0, st>>>(dst, v);
    return cudaGetLastError();
}

// Which kernel for a launch of M rows.  Measured on B200: v4's pipelined
// tiles win for one or two rows (one stream at 740 keys: 1.605 vs 1.641
// ms/token; 8192 keys: 29.6 vs 39.3 us), v3's one 64-key split per CTA for
// many rows of short contexts (8 streams at 40..740 keys: 11.5 vs 15.4 us per
// layer).  VOX_CUDA_ATTN = v3 | v4 forces one (A/B runs).
static bool attn_use_v3(int M) {
    static int forced = -1;   // 0 auto, 3, 4
    if (forced < 0) {
        const char *e = getenv("VOX_CUDA_ATTN");
        forced = (e && strcmp(e, "v3") == 0) ? 3 : (e && (strcmp(e, "v4") == 0 || strcmp(e, "deep") == 0)) ? 4 : 0;
    }
    return forced == 3 || (forced == 0 && M > 2);
}

cudaError_t launch_attn_decode(int M, const AttnParams &p, cudaStream_t st, bool pdl) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const bool v3 = attn_use_v3(M);
    static std::atomic<uint64_t> attr_set{0};   // the shared-memory opt-in is per device
    const uint64_t bit = 1ull << (dev & 63);
    if (!(attr_set.load() & bit)) {
        e = cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)sizeof(AttnShared));
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(attn_decode_v4_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)sizeof(Attn4SharedT<2>));
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(attn_decode_v4_kernel<kDeepStages>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)sizeof(Attn4SharedT<kDeepStages>));
        if (e != cudaSuccess) return e;
        attr_set.fetch_or(bit);
    }
    cudaLaunchConfig_t cfg = {};
    // CTAs per (row, KV head): no more than the partials this launch's
    // buffers hold (a prefill of fresh rows attends to few keys: S = 1)
    const bool deep = !v3 && attn_use_deep(M, p.deep_hint);
    const int g = std::min(v3 ? attn_ctas_per_head(M) : deep ? attn_deep_ctas_per_head(M) : attn4_ctas_per_head(M),
                           std::max(1, p.S));
    cfg.gridDim = dim3(g, kDecKvHeads, M);
    cfg.blockDim = dim3(128);
    cfg.dynamicSmemBytes = v3 ? sizeof(AttnShared) : deep ? sizeof(Attn4SharedT<kDeepStages>) : sizeof(Attn4SharedT<2>);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    if (v3) return cudaLaunchKernelEx(&cfg, attn_decode_kernel, p);
    return deep ? cudaLaunchKernelEx(&cfg, attn_decode_v4_kernel<kDeepStages>, p)
                : cudaLaunchKernelEx(&cfg, attn_decode_v4_kernel<2>, p);
}

// ---------------------------------------------------------------------------
// --alt selection (stream_fill_alts, voxtral.c:778-833) from device logits:
// softmax statistics over the whole vocabulary, then repeated block-wide
// scans for the most probable id >= 1000 not yet picked (ties: lowest id).
// One CTA of 1024 threads; the logits are 512 KB and stay in L2.
// ---------------------------------------------------------------------------

__device__ __forceinline__ void block_arg_reduce(float &bv, int &bi, float *sv, int *si) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (arg_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) { sv[warp] = bv; si[warp] = bi; }
    __syncthreads();
    if (warp == 0) {
        bv = (lane < (int)(blockDim.x >> 5)) ? sv[lane] : -INFINITY;
        bi = (lane < (int)(blockDim.x >> 5)) ? si[lane] : 0x7fffffff;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (arg_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
        }
        if (lane == 0) { sv[0] = bv; si[0] = bi; }
    }
    __syncthreads();
    bv = sv[0];
    bi = si[0];
    __syncthreads();
}

__global__ void __launch_bounds__(1024)
fill_alts_kernel(const float *logits, int vocab, const int *best_p, int n_alt, float cutoff,
                 int *out_ids) {
    __shared__ float sv[32];
    __shared__ int si[32];
    __shared__ float ssum[32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int best = *best_p;

    float mx = -INFINITY;
    int dummy = 0;
    for (int i = tid; i < vocab; i += blockDim.x) mx = fmaxf(mx, logits[i]);
    block_arg_reduce(mx, dummy, sv, si);

    float sum = 0.f;
    for (int i = tid; i < vocab; i += blockDim.x) sum += expf(logits[i] - mx);
    sum = warp_sum(sum);
    if (lane == 0) ssum[warp] = sum;
    __syncthreads();
    if (warp == 0) {
        float v = (lane < (int)(blockDim.x >> 5)) ? ssum[lane] : 0.f;
        v = warp_sum(v);
        if (lane == 0) ssum[0] = v;
    }
    __syncthreads();
    const float inv = 1.0f / ssum[0];
    const float pb = expf(logits[best] - mx) * inv;

    if (tid == 0) {
        out_ids[0] = best;
        for (int j = 1; j < 4; j++) out_ids[j] = -1;
    }
    if (!(pb > 0.f)) return;
    int picked[4] = {best, -1, -1, -1};
    for (int found = 1; found < n_alt; found++) {
        float bv = -1.0f;
        int bi = 0x7fffffff;
        for (int i = 1000 + tid; i < vocab; i += blockDim.x) {
            bool used = false;
#pragma unroll
            for (int j = 0; j < 4; j++) used |= (picked[j] == i);
            if (used) continue;
            const float pr = expf(logits[i] - mx) * inv;
            if (arg_better(pr, i, bv, bi)) { bv = pr; bi = i; }
        }
        block_arg_reduce(bv, bi, sv, si);
        if (bi == 0x7fffffff || bv < 0.f) break;
        if (1.0f - bv / pb > cutoff) break;
        picked[found] = bi;
        if (tid == 0) out_ids[found] = bi;
    }
}

cudaError_t launch_fill_alts(const float *logits, int vocab, const int *best, int n_alt,
                             float cutoff, int *out_ids, cudaStream_t st) {
    fill_alts_kernel<<<1, 1024, 0, st>>>(logits, vocab, best, n_alt, cutoff, out_ids);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Stand-alone interleaved-pair RoPE (vox_apply_rope, voxtral_kernels.c:502-526).
// ---------------------------------------------------------------------------
__global__ void rope_kernel(float *x, int n_heads, int head_dim, const float *cs) {
    const int half = head_dim >> 1;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_heads * half) return;
    const int h = i / half, d = i - h * half;
    float *v = x + (size_t)h * head_dim + 2 * d;
    const float c = cs[2 * d], sn = cs[2 * d + 1];
    const float a = v[0], b = v[1];
    v[0] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, sn));
    v[1] = __fadd_rn(__fmul_rn(a, sn), __fmul_rn(b, c));
}

cudaError_t launch_rope(float *x, int n_heads, int head_dim, const float *cs, cudaStream_t st) {
    const int n = n_heads * (head_dim / 2);
    rope_kernel<<<(n + 255) / 256, 256, 0, st>>>(x, n_heads, head_dim, cs);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Seeded N(0, std) bf16 fill (benchmarks): splitmix64 counter + Box-Muller.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ uint16_t f32_to_bf16_rne(float f) {
    uint32_t u = __float_as_uint(f);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

__global__ void fill_normal_bf16_kernel(uint16_t *dst, size_t n, uint64_t seed, float std) {
    const size_t pairs = (n + 1) / 2;
    for (size_t j = blockIdx.x * (size_t)blockDim.x + threadIdx.x; j < pairs;
         j += (size_t)gridDim.x * blockDim.x) {
        const uint64_t h = mix64(seed * 0xD1342543DE82EF95ull + j);
        const float u1 = ((float)(h >> 40) + 1.0f) * (1.0f / 16777217.0f);
        const float u2 = (float)((h >> 8) & 0xFFFFFFull) * (1.0f / 16777216.0f);
        const float r = sqrtf(-2.0f * logf(u1));
        float sn, cs;
        sincospif(2.0f * u2, &sn, &cs);
        dst[2 * j] = f32_to_bf16_rne(std * r * cs);
        if (2 * j + 1 < n) dst[2 * j + 1] = f32_to_bf16_rne(std * r * sn);
    }
}

cudaError_t launch_fill_normal_bf16(uint16_t *dst, size_t n, uint64_t seed, float std,
                                    cudaStream_t st) {
    fill_normal_bf16_kernel<<<148 * 8, 256, 0, st>>>(dst, n, seed, std);
    return cudaGetLastError();
}

}  // namespace vc
