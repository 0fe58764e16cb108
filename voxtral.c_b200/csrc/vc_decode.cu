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
    float k[kKeysPerSplit][kHeadDim];   // 32 KB, chunk-swizzled; the merge reuses it for its weights
    float v[kKeysPerSplit][kHeadDim];   // 32 KB
    float q[4][kHeadDim];
    float4 p4[kKeysPerSplit];           // exp(score - split max) of key j for the 4 heads
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
// split at ring slot (first + kb + j) % cap), 16 bytes per copy.  K's
// 16-byte chunk c of key j goes to chunk c ^ (j & 31): lane j reading its
// key's chunk c is conflict-free while the query chunk c is one broadcast.
__device__ __forceinline__ void attn_stage_keys(AttnShared &sh, const float *kbase, const float *vbase, int first,
                                                int kb, int cap, int j0, int j1, int tid) {
    const int n = (j1 - j0) * (kHeadDim / 4);   // 16-byte pieces per matrix
    for (int c = tid; c < n; c += 128) {
        const int j = j0 + c / (kHeadDim / 4), piece = c % (kHeadDim / 4);
        const size_t row = (size_t)((first + kb + j) % cap) * kKvDim + 4 * piece;
        cp_async16(&sh.k[j][4 * (piece ^ (j & 31))], kbase + row);
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
    const StreamSlot slt = p.slot_inline ? p.slot1 : p.slots[m];
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
            const float4 *k0 = reinterpret_cast<const float4 *>(sh.k[lane]);
            const float4 *k1 = reinterpret_cast<const float4 *>(sh.k[lane + 32]);
            float a0 = 0.f, a1 = 0.f;
#pragma unroll 8
            for (int c = 0; c < kHeadDim / 4; c++) {
                const float4 qq = q4[c];                                   // broadcast
                const float4 x0 = k0[c ^ lane], x1 = k1[c ^ lane];         // swizzled rows
                a0 = fmaf(qq.x, x0.x, a0);
                a0 = fmaf(qq.y, x0.y, a0);
                a0 = fmaf(qq.z, x0.z, a0);
                a0 = fmaf(qq.w, x0.w, a0);
                a1 = fmaf(qq.x, x1.x, a1);
                a1 = fmaf(qq.y, x1.y, a1);
                a1 = fmaf(qq.z, x1.z, a1);
                a1 = fmaf(qq.w, x1.w, a1);
            }
            float sc[2];
            sc[0] = (lane < nk) ? a0 * scale : -INFINITY;
            sc[1] = (lane + 32 < nk) ? a1 * scale : -INFINITY;
            float mx = fmaxf(sc[0], sc[1]);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            const float pa = (lane < nk) ? expf(sc[0] - mx) : 0.f;
            const float pb = (lane + 32 < nk) ? expf(sc[1] - mx) : 0.f;
            reinterpret_cast<float *>(&sh.p4[lane])[h] = pa;
            reinterpret_cast<float *>(&sh.p4[lane + 32])[h] = pb;
            const float sum = warp_sum(pa + pb);
            if (lane == 0) {
                sh.ml[h][0] = mx;
                sh.ml[h][1] = sum;
            }
        }
        __syncthreads();

        // ---- P.V: thread = dimension, 4 heads (one broadcast read of the
        // key's 4 probabilities) ----
        {
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
            for (int j = 0; j < nk; j++) {
                const float vj = sh.v[j][tid];
                const float4 pj = sh.p4[j];
                acc[0] = fmaf(pj.x, vj, acc[0]);
                acc[1] = fmaf(pj.y, vj, acc[1]);
                acc[2] = fmaf(pj.z, vj, acc[2]);
                acc[3] = fmaf(pj.w, vj, acc[3]);
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
        // the first eight partials' o go out with the (max, sum) loads: one
        // L2 round trip for the usual S <= 8 instead of three
        float4 o8[8];
#pragma unroll
        for (int u = 0; u < 8; u++)
            o8[u] = (u < S) ? __ldcg(reinterpret_cast<const float4 *>(p.part_o + (pbase + u) * kHeadDim + d4))
                            : make_float4(0.f, 0.f, 0.f, 0.f);
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
#pragma unroll
        for (int u = 0; u < 8; u++) {   // (split order, as below)
            if (u >= S) break;
            const float c = smw[hh][u];
            go[0] += o8[u].x * c;
            go[1] += o8[u].y * c;
            go[2] += o8[u].z * c;
            go[3] += o8[u].w * c;
        }
        int t = 8;
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

    const StreamSlot slt = p.slot_inline ? p.slot1 : p.slots[m];
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

// ---------------------------------------------------------------------------
// v5: keys streamed straight into registers, no shared-memory staging.
//
// A CTA of NW warps takes a contiguous range of one (row, KV head)'s keys,
// each warp a contiguous sub-range in steps of 4 keys.  Lane l holds dims
// [4l, 4l + 4) of each key's K and V row (one coalesced 512-byte load per
// row); the next step's rows are in flight while a step is computed, and a
// warp's first two steps of keys older than the launch are loaded before
// griddepcontrol.wait.  The 16 dot products of a step (4 keys x the KV
// head's 4 query heads) are summed across the warp by a halving exchange
// (8 + 4 + 2 + 1 + 1 shuffles), after which lane l holds the score of key
// l >> 3 for head (l >> 1) & 3.  Online softmax per head over the steps; the
// step's probabilities reach every lane through shared memory for P.V.  The
// warps' partials merge in shared memory; a row with several CTAs merges
// their partials in the last CTA to finish (atomic ticket, no spinning),
// with eight partials' loads in flight per thread.
// ---------------------------------------------------------------------------
constexpr int kV5Step = 4;        // keys per warp step
constexpr float kV5Lazy = 8.0f;   // log2 of the largest probability before the running max moves

// 2^x by the hardware approximation (relative error ~2^-22)
__device__ __forceinline__ float ex2f(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <int NW>
struct Attn5Shared {
    float4 pk[NW][kV5Step];                   // a step's probabilities: [key] = (4 heads)
    float4 alpha[NW];                         // a step's rescale of the running sums, per head
    float4 o[NW][4][kHeadDim / 4];            // warp partials: unnormalised o per head
    float2 ml[NW][4];                         // warp partials: (max, sum) per head
    float mw[4][kAttnSplits];                 // merge: CTA partial maxima, then their weights
    float lw[4][kAttnSplits];                 // merge: CTA partial sums
    float4 grp[NW / 4][4 * kHeadDim / 4];     // merge: the thread groups' sums
    float gl[4];                              // merge: per-head total sum
    int last;
};

__device__ __forceinline__ float4 ldcg4(const float *p) { return __ldcg(reinterpret_cast<const float4 *>(p)); }
__device__ __forceinline__ float comp4(const float4 &v, int i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}
__device__ __forceinline__ void fma4(float4 &acc, float w, const float4 &v) {
    acc.x = fmaf(w, v.x, acc.x);
    acc.y = fmaf(w, v.y, acc.y);
    acc.z = fmaf(w, v.z, acc.z);
    acc.w = fmaf(w, v.w, acc.w);
}
__device__ __forceinline__ float dot4(const float4 &a, const float4 &b) {
    return fmaf(a.w, b.w, fmaf(a.z, b.z, fmaf(a.y, b.y, a.x * b.x)));
}
// halving exchange step: of 2n values, keep the half selected by this lane's
// bit (upper when set), add the partner's copy of it, send it the other half
template <int N>
__device__ __forceinline__ void xhalve(float *a, bool upper, int mask) {
#pragma unroll
    for (int j = 0; j < N; j++) {
        const float send = upper ? a[j] : a[j + N], keep = upper ? a[j + N] : a[j];
        a[j] = keep + __shfl_xor_sync(0xffffffffu, send, mask);
    }
}

template <int NW>
__global__ void __launch_bounds__(NW * 32, NW == 4 ? 4 : 2)
attn_decode_v5_kernel(const AttnParams p) {
    __shared__ Attn5Shared<NW> sh;
    const int kvh = blockIdx.y, m = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) l2_prefetch_share(p.pf, p.pf_bytes);   // the wo GEMV's weights (this kernel leaves HBM idle)

    const StreamSlot slt = p.slot_inline ? p.slot1 : p.slots[m];
    const int n_keys = slt.n_keys;
    const int min_keys = p.min_keys > 0 ? p.min_keys : NW * 8;
    const int P = max(1, min((int)gridDim.x, (n_keys + min_keys - 1) / min_keys));   // CTAs with keys
    if ((int)blockIdx.x >= P) return;   // CTA-uniform, before any barrier
    const int c0 = (int)((long long)blockIdx.x * n_keys / P), c1 = (int)((long long)(blockIdx.x + 1) * n_keys / P);
    const int k0 = c0 + (int)((long long)warp * (c1 - c0) / NW);
    const int k1 = c0 + (int)((long long)(warp + 1) * (c1 - c0) / NW);
    const int nsteps = (k1 - k0 + kV5Step - 1) / kV5Step;
    const int first = slt.pos - n_keys + 1;   // logical position of key 0
    const int cap = slt.cap;
    const size_t layer_off = (size_t)p.layer * cap * kKvDim + kvh * kHeadDim + 4 * lane;
    const float *kbase = slt.k_ring + layer_off;
    const float *vbase = slt.v_ring + layer_off;
    const int n_old = max(0, min(slt.fresh, slt.pos) - first);   // keys [0, n_old) predate this launch
    // key j's ring row: one modulo per warp, then a conditional wrap (the
    // warp's keys span fewer than cap positions)
    const int slot0 = (first + k0) % cap;
    auto row_of = [&](int j) {
        int sl = slot0 + (j - k0);
        sl = sl >= cap ? sl - cap : sl;
        return (size_t)sl * kKvDim;
    };

    const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
    float4 kc[kV5Step], vc[kV5Step], kn[kV5Step], vn[kV5Step];   // step i, step i + 1
#pragma unroll
    for (int u = 0; u < kV5Step; u++) kc[u] = vc[u] = kn[u] = vn[u] = z4;
    // steps 0 and 1: keys older than the launch before the wait (they
    // overlap the producer kernel's tail), this launch's own after it
#pragma unroll
    for (int u = 0; u < kV5Step; u++) {
        const int j0 = k0 + u, j1 = k0 + kV5Step + u;
        if (j0 < k1 && j0 < n_old) kc[u] = ldcg4(kbase + row_of(j0)), vc[u] = ldcg4(vbase + row_of(j0));
        if (j1 < k1 && j1 < n_old) kn[u] = ldcg4(kbase + row_of(j1)), vn[u] = ldcg4(vbase + row_of(j1));
    }
    grid_dep_wait();
    grid_dep_launch();
#pragma unroll
    for (int u = 0; u < kV5Step; u++) {
        const int j0 = k0 + u, j1 = k0 + kV5Step + u;
        if (j0 < k1 && j0 >= n_old) kc[u] = ldcg4(kbase + row_of(j0)), vc[u] = ldcg4(vbase + row_of(j0));
        if (j1 < k1 && j1 >= n_old) kn[u] = ldcg4(kbase + row_of(j1)), vn[u] = ldcg4(vbase + row_of(j1));
    }
    float4 q[4];   // the KV head's 4 query heads, this lane's 4 dims
#pragma unroll
    for (int h = 0; h < 4; h++) q[h] = ldcg4(p.q + (size_t)m * kQDim + (kvh * 4 + h) * kHeadDim + 4 * lane);

    // scores in log2 units: p = 2^(s * scale * log2 e - m)
    const float scale2 = 1.4426950408889634f / sqrtf((float)kHeadDim);
    const int kl = lane >> 3, hl = (lane >> 1) & 3;   // the (key, head) whose score this lane ends with
    float m_run = -INFINITY, l_run = 0.f;              // head hl's running max (log2 units) / sum
    float4 o[4] = {z4, z4, z4, z4};                    // unnormalised output, 4 heads x this lane's dims
    float *pkw = reinterpret_cast<float *>(sh.pk[warp]);
    float *alw = reinterpret_cast<float *>(&sh.alpha[warp]);
    // step i from (ck, cv); step i + 1 goes out into (nk, nv) first (steps 0
    // and 1 went out above).  Two calls per loop pass swap the buffers.
    auto step = [&](int i, float4 *ck, float4 *cv, float4 *nk, float4 *nv) {
        if (i >= 1 && i + 1 < nsteps) {
#pragma unroll
            for (int u = 0; u < kV5Step; u++) {
                const int j = k0 + (i + 1) * kV5Step + u;
                nk[u] = j < k1 ? ldcg4(kbase + row_of(j)) : z4;
                nv[u] = j < k1 ? ldcg4(vbase + row_of(j)) : z4;
            }
        }
        float a[16];   // a[4u + h]: q_h . k_u over this lane's 4 dims
#pragma unroll
        for (int u = 0; u < kV5Step; u++)
#pragma unroll
            for (int h = 0; h < 4; h++) a[4 * u + h] = dot4(q[h], ck[u]);
        xhalve<8>(a, lane & 16, 16);
        xhalve<4>(a, lane & 8, 8);
        xhalve<2>(a, lane & 4, 4);
        xhalve<1>(a, lane & 2, 2);
        a[0] += __shfl_xor_sync(0xffffffffu, a[0], 1);
        const bool valid = k0 + i * kV5Step + kl < k1;
        const float sc = valid ? a[0] * scale2 : -INFINITY;
        float tm = fmaxf(sc, __shfl_xor_sync(0xffffffffu, sc, 8));
        tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, 16));
        // the running max moves only when a score exceeds it by more than
        // 2^8 (p stays <= 256): most steps then need no rescale
        const float nm = (tm > m_run + kV5Lazy) ? tm : m_run;   // finite: the step's first key is valid
        const float pj = valid ? ex2f(sc - nm) : 0.f;
        float ps = pj + __shfl_xor_sync(0xffffffffu, pj, 8);
        ps += __shfl_xor_sync(0xffffffffu, ps, 16);
        const bool moved = __any_sync(0xffffffffu, nm != m_run);   // warp-uniform
        float alpha = 1.0f;
        if (moved) alpha = (m_run == -INFINITY) ? 0.f : ex2f(m_run - nm);
        l_run = l_run * alpha + ps;
        m_run = nm;
        if ((lane & 1) == 0) pkw[lane >> 1] = pj;   // = pk[kl][hl]
        if (moved && (lane & 0x19) == 0) alw[hl] = alpha;   // lanes 0, 2, 4, 6
        __syncwarp();
        float4 pk[kV5Step];
#pragma unroll
        for (int u = 0; u < kV5Step; u++) pk[u] = sh.pk[warp][u];
        if (moved) {
            const float4 al = sh.alpha[warp];
#pragma unroll
            for (int h = 0; h < 4; h++) {
                const float ah = comp4(al, h);
                o[h] = make_float4(o[h].x * ah, o[h].y * ah, o[h].z * ah, o[h].w * ah);
            }
        }
        __syncwarp();   // read before the next step's writes
#pragma unroll
        for (int h = 0; h < 4; h++)
#pragma unroll
            for (int u = 0; u < kV5Step; u++) fma4(o[h], comp4(pk[u], h), cv[u]);
    };
    for (int i = 0; i < nsteps; i += 2) {
        step(i, kc, vc, kn, vn);
        if (i + 1 < nsteps) step(i + 1, kn, vn, kc, vc);
    }

    // ---- the warps' partials -> this CTA's (threads 0..127: head, 4 dims) ----
#pragma unroll
    for (int h = 0; h < 4; h++) sh.o[warp][h][lane] = o[h];
    if ((lane & 0x19) == 0) sh.ml[warp][hl] = make_float2(m_run, l_run);
    __syncthreads();
    const int hh = (tid >> 5) & 3, c = lane;   // (threads >= 128 only help with the cross-CTA merge)
    float4 co = z4;
    float cm = -INFINITY, cl = 0.f;
    if (tid < 128) {
#pragma unroll
        for (int w = 0; w < NW; w++)
            if (sh.ml[w][hh].y > 0.f) cm = fmaxf(cm, sh.ml[w][hh].x);
#pragma unroll
        for (int w = 0; w < NW; w++) {
            const float2 ml = sh.ml[w][hh];
            const float cw = ml.y > 0.f ? ex2f(ml.x - cm) : 0.f;
            cl += ml.y * cw;
            fma4(co, cw, sh.o[w][hh][c]);
        }
    }
    const int hg = kvh * 4 + hh;   // query head
    if (P == 1) {   // the row's only CTA: the output itself
        if (tid < 128) {
            const float inv = cl > 0.f ? 1.0f / cl : 0.f;
            attn_store_out(p, m, hg * kHeadDim + 4 * c, co.x * inv, co.y * inv, co.z * inv, co.w * inv);
        }
        return;
    }
    if (tid < 128) {
        const size_t pidx = ((size_t)m * kDecHeads + hg) * p.S + blockIdx.x;
        reinterpret_cast<float4 *>(p.part_o + pidx * kHeadDim)[c] = co;
        if (c == 0) {
            p.part_ml[pidx * 2] = cm;
            p.part_ml[pidx * 2 + 1] = cl;
        }
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) sh.last = (atomicAdd(&p.counters[m * kDecKvHeads + kvh], 1u) + 1u == (unsigned)P);
    __syncthreads();
    if (!sh.last) return;
    __threadfence();

    // ---- merge the P partials (last CTA of this row / KV head) ----
    for (int i = tid; i < 4 * P; i += NW * 32) {
        const int h = i / P, t = i % P;
        const size_t pidx = ((size_t)m * kDecHeads + kvh * 4 + h) * p.S + t;
        sh.mw[h][t] = __ldcg(p.part_ml + pidx * 2);
        sh.lw[h][t] = __ldcg(p.part_ml + pidx * 2 + 1);
    }
    __syncthreads();
    if (warp < 4) {   // warp h: the head's maximum, the partials' weights, the total sum
        float gm = -INFINITY;
        for (int t = lane; t < P; t += 32)
            if (sh.lw[warp][t] > 0.f) gm = fmaxf(gm, sh.mw[warp][t]);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, off));
        float gd = 0.f;
        for (int t = lane; t < P; t += 32) {
            const float w = sh.lw[warp][t] > 0.f ? ex2f(sh.mw[warp][t] - gm) : 0.f;
            gd += sh.lw[warp][t] * w;
            sh.mw[warp][t] = w;
        }
        gd = warp_sum(gd);
        if (lane == 0) sh.gl[warp] = gd;
    }
    __syncthreads();
    // thread group g (128 threads: head, 4 dims) sums partials g, g + NW/4, ...
    constexpr int G = NW / 4;
    const int g = tid >> 7;
    const float4 *src = reinterpret_cast<const float4 *>(p.part_o) + ((size_t)m * kDecHeads + hg) * p.S * (kHeadDim / 4) + c;
    float4 acc = z4;
    int t = g;
    for (; t + 7 * G < P; t += 8 * G) {   // eight loads in flight
        float4 v[8];
#pragma unroll
        for (int u = 0; u < 8; u++) v[u] = __ldcg(src + (size_t)(t + u * G) * (kHeadDim / 4));
#pragma unroll
        for (int u = 0; u < 8; u++) fma4(acc, sh.mw[hh][t + u * G], v[u]);
    }
    for (; t < P; t += G) fma4(acc, sh.mw[hh][t], __ldcg(src + (size_t)t * (kHeadDim / 4)));
    if constexpr (G > 1) {
        sh.grp[g][tid & 127] = acc;
        __syncthreads();
        if (g != 0) return;
        acc = z4;
#pragma unroll
        for (int j = 0; j < G; j++) {
            const float4 v = sh.grp[j][tid];
            acc.x += v.x, acc.y += v.y, acc.z += v.z, acc.w += v.w;
        }
    }
    const float inv = sh.gl[hh] > 0.f ? 1.0f / sh.gl[hh] : 0.f;
    attn_store_out(p, m, hg * kHeadDim + 4 * c, acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
    if (tid == 0) p.counters[m * kDecKvHeads + kvh] = 0u;
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

// The deep v4 variant: 2 tiles in flight per CTA keep ~128 KB of keys
// moving per SM, where v4's 3 CTAs x 1 tile do ~96 KB.  Only on request
// (VOX_CUDA_ATTN = deep): long contexts take v5 (attn_use_v5).
bool attn_use_deep(int M, int keys_hint) {
    (void)M;
    (void)keys_hint;
    static int forced = -1;
    if (forced < 0) {
        const char *e = getenv("VOX_CUDA_ATTN");
        forced = (e && strcmp(e, "deep") == 0) ? 1 : 0;
    }
    return forced == 1;
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

// v5 (keys in registers) for one or two rows of long contexts (the caller's
// hint of the keys per row >= kAttnDeepKeys).  Measured on B200, stand-alone
// (one row, device time after an L2 flush): 8192 keys 24.6 us against 30.7
// (v4, 3 tile buffers), 2048 keys 16.4 against 18.5; one stream's decode
// step at 740 keys ties with v4 (1.582 / 1.585 ms per token); 8 streams'
// step is slower than v3 (1.82 against 1.72 ms: v3 stages a whole 64-key
// split per CTA before griddepcontrol.wait, v5 two 4-key steps per warp).
// VOX_CUDA_ATTN = v5 forces it for every launch; VOX_CUDA_ATTN_V5_CTAS /
// _MINKEYS set its CTAs per (row, KV head) and the fewest keys per CTA.
static bool attn_use_v5(int M, int keys_hint) {
    static int forced = -1;
    if (forced < 0) {
        const char *e = getenv("VOX_CUDA_ATTN");
        forced = (e && strcmp(e, "v5") == 0) ? 1 : (e && *e) ? 0 : 2;
    }
    if (forced != 2) return forced == 1;
    return M <= 2 && keys_hint >= kAttnDeepKeys;
}

static int env_pos(const char *name) {
    const char *e = getenv(name);
    return (e && atoi(e) > 0) ? atoi(e) : 0;
}

static cudaError_t launch_attn_v5(int M, const AttnParams &p, cudaStream_t st, bool pdl, int dev) {
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    // one or two rows (long contexts): 8-warp CTAs, two per SM over the KV
    // heads; more rows: 4-warp CTAs, 16 per (row, KV head) at most
    const bool wide = M <= 2;
    int g = wide ? std::max(1, 2 * sms / (kDecKvHeads * M)) : 16;
    if (env_pos("VOX_CUDA_ATTN_V5_CTAS")) g = env_pos("VOX_CUDA_ATTN_V5_CTAS");
    g = std::min(g, std::max(1, std::min(p.S, kAttnSplits)));
    AttnParams q = p;
    q.min_keys = env_pos("VOX_CUDA_ATTN_V5_MINKEYS") ? env_pos("VOX_CUDA_ATTN_V5_MINKEYS") : wide ? 64 : 32;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(g, kDecKvHeads, M);
    cfg.blockDim = dim3(wide ? 256 : 128);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return wide ? cudaLaunchKernelEx(&cfg, attn_decode_v5_kernel<8>, q)
                : cudaLaunchKernelEx(&cfg, attn_decode_v5_kernel<4>, q);
}

cudaError_t launch_attn_decode(int M, const AttnParams &p, cudaStream_t st, bool pdl) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (p.variant != 4 && attn_use_v5(M, p.deep_hint)) return launch_attn_v5(M, p, st, pdl, dev);
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
