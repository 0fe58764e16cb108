// vc_decode.cu - decode-step kernels besides the GEMV (vc_gemv.cu): split-K
// GQA decode attention over the KV ring, the --alt selection, stand-alone
// RoPE and the seeded bf16 fill used by benchmarks.
#include "vc_common.cuh"
#include "vc_internal.h"

#include <math.h>
#include <stdlib.h>

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
        const float o0 = go[0] * inv, o1 = go[1] * inv, o2 = go[2] * inv, o3 = go[3] * inv;
        if (p.out != nullptr)
            *reinterpret_cast<float4 *>(p.out + (size_t)m * kQDim + h * kHeadDim + d4) =
                make_float4(o0, o1, o2, o3);
        if (p.xfrag_out != nullptr) {
            xfrag_put2(p.xfrag_out, m, h * kHeadDim + d4, o0, o1);
            xfrag_put2(p.xfrag_out, m, h * kHeadDim + d4 + 2, o2, o3);
        }
        if (p.out_hilo != nullptr) {
            uint32_t h0, l0, h1, l1, h2, l2, h3, l3;
            split_bf16(o0, h0, l0);
            split_bf16(o1, h1, l1);
            split_bf16(o2, h2, l2);
            split_bf16(o3, h3, l3);
            const size_t e = (size_t)hilo_row(m) * kQDim + h * kHeadDim + d4;
            *reinterpret_cast<uint2 *>(p.out_hilo + e) = make_uint2(h0 | (h1 << 16), h2 | (h3 << 16));
            *reinterpret_cast<uint2 *>(p.out_hilo + e + (size_t)64 * kQDim) =
                make_uint2(l0 | (l1 << 16), l2 | (l3 << 16));
        }
        if (tid == 0) p.counters[m * kDecKvHeads + kvh] = 0u;
    }
}

// CTAs per (stream, KV head): each loops over splits blockIdx.x + G*i.
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

cudaError_t launch_attn_decode(int M, const AttnParams &p, cudaStream_t st, bool pdl) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    static std::atomic<uint64_t> attr_set{0};   // the shared-memory opt-in is per device
    const uint64_t bit = 1ull << (dev & 63);
    if (!(attr_set.load() & bit)) {
        e = cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)sizeof(AttnShared));
        if (e != cudaSuccess) return e;
        attr_set.fetch_or(bit);
    }
    cudaLaunchConfig_t cfg = {};
    // CTAs per (row, KV head): no more than the splits this launch can have
    // (a prefill of fresh rows attends to few keys: S = 1)
    const int g = std::min(attn_ctas_per_head(M), std::max(1, p.S));
    cfg.gridDim = dim3(g, kDecKvHeads, M);
    cfg.blockDim = dim3(128);
    cfg.dynamicSmemBytes = sizeof(AttnShared);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, attn_decode_kernel, p);
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
