// vc_decode.cu - decode-step kernels besides the GEMV (vc_gemv.cu): split-K
// GQA decode attention over the KV ring, the --alt selection, stand-alone
// RoPE and the seeded bf16 fill used by benchmarks.
#include "vc_common.cuh"
#include "vc_internal.h"

#include <math.h>
#include <stdlib.h>

namespace vc {

__device__ __forceinline__ bool arg_better(float v, int i, float bv, int bi) {
    return v > bv || (v == bv && i < bi);
}

// ---------------------------------------------------------------------------
// Split-K GQA decode attention over the KV ring (vox_causal_attention with
// seq_q = 1, voxtral_kernels.c:412-482, as called at voxtral_decoder.c:481-483).
//
// grid (S, 8 KV heads, M streams), 128 threads.  A CTA takes one KV head and
// up to 64 consecutive keys of the window; its 4 query heads share every K/V
// load.  Instead of the reference's per-key online softmax (a serial chain),
// the CTA runs three parallel passes: all scores (thread = key half-row, 16
// float4 loads in flight each), the softmax of its keys (one warp per head),
// then P.V with coalesced float4 loads of V (warp = key group, lane = 4
// dims).  Splits are merged with the usual max rescaling by the last CTA of
// each (stream, KV head) to finish (atomic ticket; no spinning).
// ---------------------------------------------------------------------------

constexpr int kKeysPerSplit = 64;

__global__ void __launch_bounds__(128)
attn_decode_kernel(const AttnParams p) {
    const int kvh = blockIdx.y, m = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    __shared__ __align__(16) float sq[4][kHeadDim];       // the 4 query heads of this KV head
    __shared__ float ssc[4][kKeysPerSplit];               // scores, then exp(score - max)
    __shared__ __align__(16) float so[4][4][kHeadDim];    // P.V per key group [group][head][dim]
    __shared__ float sml[4][2];                            // per head: (max, sum of exp)
    __shared__ float smw[4][kAttnSplits];                  // merge weights per split
    __shared__ int s_last;

    grid_dep_wait();
    grid_dep_launch();

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

    {   // queries
        const float4 v = *reinterpret_cast<const float4 *>(p.q + (size_t)m * kQDim +
                                                           (kvh * 4 + warp) * kHeadDim + 4 * lane);
        *reinterpret_cast<float4 *>(&sq[warp][4 * lane]) = v;
    }

    int n_done = 0;
    for (int s = blockIdx.x; s < S; s += gridDim.x) {
        const int kb = s * chunk;
        const int nk = max(0, min(kb + chunk, n_keys) - kb);
        // K (thread = key half-row) and V (warp = key group, lane = 4 dims) of
        // this split, all loads issued before any use
        const int jk = tid >> 1, hf = tid & 1;
        float4 kv[16], vv[16];
        if (jk < nk) {
            const int slot = (first + kb + jk) % cap;
            const float4 *kr = reinterpret_cast<const float4 *>(kbase + (size_t)slot * kKvDim + 64 * hf);
#pragma unroll
            for (int i = 0; i < 16; i++) kv[i] = __ldcg(kr + i);
        }
#pragma unroll
        for (int i = 0; i < 16; i++) {
            const int j = warp + 4 * i;
            if (j < nk) {
                const int slot = (first + kb + j) % cap;
                vv[i] = __ldcg(reinterpret_cast<const float4 *>(vbase + (size_t)slot * kKvDim) + lane);
            } else {
                vv[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
        __syncthreads();   // sq ready (first split); previous split's ssc / so consumed

        // ---- scores ----
        {
            float d[4] = {0.f, 0.f, 0.f, 0.f};
            if (jk < nk) {
#pragma unroll
                for (int h = 0; h < 4; h++) {
                    const float4 *qh = reinterpret_cast<const float4 *>(&sq[h][64 * hf]);
                    float a = 0.f;
#pragma unroll
                    for (int i = 0; i < 16; i++) {
                        const float4 q4 = qh[i];
                        a = fmaf(q4.x, kv[i].x, a);
                        a = fmaf(q4.y, kv[i].y, a);
                        a = fmaf(q4.z, kv[i].z, a);
                        a = fmaf(q4.w, kv[i].w, a);
                    }
                    d[h] = a;
                }
            }
#pragma unroll
            for (int h = 0; h < 4; h++) {
                const float t = d[h] + __shfl_xor_sync(0xffffffffu, d[h], 1);
                if (hf == 0 && jk < nk) ssc[h][jk] = t * scale;
            }
        }
        __syncthreads();

        // ---- softmax of this split's keys: warp = head ----
        {
            const int h = warp;
            const float a = (lane < nk) ? ssc[h][lane] : -INFINITY;
            const float b = (lane + 32 < nk) ? ssc[h][lane + 32] : -INFINITY;
            float mx = fmaxf(a, b);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            const float pa = (lane < nk) ? expf(a - mx) : 0.f;
            const float pb = (lane + 32 < nk) ? expf(b - mx) : 0.f;
            if (lane < nk) ssc[h][lane] = pa;
            if (lane + 32 < nk) ssc[h][lane + 32] = pb;
            const float sum = warp_sum(pa + pb);
            if (lane == 0) {
                sml[h][0] = mx;
                sml[h][1] = sum;
            }
        }
        __syncthreads();

        // ---- P.V ----
        {
            float acc[4][4];
#pragma unroll
            for (int h = 0; h < 4; h++)
#pragma unroll
                for (int c = 0; c < 4; c++) acc[h][c] = 0.f;
#pragma unroll
            for (int i = 0; i < 16; i++) {
                const int j = warp + 4 * i;
                if (j < nk) {
#pragma unroll
                    for (int h = 0; h < 4; h++) {
                        const float pw = ssc[h][j];
                        acc[h][0] = fmaf(pw, vv[i].x, acc[h][0]);
                        acc[h][1] = fmaf(pw, vv[i].y, acc[h][1]);
                        acc[h][2] = fmaf(pw, vv[i].z, acc[h][2]);
                        acc[h][3] = fmaf(pw, vv[i].w, acc[h][3]);
                    }
                }
            }
#pragma unroll
            for (int h = 0; h < 4; h++)
                *reinterpret_cast<float4 *>(&so[warp][h][4 * lane]) =
                    make_float4(acc[h][0], acc[h][1], acc[h][2], acc[h][3]);
        }
        __syncthreads();

        // ---- this split's partial: warp = head, lane = 4 dims ----
        {
            const int hh = warp, d4 = 4 * lane;
            float go[4];
#pragma unroll
            for (int c = 0; c < 4; c++)
                go[c] = so[0][hh][d4 + c] + so[1][hh][d4 + c] + so[2][hh][d4 + c] + so[3][hh][d4 + c];
            const size_t pidx = ((size_t)m * kDecHeads + kvh * 4 + hh) * p.S + s;
            *reinterpret_cast<float4 *>(p.part_o + pidx * kHeadDim + d4) = make_float4(go[0], go[1], go[2], go[3]);
            if (lane == 0) {
                p.part_ml[pidx * 2] = sml[hh][0];
                p.part_ml[pidx * 2 + 1] = sml[hh][1];
            }
        }
        n_done++;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0)
        s_last = (atomicAdd(&p.counters[m * kDecKvHeads + kvh], (unsigned)n_done) + n_done == (unsigned)S);
    __syncthreads();
    if (!s_last) return;
    __threadfence();

    // ---- merge the S splits (last CTA of this stream / KV head): warp = head ----
    {
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
            if (t < kAttnSplits) smw[hh][t] = c;
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

cudaError_t launch_attn_decode(int M, const AttnParams &p, cudaStream_t st, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(attn_ctas_per_head(M), kDecKvHeads, M);
    cfg.blockDim = dim3(128);
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
