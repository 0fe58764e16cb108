// vc_decode.cu - decode-step kernels: the fused streaming GEMV (RMSNorm
// prologue; residual / RoPE + KV-ring / SwiGLU / LM-head-argmax epilogues),
// split-K GQA decode attention over the KV ring, and the --alt selection.
//
// The GEMV is HBM-bound: every launch streams an [N, K] bf16 weight matrix
// once with 16-byte non-allocating loads (L2 evict-first), the fp32
// activations sit in shared memory, accumulation is fp32 in index order
// (bf16_matvec_fused, voxtral_kernels.c:154-195).
#include "vc_common.cuh"
#include "vc_internal.h"

#include <math.h>

namespace vc {

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kXsFloats = 11264;   // 44 KB of staged activations per CTA
constexpr int kUnroll = 4;         // 16-byte segments in flight per row per lane

// K-chunk staged per pass: the largest multiple of 256 with M*KC <= kXsFloats.
template <int M>
__host__ __device__ constexpr int gemv_kc() {
    return (kXsFloats / M) / 256 * 256;
}

template <int M, int EPI>
__host__ __device__ constexpr int gemv_rows_per_warp() {
    // Pairs of rows are needed by the RoPE (q/k pair 2d, 2d+1) and SwiGLU
    // (gate_i, up_i interleaved) epilogues.  More rows per warp re-use each
    // staged activation for more weight bytes (fewer shared-memory reads per
    // HBM byte); R*M <= 32 keeps one epilogue value per lane.
    return (M == 1) ? 4 : ((M <= 4) ? 4 : 2);
}

__device__ __forceinline__ bool arg_better(float v, int i, float bv, int bi) {
    return v > bv || (v == bv && i < bi);
}

template <int M, int EPI>
__global__ void __launch_bounds__(kGemvThreads)
gemv_kernel(const GemvParams p) {
    constexpr int R = gemv_rows_per_warp<M, EPI>();
    constexpr int KC = gemv_kc<M>();
    constexpr int HALF = M * KC / 2;  // floats per half-plane
    static_assert(R * M <= 32, "one epilogue value per lane");

    // Activations are staged as two planes: lo holds elements 8s..8s+3 of
    // each 8-element segment s, hi holds 8s+4..8s+7, so the two float4 reads
    // a lane makes per weight segment are bank-conflict free.
    __shared__ __align__(16) float xs[M * KC];
    __shared__ float s_inv[M];
    __shared__ ArgmaxPartial s_arg[kGemvWarps][M];
    __shared__ int s_last;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int row0 = (blockIdx.x * kGemvWarps + warp) * R;
    const int K = p.K, N = p.N;
    const uint64_t pol = make_evict_first_policy();

    grid_dep_wait();
    grid_dep_launch();

    if (p.norm_w != nullptr) {
        // RMSNorm prologue (voxtral_kernels.c:346-363): 1/sqrt(mean(x^2)+eps)
        for (int m = warp; m < M; m += kGemvWarps) {
            const float4 *xr = reinterpret_cast<const float4 *>(p.x + (size_t)m * p.ldx);
            float ss = 0.f;
            for (int i = lane; i < (K >> 2); i += 32) {
                float4 v = xr[i];
                ss = fmaf(v.x, v.x, ss);
                ss = fmaf(v.y, v.y, ss);
                ss = fmaf(v.z, v.z, ss);
                ss = fmaf(v.w, v.w, ss);
            }
            ss = warp_sum(ss);
            if (lane == 0) s_inv[m] = 1.0f / sqrtf(ss / (float)K + kNormEps);
        }
    }

    float acc[R][M];
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
        for (int m = 0; m < M; m++) acc[r][m] = 0.f;

    for (int k0 = 0; k0 < K; k0 += KC) {
        const int kc = min(KC, K - k0);
        const int nq = kc >> 2;  // float4s per row in this chunk
        __syncthreads();
        for (int j = tid; j < M * nq; j += kGemvThreads) {
            const int m = j / nq, c = j - m * nq;
            float4 v = *reinterpret_cast<const float4 *>(p.x + (size_t)m * p.ldx + k0 + 4 * c);
            if (p.norm_w != nullptr) {
                const float inv = s_inv[m];
                const float4 w = *reinterpret_cast<const float4 *>(p.norm_w + k0 + 4 * c);
                v.x = v.x * inv * w.x;
                v.y = v.y * inv * w.y;
                v.z = v.z * inv * w.z;
                v.w = v.w * inv * w.w;
                if (p.ada != nullptr) {  // x_norm *= (1 + ada)  (voxtral_decoder.c:489-492)
                    const float4 a = *reinterpret_cast<const float4 *>(p.ada + k0 + 4 * c);
                    v.x *= (1.0f + a.x);
                    v.y *= (1.0f + a.y);
                    v.z *= (1.0f + a.z);
                    v.w *= (1.0f + a.w);
                }
            }
            *reinterpret_cast<float4 *>(xs + (c & 1) * HALF + m * (KC / 2) + 4 * (c >> 1)) = v;
        }
        __syncthreads();

        if (row0 < N) {
            const int nseg = kc >> 3;
            const uint16_t *wrow[R];
#pragma unroll
            for (int r = 0; r < R; r++) {
                const int rr = min(row0 + r, N - 1);
                wrow[r] = p.W + (size_t)rr * K + k0;
            }
            for (int s0 = lane; s0 < nseg; s0 += 32 * kUnroll) {
                uint4 w[kUnroll][R];
#pragma unroll
                for (int u = 0; u < kUnroll; u++) {
                    const int s = s0 + 32 * u;
#pragma unroll
                    for (int r = 0; r < R; r++)
                        w[u][r] = (s < nseg) ? ldg_stream(wrow[r] + 8 * s, pol) : make_uint4(0, 0, 0, 0);
                }
#pragma unroll
                for (int u = 0; u < kUnroll; u++) {
                    const int s = s0 + 32 * u;
                    if (s < nseg) {
#pragma unroll
                        for (int m = 0; m < M; m++) {
                            const float4 a = *reinterpret_cast<const float4 *>(xs + m * (KC / 2) + 4 * s);
                            const float4 b = *reinterpret_cast<const float4 *>(xs + HALF + m * (KC / 2) + 4 * s);
#pragma unroll
                            for (int r = 0; r < R; r++) acc[r][m] = dot8(w[u][r], a, b, acc[r][m]);
                        }
                    }
                }
            }
        }
    }

#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
        for (int m = 0; m < M; m++) acc[r][m] = warp_sum(acc[r][m]);

    if constexpr (EPI == EPI_STORE || EPI == EPI_ADD || EPI == EPI_LOGITS) {
#pragma unroll
        for (int r = 0; r < R; r++)
#pragma unroll
            for (int m = 0; m < M; m++)
                if (lane == r * M + m && row0 + r < N) {
                    float v = acc[r][m];
                    if (p.bias != nullptr) v += p.bias[row0 + r];
                    float *dst = p.y + (size_t)m * p.ldy + row0 + r;
                    if constexpr (EPI == EPI_ADD) *dst += v;
                    else *dst = v;
                }
    } else if constexpr (EPI == EPI_QKV) {
        // rows [0,4096): q, [4096,5120): k, [5120,6144): v.  Pairs (2d, 2d+1)
        // of q and k are rotated by the step's (cos, sin)[d]
        // (vox_apply_rope, voxtral_kernels.c:502-526), k and v go to the ring
        // slot of the step's position (voxtral_decoder.c:474-475).
#pragma unroll
        for (int pr = 0; pr < R / 2; pr++)
#pragma unroll
            for (int m = 0; m < M; m++)
                if (lane == pr * M + m && row0 + 2 * pr < N) {
                    const int ra = row0 + 2 * pr;
                    const float va = acc[2 * pr][m], vb = acc[2 * pr + 1][m];
                    const StreamSlot sl = p.slots[m];
                    const size_t ring_row = ((size_t)p.layer * sl.cap + sl.slot) * kKvDim;
                    if (ra < kQDim + kKvDim) {
                        const int d = (ra & (kHeadDim - 1)) >> 1;
                        const float c = p.rope[m * kHeadDim + 2 * d];
                        const float sn = p.rope[m * kHeadDim + 2 * d + 1];
                        const float oa = __fsub_rn(__fmul_rn(va, c), __fmul_rn(vb, sn));
                        const float ob = __fadd_rn(__fmul_rn(va, sn), __fmul_rn(vb, c));
                        if (ra < kQDim) {
                            float *dst = p.y + (size_t)m * p.ldy + ra;
                            dst[0] = oa;
                            dst[1] = ob;
                        } else {
                            float *dst = sl.k_ring + ring_row + (ra - kQDim);
                            dst[0] = oa;
                            dst[1] = ob;
                        }
                    } else {
                        float *dst = sl.v_ring + ring_row + (ra - kQDim - kKvDim);
                        dst[0] = va;
                        dst[1] = vb;
                    }
                }
    } else if constexpr (EPI == EPI_SWIGLU) {
        // h_i = silu(gate_i) * up_i  (voxtral_kernels.c:369-374 then :34-36)
#pragma unroll
        for (int pr = 0; pr < R / 2; pr++)
#pragma unroll
            for (int m = 0; m < M; m++)
                if (lane == pr * M + m && row0 + 2 * pr < N) {
                    const float g = acc[2 * pr][m], u = acc[2 * pr + 1][m];
                    const float sg = g / (1.0f + expf(-g));
                    p.y[(size_t)m * p.ldy + ((row0 + 2 * pr) >> 1)] = sg * u;
                }
    }

    if constexpr (EPI == EPI_LOGITS) {
        // First maximum over the vocabulary (voxtral_decoder.c:507-515):
        // per-CTA partials, then the last CTA to finish reduces them.
        if (lane == 0) {
#pragma unroll
            for (int m = 0; m < M; m++) {
                float bv = -INFINITY;
                int bi = 0x7fffffff;
#pragma unroll
                for (int r = 0; r < R; r++)
                    if (row0 + r < N && arg_better(acc[r][m], row0 + r, bv, bi)) {
                        bv = acc[r][m];
                        bi = row0 + r;
                    }
                s_arg[warp][m] = {bv, bi};
            }
        }
        __syncthreads();
        if (tid < M) {
            float bv = -INFINITY;
            int bi = 0x7fffffff;
            for (int w = 0; w < kGemvWarps; w++)
                if (arg_better(s_arg[w][tid].v, s_arg[w][tid].i, bv, bi)) {
                    bv = s_arg[w][tid].v;
                    bi = s_arg[w][tid].i;
                }
            p.partials[(size_t)blockIdx.x * M + tid] = {bv, bi};
            __threadfence();
        }
        __syncthreads();
        if (tid == 0) s_last = (atomicAdd(p.counter, 1u) == gridDim.x - 1);
        __syncthreads();
        if (s_last) {
            __threadfence();
            if (warp < M) {
                float bv = -INFINITY;
                int bi = 0x7fffffff;
                for (int b = lane; b < (int)gridDim.x; b += 32) {
                    const float v = __ldcg(&p.partials[(size_t)b * M + warp].v);
                    const int i = __ldcg(&p.partials[(size_t)b * M + warp].i);
                    if (arg_better(v, i, bv, bi)) { bv = v; bi = i; }
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                    if (arg_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
                }
                if (lane == 0) p.tokens[warp] = bi;
            }
            if (tid == 0) *p.counter = 0u;
        }
    }
}

template <int M, int EPI>
static int grid_for(int N) {
    constexpr int rows = kGemvWarps * gemv_rows_per_warp<M, EPI>();
    return (N + rows - 1) / rows;
}

int gemv_grid(int M, int epi, int N) {
#define VC_GRID_CASE(MM)                                                          \
    case MM:                                                                      \
        switch (epi) {                                                            \
            case EPI_STORE: return grid_for<MM, EPI_STORE>(N);                    \
            case EPI_ADD: return grid_for<MM, EPI_ADD>(N);                        \
            case EPI_QKV: return grid_for<MM, EPI_QKV>(N);                        \
            case EPI_SWIGLU: return grid_for<MM, EPI_SWIGLU>(N);                  \
            case EPI_LOGITS: return grid_for<MM, EPI_LOGITS>(N);                  \
        }                                                                         \
        break;
    switch (M) {
        VC_GRID_CASE(1) VC_GRID_CASE(2) VC_GRID_CASE(3) VC_GRID_CASE(4)
        VC_GRID_CASE(5) VC_GRID_CASE(6) VC_GRID_CASE(7) VC_GRID_CASE(8)
    }
#undef VC_GRID_CASE
    return 0;
}

template <int M, int EPI>
static cudaError_t launch_one(const GemvParams &p, cudaStream_t st, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid_for<M, EPI>(p.N));
    cfg.blockDim = dim3(kGemvThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gemv_kernel<M, EPI>, p);
}

cudaError_t launch_gemv(int M, int epi, const GemvParams &p, cudaStream_t st, bool pdl) {
#define VC_LAUNCH_CASE(MM)                                                        \
    case MM:                                                                      \
        switch (epi) {                                                            \
            case EPI_STORE: return launch_one<MM, EPI_STORE>(p, st, pdl);         \
            case EPI_ADD: return launch_one<MM, EPI_ADD>(p, st, pdl);             \
            case EPI_QKV: return launch_one<MM, EPI_QKV>(p, st, pdl);             \
            case EPI_SWIGLU: return launch_one<MM, EPI_SWIGLU>(p, st, pdl);       \
            case EPI_LOGITS: return launch_one<MM, EPI_LOGITS>(p, st, pdl);       \
        }                                                                         \
        break;
    switch (M) {
        VC_LAUNCH_CASE(1) VC_LAUNCH_CASE(2) VC_LAUNCH_CASE(3) VC_LAUNCH_CASE(4)
        VC_LAUNCH_CASE(5) VC_LAUNCH_CASE(6) VC_LAUNCH_CASE(7) VC_LAUNCH_CASE(8)
    }
#undef VC_LAUNCH_CASE
    return cudaErrorInvalidValue;
}

// ---------------------------------------------------------------------------
// Split-K GQA decode attention over the KV ring.
//
// grid (S, 8 KV heads, M streams), 128 threads.  A CTA takes one KV head and
// one contiguous range of keys; its 4 query heads share every K/V load.
// Within a warp, 8 lanes cover one key (16 of the 128 dims each), so a warp
// walks 4 keys at a time with a 3-step shuffle reduction per score.  Each
// lane group keeps the reference's online-softmax state (running max, sum,
// weighted V; voxtral_kernels.c:440-479); groups, warps and finally the S
// splits are merged with the usual rescaling.  The last CTA of each
// (stream, KV head) merges the splits (atomic ticket, no spinning).
// ---------------------------------------------------------------------------

struct SoftState {
    float mx, den;
};

__device__ __forceinline__ void merge_scale(float ma, float da, float mb, float db, float &mn,
                                            float &ca, float &cb) {
    mn = fmaxf(ma, mb);
    ca = (da > 0.f) ? expf(ma - mn) : 0.f;
    cb = (db > 0.f) ? expf(mb - mn) : 0.f;
}

__global__ void __launch_bounds__(128)
attn_decode_kernel(const AttnParams p) {
    const int s = blockIdx.x, kvh = blockIdx.y, m = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int grp = lane >> 3, sl = lane & 7;
    __shared__ float sm_o[4][4][kHeadDim];
    __shared__ float sm_ml[4][4][2];
    __shared__ int s_last;

    grid_dep_wait();
    grid_dep_launch();

    const StreamSlot slt = p.slots[m];
    const int S = p.S;
    const int n_keys = slt.n_keys;
    const int chunk = (n_keys + S - 1) / S;
    const int kb = s * chunk;
    const int ke = min(kb + chunk, n_keys);
    const int first = slt.pos - n_keys + 1;   // logical position of key 0
    const int cap = slt.cap;
    const float scale = 1.0f / sqrtf((float)kHeadDim);

    float q[4][16];
    const float *qb = p.q + (size_t)m * kQDim + (kvh * 4) * kHeadDim + sl * 16;
#pragma unroll
    for (int hh = 0; hh < 4; hh++)
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float4 v = *reinterpret_cast<const float4 *>(qb + hh * kHeadDim + 4 * i);
            q[hh][4 * i] = v.x;
            q[hh][4 * i + 1] = v.y;
            q[hh][4 * i + 2] = v.z;
            q[hh][4 * i + 3] = v.w;
        }

    float mx[4], den[4], o[4][16];
#pragma unroll
    for (int hh = 0; hh < 4; hh++) {
        mx[hh] = -INFINITY;
        den[hh] = 0.f;
#pragma unroll
        for (int d = 0; d < 16; d++) o[hh][d] = 0.f;
    }

    const size_t layer_off = (size_t)p.layer * cap * kKvDim + kvh * kHeadDim + sl * 16;
    const float *kbase = slt.k_ring + layer_off;
    const float *vbase = slt.v_ring + layer_off;

    // The loop bound is warp-uniform (the shuffles below use the full mask);
    // a lane group past the end of the range computes on zeros and skips
    // the update.
    for (int base = kb + warp * 4; base < ke; base += 16) {
        const int i = base + grp;
        const bool valid = i < ke;
        float4 kv[4], vv[4];
        if (valid) {
            const int slot = (first + i) % cap;
            const float4 *kr = reinterpret_cast<const float4 *>(kbase + (size_t)slot * kKvDim);
            const float4 *vr = reinterpret_cast<const float4 *>(vbase + (size_t)slot * kKvDim);
#pragma unroll
            for (int j = 0; j < 4; j++) kv[j] = __ldcg(kr + j);
#pragma unroll
            for (int j = 0; j < 4; j++) vv[j] = __ldcg(vr + j);
        } else {
#pragma unroll
            for (int j = 0; j < 4; j++) kv[j] = vv[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        float sc[4];
#pragma unroll
        for (int hh = 0; hh < 4; hh++) {
            float a = 0.f;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                a = fmaf(q[hh][4 * j], kv[j].x, a);
                a = fmaf(q[hh][4 * j + 1], kv[j].y, a);
                a = fmaf(q[hh][4 * j + 2], kv[j].z, a);
                a = fmaf(q[hh][4 * j + 3], kv[j].w, a);
            }
            a += __shfl_xor_sync(0xffffffffu, a, 1);
            a += __shfl_xor_sync(0xffffffffu, a, 2);
            a += __shfl_xor_sync(0xffffffffu, a, 4);
            sc[hh] = a * scale;
        }
        const float vf[16] = {vv[0].x, vv[0].y, vv[0].z, vv[0].w, vv[1].x, vv[1].y, vv[1].z, vv[1].w,
                              vv[2].x, vv[2].y, vv[2].z, vv[2].w, vv[3].x, vv[3].y, vv[3].z, vv[3].w};
        if (!valid) continue;
#pragma unroll
        for (int hh = 0; hh < 4; hh++) {
            if (sc[hh] > mx[hh]) {
                const float c = expf(mx[hh] - sc[hh]);
                den[hh] = den[hh] * c + 1.0f;
#pragma unroll
                for (int d = 0; d < 16; d++) o[hh][d] = o[hh][d] * c + vf[d];
                mx[hh] = sc[hh];
            } else {
                const float wgt = expf(sc[hh] - mx[hh]);
                den[hh] += wgt;
#pragma unroll
                for (int d = 0; d < 16; d++) o[hh][d] = fmaf(wgt, vf[d], o[hh][d]);
            }
        }
    }

    // merge the 4 lane groups of the warp
#pragma unroll
    for (int off = 8; off <= 16; off <<= 1) {
#pragma unroll
        for (int hh = 0; hh < 4; hh++) {
            const float mo = __shfl_xor_sync(0xffffffffu, mx[hh], off);
            const float dn = __shfl_xor_sync(0xffffffffu, den[hh], off);
            float mn, ca, cb;
            merge_scale(mx[hh], den[hh], mo, dn, mn, ca, cb);
            den[hh] = den[hh] * ca + dn * cb;
#pragma unroll
            for (int d = 0; d < 16; d++) {
                const float oo = __shfl_xor_sync(0xffffffffu, o[hh][d], off);
                o[hh][d] = o[hh][d] * ca + oo * cb;
            }
            mx[hh] = mn;
        }
    }
    if (grp == 0) {
#pragma unroll
        for (int hh = 0; hh < 4; hh++) {
#pragma unroll
            for (int d = 0; d < 16; d++) sm_o[warp][hh][sl * 16 + d] = o[hh][d];
            if (sl == 0) {
                sm_ml[warp][hh][0] = mx[hh];
                sm_ml[warp][hh][1] = den[hh];
            }
        }
    }
    __syncthreads();

    // merge the 4 warps; thread -> (head hh, dims 4*(tid&31)..+3)
    {
        const int hh = tid >> 5, d4 = (tid & 31) * 4;
        float gm = -INFINITY;
        for (int w = 0; w < 4; w++)
            if (sm_ml[w][hh][1] > 0.f) gm = fmaxf(gm, sm_ml[w][hh][0]);
        float gd = 0.f, go[4] = {0.f, 0.f, 0.f, 0.f};
        for (int w = 0; w < 4; w++) {
            const float dw = sm_ml[w][hh][1];
            if (dw > 0.f) {
                const float c = expf(sm_ml[w][hh][0] - gm);
                gd += dw * c;
#pragma unroll
                for (int j = 0; j < 4; j++) go[j] += sm_o[w][hh][d4 + j] * c;
            }
        }
        const int h = kvh * 4 + hh;
        const size_t pidx = ((size_t)m * kDecHeads + h) * S + s;
        *reinterpret_cast<float4 *>(p.part_o + pidx * kHeadDim + d4) = make_float4(go[0], go[1], go[2], go[3]);
        if ((tid & 31) == 0) {
            p.part_ml[pidx * 2] = gm;
            p.part_ml[pidx * 2 + 1] = gd;
        }
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = (atomicAdd(&p.counters[m * kDecKvHeads + kvh], 1u) == (unsigned)(S - 1));
    __syncthreads();
    if (!s_last) return;
    __threadfence();

    {
        const int hh = tid >> 5, d4 = (tid & 31) * 4;
        const int h = kvh * 4 + hh;
        const size_t pbase = ((size_t)m * kDecHeads + h) * S;
        float gm = -INFINITY;
        for (int t = 0; t < S; t++) {
            const float dn = __ldcg(p.part_ml + (pbase + t) * 2 + 1);
            if (dn > 0.f) gm = fmaxf(gm, __ldcg(p.part_ml + (pbase + t) * 2));
        }
        float gd = 0.f, go[4] = {0.f, 0.f, 0.f, 0.f};
        for (int t = 0; t < S; t++) {
            const float dn = __ldcg(p.part_ml + (pbase + t) * 2 + 1);
            if (dn > 0.f) {
                const float c = expf(__ldcg(p.part_ml + (pbase + t) * 2) - gm);
                gd += dn * c;
                const float4 ov = __ldcg(reinterpret_cast<const float4 *>(p.part_o + (pbase + t) * kHeadDim + d4));
                go[0] += ov.x * c;
                go[1] += ov.y * c;
                go[2] += ov.z * c;
                go[3] += ov.w * c;
            }
        }
        const float inv = (gd > 0.f) ? 1.0f / gd : 0.f;
        *reinterpret_cast<float4 *>(p.out + (size_t)m * kQDim + h * kHeadDim + d4) =
            make_float4(go[0] * inv, go[1] * inv, go[2] * inv, go[3] * inv);
        if (tid == 0) p.counters[m * kDecKvHeads + kvh] = 0u;
    }
}

cudaError_t launch_attn_decode(int M, const AttnParams &p, cudaStream_t st, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.S, kDecKvHeads, M);
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
