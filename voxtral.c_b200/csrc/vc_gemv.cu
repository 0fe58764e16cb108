// vc_gemv.cu - the decode-step "GEMV": y[M, N] = x[M, K] . W[N, K]^T for
// M = 1..8 activation rows (streams), with fused epilogues.
//
// Design (HBM-bound: every launch streams its weight matrix exactly once):
//   * Weights live in a fragment-native tiled layout built once at upload:
//     64-row blocks; inside a block, for each 16-wide k-block, the four 16x16
//     tiles are stored as the 32 lanes' mma.m16n8k16 A fragments (16 bytes per
//     lane), so a row block is one contiguous stream along K.
//   * Activations arrive pre-formatted as B fragments ("xfrag"): per k-block,
//     lane 4g+q holds stream g's values at k = 2q, 2q+1, 2q+8, 2q+9, each
//     split into bf16 hi + lo (x = hi + lo to ~2^-17).  The producer of the
//     activations (the previous kernel's epilogue, or vc_prep_xfrag) writes
//     them; an RMSNorm consumer gets x * norm_weight (* (1 + ada)) and applies
//     1/rms, a per-stream scalar, to its accumulators.  Both halves are
//     multiplied into one fp32 accumulator: fp32-level accuracy from bf16 MMAs.
//   * A CTA owns one 64-row block and one K-slice.  Thread 0 streams the slice
//     through a 5-stage shared-memory ring with cp.async.bulk (TMA bulk copies,
//     L2 evict-first) completing on mbarriers; the 8 warps each take one
//     k-block per stage (4 tiles x hi/lo = 8 MMAs).  The weight copies of the
//     first stages are issued before griddepcontrol.wait (programmatic
//     dependent launch), i.e. while the producer kernel is still running.
//   * KS K-slices of a row block form a thread-block cluster and are summed
//     through distributed shared memory by cluster rank 0, which runs the
//     epilogue.  Fixed summation order everywhere: deterministic.
//   * Every mbarrier wait is bounded (2 s of %globaltimer); on expiry the CTA
//     raises the launch's error word, which the host reads with the tokens.
#include "vc_common.cuh"
#include "vc_internal.h"

#include <math.h>
#include <stdlib.h>

namespace vc {

constexpr int kThreads = 256;
constexpr int kWarps = 8;
constexpr int kRT = 4;                   // 16-row tiles per row block
constexpr int kRowsPerCta = 16 * kRT;    // 64
constexpr int kStageKB = 8;              // k-blocks per stage (one per warp)
constexpr int kStages = 5;
constexpr int kStageW = kStageKB * kRT * 512;   // 16 KB of weights
constexpr int kStageB = kStageKB * 512;         // 4 KB of activation fragments
constexpr int kMaxKS = 8;                // cluster size limit (portable)
static_assert(kMaxKS * kRowsPerCta * 8 * 4 <= kStageW + kStageB, "cluster reduction area fits a stage");
constexpr unsigned long long kWaitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], const uint4 &a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait: false once the launch's deadline has passed.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint64_t deadline) {
    while (!mbar_try_wait(bar, parity))
        if (globaltimer() > deadline) return false;
    return true;
}

__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n"
                 "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// store v at the same shared-memory offset as `local`, in cluster CTA `rank`
__device__ __forceinline__ void st_dsmem_f32(float *local, uint32_t rank, float v) {
    uint32_t a = smem_u32(local), r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(r), "f"(v) : "memory");
}

__device__ __forceinline__ bool arg_better(float v, int i, float bv, int bi) {
    return v > bv || (v == bv && i < bi);
}

struct GemvShared {
    uint64_t full[kStages], empty[kStages];
    alignas(128) unsigned char stage[kStages][kStageW + kStageB];
    float part[kRowsPerCta][8];
    float s_inv[8];
    float s_red[kWarps][8];
    int s_redi[kWarps][8];
    int s_last;
};

template <int M, int EPI>
__global__ void __launch_bounds__(kThreads, 2)
gemv_tma_kernel(const GemvParams p) {
    extern __shared__ __align__(128) unsigned char dsm[];
    GemvShared &sh = *reinterpret_cast<GemvShared *>(dsm);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int ks = blockIdx.x, KS = gridDim.x;
    const int rb = blockIdx.y;
    const int KB = p.Kp >> 4;
    const int per = (KB + KS - 1) / KS;
    const int kb0 = ks * per;
    const int nkb = max(0, min(kb0 + per, KB) - kb0);
    const int n_it = (nkb + kStageKB - 1) / kStageKB;
    const uint64_t deadline = globaltimer() + kWaitNs;
    const uint16_t *wsrc = p.W + ((size_t)rb * KB + kb0) * (kRT * 256);
    const uint32_t *bsrc = p.xfrag + (size_t)kb0 * 128;
    bool ok = true;

    if (tid == 0) {
        for (int s = 0; s < kStages; s++) {
            mbar_init(&sh.full[s], 1);
            mbar_init(&sh.empty[s], kWarps);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    const uint64_t pol = make_evict_first_policy();    // weights: streamed once
    const uint64_t pol_x = make_evict_last_policy();   // activations: re-read by every row block
    auto stage_kbs = [&](int it) { return min(kStageKB, nkb - it * kStageKB); };
    // weights of the first stages: independent of the producer kernel
    if (tid == 0) {
        for (int it = 0; it < min(kStages, n_it); it++) {
            const int n = stage_kbs(it);
            mbar_expect_tx(&sh.full[it], (uint32_t)n * (kRT * 512 + 512));
            bulk_g2s(sh.stage[it], wsrc + (size_t)it * kStageKB * kRT * 256, (uint32_t)n * kRT * 512,
                     &sh.full[it], pol);
        }
        // the first bytes of the next weight stream, behind this CTA's own
        // first stages: HBM stays busy through this launch's reduction tail
        // and the next one's ramp
        l2_prefetch_share(p.pf, p.pf_bytes);
    }
    grid_dep_wait();
    grid_dep_launch();
    if (tid == 0) {
        for (int it = 0; it < min(kStages, n_it); it++)
            bulk_g2s(sh.stage[it] + kStageW, bsrc + (size_t)it * kStageKB * 128, (uint32_t)stage_kbs(it) * 512,
                     &sh.full[it], pol_x);
    }

    float acc[kRT][4];
#pragma unroll
    for (int t = 0; t < kRT; t++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[t][j] = 0.f;

    for (int it = 0; it < n_it; it++) {
        const int s = it % kStages;
        const uint32_t par = (uint32_t)(it / kStages) & 1u;
        // every lane polls (acquire); the decision to give up is warp-uniform
        if (!__all_sync(0xffffffffu, mbar_wait(&sh.full[s], par, deadline))) {
            ok = false;
            break;
        }
        if (warp < stage_kbs(it)) {
            const unsigned char *st = sh.stage[s];
            const uint4 b = *reinterpret_cast<const uint4 *>(st + kStageW + warp * 512 + lane * 16);
#pragma unroll
            for (int t = 0; t < kRT; t++) {
                const uint4 a = *reinterpret_cast<const uint4 *>(st + (warp * kRT + t) * 512 + lane * 16);
                mma_bf16_16816(acc[t], a, b.x, b.y);   // W . x_hi
                mma_bf16_16816(acc[t], a, b.z, b.w);   // W . x_lo
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sh.empty[s]);
        if (warp == 0) {
            // thread 0 refills this stage once all 8 warps have released it
            bool refill_ok = true;
            if (lane == 0 && it + kStages < n_it) {
                refill_ok = mbar_wait(&sh.empty[s], par, deadline);
                if (refill_ok) {
                    const int nx = it + kStages, n = stage_kbs(nx);
                    mbar_expect_tx(&sh.full[s], (uint32_t)n * (kRT * 512 + 512));
                    bulk_g2s(sh.stage[s], wsrc + (size_t)nx * kStageKB * kRT * 256,
                             (uint32_t)n * kRT * 512, &sh.full[s], pol);
                    bulk_g2s(sh.stage[s] + kStageW, bsrc + (size_t)nx * kStageKB * 128, (uint32_t)n * 512,
                             &sh.full[s], pol_x);
                }
            }
            if (!__shfl_sync(0xffffffffu, refill_ok, 0)) {
                ok = false;
                break;
            }
        }
    }
    if (!ok) {
        // report, then let copies that may still be in flight land before
        // the CTA (and its shared memory) goes away
        if (lane == 0) atomicExch(p.err, 1u);
        const uint64_t grace = globaltimer() + 10000000ull;
        while (globaltimer() < grace) {
        }
    }
    __syncthreads();   // all stages consumed: the ring is reused below
    // tell the cluster this CTA's ring is free (its peers will write into it)
    if (KS > 1) asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");

    // ---- reduce the 8 warps (fixed order) ----
    float *red = reinterpret_cast<float *>(sh.stage[0]);   // [8 warps][4 tiles][32 lanes][4]
#pragma unroll
    for (int t = 0; t < kRT; t++)
#pragma unroll
        for (int j = 0; j < 4; j++) red[((warp * kRT + t) * 32 + lane) * 4 + j] = acc[t][j];
    __syncthreads();
    for (int e = tid; e < kRT * 32 * 4; e += kThreads) {
        float v = 0.f;
        for (int w = 0; w < kWarps; w++) v += red[w * kRT * 128 + e];
        const int t = e >> 7, ln = (e >> 2) & 31, j = e & 3;
        const int g = ln >> 2, q = ln & 3;
        sh.part[t * 16 + g + ((j >> 1) << 3)][2 * q + (j & 1)] = v;
    }
    __syncthreads();

    // ---- reduce the KS slices of the cluster into rank 0: each peer stores
    // its partial into rank 0's (drained) ring; rank 0 sums in rank order ----
    if (KS > 1) {
        asm volatile("barrier.cluster.wait.aligned;" ::: "memory");   // all rings drained
        const uint32_t rank = cluster_ctarank();
        float *area = reinterpret_cast<float *>(sh.stage[1]);         // [KS][64*8]
        if (rank != 0)
            for (int e = tid; e < kRowsPerCta * 8; e += kThreads)
                st_dsmem_f32(area + rank * (kRowsPerCta * 8) + e, 0u, (&sh.part[0][0])[e]);
        cluster_sync_all();   // the peers' stores are visible in rank 0
        if (rank != 0) return;
        for (int e = tid; e < kRowsPerCta * 8; e += kThreads) {
            float v = (&sh.part[0][0])[e];
            for (int r = 1; r < KS; r++) v += area[r * (kRowsPerCta * 8) + e];
            (&sh.part[0][0])[e] = v;
        }
        __syncthreads();
    }
    if (warp == 0) {
        // RMSNorm consumer (voxtral_kernels.c:346-363): each stream's
        // 1/sqrt(mean(x^2) + eps) from the producer's per-row-block sums of
        // x^2.  Lane = (stream lane & 7, part group lane >> 3): four loads in
        // flight per stream; the groups' sums are added in a fixed order.
        float ss = 0.f;
        const int sm = lane & 7;
        if (p.ss_in != nullptr && sm < M)
            for (int j = lane >> 3; j < p.ss_parts; j += 4) ss += __ldcg(p.ss_in + sm * p.ss_parts + j);
        ss += __shfl_xor_sync(0xffffffffu, ss, 8);
        ss += __shfl_xor_sync(0xffffffffu, ss, 16);
        if (lane < 8) sh.s_inv[lane] = (p.ss_in != nullptr && lane < M) ? 1.0f / sqrtf(ss / (float)p.K + kNormEps) : 1.0f;
    }
    __syncthreads();

    // ---- epilogue: thread -> stream m = tid & 7, row pair (2pp, 2pp+1) ----
    const int m = tid & 7, pp = tid >> 3;
    const int r0 = rb * kRowsPerCta + 2 * pp;
    const bool active = (m < M) && (r0 < p.N);
    const bool has1 = r0 + 1 < p.N;
    float v0 = sh.part[2 * pp][m] * sh.s_inv[m];
    float v1 = sh.part[2 * pp + 1][m] * sh.s_inv[m];

    if constexpr (EPI == EPI_STORE || EPI == EPI_ADD || EPI == EPI_LOGITS) {
        float ss = 0.f;
        if (active) {
            if (p.bias != nullptr) {
                v0 += p.bias[r0];
                if (has1) v1 += p.bias[r0 + 1];
            }
            float *dst = p.y + (size_t)m * p.ldy + r0;
            if constexpr (EPI == EPI_ADD) {
                v0 += dst[0];
                if (has1) v1 += dst[1];
            }
            dst[0] = v0;
            if (has1) dst[1] = v1;
            if (!has1) v1 = 0.f;
            ss = v0 * v0 + v1 * v1;
            if constexpr (EPI == EPI_ADD) {
                // the next GEMV's activations: y * g_next as B fragments
                if (p.xfrag_out != nullptr) {
                    const float g0 = p.g_next ? p.g_next[r0] : 1.0f;
                    const float g1 = (p.g_next && has1) ? p.g_next[r0 + 1] : 1.0f;
                    xfrag_put2(p.xfrag_out, m, r0, v0 * g0, v1 * g1);
                }
            }
        }
        if constexpr (EPI == EPI_ADD) {
            // per-row-block sum of squares of the new residual, for the next
            // RMSNorm (fixed-order sums: deterministic)
            if (p.ss_out != nullptr) {
                ss += __shfl_xor_sync(0xffffffffu, ss, 8);
                ss += __shfl_xor_sync(0xffffffffu, ss, 16);
                if (lane < 8) sh.s_red[warp][lane] = ss;
                __syncthreads();
                if (tid < M) {
                    float t = 0.f;
                    for (int w = 0; w < kWarps; w++) t += sh.s_red[w][tid];
                    p.ss_out[tid * gridDim.y + rb] = t;
                }
            }
        }
        if constexpr (EPI == EPI_LOGITS) {
            // first maximum over the vocabulary (voxtral_decoder.c:507-515)
            float bv = -INFINITY;
            int bi = 0x7fffffff;
            if (active) {
                bv = v0;
                bi = r0;
                if (has1 && v1 > bv) { bv = v1; bi = r0 + 1; }
            }
#pragma unroll
            for (int o = 8; o <= 16; o <<= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (arg_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
            }
            if (lane < 8) {
                sh.s_red[warp][lane] = bv;
                sh.s_redi[warp][lane] = bi;
            }
            __syncthreads();
            if (tid < M) {
                float b = -INFINITY;
                int ib = 0x7fffffff;
                for (int w = 0; w < kWarps; w++)
                    if (arg_better(sh.s_red[w][tid], sh.s_redi[w][tid], b, ib)) {
                        b = sh.s_red[w][tid];
                        ib = sh.s_redi[w][tid];
                    }
                p.partials[(size_t)rb * M + tid] = {b, ib};
                __threadfence();
            }
            __syncthreads();
            if (tid == 0) sh.s_last = (atomicAdd(p.counter, 1u) == gridDim.y - 1);
            __syncthreads();
            if (sh.s_last) {
                __threadfence();
                if (warp < M) {
                    // 2048 partials at the 4B vocabulary: 8 loads in flight per
                    // lane (one 8-byte (value, index) load each), not one
                    float b = -INFINITY;
                    int ib = 0x7fffffff;
                    const int G = (int)gridDim.y;
                    const int2 *pp = reinterpret_cast<const int2 *>(p.partials);
                    for (int j0 = lane; j0 < G; j0 += 32 * 8) {
                        int2 t[8];
#pragma unroll
                        for (int u = 0; u < 8; u++) {
                            const int j = j0 + 32 * u;
                            t[u] = j < G ? __ldcg(pp + (size_t)j * M + warp) : make_int2(__float_as_int(-INFINITY),
                                                                                          0x7fffffff);
                        }
#pragma unroll
                        for (int u = 0; u < 8; u++) {
                            const float v = __int_as_float(t[u].x);
                            if (arg_better(v, t[u].y, b, ib)) { b = v; ib = t[u].y; }
                        }
                    }
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) {
                        const float ov = __shfl_xor_sync(0xffffffffu, b, o);
                        const int oi = __shfl_xor_sync(0xffffffffu, ib, o);
                        if (arg_better(ov, oi, b, ib)) { b = ov; ib = oi; }
                    }
                    if (lane == 0) {
                        p.tokens[warp] = ib;
                        if (p.tokens_to != nullptr) {
                            int *dst = *p.tokens_to;   // the caller's buffer of this step
                            if (dst != nullptr) dst[warp] = ib;
                        }
                    }
                }
                if (tid == 0) *p.counter = 0u;
            }
        }
    } else if constexpr (EPI == EPI_QKV) {
        // rows [0,4096): q, [4096,5120): k, [5120,6144): v.  q and k pairs
        // (2d, 2d+1) are rotated by the step's (cos, sin)[d] (vox_apply_rope,
        // voxtral_kernels.c:502-526); k and v go to the ring slot of the
        // step's position (voxtral_decoder.c:474-475).
        if (active) {
            const StreamSlot sl = p.slots[m];
            const size_t ring_row = ((size_t)p.layer * sl.cap + sl.slot) * kKvDim;
            if (r0 < kQDim + kKvDim) {
                const int d = (r0 & (kHeadDim - 1)) >> 1;
                const float cs = p.rope[m * kHeadDim + 2 * d];
                const float sn = p.rope[m * kHeadDim + 2 * d + 1];
                const float oa = __fsub_rn(__fmul_rn(v0, cs), __fmul_rn(v1, sn));
                const float ob = __fadd_rn(__fmul_rn(v0, sn), __fmul_rn(v1, cs));
                float *dst = (r0 < kQDim) ? p.y + (size_t)m * p.ldy + r0
                                          : sl.k_ring + ring_row + (r0 - kQDim);
                dst[0] = oa;
                dst[1] = ob;
            } else {
                float *dst = sl.v_ring + ring_row + (r0 - kQDim - kKvDim);
                dst[0] = v0;
                dst[1] = v1;
            }
        }
    } else if constexpr (EPI == EPI_SWIGLU) {
        // rows (2i, 2i+1) = (gate_i, up_i): h_i = silu(g) * u
        // (voxtral_kernels.c:369-374, then :34-36), written as the w2 GEMV's
        // B fragments
        if (active) {
            const float sg = v0 / (1.0f + expf(-v0));
            xfrag_put1(p.xfrag_out, m, r0 >> 1, sg * v1);
        }
    }
}

// ---------------------------------------------------------------------------
// Activations -> B fragments (for the first GEMV of a chain and for the
// general matmul entry): xfrag = x * g, plus per-64-row-block sums of x^2
// when ss_out is given.  grid = ceil(K / 64), 256 threads.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
prep_xfrag_kernel(const float *x, int M, int K, int ldx, const float *g, uint32_t *xfrag, float *ss_out) {
    __shared__ float s_red[8][8];
    grid_dep_wait();
    grid_dep_launch();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int m = tid & 7, pp = tid >> 3;
    const int k0 = blockIdx.x * 64 + 2 * pp;
    float ss = 0.f;
    if (m < M && k0 < K) {
        const float v0 = x[(size_t)m * ldx + k0];
        const float v1 = (k0 + 1 < K) ? x[(size_t)m * ldx + k0 + 1] : 0.f;
        ss = v0 * v0 + v1 * v1;
        const float g0 = g ? g[k0] : 1.0f, g1 = (g && k0 + 1 < K) ? g[k0 + 1] : 1.0f;
        xfrag_put2(xfrag, m, k0, v0 * g0, v1 * g1);
    }
    if (ss_out != nullptr) {
        ss += __shfl_xor_sync(0xffffffffu, ss, 8);
        ss += __shfl_xor_sync(0xffffffffu, ss, 16);
        if (lane < 8) s_red[warp][lane] = ss;
        __syncthreads();
        if (tid < M) {
            float t = 0.f;
            for (int w = 0; w < 8; w++) t += s_red[w][tid];
            ss_out[tid * gridDim.x + blockIdx.x] = t;
        }
    }
}

cudaError_t launch_prep_xfrag(const float *x, int M, int K, int ldx, const float *g, uint32_t *xfrag,
                              float *ss_out, cudaStream_t st, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((K + 63) / 64);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, prep_xfrag_kernel, x, M, K, ldx, g, xfrag, ss_out);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

int gemv_row_blocks(int N) { return (N + kRowsPerCta - 1) / kRowsPerCta; }

// K-slices per row block.  Measured on B200 (launch lists of the decode
// step): ~1.3 CTAs per SM (192 CTAs) is the sweet spot - enough weight bytes
// in flight, a single wave, small slice clusters; more slices add cluster
// and epilogue cost, fewer leave SMs idle.
int gemv_k_slices(int N, int Kp) {
    static int target = 0, max_ks = -1;
    if (target == 0) {
        int dev = 0, sms = 148;
        if (cudaGetDevice(&dev) == cudaSuccess)
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        target = (sms * 4) / 3;
        // tuning knob: VOX_CUDA_GEMV_MAXKS caps the K-split (default 6)
        const char *e = getenv("VOX_CUDA_GEMV_MAXKS");
        max_ks = (e && atoi(e) >= 1 && atoi(e) <= kMaxKS) ? atoi(e) : 6;
    }
    const int KB = Kp / 16;
    const int rb = gemv_row_blocks(N);
    int ks = (target + rb / 2) / rb;
    if (ks > max_ks) ks = max_ks;
    const int max_by_k = (KB + kStageKB - 1) / kStageKB;   // >= one stage per slice
    if (ks > max_by_k) ks = max_by_k;
    if (ks < 1) ks = 1;
    // every slice must own at least one k-block
    while (ks > 1 && (KB + ks - 1) / ks * (ks - 1) >= KB) ks--;
    return ks;
}

int gemv_grid(int /*M*/, int /*epi*/, int N) { return gemv_row_blocks(N); }

size_t xfrag_bytes(int K) { return (size_t)((K + 15) / 16) * 512; }

template <int M, int EPI>
static cudaError_t launch_one(const GemvParams &p, cudaStream_t st, bool pdl) {
    static bool attr_set = false;   // benign race: same value written
    const int smem = (int)sizeof(GemvShared);
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(gemv_tma_kernel<M, EPI>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    const int KS = gemv_k_slices(p.N, p.Kp);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(KS, gemv_row_blocks(p.N));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (pdl) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        na++;
    }
    if (KS > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = KS;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = 1;
        na++;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, gemv_tma_kernel<M, EPI>, p);
}

cudaError_t launch_gemv(int M, int epi, const GemvParams &p, cudaStream_t st, bool pdl) {
    if (p.Kp % 16 != 0 || p.Kp < p.K || p.K <= 0 || p.N <= 0 || !p.xfrag || !p.err)
        return cudaErrorInvalidValue;
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
// Weight layout: row-major [N, K] bf16 -> 64-row blocks; inside a block, per
// 16-wide k-block, tiles t = 0..3 (rows 16t..16t+15 of the block) as the 32
// lanes' A fragments of mma.m16n8k16 (lane = 4g + q holds rows g, g+8 and
// columns 2q, 2q+1, 2q+8, 2q+9).  Rows past N and columns past K are zero.
// ---------------------------------------------------------------------------

__global__ void tile_weights_kernel(uint16_t *dst, const uint16_t *src, int N, int K, int Np, int Kp) {
    const int KB = Kp >> 4;
    const size_t n_lanes = (size_t)(Np >> 4) * KB * 32;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n_lanes;
         i += (size_t)gridDim.x * blockDim.x) {
        const int lane = (int)(i & 31);
        const size_t tile = i >> 5;                 // (rb, kb, t) with t fastest
        const int t = (int)(tile & 3);
        const size_t rbkb = tile >> 2;
        const int kb = (int)(rbkb % KB);
        const int rblk = (int)(rbkb / KB);
        const int g = lane >> 2, q = lane & 3;
        const int ra = rblk * 64 + t * 16 + g, rbw = ra + 8;
        const int k0 = kb * 16 + 2 * q;
        auto at = [&](int r, int k) -> uint32_t {
            return (r < N && k < K) ? (uint32_t)src[(size_t)r * K + k] : 0u;
        };
        uint4 v;
        v.x = at(ra, k0) | (at(ra, k0 + 1) << 16);
        v.y = at(rbw, k0) | (at(rbw, k0 + 1) << 16);
        v.z = at(ra, k0 + 8) | (at(ra, k0 + 9) << 16);
        v.w = at(rbw, k0 + 8) | (at(rbw, k0 + 9) << 16);
        reinterpret_cast<uint4 *>(dst)[i] = v;
    }
}

cudaError_t launch_tile_weights(uint16_t *dst, const uint16_t *src, int N, int K, int Np, int Kp,
                                cudaStream_t st) {
    if (Np % kRowsPerCta != 0 || Kp % 16 != 0) return cudaErrorInvalidValue;
    tile_weights_kernel<<<148 * 16, 256, 0, st>>>(dst, src, N, K, Np, Kp);
    return cudaGetLastError();
}

// One thread per pair of columns (k, k+1) of one row: the pair is one 32-bit
// word of the tiled layout (the inverse of tile_weights_kernel's mapping).
__global__ void embed_tokens_kernel(float *x, const float *const *row_ptrs, const float *rows, size_t row_stride,
                                    const int *tokens, int n, const uint16_t *E, int vocab, int K,
                                    unsigned *err) {
    const int m = blockIdx.y;
    const int k = 2 * (blockIdx.x * blockDim.x + threadIdx.x);
    if (m >= n || k >= K) return;
    const int tok = tokens[m];
    const bool valid = tok >= 0 && tok < vocab;
    float e0 = 0.f, e1 = 0.f;
    if (valid) {
        const int KB = (K + 15) >> 4;
        const int t = (tok >> 4) & 3, rr = tok & 15, g = rr & 7, hi = rr >> 3;
        const int kb = k >> 4, kk = k & 15, q = (kk & 7) >> 1, khalf = kk >> 3;
        const size_t word = ((((size_t)(tok >> 6) * KB + kb) * 4 + t) * 32 + g * 4 + q) * 4 + khalf * 2 + hi;
        const uint32_t v = reinterpret_cast<const uint32_t *>(E)[word];
        e0 = __uint_as_float(v << 16);
        e1 = __uint_as_float(v & 0xffff0000u);
    } else if (k == 0 && err) {
        atomicOr(err, 2u);
    }
    const float *r = row_ptrs ? row_ptrs[m] : (rows ? rows + (size_t)m * row_stride : nullptr);
    float a0 = 0.f, a1 = 0.f;
    if (r) {
        a0 = r[k];
        if (k + 1 < K) a1 = r[k + 1];
    }
    x[(size_t)m * K + k] = a0 + e0;
    if (k + 1 < K) x[(size_t)m * K + k + 1] = a1 + e1;
}

cudaError_t launch_embed_tokens(float *x, const float *const *row_ptrs, const float *rows, size_t row_stride,
                                const int *tokens, int n, const uint16_t *E, int vocab, int K,
                                unsigned *err, cudaStream_t st) {
    if (n <= 0 || K <= 0 || (K & 1)) return cudaErrorInvalidValue;
    dim3 grid((K / 2 + 255) / 256, n);
    embed_tokens_kernel<<<grid, 256, 0, st>>>(x, row_ptrs, rows, row_stride, tokens, n, E, vocab, K, err);
    return cudaGetLastError();
}

}  // namespace vc
