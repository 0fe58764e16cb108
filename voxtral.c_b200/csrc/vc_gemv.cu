// vc_gemv.cu - the decode-step "GEMV": y[M, N] = x[M, K] . W[N, K]^T for
// M = 1..8 activation rows (streams), with fused prologues and epilogues.
//
// Design (HBM-bound; every launch streams its weight matrix exactly once):
//   * Weights live in a fragment-native tiled layout (built once at upload):
//     16x16 bf16 tiles, each stored as the 32 lanes' mma.m16n8k16 A fragments
//     (16 bytes per lane), tiles of a 16-row band contiguous along K.  One
//     coalesced 16-byte non-allocating load per lane per tile feeds an MMA
//     directly - no shared-memory staging and no shuffles for the weights.
//   * Activations (fp32) are staged once per CTA in shared memory as B
//     fragments, split into bf16 hi + lo parts (x = hi + lo to 2^-17), and
//     both parts are multiplied into one fp32 accumulator, so the result has
//     fp32-level accuracy (<= ~1e-5 relative) although the tensor core only
//     takes bf16.  The 8 MMA columns are the (up to) 8 streams.
//   * A CTA owns 64 output rows (4 row tiles x 2 warps along K) and one
//     K-slice; the KS slices of a row block form a thread-block cluster and
//     are reduced through distributed shared memory by cluster rank 0, which
//     then runs the epilogue.  Deterministic: fixed summation order, no
//     atomics on data.
//   * Programmatic dependent launch: each CTA issues its first weight loads
//     before waiting for the producer of its activations.
#include "vc_common.cuh"
#include "vc_internal.h"

#include <math.h>

namespace vc {

constexpr int kThreads = 256;
constexpr int kWarps = 8;
constexpr int kRT = 4;                 // row tiles per CTA
constexpr int kWK = 2;                 // warps per row tile (split along K)
constexpr int kRowsPerCta = 16 * kRT;  // 64
constexpr int kChunkKB = 80;           // k-blocks (16 wide) of x staged per pass: 40 KB
constexpr int kU = 8;                  // weight tiles in flight per warp
constexpr int kMaxKS = 8;              // cluster size limit (portable)

static_assert(kRT * kWK == kWarps, "warp layout");

__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], const uint4 &a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t bf16_bits_rn(float f) {
    uint32_t u = __float_as_uint(f);
    u += 0x7FFFu + ((u >> 16) & 1u);   // finite inputs only
    return u >> 16;
}

// (hi, lo) bf16 split of two values, packed as the mma B-fragment register.
__device__ __forceinline__ void split2(float v0, float v1, uint32_t &hi, uint32_t &lo) {
    const uint32_t h0 = bf16_bits_rn(v0), h1 = bf16_bits_rn(v1);
    const float r0 = v0 - __uint_as_float(h0 << 16);
    const float r1 = v1 - __uint_as_float(h1 << 16);
    hi = h0 | (h1 << 16);
    lo = bf16_bits_rn(r0) | (bf16_bits_rn(r1) << 16);
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

__device__ __forceinline__ float ld_dsmem_f32(const float *local, uint32_t rank) {
    uint32_t a = (uint32_t)__cvta_generic_to_shared(local), r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(r) : "memory");
    return v;
}

__device__ __forceinline__ bool arg_better(float v, int i, float bv, int bi) {
    return v > bv || (v == bv && i < bi);
}

struct GemvShared {
    uint4 xs[kChunkKB * 32];            // B fragments (hi.x, hi.y, lo.x, lo.y) per (kblock, lane)
    float red[kWarps][32][4];           // per-warp D fragments (split-K within the CTA)
    float part[kRowsPerCta][8];         // this CTA's [rows][streams] partial
    float s_inv[8];
    float s_red[kWarps][8];
    int s_redi[kWarps][8];
    int s_last;
};

template <int M, int EPI>
__global__ void __launch_bounds__(kThreads)
gemv_mma_kernel(const GemvParams p) {
    __shared__ __align__(16) GemvShared sh;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int ks = blockIdx.x, KS = gridDim.x;
    const int rb = blockIdx.y;                        // 64-row block
    const int rt_local = warp / kWK, wk = warp % kWK;
    const int rt = rb * kRT + rt_local;               // 16-row tile
    const int KBp = p.Kp >> 4;                        // k-blocks per row (padded)
    // this CTA's k-block slice
    const int per = (KBp + KS - 1) / KS;
    const int kb0 = ks * per;
    const int kb1 = min(kb0 + per, KBp);
    const uint64_t pol = make_evict_first_policy();
    const uint16_t *wt = p.W + ((size_t)rt * KBp) * 256 + lane * 8;

    // ---- prefetch the first weight tiles (independent of the producer) ----
    uint4 a[kU];
    const int my_first = kb0 + wk;                   // this warp's k-blocks: my_first + kWK*i
    const int n_my = (kb1 > my_first) ? (kb1 - my_first + kWK - 1) / kWK : 0;
#pragma unroll
    for (int u = 0; u < kU; u++)
        a[u] = (u < n_my) ? ldg_stream(wt + (size_t)(my_first + kWK * u) * 256, pol) : make_uint4(0, 0, 0, 0);

    grid_dep_wait();
    grid_dep_launch();

    // ---- RMSNorm statistics (voxtral_kernels.c:346-363) ----
    if (p.norm_w != nullptr) {
        if (p.ss_in != nullptr) {
            if (tid < M) {
                float ss = 0.f;
                for (int j = 0; j < p.ss_parts; j++) ss += p.ss_in[tid * p.ss_parts + j];
                sh.s_inv[tid] = 1.0f / sqrtf(ss / (float)p.K + kNormEps);
            }
        } else {
            for (int m = warp; m < M; m += kWarps) {
                const float *xr = p.x + (size_t)m * p.ldx;
                float ss = 0.f;
                for (int i = lane; i < p.K; i += 32) ss = fmaf(xr[i], xr[i], ss);
                ss = warp_sum(ss);
                if (lane == 0) sh.s_inv[m] = 1.0f / sqrtf(ss / (float)p.K + kNormEps);
            }
        }
    }

    float c[4] = {0.f, 0.f, 0.f, 0.f};
    int done = 0;   // k-blocks of this warp consumed so far
    for (int c0 = kb0; c0 < kb1; c0 += kChunkKB) {
        const int c1 = min(c0 + kChunkKB, kb1);
        __syncthreads();   // previous chunk consumed; s_inv visible
        // ---- stage x[:, 16*c0 .. 16*c1) as split B fragments ----
        for (int item = tid; item < (c1 - c0) * 32; item += kThreads) {
            const int kbl = item >> 5, t = item & 31;
            const int g = t >> 2, q = t & 3;
            uint4 v = make_uint4(0, 0, 0, 0);
            if (g < M) {
                const int k = (c0 + kbl) * 16 + 2 * q;
                const float *xr = p.x + (size_t)g * p.ldx;
                float x0 = (k < p.K) ? xr[k] : 0.f, x1 = (k + 1 < p.K) ? xr[k + 1] : 0.f;
                float x8 = (k + 8 < p.K) ? xr[k + 8] : 0.f, x9 = (k + 9 < p.K) ? xr[k + 9] : 0.f;
                if (p.norm_w != nullptr) {
                    const float inv = sh.s_inv[g];
                    if (k < p.K) x0 = x0 * inv * p.norm_w[k];
                    if (k + 1 < p.K) x1 = x1 * inv * p.norm_w[k + 1];
                    if (k + 8 < p.K) x8 = x8 * inv * p.norm_w[k + 8];
                    if (k + 9 < p.K) x9 = x9 * inv * p.norm_w[k + 9];
                    if (p.ada != nullptr) {  // x_norm *= (1 + ada)  (voxtral_decoder.c:489-492)
                        if (k < p.K) x0 *= (1.0f + p.ada[k]);
                        if (k + 1 < p.K) x1 *= (1.0f + p.ada[k + 1]);
                        if (k + 8 < p.K) x8 *= (1.0f + p.ada[k + 8]);
                        if (k + 9 < p.K) x9 *= (1.0f + p.ada[k + 9]);
                    }
                }
                split2(x0, x1, v.x, v.z);
                split2(x8, x9, v.y, v.w);
            }
            sh.xs[item] = v;
        }
        __syncthreads();

        // ---- stream this warp's weight tiles of the chunk through the MMA ----
        const int n_chunk = (c1 > my_first + kWK * done) ? (c1 - (my_first + kWK * done) + kWK - 1) / kWK : 0;
        for (int i = 0; i < n_chunk; i += kU) {
            if (!(c0 == kb0 && i == 0)) {
#pragma unroll
                for (int u = 0; u < kU; u++) {
                    const int kb = my_first + kWK * (done + i + u);
                    a[u] = (i + u < n_chunk) ? ldg_stream(wt + (size_t)kb * 256, pol) : make_uint4(0, 0, 0, 0);
                }
            }
#pragma unroll
            for (int u = 0; u < kU; u++) {
                if (i + u < n_chunk) {
                    const int kb = my_first + kWK * (done + i + u);
                    const uint4 b = sh.xs[(kb - c0) * 32 + lane];
                    mma_bf16_16816(c, a[u], b.x, b.y);   // W . x_hi
                    mma_bf16_16816(c, a[u], b.z, b.w);   // W . x_lo
                }
            }
        }
        done += n_chunk;
    }

    // ---- reduce the kWK warps of each row tile (fixed order) ----
    if (wk != 0) {
#pragma unroll
        for (int j = 0; j < 4; j++) sh.red[warp][lane][j] = c[j];
    }
    __syncthreads();
    if (wk == 0) {
        for (int w2 = 1; w2 < kWK; w2++)
#pragma unroll
            for (int j = 0; j < 4; j++) c[j] += sh.red[warp + w2][lane][j];
        const int g = lane >> 2, q = lane & 3;
        float *pr = &sh.part[rt_local * 16][0];
        pr[g * 8 + 2 * q] = c[0];
        pr[g * 8 + 2 * q + 1] = c[1];
        pr[(g + 8) * 8 + 2 * q] = c[2];
        pr[(g + 8) * 8 + 2 * q + 1] = c[3];
    }
    __syncthreads();

    // ---- reduce the KS slices of the cluster into rank 0 ----
    if (KS > 1) {
        cluster_sync_all();
        if (cluster_ctarank() == 0) {
            for (int e = tid; e < kRowsPerCta * 8; e += kThreads) {
                float v = (&sh.part[0][0])[e];
                for (int r = 1; r < KS; r++) v += ld_dsmem_f32(&sh.part[0][0] + e, (uint32_t)r);
                (&sh.part[0][0])[e] = v;
            }
        }
        cluster_sync_all();   // peers keep their shared memory until rank 0 has read it
        if (cluster_ctarank() != 0) return;
        __syncthreads();
    }

    // ---- epilogue: thread -> stream m = tid & 7, row pair (2pp, 2pp+1) ----
    const int m = tid & 7, pp = tid >> 3;
    const int r0 = rb * kRowsPerCta + 2 * pp;         // global row of the pair
    const bool active = (m < M) && (r0 < p.N);
    float v0 = sh.part[2 * pp][m], v1 = sh.part[2 * pp + 1][m];

    if constexpr (EPI == EPI_STORE || EPI == EPI_ADD || EPI == EPI_LOGITS) {
        float ss = 0.f;
        if (active) {
            if (p.bias != nullptr) {
                v0 += p.bias[r0];
                if (r0 + 1 < p.N) v1 += p.bias[r0 + 1];
            }
            float *dst = p.y + (size_t)m * p.ldy + r0;
            if constexpr (EPI == EPI_ADD) {
                v0 += dst[0];
                if (r0 + 1 < p.N) v1 += dst[1];
            }
            dst[0] = v0;
            if (r0 + 1 < p.N) dst[1] = v1;
            ss = v0 * v0 + ((r0 + 1 < p.N) ? v1 * v1 : 0.f);
        }
        if constexpr (EPI == EPI_ADD) {
            // per-row-block sum of squares of the new residual, consumed by the
            // next RMSNorm prologue (fixed-order sums: deterministic)
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
                if (r0 + 1 < p.N && v1 > bv) { bv = v1; bi = r0 + 1; }
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
                    float b = -INFINITY;
                    int ib = 0x7fffffff;
                    for (int j = lane; j < (int)gridDim.y; j += 32) {
                        const float v = __ldcg(&p.partials[(size_t)j * M + warp].v);
                        const int i = __ldcg(&p.partials[(size_t)j * M + warp].i);
                        if (arg_better(v, i, b, ib)) { b = v; ib = i; }
                    }
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) {
                        const float ov = __shfl_xor_sync(0xffffffffu, b, o);
                        const int oi = __shfl_xor_sync(0xffffffffu, ib, o);
                        if (arg_better(ov, oi, b, ib)) { b = ov; ib = oi; }
                    }
                    if (lane == 0) p.tokens[warp] = ib;
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
        // (voxtral_kernels.c:369-374, then :34-36)
        if (active) {
            const float sg = v0 / (1.0f + expf(-v0));
            p.y[(size_t)m * p.ldy + (r0 >> 1)] = sg * v1;
        }
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

int gemv_row_blocks(int N) { return (N + kRowsPerCta - 1) / kRowsPerCta; }

int gemv_k_slices(int N, int Kp) {
    const int KB = Kp / 16;
    const int rb = gemv_row_blocks(N);
    int ks = (KB + 63) / 64;                       // <= 1024 k per slice
    const int fill = (2 * 148 + rb - 1) / rb;       // >= ~2 CTAs per SM
    if (fill > ks) ks = fill;
    if (ks > kMaxKS) ks = kMaxKS;
    if (ks > KB / kWK) ks = KB / kWK > 0 ? KB / kWK : 1;   // every warp gets >= 1 k-block
    if (ks < 1) ks = 1;
    return ks;
}

int gemv_grid(int /*M*/, int /*epi*/, int N) { return gemv_row_blocks(N); }

template <int M, int EPI>
static cudaError_t launch_one(const GemvParams &p, cudaStream_t st, bool pdl) {
    const int KS = gemv_k_slices(p.N, p.Kp);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(KS, gemv_row_blocks(p.N));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = 0;
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
    return cudaLaunchKernelEx(&cfg, gemv_mma_kernel<M, EPI>, p);
}

cudaError_t launch_gemv(int M, int epi, const GemvParams &p, cudaStream_t st, bool pdl) {
    if (p.Kp % 16 != 0 || p.Kp < p.K || p.K <= 0 || p.N <= 0) return cudaErrorInvalidValue;
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
// Weight layout: row-major [N, K] bf16 -> fragment-native tiles.  Tile
// (rt, kb) holds rows 16rt..16rt+15, columns 16kb..16kb+15 as the 32 lanes'
// A fragments of mma.m16n8k16 (lane = 4g + q holds rows g and g+8, columns
// 2q, 2q+1, 2q+8, 2q+9); rows beyond N and columns beyond K are zero.
// ---------------------------------------------------------------------------

__global__ void tile_weights_kernel(uint16_t *dst, const uint16_t *src, int N, int K, int Np, int Kp) {
    const int KB = Kp >> 4;
    const size_t n_lanes = (size_t)(Np >> 4) * KB * 32;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n_lanes;
         i += (size_t)gridDim.x * blockDim.x) {
        const int lane = (int)(i & 31);
        const size_t tile = i >> 5;
        const int kb = (int)(tile % KB);
        const int rt = (int)(tile / KB);
        const int g = lane >> 2, q = lane & 3;
        const int ra = rt * 16 + g, rb = ra + 8;
        const int k0 = kb * 16 + 2 * q;
        auto at = [&](int r, int k) -> uint16_t {
            return (r < N && k < K) ? src[(size_t)r * K + k] : (uint16_t)0;
        };
        uint4 v;
        v.x = at(ra, k0) | ((uint32_t)at(ra, k0 + 1) << 16);
        v.y = at(rb, k0) | ((uint32_t)at(rb, k0 + 1) << 16);
        v.z = at(ra, k0 + 8) | ((uint32_t)at(ra, k0 + 9) << 16);
        v.w = at(rb, k0 + 8) | ((uint32_t)at(rb, k0 + 9) << 16);
        reinterpret_cast<uint4 *>(dst)[i] = v;
    }
}

cudaError_t launch_tile_weights(uint16_t *dst, const uint16_t *src, int N, int K, int Np, int Kp,
                                cudaStream_t st) {
    tile_weights_kernel<<<148 * 16, 256, 0, st>>>(dst, src, N, K, Np, Kp);
    return cudaGetLastError();
}

}  // namespace vc
