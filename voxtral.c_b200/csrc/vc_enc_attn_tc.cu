// vc_enc_attn_tc.cu - encoder sliding-window attention on the tcgen05 tensor
// cores (vox_causal_attention for seq_q = new_len, window 750, 32 heads x 64,
// voxtral_kernels.c:412-482 as called at voxtral_encoder.c:574-576).
//
// One CTA = 128 query rows of one head (TMEM lane = query row), 192 or 320
// threads, three CTAs per SM (73 KB shared memory, 128 TMEM columns) so that
// a 1500-row chunk's 12 x 32 tiles run in one wave:
//   warp 0 (one thread)  TMA: the Q tile once, then 64-key blocks of K and V
//                        from the fp16 ring: K into a 3-deep ring (a slot is
//                        free once its S MMA completes), V into a 2-deep one
//                        (free once its P.V MMA completes)
//   warp 1 (one thread)  MMAs: S_b = Q K_b^T (M 128, N 64, K 64) into TMEM
//                        columns [0,64); O += P_b V_b (M 128, N 64, K 64, V
//                        an MN-major operand) accumulating in columns [64,128)
//   warps 2-5 (2-9)      softmax, one (two) warp(s) per TMEM lane quarter,
//                        thread = row, each warp 64 (32) of the block's 64 key
//                        columns: tcgen05.ld of its columns of S_b, mask (the row's own
//                        window [pos - 749, pos]), the row's block max over
//                        both halves (exchanged through shared memory under a
//                        64-thread named barrier per quarter), its half of
//                        P_b = 2^(s - m) as fp16 into shared memory (the A
//                        operand of the O MMA), its half's row sum in fp32;
//                        at the end its 32 columns of O / l (l summed over
//                        both halves) as fp16 (or bf16) for the wo GEMM
// The running max m of a row moves only when a block's max exceeds it by more
// than 2^8 (P stays <= 256, exact enough in fp16 and fp32); then the thread
// rescales its O row in TMEM (tcgen05.ld / st) and its sum after writing
// P_b.  As soon as the softmax warps have read S_b into registers the MMA
// warp issues S_{b+1} (S has one TMEM buffer), so that MMA overlaps the
// exponentials of block b; once P_b is in shared memory it issues
// O += P_b V_b.  The softmax takes the max of S_{b+1} before it waits for that
// O MMA (whose completion also frees P).  Key blocks start at multiples of 64
// positions and the ring capacity is a multiple of 128, so a block never
// wraps in the ring.  Every mbarrier wait is bounded (2 s of %globaltimer);
// on expiry the CTA raises the error word and exits after a grace period;
// the softmax warps then run their remaining blocks with every wait failing
// at once, so both warps of a pair reach every named barrier.
// Key split (chunks with few row tiles, e.g. 100 rows = 32 tiles): blockIdx.z
// takes consecutive key blocks of the tile's range; the softmax threads leave
// their row's unnormalised o, running max and sum in a workspace, and the
// last of the tile's ksplit CTAs to finish (atomic ticket) merges them.
#include "vc_common.cuh"
#include "vc_internal.h"
#include "vc_tc.cuh"

#include <cuda_fp16.h>
#include <math.h>
#include <stdlib.h>

#include <atomic>
#include <mutex>

namespace vc {

using namespace tc;

constexpr int kFaRows = 128;      // query rows per CTA = TMEM lanes
constexpr int kFaKeys = 64;       // keys per block
// softmax warps: NH (1 or 2) per TMEM lane quarter; 64 + 128 NH threads
constexpr int fa_threads(int nh) { return 64 + 128 * nh; }
constexpr int kFaTmemCols = 128;  // S [0,64), O [64,128)
constexpr uint64_t kFaWaitNs = 2000000000ull;
constexpr float kFaRescale = 8.0f;   // log2 of the largest P before the max moves
constexpr int kFaKStages = 3;        // K ring depth
constexpr int kFaVStages = 2;        // V ring depth
constexpr int kFaPartFloats = kEncHeadDim + 4;   // a key split's row partial: o, max, sum (16-byte rows)
constexpr int kFaMaxSplit = 8;                   // key splits at most
constexpr size_t kFaSpreadSmem = 120 * 1024;     // > half an SM's shared memory: one CTA per SM

struct FaSmem {
    unsigned char q[kFaRows * 128];                // Q [128 rows][64 dims] fp16, 128-byte swizzle
    unsigned char k[kFaKStages][kFaKeys * 128];    // K blocks [64 keys][64 dims]
    unsigned char v[kFaVStages][kFaKeys * 128];    // V blocks [64 keys][64 dims] (MN-major B of P.V)
    unsigned char p[kFaRows * 128];                // P [128 rows][64 keys], K-major
    uint64_t q_full, s_full, s_free, p_full, o_full;
    uint64_t k_full[kFaKStages], k_empty[kFaKStages];
    uint64_t v_full[kFaVStages], v_empty[kFaVStages];
    uint32_t tmem;
    float mx[2][kFaRows];   // the two halves' row maxima (then row sums)
    int last;   // key split: this CTA merges
};

// Instruction descriptor, kind::f16 with fp16 A and B (format 0), fp32 D;
// b_mn: B is MN-major (bit 16).
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, bool b_mn) {
    return (1u << 4) | (b_mn ? (1u << 16) : 0u) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Shared-memory descriptor of an MN-major operand in the 128-byte-swizzle
// canonical layout whose MN extent is one 64-element atom: rows of 128 bytes
// along K, 8-row groups 1024 bytes apart (stride byte offset); the leading
// byte offset (between MN atoms) is unused at this width.
__device__ __forceinline__ uint64_t smem_desc_sw128_mn(const void *p) {
    const uint64_t addr = smem_u32(p);
    return ((addr >> 4) & 0x3FFFull) | ((uint64_t)(16384 >> 4) << 16) | ((uint64_t)(1024 >> 4) << 32) |
           (1ull << 46) | (2ull << 61);
}

// barrier `id` over `n` threads (whole warps; id 0 is __syncthreads')
__device__ __forceinline__ void named_bar_sync(int id, int n) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ uint32_t half2_bits(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// the output pair as fp16 (f16) or bf16
__device__ __forceinline__ uint32_t out16x2(float a, float b, int f16) {
    return f16 ? half2_bits(a, b) : (bf16_bits_rn(a) | (bf16_bits_rn(b) << 16));
}

template <int NH>
__global__ void __launch_bounds__(64 + 128 * NH, 3)
enc_attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const EncAttnParams p) {
    extern __shared__ __align__(1024) unsigned char fa_smem_raw[];
    FaSmem &sh = *reinterpret_cast<FaSmem *>(fa_smem_raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r0 = blockIdx.x * kFaRows, head = blockIdx.y;
    const uint64_t deadline = globaltimer() + kFaWaitNs;
    bool ok = (smem_u32(fa_smem_raw) & 1023u) == 0;   // the swizzled tiles need 1024-byte alignment

    if (threadIdx.x == 0) {
        mbar_init(&sh.q_full, 1);
        mbar_init(&sh.s_full, 1);
        mbar_init(&sh.s_free, 4 * NH);   // one arrival per softmax warp
        mbar_init(&sh.p_full, 4 * NH);
        mbar_init(&sh.o_full, 1);
        for (int i = 0; i < kFaKStages; i++) {
            mbar_init(&sh.k_full[i], 1);
            mbar_init(&sh.k_empty[i], 1);
        }
        for (int i = 0; i < kFaVStages; i++) {
            mbar_init(&sh.v_full[i], 1);
            mbar_init(&sh.v_empty[i], 1);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        prefetch_tensormap(&tmQ);
        prefetch_tensormap(&tmK);
        prefetch_tensormap(&tmV);
    }
    if (warp == 1) {
        tmem_alloc(&sh.tmem, kFaTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sh.tmem;

    grid_dep_wait();
    grid_dep_launch();

    const int M = p.M;
    const int pos0 = p.pos0_dev ? *p.pos0_dev : p.pos0;
    const int p_first = pos0 + r0;
    const int p_last = pos0 + min(r0 + kFaRows, M) - 1;
    const int kall = max(0, p_first - (kEncWindow - 1)) / kFaKeys * kFaKeys;
    const int nball = (p_last - kall) / kFaKeys + 1;
    // this CTA's key blocks: all, or split z of KZ (possibly none)
    const int KZ = p.ksplit > 1 ? p.ksplit : 1, z = blockIdx.z;
    // the KZ splits are one cluster (rank = z); launched with two softmax warps per quarter
    const bool KCL = NH == 2 && KZ > 1 && p.kcluster > 1;
    const int bz0 = z * nball / KZ, bz1 = (z + 1) * nball / KZ;
    const int kstart = kall + bz0 * kFaKeys;
    const int nb = bz1 - bz0;

    if (!ok) {
        // misaligned shared memory: nothing was issued
    } else if (warp == 0) {
        if (lane == 0) {
            uint64_t pol;
            asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
            if (nb > 0) {
                mbar_expect_tx(&sh.q_full, kFaRows * 128);
                tma_load_2d(sh.q, &tmQ, head * kEncHeadDim, r0, &sh.q_full, pol);
            }
            for (int b = 0; b < nb; b++) {
                const int kbuf = b % kFaKStages, vbuf = b % kFaVStages;
                const int slot = (kstart + b * kFaKeys) % p.cap;
                if (b >= kFaKStages &&
                    !mbar_wait(&sh.k_empty[kbuf], ((b / kFaKStages) + 1) & 1u, deadline)) {
                    ok = false;
                    break;
                }
                mbar_expect_tx(&sh.k_full[kbuf], kFaKeys * 128);
                tma_load_2d(sh.k[kbuf], &tmK, head * kEncHeadDim, slot, &sh.k_full[kbuf], pol);
                if (b >= kFaVStages &&
                    !mbar_wait(&sh.v_empty[vbuf], ((b / kFaVStages) + 1) & 1u, deadline)) {
                    ok = false;
                    break;
                }
                mbar_expect_tx(&sh.v_full[vbuf], kFaKeys * 128);
                tma_load_2d(sh.v[vbuf], &tmV, head * kEncHeadDim, slot, &sh.v_full[vbuf], pol);
            }
            // tail: the last releases of every buffer have arrived
            for (int b = nb > kFaKStages ? nb - kFaKStages : 0; b < nb && ok; b++)
                ok = mbar_wait(&sh.k_empty[b % kFaKStages], (b / kFaKStages) & 1u, deadline);
            for (int b = nb > kFaVStages ? nb - kFaVStages : 0; b < nb && ok; b++)
                ok = mbar_wait(&sh.v_empty[b % kFaVStages], (b / kFaVStages) & 1u, deadline);
        }
    } else if (warp == 1) {
        // MMA issue order: S_0; then per block b: S_{b+1} once the softmax
        // has read S_b (and K_{b+1} is in), then O += P_b V_b once P_b is in
        // shared memory (and V_b is in).
        if (lane == 0) {
            constexpr uint32_t id_s = idesc_f16(kFaRows, kFaKeys, false);
            constexpr uint32_t id_o = idesc_f16(kFaRows, kEncHeadDim, true);
            auto issue_s = [&](int b) -> bool {
                const int kbuf = b % kFaKStages;
                if (!mbar_wait(&sh.k_full[kbuf], (b / kFaKStages) & 1u, deadline)) return false;
                tc_fence_after();
                const uint64_t a0 = smem_desc_sw128(sh.q), b0 = smem_desc_sw128(sh.k[kbuf]);
#pragma unroll
                for (int k = 0; k < kEncHeadDim / 16; k++)   // +32 bytes per K=16 step
                    tc_mma_f16(tmem, a0 + 2 * k, b0 + 2 * k, id_s, k != 0 ? 1u : 0u);
                tc_commit(&sh.s_full);
                tc_commit(&sh.k_empty[kbuf]);
                return true;
            };
            ok = nb == 0 || (mbar_wait(&sh.q_full, 0u, deadline) && issue_s(0));
            for (int b = 0; b < nb && ok; b++) {
                if (b + 1 < nb) {
                    // S is one TMEM buffer: S_{b+1} after the softmax's read of S_b
                    if (!mbar_wait(&sh.s_free, b & 1u, deadline)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    if (!issue_s(b + 1)) {
                        ok = false;
                        break;
                    }
                }
                const int vbuf = b % kFaVStages;
                if (!mbar_wait(&sh.p_full, b & 1u, deadline) ||
                    !mbar_wait(&sh.v_full[vbuf], (b / kFaVStages) & 1u, deadline)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint64_t a0 = smem_desc_sw128(sh.p);
#pragma unroll
                for (int t = 0; t < kFaKeys / 16; t++) {   // 4 steps of 16 keys
                    const uint64_t bv = smem_desc_sw128_mn(sh.v[vbuf] + t * 16 * 128);
                    tc_mma_f16(tmem + kFaKeys, a0 + 2 * t, bv, id_o, (b | t) != 0 ? 1u : 0u);
                }
                tc_commit(&sh.o_full);
                tc_commit(&sh.v_empty[vbuf]);
            }
        }
    } else {
        // ---- softmax: NH warps per TMEM lane quarter, thread = query row,
        // each warp CW of the 64 key columns (and of O) ----
        constexpr int CW = kFaKeys / NH;
        const int q = warp & 3, half = NH == 2 ? (warp - 2) >> 2 : 0;
        const int row = 32 * q + lane;
        const int pr = pos0 + r0 + row;                     // this row's logical position
        const uint32_t tl = tmem + ((uint32_t)(32 * q) << 16);
        const uint32_t ts = tl + (uint32_t)(half * CW);               // this warp's S columns
        const uint32_t to = tl + (uint32_t)(kFaKeys + half * CW);     // and O columns
        const float sl2 = 0.18033688011112042f;              // (1 / sqrt(64)) * log2(e)
        float m = -INFINITY, l = 0.f;                        // l: this half's columns only
        for (int b = 0; b < nb; b++) {
            const bool got = mbar_wait(&sh.s_full, b & 1u, deadline);
            if (!__all_sync(0xffffffffu, got)) {
                ok = false;
            }
            tc_fence_after();
            float sv[CW];   // S_b columns half*CW .. half*CW+CW-1
#pragma unroll
            for (int c2 = 0; c2 < CW; c2 += 32) tmem_ld32(ts + (uint32_t)c2, *reinterpret_cast<float(*)[32]>(sv + c2));
            // S_b is in registers: the MMA warp may overwrite S with S_{b+1}
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sh.s_free);
            const int kb0 = kstart + b * kFaKeys + half * CW;
            // every key of the block inside every valid row's window: no mask;
            // else key offset c is valid for this row iff (unsigned)(c - lo) <= 749
            const bool full = kstart + b * kFaKeys >= p_last - (kEncWindow - 1) &&
                              kstart + b * kFaKeys + kFaKeys - 1 <= p_first;
            const int lo = pr - (kEncWindow - 1) - kb0;
            if (!full) {
#pragma unroll
                for (int j = 0; j < CW; j++)
                    if ((unsigned)(j - lo) > (unsigned)(kEncWindow - 1)) sv[j] = -INFINITY;
            }
            float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
            for (int j = 0; j < CW; j++) mx4[j & 3] = fmaxf(mx4[j & 3], sv[j]);
            float mb = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
            if constexpr (NH == 2) {   // the row's block maximum over both halves (pair barrier q + 1)
                sh.mx[half][row] = mb;
                named_bar_sync(1 + q, 64);
                mb = fmaxf(sh.mx[0][row], sh.mx[1][row]);
            }
            mb *= sl2;
            // move the running max only when this block's max exceeds it by > 2^8
            const bool move = mb > m + kFaRescale;
            float factor = 1.f;
            if (move) {
                factor = (m == -INFINITY) ? 0.f : fast_exp2(m - mb);
                m = mb;
                l *= factor;
            }
            // O += P_{b-1} V_{b-1} complete: P is free and O can be rescaled
            if (b > 0) {
                const bool got_o = mbar_wait(&sh.o_full, (b - 1) & 1u, deadline);
                if (!__all_sync(0xffffffffu, got_o)) ok = false;
                tc_fence_after();
            }
            const float base = (m == -INFINITY) ? 0.f : m;
            // P = 2^(s * sl2 - m) as fp16, row sum in fp32 (4 chains)
            float rs4[4] = {0.f, 0.f, 0.f, 0.f};
            unsigned char *ph = sh.p + row * 128;
#pragma unroll
            for (int c = 0; c < CW; c += 8) {
                uint32_t h[4];
#pragma unroll
                for (int j = 0; j < 8; j += 2) {
                    const float ea = fast_exp2(fmaf(sv[c + j], sl2, -base));
                    const float eb = fast_exp2(fmaf(sv[c + j + 1], sl2, -base));
                    rs4[(j >> 1) & 3] += ea + eb;
                    h[j >> 1] = half2_bits(ea, eb);
                }
                const int chunk = (half * CW + c) >> 3;
                *reinterpret_cast<uint4 *>(ph + 16 * (chunk ^ (row & 7))) = make_uint4(h[0], h[1], h[2], h[3]);
            }
            l += (rs4[0] + rs4[1]) + (rs4[2] + rs4[3]);
            // rows whose max moved rescale their O row (after P, so S is dead)
            if (b > 0 && __any_sync(0xffffffffu, move)) {
#pragma unroll
                for (int c2 = 0; c2 < CW; c2 += 32) {
                    float ov[32];
                    tmem_ld32(to + (uint32_t)c2, ov);
#pragma unroll
                    for (int j = 0; j < 32; j++) ov[j] *= factor;
                    tmem_st32(to + (uint32_t)c2, ov);
                }
            }
            fence_async_smem();   // P visible to the tensor core
            tc_fence_before();    // S / O accesses ordered before the next MMAs
            __syncwarp();
            if (lane == 0) mbar_arrive(&sh.p_full);
        }
        // the last O MMA, then o / l as fp16 (the wo GEMM's A operand)
        bool got_o = ok && (nb == 0 || mbar_wait(&sh.o_full, (nb - 1) & 1u, deadline));
        if (!__all_sync(0xffffffffu, got_o)) ok = false;
        float lt = l;
        if constexpr (NH == 2) {   // the row's sum over both halves (pair barrier q + 1)
            sh.mx[half][row] = l;
            named_bar_sync(1 + q, 64);
            lt = sh.mx[0][row] + sh.mx[1][row];
        }
        uint16_t *dst = p.out + (size_t)(r0 + row) * kEncQkv + head * kEncHeadDim + half * CW;
        const bool rv = r0 + row < M;
        if (ok && KZ == 1) {
            tc_fence_after();
            const float il = (lt > 0.f) ? 1.0f / lt : 0.f;
#pragma unroll
            for (int c2 = 0; c2 < CW; c2 += 32) {
                float ov[32];
                tmem_ld32(to + (uint32_t)c2, ov);
                if (rv) {
#pragma unroll
                    for (int j = 0; j < 32; j += 8)
                        *reinterpret_cast<uint4 *>(dst + c2 + j) =
                            make_uint4(out16x2(ov[j] * il, ov[j + 1] * il, p.f16),
                                       out16x2(ov[j + 2] * il, ov[j + 3] * il, p.f16),
                                       out16x2(ov[j + 4] * il, ov[j + 5] * il, p.f16),
                                       out16x2(ov[j + 6] * il, ov[j + 7] * il, p.f16));
                }
            }
        } else if (KCL) {
            // this split's row partial into its drained Q / K tiles: [128 rows]
            // x (64 o, max, sum, 2 unused); merged after the cluster barrier
            float *pt = reinterpret_cast<float *>(fa_smem_raw) + row * kFaPartFloats;
            if (ok && nb > 0) tc_fence_after();
#pragma unroll
            for (int c2 = 0; c2 < CW; c2 += 32) {
                float ov[32];
                if (nb > 0) tmem_ld32(to + (uint32_t)c2, ov);   // (warp-uniform)
                else {
#pragma unroll
                    for (int j = 0; j < 32; j++) ov[j] = 0.f;
                }
#pragma unroll
                for (int j = 0; j < 32; j += 4)
                    *reinterpret_cast<float4 *>(pt + half * CW + c2 + j) =
                        make_float4(ov[j], ov[j + 1], ov[j + 2], ov[j + 3]);
            }
            if (half == 0) *reinterpret_cast<float2 *>(pt + kEncHeadDim) = make_float2(m, lt);
        } else if (KZ > 1) {
            // this split's row partial: o (64 fp32), then (max, sum)
            const size_t pr_idx = ((size_t)z * M + (r0 + row)) * kEncHeads + head;
            float *po = p.part + pr_idx * kFaPartFloats;
            if (ok && nb > 0) tc_fence_after();
#pragma unroll
            for (int c2 = 0; c2 < CW; c2 += 32) {
                float ov[32];
                if (nb > 0) tmem_ld32(to + (uint32_t)c2, ov);   // (warp-uniform)
                else {
#pragma unroll
                    for (int j = 0; j < 32; j++) ov[j] = 0.f;
                }
                if (rv) {
#pragma unroll
                    for (int j = 0; j < 32; j += 4)
                        __stcg(reinterpret_cast<float4 *>(po + half * CW + c2 + j),
                               make_float4(ov[j], ov[j + 1], ov[j + 2], ov[j + 3]));
                }
            }
            if (rv && half == 0) __stcg(reinterpret_cast<float2 *>(po + kEncHeadDim), make_float2(m, lt));
            __threadfence();
            named_bar_sync(5, 128 * NH);   // every softmax warp
            if (threadIdx.x == 64) {
                const unsigned t = atomicAdd(&p.cnt[blockIdx.x * kEncHeads + head], 1u);
                sh.last = (t + 1u == (unsigned)KZ) ? 1 : 0;
            }
            named_bar_sync(5, 128 * NH);
            if (sh.last) {
                __threadfence();
                if (rv) {
                    // max over the splits that saw keys, then the weighted sums in split order
                    float mz[kFaMaxSplit], lz[kFaMaxSplit];
                    float gm = -INFINITY;
#pragma unroll
                    for (int s2 = 0; s2 < kFaMaxSplit; s2++) {
                        mz[s2] = -INFINITY;
                        lz[s2] = 0.f;
                        if (s2 < KZ) {
                            const float2 v = __ldcg(reinterpret_cast<const float2 *>(
                                p.part + (((size_t)s2 * M + (r0 + row)) * kEncHeads + head) * kFaPartFloats +
                                kEncHeadDim));
                            mz[s2] = v.x;
                            lz[s2] = v.y;
                            if (v.y > 0.f) gm = fmaxf(gm, v.x);
                        }
                    }
                    float gl = 0.f, wz[kFaMaxSplit];
#pragma unroll
                    for (int s2 = 0; s2 < kFaMaxSplit; s2++) {
                        wz[s2] = (s2 < KZ && lz[s2] > 0.f) ? fast_exp2(mz[s2] - gm) : 0.f;
                        gl += lz[s2] * wz[s2];
                    }
                    const float il = gl > 0.f ? 1.0f / gl : 0.f;
#pragma unroll
                    for (int c = 0; c < CW; c += 16) {   // this warp's columns
                        float4 acc[4] = {};
#pragma unroll
                        for (int s2 = 0; s2 < kFaMaxSplit; s2++) {
                            if (s2 >= KZ) break;
                            const float4 *src = reinterpret_cast<const float4 *>(
                                p.part + (((size_t)s2 * M + (r0 + row)) * kEncHeads + head) * kFaPartFloats +
                                half * CW + c);
                            const float w = wz[s2];
#pragma unroll
                            for (int j = 0; j < 4; j++) {
                                const float4 v = __ldcg(src + j);
                                acc[j].x = fmaf(w, v.x, acc[j].x);
                                acc[j].y = fmaf(w, v.y, acc[j].y);
                                acc[j].z = fmaf(w, v.z, acc[j].z);
                                acc[j].w = fmaf(w, v.w, acc[j].w);
                            }
                        }
#pragma unroll
                        for (int j = 0; j < 4; j += 2)
                            *reinterpret_cast<uint4 *>(dst + c + 4 * j) =
                                make_uint4(out16x2(acc[j].x * il, acc[j].y * il, p.f16),
                                           out16x2(acc[j].z * il, acc[j].w * il, p.f16),
                                           out16x2(acc[j + 1].x * il, acc[j + 1].y * il, p.f16),
                                           out16x2(acc[j + 1].z * il, acc[j + 1].w * il, p.f16));
                    }
                }
                if (threadIdx.x == 64) p.cnt[blockIdx.x * kEncHeads + head] = 0u;
            }
        }
    }

    if (KCL) {
        // every split's partial is in its CTA's shared memory (every thread of
        // every CTA arrives, whatever failed before: no CTA waits forever);
        // rank z merges the tile rows r with r % KZ == z: the maximum over the
        // splits that saw keys, then the weighted sums in split order (the
        // same arithmetic as the workspace merge)
        cluster_sync_all();
        if (warp >= 2 && ok) {
            constexpr int CW = kFaKeys / NH;
            const int q = warp & 3, half = NH == 2 ? (warp - 2) >> 2 : 0;
            const int row = 32 * q + lane;
            if (row % KZ == z && r0 + row < M) {
                const uint32_t base = smem_u32(reinterpret_cast<float *>(fa_smem_raw) + row * kFaPartFloats);
                float mz[kFaMaxSplit], lz[kFaMaxSplit];
                float gm = -INFINITY;
#pragma unroll
                for (int s2 = 0; s2 < kFaMaxSplit; s2++) {
                    mz[s2] = -INFINITY;
                    lz[s2] = 0.f;
                    if (s2 < KZ) {
                        const float2 v = ld_dsmem_f2(mapa_shared(base + 4u * kEncHeadDim, (uint32_t)s2));
                        mz[s2] = v.x;
                        lz[s2] = v.y;
                        if (v.y > 0.f) gm = fmaxf(gm, v.x);
                    }
                }
                float gl = 0.f, wz[kFaMaxSplit];
#pragma unroll
                for (int s2 = 0; s2 < kFaMaxSplit; s2++) {
                    wz[s2] = (s2 < KZ && lz[s2] > 0.f) ? fast_exp2(mz[s2] - gm) : 0.f;
                    gl += lz[s2] * wz[s2];
                }
                const float il = gl > 0.f ? 1.0f / gl : 0.f;
                uint16_t *dst = p.out + (size_t)(r0 + row) * kEncQkv + head * kEncHeadDim + half * CW;
#pragma unroll
                for (int c = 0; c < CW; c += 16) {   // this thread's columns
                    float4 acc[4] = {};
#pragma unroll
                    for (int s2 = 0; s2 < kFaMaxSplit; s2++) {
                        if (s2 >= KZ) break;
                        const uint32_t src = mapa_shared(base + 4u * (half * CW + c), (uint32_t)s2);
                        const float w = wz[s2];
#pragma unroll
                        for (int j = 0; j < 4; j++) {
                            const float4 v = ld_dsmem_f4(src + 16u * j);
                            acc[j].x = fmaf(w, v.x, acc[j].x);
                            acc[j].y = fmaf(w, v.y, acc[j].y);
                            acc[j].z = fmaf(w, v.z, acc[j].z);
                            acc[j].w = fmaf(w, v.w, acc[j].w);
                        }
                    }
#pragma unroll
                    for (int j = 0; j < 4; j += 2)
                        *reinterpret_cast<uint4 *>(dst + c + 4 * j) =
                            make_uint4(out16x2(acc[j].x * il, acc[j].y * il, p.f16),
                                       out16x2(acc[j].z * il, acc[j].w * il, p.f16),
                                       out16x2(acc[j + 1].x * il, acc[j + 1].y * il, p.f16),
                                       out16x2(acc[j + 1].z * il, acc[j + 1].w * il, p.f16));
                }
            }
        }
        cluster_sync_all();   // no CTA leaves while a peer still reads its partials
    }
    if (!__all_sync(0xffffffffu, ok)) ok = false;
    if (!ok) {
        if (lane == 0 && p.err) atomicExch(p.err, 1u);
        const uint64_t grace = globaltimer() + 10000000ull;   // let in-flight copies / MMAs land
        while (globaltimer() < grace) {
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kFaTmemCols);
    }
}

namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn fa_encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *q = nullptr;
        cudaDriverEntryPointQueryResult r;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &q, cudaEnableDefault, &r) == cudaSuccess &&
            r == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)q;
    });
    return fn;
}

// fp16 [rows][2048], box box_rows x 64 columns (one head), 128-byte swizzle
bool fa_map(CUtensorMap *m, const void *ptr, int rows, int box_rows) {
    EncodeTiledFn fn = fa_encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)kEncQkv, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)kEncQkv * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kEncHeadDim, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(ptr), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

// Key splits for an M-row chunk, off unless VOX_CUDA_ENC_ATTN_KSPLIT = n
// (n <= 8) asks for them: a 100-row chunk has 32 tiles (one per head) of ~14
// key blocks each, and splitting the blocks over up to n CTAs fills more
// SMs, as long as the partials fit the workspace.  Measured per 32-layer
// chunk (one CTA per SM): 100 rows 2.15 ms unsplit, 2.18 ms at 2 splits,
// 2.20 ms at 4; 500 rows 3.22 / 3.59 / 3.81 ms.  The per-tile merge (a
// fence, a ticket, four dependent L2 round trips) costs more than the
// shorter key loop saves.
int enc_attn_ksplit(int M, size_t ws_floats) {
    const char *e = getenv("VOX_CUDA_ENC_ATTN_KSPLIT");
    const int cap = (e && atoi(e) >= 1) ? std::min(atoi(e), kFaMaxSplit) : 1;
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int tiles = (M + kFaRows - 1) / kFaRows * kEncHeads;
    int ks = std::min(cap, std::max(1, 3 * sms / tiles));
    while (ks > 1 && (size_t)ks * M * kEncHeads * kFaPartFloats > ws_floats) ks--;
    return ks;
}

namespace {

// Clusters of kz spread CTAs (one per SM, two softmax warps per lane
// quarter) the device runs at once; cached per cluster size, 0 if unknown.
int fa_max_clusters(int kz) {
    static std::atomic<int> cache[kFaMaxSplit + 1];
    if (kz < 2 || kz > kFaMaxSplit) return 0;
    int c = cache[kz].load();
    if (c == 0) {
        int n = 0;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(1, kEncHeads, kz);
        cfg.blockDim = dim3(fa_threads(2));
        cfg.dynamicSmemBytes = std::max(sizeof(FaSmem), kFaSpreadSmem);
        cudaLaunchAttribute a[1];
        a[0].id = cudaLaunchAttributeClusterDimension;
        a[0].val.clusterDim.x = 1;
        a[0].val.clusterDim.y = 1;
        a[0].val.clusterDim.z = kz;
        cfg.attrs = a;
        cfg.numAttrs = 1;
        if (cudaFuncSetAttribute(enc_attn_tc_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)cfg.dynamicSmemBytes) != cudaSuccess ||
            cudaOccupancyMaxActiveClusters(&n, enc_attn_tc_kernel<2>, &cfg) != cudaSuccess) {
            cudaGetLastError();
            n = 0;
        }
        c = n > 0 ? n : -1;
        cache[kz].store(c);
    }
    return c > 0 ? c : 0;
}

// Cluster key split for an M-row chunk (p.kcluster = 1, no workspace split):
// when the (row tile, head) tiles fill at most half the SMs, each tile's key
// blocks go to kz CTAs of one cluster (>= 2 blocks each, every cluster
// resident at once), merged through distributed shared memory.
// VOX_CUDA_ENC_ATTN_CLUSTER = -1 turns it off, n >= 2 caps kz.
int fa_cluster_split(int M, int sms) {
    const char *e = getenv("VOX_CUDA_ENC_ATTN_CLUSTER");
    const int env = (e && *e) ? atoi(e) : 0;
    if (env < 0) return 1;
    const int tiles = (M + kFaRows - 1) / kFaRows * kEncHeads;
    if (2 * tiles > sms) return 1;
    const int nball = (M - 1 + kEncWindow - 1 + kFaKeys - 1) / kFaKeys + 1;   // at most
    int kz = std::min(std::min(kFaMaxSplit, sms / tiles), nball / 2);
    if (env >= 2) kz = std::min(kz, env);
    while (kz >= 2 && tiles > fa_max_clusters(kz)) kz--;
    return kz >= 2 ? kz : 1;
}

}  // namespace

bool enc_attn_tc_supported(const EncAttnParams &p) {
    return p.cap % kEncRingAlign == 0 && p.cap >= p.M + kEncWindow - 1 && p.err != nullptr &&
           ((uintptr_t)p.q & 15) == 0 && ((uintptr_t)p.k_ring & 15) == 0 && ((uintptr_t)p.v_ring & 15) == 0 &&
           ((uintptr_t)p.out & 15) == 0;
}

cudaError_t launch_enc_attn_tc(const EncAttnParams &p_in, cudaStream_t st, bool pdl) {
    EncAttnParams p = p_in;
    if (p.M <= 0 || !enc_attn_tc_supported(p)) return cudaErrorInvalidValue;
    CUtensorMap mq, mk, mv;
    if (!fa_map(&mq, p.q, p.M, kFaRows) || !fa_map(&mk, p.k_ring, p.cap, kFaKeys) ||
        !fa_map(&mv, p.v_ring, p.cap, kFaKeys))
        return cudaErrorInvalidValue;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    static std::atomic<uint64_t> attr_set{0};   // the shared-memory opt-in is per device
    const uint64_t bit = 1ull << (dev & 63);
    if (!(attr_set.load() & bit)) {
        e = cudaFuncSetAttribute(enc_attn_tc_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)std::max(sizeof(FaSmem), kFaSpreadSmem));
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(enc_attn_tc_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)std::max(sizeof(FaSmem), kFaSpreadSmem));
        if (e != cudaSuccess) return e;
        attr_set.fetch_or(bit);
    }
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (p.ksplit <= 1 && p.kcluster == 1) {
        p.ksplit = fa_cluster_split(p.M, sms);
        p.kcluster = p.ksplit > 1 ? p.ksplit : 0;
    } else {
        p.kcluster = 0;
    }
    const int kz = p.ksplit > 1 ? p.ksplit : 1;
    if (kz > 1 && !p.kcluster &&
        (kz > kFaMaxSplit || !p.part || !p.cnt || (p.M + kFaRows - 1) / kFaRows * kEncHeads > kTcSplitCounters))
        return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    const int ctas = (p.M + kFaRows - 1) / kFaRows * kEncHeads * kz;
    cfg.gridDim = dim3((p.M + kFaRows - 1) / kFaRows, kEncHeads, kz);
    // A launch with no more CTAs than SMs reserves enough shared memory for
    // one CTA per SM: launched early (programmatic dependent launch) while
    // the q|k|v GEMM still holds most SMs, its CTAs would otherwise pack
    // three to an SM on the few free ones and share their issue slots.  Such
    // a CTA alone on its SM splits the softmax over two warps per TMEM lane
    // quarter (NH = 2; VOX_CUDA_ENC_ATTN_NH = 1 | 2 forces one).
    // (a cluster split always spreads, two softmax warps per quarter: the
    // cluster residency was checked for that shape; launches that share the
    // SMs with other streams' launches do not spread: measured for 8 streams
    // x 100 rows, 4.40 -> 4.03 ms per batched round)
    const char *sp = getenv("VOX_CUDA_ENC_ATTN_SPREAD");
    const bool spread = p.kcluster ? true : sp ? atoi(sp) != 0 : !p.shared_sms && ctas <= sms;
    const char *nh_env = getenv("VOX_CUDA_ENC_ATTN_NH");
    const int nh = p.kcluster                                          ? 2
                   : (nh_env && (atoi(nh_env) == 1 || atoi(nh_env) == 2)) ? atoi(nh_env)
                   : spread                                            ? 2
                                                                       : 1;
    cfg.blockDim = dim3(fa_threads(nh));
    cfg.dynamicSmemBytes = spread ? std::max(sizeof(FaSmem), kFaSpreadSmem) : sizeof(FaSmem);
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (pdl) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        na++;
    }
    if (p.kcluster) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = 1;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = kz;
        na++;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return nh == 2 ? cudaLaunchKernelEx(&cfg, enc_attn_tc_kernel<2>, mq, mk, mv, p)
                   : cudaLaunchKernelEx(&cfg, enc_attn_tc_kernel<1>, mq, mk, mv, p);
}

}  // namespace vc

