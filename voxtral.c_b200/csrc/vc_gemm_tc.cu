// vc_gemm_tc.cu - tcgen05 tensor-core GEMM for the encoder chunk, the adapter
// and M > 8 matmuls: C[M, N] = A[M, K] . W[N, K]^T with bf16 A and W (both
// K-major, row-major as stored), fp32 accumulation in TMEM, fused epilogues.
//
// Persistent: one CTA per SM walks the 128 x BN output tiles t = blockIdx.x,
// blockIdx.x + gridDim.x, ... (row tiles fastest, so the CTAs of one wave
// share W tiles in L2).
//   warp 0 (one thread)  TMA producer: 128x64 A and BNx64 W tiles, 128-byte
//                        swizzle, into a STAGES-deep shared-memory ring that
//                        runs on across tiles
//   warp 1 (one thread)  tcgen05.mma issuer (M=128, N=BN, K=16, cta_group::1)
//                        into one of two TMEM accumulators (2 x BN fp32
//                        columns); tcgen05.commit releases ring stages and
//                        hands a finished accumulator to the epilogue
//   warps 2-9            epilogue, two warps per 32-lane TMEM quarter (warp
//                        id mod 4 selects the quarter), each taking half of
//                        the columns: tcgen05.ld (32 columns per load), bias /
//                        residual / activation / RoPE, 16-byte stores; then
//                        the accumulator goes back to the issuer, so the
//                        epilogue of tile i overlaps the MMAs of tile i + 1
// Every mbarrier wait is bounded (2 s of %globaltimer); on expiry the CTA sets
// the launch's error word and exits after a grace period for in-flight copies.
#include "vc_common.cuh"
#include "vc_internal.h"
#include "vc_tc.cuh"

#include <cuda_fp16.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <unordered_map>

namespace vc {

using namespace tc;

constexpr int kEpiWarps = 8;                 // two per TMEM lane quarter, each half the columns
constexpr int kTcThreads = 64 + 32 * kEpiWarps;
constexpr int kBM = 128;
constexpr int kBK = 64;                     // one 128-byte swizzle row of bf16
constexpr int kEpiCols = 32;                // accumulator columns per tcgen05.ld
constexpr int kStageBytes = 32 * 128;       // a warp's staging tile: 32 rows x 128 bytes
constexpr int kTcMaxSplit = 4;              // split-K slices at most
constexpr int kTcSplitMinKB = 32;           // split-K only for K >= 32 k-blocks (2048)
constexpr uint64_t kTcWaitNs = 2000000000ull;

template <int BN>
struct TcCfg {
    static constexpr int kABytes = kBM * kBK * 2;
    static constexpr int kBBytes = BN * kBK * 2;
    // as many stages as fit 192 KB, at most 6 (BN 64 / 128: 6, 192 / 256: 4)
    static constexpr int kStages = (196608 / (kABytes + kBBytes)) < 6 ? (196608 / (kABytes + kBBytes)) : 6;
    // two accumulators of BN columns; the allocation is a power of two
    static constexpr int kTmemCols = (2 * BN <= 128) ? 128 : (2 * BN <= 256) ? 256 : 512;
    static constexpr int kSmem = kStages * (kABytes + kBBytes) + kEpiWarps * kStageBytes + 1024 /*align*/ +
                                 256 /*barriers*/ + 512 /*row scales of a cluster split*/;
};

__device__ __forceinline__ float gelu_tanh(float v) {
    // tanh-approximated GELU (vox_gelu, voxtral_kernels.c:376-384)
    const float x3 = v * v * v;
    const float inner = 0.7978845608028654f * (v + 0.044715f * x3);
    return 0.5f * v * (1.0f + tanhf(inner));
}

// SiLU with the fast exp / divide intrinsics: a few ulp of fp32, far below the
// bf16 rounding of the product that follows.  g -> -inf gives -0.
__device__ __forceinline__ float silu_fast(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
    return bf16_bits_rn(a) | (bf16_bits_rn(b) << 16);
}

// fp16 operands and rings (the encoder, its adapter, the conv stem's GEMMs)
// convert with saturation: a value beyond fp16's finite range becomes
// +-65504 rather than inf (NaN stays NaN).  One instruction, as the plain
// conversion.  Two kinds of event are counted (vox_cuda_fp16_saturations):
// a SwiGLU output chunk with a clamped value - the product silu(g) * u is
// where the encoder's magnitudes peak - and a residual row that reached a
// norm pass with a non-finite value.  Per-element checks elsewhere cost ~10%
// of the chunk and catch nothing these two do not.
__device__ unsigned long long g_f16_sat_gemm;

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
    uint32_t r;   // the first source lands in the upper half: (b, a) puts a in .x
    asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
    return r;
}
// Running per-half maximum of |v| over packed fp16 pairs (sign bits masked):
// one chunk is clamped when a half reached 65504 (0x7BFF; NaN sorts above).
__device__ __forceinline__ uint32_t f16x2_absmax(uint32_t m, uint32_t w) {
    return __vmaxu2(m, w & 0x7FFF7FFFu);
}
__device__ __forceinline__ void count_clamped(uint32_t absmax) {
    if (__vcmpgeu2(absmax, 0x7BFF7BFFu)) atomicAdd(&g_f16_sat_gemm, 1ull);
}

// two 16-bit operand values (the next GEMM's A): fp16 or bf16
__device__ __forceinline__ uint32_t pack16x2(float a, float b, int f16) {
    return f16 ? pack_half2(a, b) : pack_bf16x2(a, b);
}
__device__ __forceinline__ uint16_t bits16(float a, int f16) {
    return f16 ? (uint16_t)(pack_half2(a, 0.0f) & 0xFFFFu) : (uint16_t)bf16_bits_rn(a);
}

// v = hi + lo in bf16: hi = bf16(v), lo = bf16(v - hi) (~2^-17 relative)
__device__ __forceinline__ float bf16_hi_f(float v) { return __uint_as_float(bf16_bits_rn(v) << 16); }
__device__ __forceinline__ uint32_t pack_bf16_lo2(float a, float b) {
    return pack_bf16x2(a - bf16_hi_f(a), b - bf16_hi_f(b));
}

__device__ __forceinline__ void st16(void *dst, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    *reinterpret_cast<uint4 *>(dst) = make_uint4(a, b, c, d);
}

// Per-thread facts of one tile row, fixed across its column chunks.
struct EpiRow {
    int row;        // output row (this thread's TMEM lane)
    int pos;        // TC_QKV_ENC: logical position of the row
    size_t slot;    // TC_QKV_ENC: ring slot of the row
    uint16_t *ek, *ev;   // TC_QKV_ENC: the row's rings (this layer)
    int ecap;            // TC_QKV_ENC: their capacity
    float *kd, *vd; // TC_QKV_DEC: the row's K / V ring rows (this layer)
    float rs;       // ss_in: the row's 1 / rms (else 1)
};

// 1 / sqrt(mean square + eps) of a row from its per-32-column-chunk sums of
// squares (K / 32 chunks, summed in chunk order: the same value whatever
// the producer's tile width); sixteen loads in flight
__device__ __forceinline__ float row_inv_rms(const float *ss, int ld, int row, int K) {
    const int nch = K / kEpiCols;
    float acc = 0.f;
    int c = 0;
    for (; c + 16 <= nch; c += 16) {
        float t[16];
#pragma unroll
        for (int u = 0; u < 16; u++) t[u] = __ldcg(ss + (size_t)(c + u) * ld + row);
#pragma unroll
        for (int u = 0; u < 16; u++) acc += t[u];
    }
    for (; c < nch; c++) acc += __ldcg(ss + (size_t)c * ld + row);
    return 1.0f / sqrtf(acc / (float)K + kNormEps);
}

// The per-row facts of TC_QKV_ENC / TC_QKV_DEC for output row `row`.
template <int EPI>
__device__ __forceinline__ EpiRow epi_row(const TcGemmParams &p, int row) {
    EpiRow er;
    er.row = row;
    er.pos = 0;
    er.slot = 0;
    er.kd = er.vd = nullptr;
    er.ek = er.ev = nullptr;
    er.ecap = 0;
    er.rs = 1.0f;   // (ss_in: set by the caller, computed before the accumulator is ready)
    if constexpr (EPI == TC_QKV_ENC) {
        if (p.segs) {   // several streams' rows: the row's segment (row0 ascending)
            int s = 0;
            while (s + 1 < p.n_segs && row >= p.segs[s + 1].row0) s++;
            const EncSeg g = p.segs[s];
            er.pos = *g.pos0_dev + (row - g.row0);
            er.ecap = g.cap;
            const size_t lo = (size_t)p.layer * g.cap * kEncQkv;
            er.ek = g.k_ring + lo;
            er.ev = g.v_ring + lo;
        } else {
            er.pos = (p.pos0_dev ? *p.pos0_dev : p.pos0) + row;
            er.ecap = p.cap;
            er.ek = p.k_ring;
            er.ev = p.v_ring;
        }
        er.slot = (size_t)(er.pos % er.ecap);
    }
    if constexpr (EPI == TC_QKV_DEC) {
        if (row < p.M) {
            const StreamSlot sl = p.slots[row];
            const size_t off = ((size_t)p.layer * sl.cap + sl.slot) * kKvDim;
            er.kd = sl.k_ring + off;
            er.vd = sl.v_ring + off;
        }
    }
    return er;
}

// Decoder q|k RoPE of one row's 16 pairs at pair indices d0..d0+15 of a
// 128-wide head (vox_apply_rope, voxtral_kernels.c:505-526, as the prefill
// applies it, voxtral_decoder.c:303-306), cos / sin from the row's table.
__device__ __forceinline__ void dec_rope_chunk(const TcGemmParams &p, const EpiRow &er, int d0, float (&v)[kEpiCols]) {
    const float4 *t = reinterpret_cast<const float4 *>(p.rope_rows + (size_t)er.row * kHeadDim + 2 * d0);
    float4 cs[kEpiCols / 4];
#pragma unroll
    for (int i = 0; i < kEpiCols / 4; i++) cs[i] = __ldg(t + i);   // (cos, sin) of 2 pairs each
#pragma unroll
    for (int i = 0; i < kEpiCols / 4; i++) {
        const float c0 = cs[i].x, s0 = cs[i].y, c1 = cs[i].z, s1 = cs[i].w;
        float a = v[4 * i], b = v[4 * i + 1];
        v[4 * i] = __fsub_rn(__fmul_rn(a, c0), __fmul_rn(b, s0));
        v[4 * i + 1] = __fadd_rn(__fmul_rn(a, s0), __fmul_rn(b, c0));
        a = v[4 * i + 2], b = v[4 * i + 3];
        v[4 * i + 2] = __fsub_rn(__fmul_rn(a, c1), __fmul_rn(b, s1));
        v[4 * i + 3] = __fadd_rn(__fmul_rn(a, s1), __fmul_rn(b, c1));
    }
}

// The q|k|v region of decoder column col0 (32-column chunks never straddle
// two): [0,4096) q (RoPE), [4096,5120) k (RoPE), [5120,6144) v.
__device__ __forceinline__ int dec_qkv_apply(const TcGemmParams &p, const EpiRow &er, float (&v)[kEpiCols], int col0) {
    if (col0 >= kQDim + kKvDim) return 2;
    dec_rope_chunk(p, er, (col0 & (kHeadDim - 1)) >> 1, v);
    return col0 < kQDim ? 0 : 1;
}

__device__ __forceinline__ float *dec_qkv_dst(const TcGemmParams &p, const EpiRow &er, int col0, int region) {
    return region == 0 ? p.q32 + (size_t)er.row * kQDim + col0
           : region == 1 ? er.kd + (col0 - kQDim)
                         : er.vd + (col0 - kQDim - kKvDim);
}

// Encoder q|k RoPE of one row's 16 pairs (v[2i], v[2i+1]) at pair indices
// d0..d0+15 of a head (vox_apply_rope, voxtral_kernels.c:505-526; cos/sin as
// in :488-503).  The table holds a cos plane and a sin plane, [32][rope_ld]
// each, indexed by row, so a warp's 32 rows read 32 consecutive floats; all
// 32 loads are issued before the first use.
__device__ __forceinline__ void enc_rope_chunk(const TcGemmParams &p, const EpiRow &er, int d0, float (&v)[kEpiCols]) {
    float cs[kEpiCols / 2], sn[kEpiCols / 2];
    if (p.rope) {
        const float *cp = p.rope + (size_t)d0 * p.rope_ld + er.row;
        const float *sp = p.rope + (size_t)(kEncHeadDim / 2 + d0) * p.rope_ld + er.row;
#pragma unroll
        for (int i = 0; i < kEpiCols / 2; i++) {
            cs[i] = __ldg(cp + (size_t)i * p.rope_ld);
            sn[i] = __ldg(sp + (size_t)i * p.rope_ld);
        }
    } else {   // angle = pos * inv_freq exactly as the host formula
#pragma unroll
        for (int i = 0; i < kEpiCols / 2; i++) sincosf((float)er.pos * p.inv_freq[d0 + i], &sn[i], &cs[i]);
    }
#pragma unroll
    for (int i = 0; i < kEpiCols / 2; i++) {
        const float a = v[2 * i], b = v[2 * i + 1];
        v[2 * i] = __fsub_rn(__fmul_rn(a, cs[i]), __fmul_rn(b, sn[i]));
        v[2 * i + 1] = __fadd_rn(__fmul_rn(a, sn[i]), __fmul_rn(b, cs[i]));
    }
}

// v[j] += bias[col0 + j] for the columns inside N
__device__ __forceinline__ void add_bias(float (&v)[kEpiCols], const float *bias, int col0, int N) {
    if (!bias) return;
    if (col0 + kEpiCols <= N) {
#pragma unroll
        for (int j = 0; j < kEpiCols; j += 4) {
            const float4 b = __ldg(reinterpret_cast<const float4 *>(bias + col0 + j));
            v[j] += b.x, v[j + 1] += b.y, v[j + 2] += b.z, v[j + 3] += b.w;
        }
    } else {
#pragma unroll
        for (int j = 0; j < kEpiCols; j++)
            if (col0 + j < N) v[j] += __ldg(bias + col0 + j);
    }
}

// The q|k|v region of encoder column col0 (32-column chunks never straddle two):
// [0,2048) q (+bias, RoPE), [2048,4096) k (RoPE), [4096,6144) v (+bias)
// (voxtral_encoder.c:542-559).  Applies bias and RoPE to v in place.
__device__ __forceinline__ int qkv_apply(const TcGemmParams &p, const EpiRow &er, float (&v)[kEpiCols], int col0) {
    if (col0 < 2 * kEncQkv) {
        if (col0 < kEncQkv) add_bias(v, p.bias, col0, kEncQkv);
        enc_rope_chunk(p, er, (col0 & (kEncHeadDim - 1)) >> 1, v);
        return col0 < kEncQkv ? 0 : 1;
    }
    add_bias(v, p.bias2, col0 - 2 * kEncQkv, kEncQkv);
    return 2;
}

// ss_in: the accumulator row times the row's 1 / rms (the consumer half of
// the folded RMSNorm)
template <int EPI>
__device__ __forceinline__ void scale_row(const TcGemmParams &p, const EpiRow &er, float (&v)[kEpiCols]) {
    if constexpr (EPI == TC_QKV_ENC || EPI == TC_SWIGLU || EPI == TC_QKV_DEC) {
        if (p.ss_in) {
#pragma unroll
            for (int j = 0; j < kEpiCols; j++) v[j] *= er.rs;
        }
    }
}

// TC_RESID with xn_out: the updated residual chunk v (32 columns from col0,
// all inside N) -> its sum of squares and fp16(v * gain) (the producer half
// of the folded RMSNorm, vox_rms_norm at voxtral_kernels.c:346-363)
__device__ __forceinline__ void norm_prep_chunk(const TcGemmParams &p, int row, int col0, const float (&v)[kEpiCols]) {
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < kEpiCols; j++) ss = fmaf(v[j], v[j], ss);
    p.ss_out[(size_t)(col0 / kEpiCols) * p.ss_ld + row] = ss;
    if (p.hilo) {   // split activations: bf16 hi / lo rows of x * gain
        uint32_t hh[kEpiCols / 2], ll[kEpiCols / 2];
#pragma unroll
        for (int j = 0; j < kEpiCols; j += 4) {
            const float4 g = __ldg(reinterpret_cast<const float4 *>(p.xn_gain + col0 + j));
            const float a = v[j] * g.x, b = v[j + 1] * g.y, c = v[j + 2] * g.z, d = v[j + 3] * g.w;
            hh[j >> 1] = pack_bf16x2(a, b), hh[(j >> 1) + 1] = pack_bf16x2(c, d);
            ll[j >> 1] = pack_bf16_lo2(a, b), ll[(j >> 1) + 1] = pack_bf16_lo2(c, d);
        }
        uint16_t *oh = p.xn_out + (size_t)hilo_row(row) * p.ldo + col0;
        uint16_t *ol = oh + (size_t)64 * p.ldo;
#pragma unroll
        for (int j = 0; j < kEpiCols; j += 8) {
            st16(oh + j, hh[j >> 1], hh[(j >> 1) + 1], hh[(j >> 1) + 2], hh[(j >> 1) + 3]);
            st16(ol + j, ll[j >> 1], ll[(j >> 1) + 1], ll[(j >> 1) + 2], ll[(j >> 1) + 3]);
        }
        return;
    }
    uint32_t h[kEpiCols / 2], mx = 0;
#pragma unroll
    for (int j = 0; j < kEpiCols; j += 4) {
        const float4 g = __ldg(reinterpret_cast<const float4 *>(p.xn_gain + col0 + j));
        h[j >> 1] = pack_half2(v[j] * g.x, v[j + 1] * g.y);
        h[(j >> 1) + 1] = pack_half2(v[j + 2] * g.z, v[j + 3] * g.w);
        mx = f16x2_absmax(mx, h[j >> 1]);
        mx = f16x2_absmax(mx, h[(j >> 1) + 1]);
    }
    count_clamped(mx);
    uint16_t *o = p.xn_out + (size_t)row * p.ldo + col0;
#pragma unroll
    for (int j = 0; j < kEpiCols; j += 8) st16(o + j, h[j >> 1], h[(j >> 1) + 1], h[(j >> 1) + 2], h[(j >> 1) + 3]);
}

// Direct stores of one row's chunk [col0, col0 + 32), all inside N, 16-byte
// aligned destinations (p.vec).  TC_QKV_ENC: bias / RoPE already applied.
template <int EPI>
__device__ __forceinline__ void epi_vec(const TcGemmParams &p, const EpiRow &er, float (&v)[kEpiCols], int col0,
                                        int region) {
    const int row = er.row;
    if constexpr (EPI == TC_STORE || EPI == TC_RESID) {
        add_bias(v, p.bias, col0, p.N);
        float *o = p.out + (size_t)row * p.ldo + col0;
        if constexpr (EPI == TC_RESID) {
#pragma unroll
            for (int j = 0; j < kEpiCols; j += 4) {
                const float4 r = *reinterpret_cast<const float4 *>(o + j);
                v[j] += r.x, v[j + 1] += r.y, v[j + 2] += r.z, v[j + 3] += r.w;
            }
        }
        if (p.act == 1) {
#pragma unroll
            for (int j = 0; j < kEpiCols; j++) v[j] = gelu_tanh(v[j]);
        }
        if (p.out_bf16) {
            uint16_t *ob = p.out_bf16 + (size_t)row * p.ldo_bf16 + col0;
#pragma unroll
            for (int j = 0; j < kEpiCols; j += 8)
                st16(ob + j, pack16x2(v[j], v[j + 1], p.f16), pack16x2(v[j + 2], v[j + 3], p.f16),
                     pack16x2(v[j + 4], v[j + 5], p.f16), pack16x2(v[j + 6], v[j + 7], p.f16));
        } else {
#pragma unroll
            for (int j = 0; j < kEpiCols; j += 4)
                *reinterpret_cast<float4 *>(o + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        }
        if constexpr (EPI == TC_RESID) {
            if (p.xn_out) norm_prep_chunk(p, row, col0, v);
        }
    } else if constexpr (EPI == TC_SWIGLU) {
        // columns (2i, 2i+1) = (gate_i, up_i) -> h_i = silu(g) * u
        // (voxtral_kernels.c:369-374, then :34-36), bf16 for the next GEMM
        uint32_t h[kEpiCols / 4], clamp = 0;
#pragma unroll
        for (int j = 0; j < kEpiCols; j += 4) {
            h[j >> 2] = pack16x2(silu_fast(v[j]) * v[j + 1], silu_fast(v[j + 2]) * v[j + 3], p.f16);
            clamp = f16x2_absmax(clamp, h[j >> 2]);
        }
        if (p.f16) count_clamped(clamp);
        const int orow = p.out_hilo ? hilo_row(row) : row;
        uint16_t *o = p.out_bf16 + (size_t)orow * p.ldo_bf16 + (col0 >> 1);
#pragma unroll
        for (int j = 0; j < kEpiCols / 4; j += 4) st16(o + 2 * j, h[j], h[j + 1], h[j + 2], h[j + 3]);
        if (p.out_hilo) {   // the lo rows for a split-activation consumer (bf16 only)
            float hv[kEpiCols / 2];
#pragma unroll
            for (int j = 0; j < kEpiCols; j += 2) hv[j >> 1] = silu_fast(v[j]) * v[j + 1];
            uint16_t *ol = p.out_bf16 + (size_t)(orow + 64) * p.ldo_bf16 + (col0 >> 1);
#pragma unroll
            for (int j = 0; j < kEpiCols / 2; j += 8)
                st16(ol + j, pack_bf16_lo2(hv[j], hv[j + 1]), pack_bf16_lo2(hv[j + 2], hv[j + 3]),
                     pack_bf16_lo2(hv[j + 4], hv[j + 5]), pack_bf16_lo2(hv[j + 6], hv[j + 7]));
        }
    } else if constexpr (EPI == TC_QKV_DEC) {
        float *dst = dec_qkv_dst(p, er, col0, region);
#pragma unroll
        for (int j = 0; j < kEpiCols; j += 4)
            *reinterpret_cast<float4 *>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
    } else if constexpr (EPI == TC_QKV_ENC) {
        uint16_t *dst = region == 0   ? p.q_out + (size_t)row * kEncQkv + col0
                        : region == 1 ? er.ek + er.slot * kEncQkv + (col0 - kEncQkv)
                                      : er.ev + er.slot * kEncQkv + (col0 - 2 * kEncQkv);
#pragma unroll
        for (int j = 0; j < kEpiCols; j += 8)
            st16(dst + j, pack_half2(v[j], v[j + 1]), pack_half2(v[j + 2], v[j + 3]), pack_half2(v[j + 4], v[j + 5]),
                 pack_half2(v[j + 6], v[j + 7]));
    }
}

// Element-wise direct stores for a chunk that reaches past N or whose
// destinations are not 16-byte aligned.  TC_QKV_ENC: bias / RoPE applied.
template <int EPI>
__device__ __forceinline__ void epi_scalar(const TcGemmParams &p, const EpiRow &er, float (&v)[kEpiCols], int col0,
                                           int region) {
    const int row = er.row;
    if constexpr (EPI == TC_STORE || EPI == TC_RESID) {
        add_bias(v, p.bias, col0, p.N);
        float *o = p.out + (size_t)row * p.ldo + col0;
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < kEpiCols; j++) {
            if (col0 + j >= p.N) break;
            float x = v[j];
            if constexpr (EPI == TC_RESID) x += o[j];
            if (p.act == 1) x = gelu_tanh(x);
            if (p.out_bf16) p.out_bf16[(size_t)row * p.ldo_bf16 + col0 + j] = bits16(x, p.f16);
            else o[j] = x;
            if constexpr (EPI == TC_RESID) {
                if (p.xn_out) {
                    ss = fmaf(x, x, ss);
                    const float xg = x * __ldg(p.xn_gain + col0 + j);
                    p.xn_out[(size_t)row * p.ldo + col0 + j] = bits16(xg, 1);
                    if (!(fabsf(xg) < 65504.0f)) atomicAdd(&g_f16_sat_gemm, 1ull);
                }
            }
        }
        if constexpr (EPI == TC_RESID) {
            if (p.xn_out) p.ss_out[(size_t)(col0 / kEpiCols) * p.ss_ld + row] = ss;
        }
    } else if constexpr (EPI == TC_SWIGLU) {
        const int orow = p.out_hilo ? hilo_row(row) : row;
        uint16_t *o = p.out_bf16 + (size_t)orow * p.ldo_bf16 + (col0 >> 1);
#pragma unroll
        for (int j = 0; j < kEpiCols; j += 2) {
            if (col0 + j + 1 >= p.N) break;
            const float h = silu_fast(v[j]) * v[j + 1];
            o[j >> 1] = bits16(h, p.f16);
            if (p.f16 && !(fabsf(h) < 65504.0f)) atomicAdd(&g_f16_sat_gemm, 1ull);
            if (p.out_hilo)
                p.out_bf16[(size_t)(orow + 64) * p.ldo_bf16 + ((col0 + j) >> 1)] =
                    (uint16_t)bf16_bits_rn(h - bf16_hi_f(h));
        }
    } else if constexpr (EPI == TC_QKV_DEC) {
        float *dst = dec_qkv_dst(p, er, col0, region);
#pragma unroll
        for (int j = 0; j < kEpiCols; j++) dst[j] = v[j];
    } else if constexpr (EPI == TC_QKV_ENC) {
        uint16_t *dst = region == 0   ? p.q_out + (size_t)row * kEncQkv + col0
                        : region == 1 ? er.ek + er.slot * kEncQkv + (col0 - kEncQkv)
                                      : er.ev + er.slot * kEncQkv + (col0 - 2 * kEncQkv);
#pragma unroll
        for (int j = 0; j < kEpiCols; j += 2)
            *reinterpret_cast<uint32_t *>(dst + j) = pack_half2(v[j], v[j + 1]);
    }
}

// Tensor maps of the TMA-store epilogue (p.tma_out): o = the output (q for
// TC_QKV_ENC), k / v = this layer's rings.
struct EpiMaps {
    const CUtensorMap *o, *k, *v;
};

// TMA-store epilogue of one warp's 32 rows x 32 accumulator columns: stage
// the converted chunk in shared memory (`stg`, 4 KB, swizzled to the map's
// span) and let lane 0 store it, or add it (TC_RESID).  Rows / columns past
// the map's extent are not written.  The ring rows of TC_QKV_ENC are written
// this way only when the warp's 32 rows are all valid and do not wrap.
template <int EPI>
__device__ __forceinline__ void epi_tma(const TcGemmParams &p, const EpiMaps &mp, const EpiRow &er,
                                        float (&v)[kEpiCols], int row0, int col0, int lane, unsigned char *stg) {
    if constexpr (EPI == TC_QKV_DEC) {
        return;   // launch_tc_gemm never enables TMA stores for it
    }
    int region = 0;
    if constexpr (EPI == TC_QKV_ENC) {
        region = qkv_apply(p, er, v, col0);
        if (region != 0) {
            const int slot0 = __shfl_sync(0xffffffffu, (int)er.slot, 0);
            if (row0 + 32 > p.M || slot0 + 32 > p.cap) {   // tail rows or wrap: direct stores
                if (er.row < p.M) epi_vec<EPI>(p, er, v, col0, region);
                return;
            }
        }
    } else {
        add_bias(v, p.bias, col0, p.N);
        if constexpr (EPI == TC_STORE) {
            if (p.act == 1) {
#pragma unroll
                for (int j = 0; j < kEpiCols; j++) v[j] = gelu_tanh(v[j]);
            }
        }
    }
    if (lane == 0) bulk_wait_read_all();   // the previous store has read the staging tile
    __syncwarp();
    if constexpr (EPI == TC_SWIGLU) {
        uint32_t h[kEpiCols / 4], clamp = 0;
#pragma unroll
        for (int j = 0; j < kEpiCols; j += 4) {
            h[j >> 2] = pack16x2(silu_fast(v[j]) * v[j + 1], silu_fast(v[j + 2]) * v[j + 3], p.f16);
            clamp = f16x2_absmax(clamp, h[j >> 2]);
        }
        if (p.f16) count_clamped(clamp);
        swz_put<32>(stg, lane, 0, make_uint4(h[0], h[1], h[2], h[3]));
        swz_put<32>(stg, lane, 1, make_uint4(h[4], h[5], h[6], h[7]));
    } else if (EPI == TC_QKV_ENC || p.out_bf16) {   // 16-bit outputs, 64-byte rows
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const float *w = v + 8 * c;
            const uint4 u = EPI == TC_QKV_ENC
                                ? make_uint4(pack_half2(w[0], w[1]), pack_half2(w[2], w[3]), pack_half2(w[4], w[5]),
                                             pack_half2(w[6], w[7]))
                                : make_uint4(pack16x2(w[0], w[1], p.f16), pack16x2(w[2], w[3], p.f16),
                                             pack16x2(w[4], w[5], p.f16), pack16x2(w[6], w[7], p.f16));
            swz_put<64>(stg, lane, c, u);
        }
    } else {   // fp32 outputs, 128-byte rows
#pragma unroll
        for (int c = 0; c < 8; c++)
            swz_put<128>(stg, lane, c,
                         make_uint4(__float_as_uint(v[4 * c]), __float_as_uint(v[4 * c + 1]),
                                    __float_as_uint(v[4 * c + 2]), __float_as_uint(v[4 * c + 3])));
    }
    fence_async_smem();
    __syncwarp();
    if (lane == 0) {
        if constexpr (EPI == TC_SWIGLU) {
            tma_store_2d(mp.o, stg, col0 >> 1, row0);
        } else if constexpr (EPI == TC_RESID) {
            tma_reduce_add_2d(mp.o, stg, col0, row0);
        } else if constexpr (EPI == TC_QKV_ENC) {
            if (region == 0) tma_store_2d(mp.o, stg, col0, row0);
            else tma_store_2d(region == 1 ? mp.k : mp.v, stg, col0 - region * kEncQkv, (int)er.slot);
        } else {
            tma_store_2d(mp.o, stg, col0, row0);
        }
        bulk_commit();
    }
}

// TC_RESID with the folded norm (direct stores): the warp's half of the BN
// columns of its 32 rows, 32 columns per step.  Every step's residual line
// (128 bytes of the row) is prefetched into L1 first, and each step issues
// its residual loads before its accumulator read, so the L2 latency of the
// read-modify-write overlaps; then x, fp16(x * gain) and the chunk sums.
template <int BN>
__device__ __forceinline__ void resid_norm_tile(const TcGemmParams &p, uint32_t tbase, int row, int n0, int half,
                                                bool rv) {
    constexpr int kSteps = BN / 2 / kEpiCols;
    const int c0 = half * (BN / 2);
    float *xr = p.out + (size_t)row * p.ldo + n0 + c0;
    if (rv) {
#pragma unroll
        for (int i = 0; i < kSteps; i++)
            if (n0 + c0 + i * kEpiCols < p.N) asm volatile("prefetch.global.L1 [%0];" ::"l"(xr + i * kEpiCols));
    }
#pragma unroll 1
    for (int i = 0; i < kSteps; i++) {
        const int c = c0 + i * kEpiCols, col0 = n0 + c;
        const bool in = rv && col0 < p.N;
        float4 r[kEpiCols / 4];
#pragma unroll
        for (int j = 0; j < kEpiCols / 4; j++)
            r[j] = in ? *reinterpret_cast<const float4 *>(xr + i * kEpiCols + 4 * j) : make_float4(0.f, 0.f, 0.f, 0.f);
        float v[kEpiCols];
        tmem_ld32(tbase + (uint32_t)c, v);   // warp-collective: before any branch
        if (!in) continue;
        add_bias(v, p.bias, col0, p.N);
#pragma unroll
        for (int j = 0; j < kEpiCols / 4; j++)
            v[4 * j] += r[j].x, v[4 * j + 1] += r[j].y, v[4 * j + 2] += r[j].z, v[4 * j + 3] += r[j].w;
        float *o = xr + i * kEpiCols;
#pragma unroll
        for (int j = 0; j < kEpiCols; j += 4)
            *reinterpret_cast<float4 *>(o + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        norm_prep_chunk(p, row, col0, v);
    }
}

// TC_RESID with the folded norm when the stage ring is drained (the CTA's
// last tile, or a cluster split's reduction): the warp's residual chunks
// (32 rows x 32 fp32 columns each) arrive by TMA in the 128-byte swizzle
// into `t` (already issued on the warp's barrier); the updated rows go back
// into the same tile, fp16(x * gain) into `t16` (64-byte swizzle), and both
// leave by TMA stores (whole lines; rows past M are clipped); the chunk sums
// of squares are stored per row.  The same arithmetic as resid_norm_tile and
// norm_prep_chunk: x = (acc + bias) + residual, one fp16 rounding of x * gain.
__device__ __forceinline__ void resid_fold_chunk_tma(const TcGemmParams &p, const EpiMaps &mp, float (&v)[kEpiCols],
                                                     int row0, int col0, int lane, unsigned char *t,
                                                     unsigned char *t16) {
    add_bias(v, p.bias, col0, p.N);
    const bool rv = row0 + lane < p.M;
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < kEpiCols / 4; j++) {
        float4 *a = reinterpret_cast<float4 *>(t + lane * 128 + 16 * (j ^ (lane & 7)));
        const float4 r = *a;
        v[4 * j] += r.x, v[4 * j + 1] += r.y, v[4 * j + 2] += r.z, v[4 * j + 3] += r.w;
        *a = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    }
#pragma unroll
    for (int j = 0; j < kEpiCols; j++) ss = fmaf(v[j], v[j], ss);
    if (rv) p.ss_out[(size_t)(col0 / kEpiCols) * p.ss_ld + row0 + lane] = ss;
    uint32_t h[kEpiCols / 2], mx = 0;
#pragma unroll
    for (int j = 0; j < kEpiCols; j += 4) {
        const float4 g = __ldg(reinterpret_cast<const float4 *>(p.xn_gain + col0 + j));
        h[j >> 1] = pack_half2(v[j] * g.x, v[j + 1] * g.y);
        h[(j >> 1) + 1] = pack_half2(v[j + 2] * g.z, v[j + 3] * g.w);
        mx = f16x2_absmax(mx, h[j >> 1]);
        mx = f16x2_absmax(mx, h[(j >> 1) + 1]);
    }
    if (rv) count_clamped(mx);
#pragma unroll
    for (int c = 0; c < 4; c++) swz_put<64>(t16, lane, c, make_uint4(h[4 * c], h[4 * c + 1], h[4 * c + 2], h[4 * c + 3]));
    fence_async_smem();
    __syncwarp();
    if (lane == 0) {
        tma_store_2d(mp.o, t, col0, row0);
        tma_store_2d(mp.k, t16, col0, row0);
    }
}

// issue the residual loads of the warp's chunks [col0, col0 + 32 n) of rows
// row0.. (lane 0); the number of chunks inside N, 0 when none is loaded
__device__ __forceinline__ int resid_fold_issue(const TcGemmParams &p, const EpiMaps &mp, int row0, int col0,
                                                int n, int lane, unsigned char *buf, uint64_t *bar) {
    if (row0 >= p.M) return 0;
    int nin = 0;
    while (nin < n && col0 + nin * kEpiCols < p.N) nin++;
    if (lane == 0 && nin > 0) {
        mbar_expect_tx(bar, (uint32_t)(nin * kStageBytes));
        for (int i = 0; i < nin; i++) tma_load_2d_plain(buf + i * kStageBytes, mp.o, col0 + i * kEpiCols, row0, bar);
    }
    return nin;
}

template <int BN>
__device__ __forceinline__ bool resid_fold_tile_tma(const TcGemmParams &p, const EpiMaps &mp, uint32_t tbase,
                                                    int row0, int n0, int half, int lane, unsigned char *buf,
                                                    unsigned char *buf16, uint64_t *bar, uint64_t deadline) {
    constexpr int kSteps = BN / 2 / kEpiCols;
    const int c0 = half * (BN / 2);
    const int nin = resid_fold_issue(p, mp, row0, n0 + c0, kSteps, lane, buf, bar);
    bool got = true;
    if (nin > 0) got = __all_sync(0xffffffffu, mbar_wait(bar, 0, deadline));
#pragma unroll 1
    for (int i = 0; i < kSteps; i++) {
        float v[kEpiCols];
        tmem_ld32(tbase + (uint32_t)(c0 + i * kEpiCols), v);   // warp-collective: before any branch
        if (i < nin && got)
            resid_fold_chunk_tma(p, mp, v, row0, n0 + c0 + i * kEpiCols, lane, buf + i * kStageBytes,
                                 buf16 + i * (kStageBytes / 2));
    }
    if (lane == 0 && nin > 0) bulk_commit();
    return got;
}

// The epilogue of one accumulator for one epilogue warp: this thread's row
// (its TMEM lane) and the warp's half of the BN columns from n0, 32 columns
// per tcgen05.ld.  row0 = the warp's first row.
template <int BN, int EPI>
__device__ __forceinline__ void epilogue_tile(const TcGemmParams &p, const EpiMaps &mp, uint32_t tbase, int row0,
                                              int n0, int half, int lane, unsigned char *stg, float rs = 1.0f) {
    static_assert(BN % (2 * kEpiCols) == 0, "each epilogue warp takes whole 32-column chunks");
    EpiRow er = epi_row<EPI>(p, row0 + lane);
    er.rs = rs;
    const bool rv = er.row < p.M;
    if constexpr (EPI == TC_RESID) {
        if (p.xn_out && p.vec && !p.tma_out) {
            resid_norm_tile<BN>(p, tbase, er.row, n0, half, rv);
            return;
        }
    }
#pragma unroll 1
    for (int c = half * (BN / 2); c < (half + 1) * (BN / 2); c += kEpiCols) {
        float v[kEpiCols];
        tmem_ld32(tbase + (uint32_t)c, v);   // warp-collective: before any branch
        const int col0 = n0 + c;
        if (col0 >= p.N) continue;           // warp-uniform
        scale_row<EPI>(p, er, v);
        if (p.tma_out) {
            epi_tma<EPI>(p, mp, er, v, row0, col0, lane, stg);
            continue;
        }
        if (!rv) continue;
        int region = 0;
        if constexpr (EPI == TC_QKV_ENC) region = qkv_apply(p, er, v, col0);
        if constexpr (EPI == TC_QKV_DEC) region = dec_qkv_apply(p, er, v, col0);
        if (p.vec && col0 + kEpiCols <= p.N) epi_vec<EPI>(p, er, v, col0, region);
        else epi_scalar<EPI>(p, er, v, col0, region);
    }
}

// Split-K workspace: one region of 32 rows x BN/2 columns per (slice ks,
// tile t, epilogue warp), the warp's TMEM lane quarter q and column half.
// Inside a region, column chunk cc (32 columns) holds 8 float4 groups, each
// with the 32 lanes' float4s side by side: every warp-wide store or load
// covers 512 consecutive bytes.  All rows and chunks below N are written
// (rows past M hold the products of zero-filled A rows and are never used).
__device__ __forceinline__ size_t split_region(int ks, int t, int tiles, int q, int half, int bn) {
    return (((size_t)ks * tiles + t) * kEpiWarps + half * 4 + q) * (size_t)(16 * bn);
}

// Split-K: one warp's 32 rows x BN/2 columns of slice ks -> its region.
template <int BN>
__device__ __forceinline__ void split_partial(const TcGemmParams &p, uint32_t tbase, int q, int n0, int half,
                                              int lane, int ks, int t, int tiles) {
    float4 *dst = reinterpret_cast<float4 *>(p.ws + split_region(ks, t, tiles, q, half, BN)) + lane;
#pragma unroll 1
    for (int c = half * (BN / 2); c < (half + 1) * (BN / 2); c += kEpiCols) {
        float v[kEpiCols];
        tmem_ld32(tbase + (uint32_t)c, v);   // warp-collective: before any branch
        if (n0 + c >= p.N) continue;          // warp-uniform
        float4 *d = dst + (size_t)((c - half * (BN / 2)) / kEpiCols) * (kEpiCols / 4) * 32;
#pragma unroll
        for (int j = 0; j < kEpiCols / 4; j++)
            __stcg(d + 32 * j, make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]));
    }
}

// Split-K: sum the KS slices of the sub-tile in slice order (the same sum
// whichever slice finished last) and run the epilogue on it.
template <int BN, int EPI>
__device__ __forceinline__ void split_finish(const TcGemmParams &p, const EpiMaps &mp, int row0, int n0, int half,
                                             int lane, unsigned char *stg, int KS, int q, int t, int tiles,
                                             float rs = 1.0f) {
    EpiRow er = epi_row<EPI>(p, row0 + lane);
    er.rs = rs;
    const bool rv = er.row < p.M;
    const size_t slice = (size_t)tiles * kEpiWarps * 16 * BN;   // floats between slices
    const float4 *src0 = reinterpret_cast<const float4 *>(p.ws + split_region(0, t, tiles, q, half, BN)) + lane;
#pragma unroll 1
    for (int c = half * (BN / 2); c < (half + 1) * (BN / 2); c += kEpiCols) {
        const int col0 = n0 + c;
        if (col0 >= p.N) continue;   // warp-uniform
        float v[kEpiCols];
#pragma unroll
        for (int j = 0; j < kEpiCols; j++) v[j] = 0.f;
        if (rv) {
            const float4 *src = src0 + (size_t)((c - half * (BN / 2)) / kEpiCols) * (kEpiCols / 4) * 32;
            // two slices in flight: the loads of slice s+1 are issued before
            // the adds of slice s (the adds stay in slice order)
            float4 cur[kEpiCols / 4], nxt[kEpiCols / 4];
#pragma unroll
            for (int j = 0; j < kEpiCols / 4; j++) cur[j] = __ldcg(src + 32 * j);
            for (int s = 0; s < KS; s++) {
                if (s + 1 < KS) {
                    const float4 *nsrc = src + (size_t)(s + 1) * (slice / 4);
#pragma unroll
                    for (int j = 0; j < kEpiCols / 4; j++) nxt[j] = __ldcg(nsrc + 32 * j);
                }
#pragma unroll
                for (int j = 0; j < kEpiCols / 4; j++)
                    v[4 * j] += cur[j].x, v[4 * j + 1] += cur[j].y, v[4 * j + 2] += cur[j].z,
                        v[4 * j + 3] += cur[j].w;
#pragma unroll
                for (int j = 0; j < kEpiCols / 4; j++) cur[j] = nxt[j];
            }
        }
        scale_row<EPI>(p, er, v);
        if (p.tma_out) {
            epi_tma<EPI>(p, mp, er, v, row0, col0, lane, stg);
            continue;
        }
        if (!rv) continue;
        int region = 0;
        if constexpr (EPI == TC_QKV_ENC) region = qkv_apply(p, er, v, col0);
        if constexpr (EPI == TC_QKV_DEC) region = dec_qkv_apply(p, er, v, col0);
        if (p.vec && col0 + kEpiCols <= p.N) epi_vec<EPI>(p, er, v, col0, region);
        else epi_scalar<EPI>(p, er, v, col0, region);
    }
}

// ---- split activations (p.hilo): accumulator rows r (hi) and r + 64 (lo)
// of a tile belong to output row tm * 64 + r.  TMEM lane quarters 0, 1 hold
// the hi rows, 2, 3 the lo rows; the epilogue warp of lo quarter q + 2 hands
// its chunk to the warp of quarter q (same column half) through shared
// memory, paced by two shared-memory counters per pair (chunks staged,
// chunks consumed) whose waits are bounded like every other wait.

// lane 0 spins until *f == want (or the deadline passes); warp-uniform result
__device__ __forceinline__ bool flag_wait(volatile int *f, int want, uint64_t deadline, int lane) {
    int bad = 0;
    if (lane == 0) {
        while (*f != want)
            if (globaltimer() > deadline) {
                bad = 1;
                break;
            }
        __threadfence_block();
    }
    return __shfl_sync(0xffffffffu, bad, 0) == 0;
}

// The direct-store epilogue of one finished output chunk (token rows).
template <int EPI>
__device__ __forceinline__ void epi_direct(const TcGemmParams &p, const EpiRow &er, float (&v)[kEpiCols], int col0) {
    int region = 0;
    if constexpr (EPI == TC_QKV_ENC) region = qkv_apply(p, er, v, col0);
    if constexpr (EPI == TC_QKV_DEC) region = dec_qkv_apply(p, er, v, col0);
    if (p.vec && col0 + kEpiCols <= p.N) epi_vec<EPI>(p, er, v, col0, region);
    else epi_scalar<EPI>(p, er, v, col0, region);
}

// One accumulator of a split-activation tile: warp quarter q, column half.
// xch: the pair's exchange tile (the lo warp's staging area, 32 x 32 fp32,
// column-major so both sides access it without bank conflicts); flg: the
// pair's counters {staged, consumed}; seq: chunks exchanged so far by this
// pair.  Returns false when a wait expired.
template <int BN, int EPI>
__device__ __forceinline__ bool epilogue_pair(const TcGemmParams &p, uint32_t tbase, int tm, int n0, int q, int half,
                                              int lane, float *xch, volatile int *flg, int &seq, uint64_t deadline,
                                              float rs = 1.0f) {
    const bool hi = q < 2;
    EpiRow er = epi_row<EPI>(p, tm * 64 + 32 * (q & 1) + lane);
    er.rs = rs;
    const bool rv = er.row < p.M;
#pragma unroll 1
    for (int c = half * (BN / 2); c < (half + 1) * (BN / 2); c += kEpiCols) {
        float v[kEpiCols];
        tmem_ld32(tbase + (uint32_t)c, v);   // warp-collective: before any branch
        const int col0 = n0 + c;
        if (col0 >= p.N) continue;           // the same for both warps of the pair
        if (!hi) {
            if (!flag_wait(&flg[1], seq, deadline, lane)) return false;   // previous chunk consumed
#pragma unroll
            for (int j = 0; j < kEpiCols; j++) xch[j * 32 + lane] = v[j];
            __syncwarp();
            if (lane == 0) {
                __threadfence_block();
                flg[0] = seq + 1;
            }
            seq++;
            continue;
        }
        if (!flag_wait(&flg[0], seq + 1, deadline, lane)) return false;   // this chunk staged
        __syncwarp();
#pragma unroll
        for (int j = 0; j < kEpiCols; j++) v[j] += xch[j * 32 + lane];
        __syncwarp();
        if (lane == 0) {
            __threadfence_block();
            flg[1] = seq + 1;
        }
        seq++;
        scale_row<EPI>(p, er, v);
        if (rv) epi_direct<EPI>(p, er, v, col0);
    }
    return true;
}

// Split-K finish of one pair's 32 output rows x BN/2 columns: the slices of
// the hi (lane quarter qq) and the lo (quarter qq + 2) accumulator rows
// summed in slice order.
template <int BN, int EPI>
__device__ __forceinline__ void split_finish_pair(const TcGemmParams &p, int tm, int qq, int n0, int half, int lane,
                                                  int KS, int t, int tiles, float rs = 1.0f) {
    EpiRow er = epi_row<EPI>(p, tm * 64 + 32 * qq + lane);
    er.rs = rs;
    if (er.row >= p.M) return;
    const size_t slice = (size_t)tiles * kEpiWarps * 16 * BN / 4;   // float4s between slices
    const float4 *hi0 = reinterpret_cast<const float4 *>(p.ws + split_region(0, t, tiles, qq, half, BN)) + lane;
    const float4 *lo0 = reinterpret_cast<const float4 *>(p.ws + split_region(0, t, tiles, qq + 2, half, BN)) + lane;
#pragma unroll 1
    for (int c = half * (BN / 2); c < (half + 1) * (BN / 2); c += kEpiCols) {
        const int col0 = n0 + c;
        if (col0 >= p.N) continue;
        const size_t cc = (size_t)((c - half * (BN / 2)) / kEpiCols) * (kEpiCols / 4) * 32;
        float v[kEpiCols];
#pragma unroll
        for (int j = 0; j < kEpiCols; j++) v[j] = 0.f;
        for (int s = 0; s < KS; s++) {
            const float4 *a = hi0 + (size_t)s * slice + cc;
            const float4 *b = lo0 + (size_t)s * slice + cc;
#pragma unroll
            for (int j = 0; j < kEpiCols / 4; j++) {
                const float4 x = __ldcg(a + 32 * j);
                const float4 y = __ldcg(b + 32 * j);
                v[4 * j] += x.x + y.x, v[4 * j + 1] += x.y + y.y, v[4 * j + 2] += x.z + y.z,
                    v[4 * j + 3] += x.w + y.w;
            }
        }
        scale_row<EPI>(p, er, v);
        epi_direct<EPI>(p, er, v, col0);
    }
}

// ---- cluster split-K (one row tile, p.cluster): the KS K slices of a tile
// are the KS CTAs of a thread-block cluster.  Each stages its fp32 partial in
// its drained stage ring, 32 x 32 chunks lane-contiguous ([8 float4][32
// lanes], the epilogue warp's region); after a cluster barrier the 8 x KS
// epilogue warps of the cluster split the tile's chunks, each summing one
// chunk over the KS CTAs (distributed shared memory, rank order: the same
// sum whichever CTA reads) and running the epilogue on it.

// split activations: chunks uh (hi rows) and ul (lo rows) summed over the KS
// CTAs, hi + lo per slice, in rank order
template <int BN>
__device__ __forceinline__ void cl_sum_chunk_pair(const float4 *part, int uh, int ul, int KS, int lane,
                                                  float (&v)[kEpiCols]) {
    const uint32_t bh = smem_u32(part + (size_t)uh * 256 + lane), bl = smem_u32(part + (size_t)ul * 256 + lane);
#pragma unroll
    for (int j = 0; j < kEpiCols; j++) v[j] = 0.f;
    for (int r = 0; r < KS; r++) {
        const uint32_t rh = mapa_shared(bh, (uint32_t)r), rl = mapa_shared(bl, (uint32_t)r);
#pragma unroll
        for (int j = 0; j < kEpiCols / 4; j++) {
            const float4 x = ld_dsmem_f4(rh + 512u * j), y = ld_dsmem_f4(rl + 512u * j);
            v[4 * j] += x.x + y.x, v[4 * j + 1] += x.y + y.y, v[4 * j + 2] += x.z + y.z, v[4 * j + 3] += x.w + y.w;
        }
    }
}

// this warp's chunks (of its column half) of the accumulator -> its region
template <int BN>
__device__ __forceinline__ void cl_stage_partial(uint32_t tbase, float4 *part, int ew, int half, int lane) {
#pragma unroll 1
    for (int cc = 0; cc < BN / 64; cc++) {
        float v[kEpiCols];
        tmem_ld32(tbase + (uint32_t)(half * (BN / 2) + cc * kEpiCols), v);
        float4 *d = part + (size_t)(ew * (BN / 64) + cc) * 256 + lane;
#pragma unroll
        for (int j = 0; j < kEpiCols / 4; j++) d[32 * j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    }
}

// chunk uu of the tile summed over the KS CTAs, in rank order
template <int BN>
__device__ __forceinline__ void cl_sum_chunk(const float4 *part, int uu, int KS, int lane, float (&v)[kEpiCols]) {
    const uint32_t base = smem_u32(part + (size_t)uu * 256 + lane);
#pragma unroll
    for (int j = 0; j < kEpiCols; j++) v[j] = 0.f;
    for (int r = 0; r < KS; r++) {
        float4 a[kEpiCols / 4];
        const uint32_t ra = mapa_shared(base, (uint32_t)r);
#pragma unroll
        for (int j = 0; j < kEpiCols / 4; j++) a[j] = ld_dsmem_f4(ra + 512u * j);
#pragma unroll
        for (int j = 0; j < kEpiCols / 4; j++) {
            v[4 * j] += a[j].x, v[4 * j + 1] += a[j].y, v[4 * j + 2] += a[j].z, v[4 * j + 3] += a[j].w;
        }
    }
}

template <int BN, int EPI, bool HILO = false>
__global__ void __launch_bounds__(kTcThreads, 1)
tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmO, const __grid_constant__ CUtensorMap tmK,
               const __grid_constant__ CUtensorMap tmV, const TcGemmParams p) {
    using Cfg = TcCfg<BN>;
    constexpr int S = Cfg::kStages;
    extern __shared__ unsigned char smem_raw[];
    unsigned char *smem = (unsigned char *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    unsigned char *sA = smem;
    unsigned char *sB = smem + S * Cfg::kABytes;
    unsigned char *sStage = sB + S * Cfg::kBBytes;   // [kEpiWarps][kStageBytes] epilogue staging
    uint64_t *full = reinterpret_cast<uint64_t *>(sStage + kEpiWarps * kStageBytes);
    uint64_t *empty = full + S;
    uint64_t *tfull = empty + S;     // [2] accumulator b holds a finished tile
    uint64_t *tempty = tfull + 2;    // [2] accumulator b was drained by the epilogue
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tempty + 2);
    volatile int *pair_flags = reinterpret_cast<volatile int *>(tmem_slot + 1);   // HILO: [4 pairs][2]
    float *rs_s = reinterpret_cast<float *>(reinterpret_cast<unsigned char *>(full) + 256);   // [128]
    // the folded norm's residual loads: one barrier per epilogue warp, used once
    uint64_t *ebar = reinterpret_cast<uint64_t *>(reinterpret_cast<unsigned char *>(full) + 192);
    static_assert((2 * S + 4) * 8 + 4 + 32 <= 192, "barrier block overlaps the residual-load barriers");
    // the folded norm's tiles fit the drained ring: a last tile's fp32 + fp16
    // chunks, and (cluster splits: 64- or 128-wide) the partials + one chunk per warp
    static_assert(BN * 768 <= S * (Cfg::kABytes + Cfg::kBBytes), "fold tiles exceed the stage ring");
    static_assert(BN > 128 || BN * 512 + kEpiWarps * kStageBytes * 3 / 2 <= S * (Cfg::kABytes + Cfg::kBBytes),
                  "cluster fold tiles exceed the stage ring");

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool CL = p.cluster != 0;   // cluster split-K: one unit per CTA
    // row tiles: 128 output rows, or (HILO) 64 output rows = 128 A rows [hi; lo]
    const int MT = HILO ? (p.M + 63) / 64 : (p.M + kBM - 1) / kBM;
    const int tiles = MT * ((p.N + BN - 1) / BN);
    const int KB = (p.K + kBK - 1) / kBK;
    const int KS = p.ksplit > 1 ? p.ksplit : 1;   // K slices per tile (split-K)
    const int units = tiles * KS;
    const uint64_t deadline = globaltimer() + kTcWaitNs;
    bool ok = true;
    int cl_fold = 0;   // cluster split, folded norm: this warp's residual chunk is on its way

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], kEpiWarps);    // one arrival per epilogue warp
        }
        for (int i = 0; i < 8; i++) pair_flags[i] = 0;
        for (int w = 0; w < kEpiWarps; w++) mbar_init(&ebar[w], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        prefetch_tensormap(&tmA);
        prefetch_tensormap(&tmB);
        if (p.tma_out || p.fold_tma) prefetch_tensormap(&tmO);
        if (p.fold_tma) prefetch_tensormap(&tmK);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, Cfg::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // A and W are both re-read by other tiles (A by every column tile, W by
    // every row tile); keep both in L2.
    uint64_t pol = 0;
    // The first unit's first S weight stages go out before the dependency
    // wait: W is never written by the kernel this launch depends on (every
    // programmatic-dependent launch passes resident weights), so the weight
    // stream overlaps the previous kernel's tail; A follows the wait.
    int pre = 0;
    if (threadIdx.x == 0) {
        asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
        if ((int)blockIdx.x < units) {
            const int t = (int)blockIdx.x / KS, ks = (int)blockIdx.x % KS, n0 = (t / MT) * BN;
            const int kb0 = ks * KB / KS, nkb = (ks + 1) * KB / KS - kb0;
            pre = nkb < S ? nkb : S;
            for (int s = 0; s < pre; s++) {
                mbar_expect_tx(&full[s], Cfg::kABytes + Cfg::kBBytes);
                tma_load_2d(sB + s * Cfg::kBBytes, &tmB, (kb0 + s) * kBK, n0, &full[s], pol);
            }
        }
    }

    grid_dep_wait();
    grid_dep_launch();

    if (warp == 0) {
        if (lane == 0) {
            uint32_t it = 0;
            for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
                const int t = u / KS, ks = u % KS;
                const int m0 = (t % MT) * kBM, n0 = (t / MT) * BN;
                for (int kb = ks * KB / KS; kb < (ks + 1) * KB / KS; kb++, it++) {
                    const int s = it % S;
                    if (it < (uint32_t)pre) {   // its W is in flight already
                        tma_load_2d(sA + s * Cfg::kABytes, &tmA, kb * kBK, m0, &full[s], pol);
                        continue;
                    }
                    if (it >= (uint32_t)S && !mbar_wait(&empty[s], ((it / S) + 1) & 1u, deadline)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(&full[s], Cfg::kABytes + Cfg::kBBytes);
                    tma_load_2d(sA + s * Cfg::kABytes, &tmA, kb * kBK, m0, &full[s], pol);
                    tma_load_2d(sB + s * Cfg::kBBytes, &tmB, kb * kBK, n0, &full[s], pol);
                }
            }
            // tail: every stage's last release has arrived before the CTA can exit
            for (uint32_t j = it > (uint32_t)S ? it - S : 0; j < it && ok; j++)
                ok = mbar_wait(&empty[j % S], (j / S) & 1u, deadline);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // kind::f16 operand formats: bf16 (1) or fp16 (0) for A (bits 7-9) and B (10-12)
            const uint32_t idesc = p.f16 ? (idesc_bf16(kBM, BN) & ~((1u << 7) | (1u << 10))) : idesc_bf16(kBM, BN);
            uint32_t it = 0, lt = 0;
            for (int u = blockIdx.x; u < units && ok; u += gridDim.x, lt++) {
                const int ks = u % KS, kb_first = ks * KB / KS;
                const uint32_t b = lt & 1u;
                if (lt >= 2 && !mbar_wait(&tempty[b], ((lt >> 1) + 1) & 1u, deadline)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + b * (Cfg::kTmemCols / 2);   // accumulator b at half the allocation
                for (int kb = kb_first; kb < (ks + 1) * KB / KS; kb++, it++) {
                    const int s = it % S;
                    if (!mbar_wait(&full[s], (it / S) & 1u, deadline)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t a0 = smem_desc_sw128(sA + s * Cfg::kABytes);
                    const uint64_t b0 = smem_desc_sw128(sB + s * Cfg::kBBytes);
#pragma unroll
                    for (int k = 0; k < kBK / 16; k++)   // +32 bytes (2 x 16) per K=16 step
                        tc_mma_bf16(d, a0 + 2 * k, b0 + 2 * k, idesc, (kb != kb_first || k != 0) ? 1u : 0u);
                    tc_commit(&empty[s]);
                }
                if (ok) tc_commit(&tfull[b]);
            }
        }
    } else {
        // ---- epilogue: warp quarter q owns TMEM lanes 32q..32q+31 = tile rows ----
        const int q = warp & 3, half = (warp - 2) >> 2;   // TMEM lane quarter, column half
        const EpiMaps mp = {&tmO, &tmK, &tmV};
        unsigned char *stg = sStage + (warp - 2) * kStageBytes;
        int pair_seq = 0;   // HILO: chunks this warp's pair has exchanged
        uint32_t lt = 0;
        for (int u = blockIdx.x; u < units; u += gridDim.x, lt++) {
            const int t = u / KS, ks = u % KS;
            const uint32_t b = lt & 1u;
            // ss_in: the row's 1 / rms while the accumulator is still being
            // summed (with split-K whichever slice finishes last scales)
            float rs = 1.0f;
            if constexpr (EPI == TC_QKV_ENC || EPI == TC_SWIGLU || EPI == TC_QKV_DEC) {
                // (HILO: the pair's output rows; either warp may finish them)
                const int r = HILO ? (t % MT) * 64 + 32 * (q & 1) + lane : (t % MT) * kBM + 32 * q + lane;
                if (p.ss_in && r < p.M) rs = row_inv_rms(p.ss_in, p.ss_ld, r, p.K);
            }
            const bool got = mbar_wait(&tfull[b], (lt >> 1) & 1u, deadline);
            if (!__all_sync(0xffffffffu, got)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const int m0 = (t % MT) * kBM, n0 = (t / MT) * BN;
            const uint32_t tb = tmem + ((uint32_t)(32 * q) << 16) + b * (Cfg::kTmemCols / 2);
            if constexpr (HILO) {
                if (CL) {   // this slice's hi / lo partials into the drained ring (summed after the barrier)
                    cl_stage_partial<BN>(tb, reinterpret_cast<float4 *>(smem), warp - 2, half, lane);
                    if (half == 0) rs_s[32 * q + lane] = rs;
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tempty[b]);
                } else if (KS == 1) {
                    // the lo warp of the pair (warp - 2 for a hi warp) stages its chunks
                    float *xch = reinterpret_cast<float *>(sStage + ((q < 2 ? warp - 2 : warp) - 2) * kStageBytes);
                    if (!epilogue_pair<BN, EPI>(p, tb, t % MT, n0, q, half, lane, xch,
                                                pair_flags + 2 * (half * 2 + (q & 1)), pair_seq, deadline, rs)) {
                        ok = false;
                        break;
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tempty[b]);
                } else {
                    split_partial<BN>(p, tb, q, n0, half, lane, ks, t, tiles);
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tempty[b]);
                    // the pair's 2 x KS partials: the last to arrive finishes the rows
                    __threadfence();
                    __syncwarp();
                    const int pair = half * 2 + (q & 1);
                    unsigned prev = 0;
                    if (lane == 0) prev = atomicAdd(&p.ws_cnt[t * 4 + pair], 1u);
                    prev = __shfl_sync(0xffffffffu, prev, 0);
                    if (prev == (unsigned)(2 * KS - 1)) {
                        __threadfence();
                        split_finish_pair<BN, EPI>(p, t % MT, q & 1, n0, half, lane, KS, t, tiles, rs);
                        if (lane == 0) p.ws_cnt[t * 4 + pair] = 0u;
                    }
                }
                continue;
            }
            if (CL) {   // this slice's partial into the drained ring; the epilogue runs after the cluster barrier
                cl_stage_partial<BN>(tb, reinterpret_cast<float4 *>(smem), warp - 2, half, lane);
                if (half == 0) rs_s[32 * q + lane] = rs;
                if constexpr (EPI == TC_RESID) {
                    if (p.fold_tma) {   // the residual of this warp's first reduced chunk, behind the partials
                        const int uu = (warp - 2) * KS + ks;
                        if (uu < kEpiWarps * (BN / 64)) {
                            const int ew = uu / (BN / 64), cc = uu % (BN / 64);
                            cl_fold = resid_fold_issue(p, mp, m0 + 32 * ((ew + 2) & 3),
                                                       n0 + (ew >> 2) * (BN / 2) + cc * kEpiCols, 1, lane,
                                                       smem + BN * 512 + (warp - 2) * kStageBytes, &ebar[warp - 2]);
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[b]);
            } else if (KS == 1) {
                bool done = false;
                if constexpr (EPI == TC_RESID) {
                    if (p.fold_tma && u + (int)gridDim.x >= units) {
                        // the CTA's last tile: the drained stage ring holds the residual tiles
                        // (fp32 tiles [0, BN * 512), fp16 tiles [BN * 512, BN * 768) of the ring)
                        if (!resid_fold_tile_tma<BN>(p, mp, tb, m0 + 32 * q, n0, half, lane,
                                                     smem + (warp - 2) * (BN / 64) * kStageBytes,
                                                     smem + BN * 512 + (warp - 2) * (BN / 64) * (kStageBytes / 2),
                                                     &ebar[warp - 2], deadline)) {
                            ok = false;
                            break;
                        }
                        done = true;
                    }
                }
                if (!done) epilogue_tile<BN, EPI>(p, mp, tb, m0 + 32 * q, n0, half, lane, stg, rs);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[b]);
            } else {
                // this split's partial of the warp's 32 x BN/2 sub-tile -> workspace
                split_partial<BN>(p, tb, q, n0, half, lane, ks, t, tiles);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[b]);   // the accumulator is free already
                // the last of the KS partials of this sub-tile sums them (fixed
                // order) and runs the epilogue
                __threadfence();
                __syncwarp();
                unsigned prev = 0;
                if (lane == 0) prev = atomicAdd(&p.ws_cnt[t * kEpiWarps + (warp - 2)], 1u);
                prev = __shfl_sync(0xffffffffu, prev, 0);
                if (prev == (unsigned)(KS - 1)) {
                    __threadfence();
                    split_finish<BN, EPI>(p, mp, m0 + 32 * q, n0, half, lane, stg, KS, q, t, tiles, rs);
                    if (lane == 0) p.ws_cnt[t * kEpiWarps + (warp - 2)] = 0u;
                }
            }
        }
    }

    if (CL) {
        // every slice's partial is in its CTA's shared memory (every thread of
        // every CTA arrives, whatever failed before: no CTA waits forever)
        cluster_sync_all();
        if (warp >= 2 && ok) {
            const int t = (int)blockIdx.x / KS, rank = (int)blockIdx.x % KS;
            const int m0 = (t % MT) * kBM, n0 = (t / MT) * BN;
            const EpiMaps mp = {&tmO, &tmK, &tmV};
            unsigned char *stg = sStage + (warp - 2) * kStageBytes;
            constexpr int U = kEpiWarps * (BN / 64);   // 32 x 32 chunks of the tile
            if constexpr (HILO) {
                // output chunks: 2 row quarters (hi rows 32 qq.., lo rows 64 + 32 qq..)
                // x 2 column halves x BN / 64; each sums its hi and lo partials
                // over the KS CTAs, hi + lo per slice in slice order (as the
                // workspace split's split_finish_pair)
                constexpr int C2 = BN / 64;
                for (int uu = (warp - 2) * KS + rank; uu < 4 * C2; uu += kEpiWarps * KS) {
                    const int qq = uu / (2 * C2), hf = (uu / C2) & 1, cc = uu % C2;
                    const int col0 = n0 + hf * (BN / 2) + cc * kEpiCols;
                    float v[kEpiCols];
                    cl_sum_chunk_pair<BN>(reinterpret_cast<const float4 *>(smem), (4 * hf + qq + 2) * C2 + cc,
                                          (4 * hf + qq) * C2 + cc, KS, lane, v);
                    if (col0 >= p.N) continue;   // warp-uniform
                    EpiRow er = epi_row<EPI>(p, (t % MT) * 64 + 32 * qq + lane);
                    er.rs = rs_s[32 * qq + lane];
                    if (er.row >= p.M) continue;
                    scale_row<EPI>(p, er, v);
                    epi_direct<EPI>(p, er, v, col0);
                }
            }
            for (int uu = (warp - 2) * KS + rank; !HILO && uu < U; uu += kEpiWarps * KS) {
                const int ew = uu / (BN / 64), cc = uu % (BN / 64);
                const int q = (ew + 2) & 3, half = ew >> 2;   // the writing warp's lane quarter / half
                const int row0 = m0 + 32 * q, col0 = n0 + half * (BN / 2) + cc * kEpiCols;
                float v[kEpiCols];
                cl_sum_chunk<BN>(reinterpret_cast<const float4 *>(smem), uu, KS, lane, v);
                if (col0 >= p.N) continue;   // warp-uniform
                if constexpr (EPI == TC_RESID) {
                    if (cl_fold && uu == (warp - 2) * KS + rank) {   // the chunk whose residual was loaded
                        if (!__all_sync(0xffffffffu, mbar_wait(&ebar[warp - 2], 0, deadline))) {
                            ok = false;
                            break;
                        }
                        resid_fold_chunk_tma(p, mp, v, row0, col0, lane, smem + BN * 512 + (warp - 2) * kStageBytes,
                                             smem + BN * 512 + kEpiWarps * kStageBytes +
                                                 (warp - 2) * (kStageBytes / 2));
                        if (lane == 0) bulk_commit();
                        continue;
                    }
                }
                EpiRow er = epi_row<EPI>(p, row0 + lane);
                er.rs = rs_s[32 * q + lane];
                scale_row<EPI>(p, er, v);
                if (p.tma_out) {
                    epi_tma<EPI>(p, mp, er, v, row0, col0, lane, stg);
                    continue;
                }
                if (er.row >= p.M) continue;
                int region = 0;
                if constexpr (EPI == TC_QKV_ENC) region = qkv_apply(p, er, v, col0);
                if constexpr (EPI == TC_QKV_DEC) region = dec_qkv_apply(p, er, v, col0);
                if (p.vec && col0 + kEpiCols <= p.N) epi_vec<EPI>(p, er, v, col0, region);
                else epi_scalar<EPI>(p, er, v, col0, region);
            }
        }
        cluster_sync_all();   // no CTA leaves while a peer still reads its partial
    }
    if (warp >= 2 && lane == 0 && (p.tma_out || p.fold_tma)) bulk_wait_all();   // epilogue stores complete
    if (!__all_sync(0xffffffffu, ok)) ok = false;
    if (!ok) {
        if (lane == 0) atomicExch(p.err, 1u);
        const uint64_t grace = globaltimer() + 10000000ull;   // let in-flight copies / MMAs land
        while (globaltimer() < grace) {
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, Cfg::kTmemCols);
    }
}


// ---------------------------------------------------------------------------
// CTA-pair variant: a cluster of two CTAs computes a 256 x BN tile with
// cta_group::2 MMAs (M = 256).  CTA r loads A rows [m0 + 128 r, +128) and W
// rows [n0 + r BN/2, +BN/2) into its own shared memory; both halves land on
// rank 0's `full` barrier; rank 0 issues the MMAs, which read A and W from
// both CTAs and write each CTA's 128 rows x BN columns to that CTA's TMEM.
// Per SM, a k-block moves (128 + BN/2) x 64 operand elements instead of
// (128 + BN) x 64, a third less L2 -> shared memory traffic at BN = 256.
// Both CTAs run the epilogue over their own rows; accumulator releases go to
// rank 0's `tempty`.  No load is multicast.
// ---------------------------------------------------------------------------
template <int BN>
struct Tc2Cfg {
    static constexpr int kABytes = kBM * kBK * 2;
    static constexpr int kBBytes = (BN / 2) * kBK * 2;
    static constexpr int kStages = (196608 / (kABytes + kBBytes)) < 8 ? (196608 / (kABytes + kBBytes)) : 8;
    static constexpr int kTmemCols = 2 * BN;
    static constexpr int kSmem =
        kStages * (kABytes + kBBytes) + kEpiWarps * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;
};

template <int BN, int EPI>
__global__ void __launch_bounds__(kTcThreads, 1)
tc_gemm2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmO, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, const TcGemmParams p) {
    using Cfg = Tc2Cfg<BN>;
    constexpr int S = Cfg::kStages;
    extern __shared__ unsigned char smem_raw[];
    unsigned char *smem = (unsigned char *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    unsigned char *sA = smem;
    unsigned char *sB = smem + S * Cfg::kABytes;
    unsigned char *sStage = sB + S * Cfg::kBBytes;   // [kEpiWarps][kStageBytes] epilogue staging
    uint64_t *full = reinterpret_cast<uint64_t *>(sStage + kEpiWarps * kStageBytes);   // used on rank 0
    uint64_t *empty = full + S;
    uint64_t *tfull = empty + S;      // [2]
    uint64_t *tempty = tfull + 2;     // [2], used on rank 0
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tempty + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const int cl = blockIdx.x >> 1, ncl = gridDim.x >> 1;
    const int MT = (p.M + 2 * kBM - 1) / (2 * kBM);
    const int tiles = MT * ((p.N + BN - 1) / BN);
    const int KB = (p.K + kBK - 1) / kBK;
    const uint64_t deadline = globaltimer() + kTcWaitNs;
    bool ok = true;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 2 * kEpiWarps);    // epilogue warps of both CTAs
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        prefetch_tensormap(&tmA);
        prefetch_tensormap(&tmB);
        if (p.tma_out) prefetch_tensormap(&tmO);
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, Cfg::kTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync_all();   // barriers of both CTAs initialised, TMEM allocated
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    grid_dep_wait();
    grid_dep_launch();

    if (warp == 0) {
        if (lane == 0) {
            uint64_t pol;
            asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
            uint32_t it = 0;
            for (int t = cl; t < tiles && ok; t += ncl) {
                const int m0 = (t % MT) * 2 * kBM + (int)rank * kBM;
                const int nb = (t / MT) * BN + (int)rank * (BN / 2);
                for (int kb = 0; kb < KB; kb++, it++) {
                    const int s = it % S;
                    if (it >= (uint32_t)S && !mbar_wait(&empty[s], ((it / S) + 1) & 1u, deadline)) {
                        ok = false;
                        break;
                    }
                    if (rank == 0) mbar_expect_tx(&full[s], 2 * (Cfg::kABytes + Cfg::kBBytes));
                    const uint32_t fb = mapa_shared(smem_u32(&full[s]), 0);
                    tma_load_2d_pair(sA + s * Cfg::kABytes, &tmA, kb * kBK, m0, fb, pol);
                    tma_load_2d_pair(sB + s * Cfg::kBBytes, &tmB, kb * kBK, nb, fb, pol);
                }
            }
            // tail: every stage's last release (committed by rank 0) has arrived
            for (uint32_t j = it > (uint32_t)S ? it - S : 0; j < it && ok; j++)
                ok = mbar_wait(&empty[j % S], (j / S) & 1u, deadline);
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            const uint32_t idesc =
                p.f16 ? (idesc_bf16(2 * kBM, BN) & ~((1u << 7) | (1u << 10))) : idesc_bf16(2 * kBM, BN);
            uint32_t it = 0, lt = 0;
            for (int t = cl; t < tiles && ok; t += ncl, lt++) {
                const uint32_t b = lt & 1u;
                if (lt >= 2 && !mbar_wait(&tempty[b], ((lt >> 1) + 1) & 1u, deadline)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + b * BN;
                for (int kb = 0; kb < KB; kb++, it++) {
                    const int s = it % S;
                    if (!mbar_wait(&full[s], (it / S) & 1u, deadline)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t a0 = smem_desc_sw128(sA + s * Cfg::kABytes);
                    const uint64_t b0 = smem_desc_sw128(sB + s * Cfg::kBBytes);
#pragma unroll
                    for (int k = 0; k < kBK / 16; k++)
                        tc_mma_bf16_pair(d, a0 + 2 * k, b0 + 2 * k, idesc, (kb | k) != 0 ? 1u : 0u);
                    tc_commit_pair_both(&empty[s]);
                }
                if (!ok) break;
                tc_commit_pair_both(&tfull[b]);
            }
        }
    } else {
        const int q = warp & 3, half = (warp - 2) >> 2;   // TMEM lane quarter, column half
        const EpiMaps mp = {&tmO, &tmK, &tmV};
        unsigned char *stg = sStage + (warp - 2) * kStageBytes;
        const uint32_t te0 = mapa_shared(smem_u32(&tempty[0]), 0);
        const uint32_t te1 = mapa_shared(smem_u32(&tempty[1]), 0);
        uint32_t lt = 0;
        for (int t = cl; t < tiles; t += ncl, lt++) {
            const uint32_t b = lt & 1u;
            const bool got = mbar_wait(&tfull[b], (lt >> 1) & 1u, deadline);
            if (!__all_sync(0xffffffffu, got)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const int m0 = (t % MT) * 2 * kBM + (int)rank * kBM, n0 = (t / MT) * BN;
            epilogue_tile<BN, EPI>(p, mp, tmem + ((uint32_t)(32 * q) << 16) + b * BN, m0 + 32 * q, n0, half, lane,
                                   stg);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(b ? te1 : te0);
        }
    }

    if (warp >= 2 && lane == 0 && p.tma_out) bulk_wait_all();   // epilogue stores complete
    if (!__all_sync(0xffffffffu, ok)) ok = false;
    if (!ok) {
        if (lane == 0) atomicExch(p.err, 1u);
        const uint64_t grace = globaltimer() + 10000000ull;   // let in-flight copies / MMAs land
        while (globaltimer() < grace) {
        }
    }
    tc_fence_before();
    cluster_sync_all();   // both CTAs done with TMEM and with each other's barriers
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, Cfg::kTmemCols);
    }
}

// ---------------------------------------------------------------------------
// host side: tensor maps and launches
// ---------------------------------------------------------------------------

namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)p;
    });
    return fn;
}

// Row-major [rows, cols] tensor (row stride `ld` elements) of `esize`-byte
// elements, box [box_rows, box_cols], given swizzle.
bool make_map_2d(CUtensorMap *m, const void *ptr, CUtensorMapDataType dt, int esize, int rows, int cols, int ld,
                 int box_cols, int box_rows, CUtensorMapSwizzle swz) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)ld * (cuuint64_t)esize};
    const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(m, dt, 2, const_cast<void *>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// bf16 row-major [rows, cols] operand, box [box_rows, 64], 128B swizzle
bool make_map(CUtensorMap *m, const void *ptr, int rows, int cols, int box_rows) {
    return make_map_2d(m, ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows, cols, cols, kBK, box_rows,
                       CU_TENSOR_MAP_SWIZZLE_128B);
}

// Output maps of the TMA-store epilogue: one warp's 32 x 32 accumulator
// chunk per box.  Returns false when the epilogue must use direct stores.
bool make_out_maps(int epi, const TcGemmParams &p, CUtensorMap *mo, CUtensorMap *mk, CUtensorMap *mv) {
    switch (epi) {
        case TC_STORE:
            if (p.out_bf16)
                return make_map_2d(mo, p.out_bf16, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p.M, p.N, p.ldo_bf16, 32, 32,
                                   CU_TENSOR_MAP_SWIZZLE_64B);
            return make_map_2d(mo, p.out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, p.M, p.N, p.ldo, 32, 32,
                               CU_TENSOR_MAP_SWIZZLE_128B);
        case TC_RESID:   // out += acc + bias as one fp32 add per element, in L2
            if (p.out_bf16 || p.act != 0) return false;
            return make_map_2d(mo, p.out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, p.M, p.N, p.ldo, 32, 32,
                               CU_TENSOR_MAP_SWIZZLE_128B);
        case TC_SWIGLU:
            return make_map_2d(mo, p.out_bf16, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p.M, p.N / 2, p.ldo_bf16, 16, 32,
                               CU_TENSOR_MAP_SWIZZLE_32B);
        case TC_QKV_ENC:   // (a batched launch's rows go to several rings: direct stores)
            if (p.N != 3 * kEncQkv || p.cap < 32 || p.segs) return false;
            return make_map_2d(mo, p.q_out, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.M, kEncQkv, kEncQkv, 32, 32,
                               CU_TENSOR_MAP_SWIZZLE_64B) &&
                   make_map_2d(mk, p.k_ring, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.cap, kEncQkv, kEncQkv, 32, 32,
                               CU_TENSOR_MAP_SWIZZLE_64B) &&
                   make_map_2d(mv, p.v_ring, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.cap, kEncQkv, kEncQkv, 32, 32,
                               CU_TENSOR_MAP_SWIZZLE_64B);
    }
    return false;
}

int device_sms(int dev) {
    static std::atomic<int> cache[64];
    if (dev >= 0 && dev < 64) {
        const int v = cache[dev].load();
        if (v) return v;
    }
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    if (dev >= 0 && dev < 64) cache[dev].store(n);
    return n;
}

bool al16(const void *p) { return ((uintptr_t)p & 15) == 0; }

template <int BN, int EPI, bool HILO = false>
cudaError_t launch_bn(const TcGemmParams &p, const void *A, const void *W, cudaStream_t st, bool pdl,
                      const CUtensorMap &mo, const CUtensorMap &mk, const CUtensorMap &mv) {
    CUtensorMap ma, mb;
    // HILO: A holds hilo_rows(M) rows (per 64 output rows, their hi then lo rows)
    const int a_rows = HILO ? hilo_rows(p.M) : p.M;
    if (!make_map(&ma, A, a_rows, p.K, kBM) || !make_map(&mb, W, p.N, p.K, BN)) return cudaErrorInvalidValue;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    // the shared-memory opt-in is per device
    static std::atomic<uint64_t> attr_set{0};
    const uint64_t bit = 1ull << (dev & 63);
    if (!(attr_set.load() & bit)) {
        e = cudaFuncSetAttribute(tc_gemm_kernel<BN, EPI, HILO>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 TcCfg<BN>::kSmem);
        if (e != cudaSuccess) return e;
        attr_set.fetch_or(bit);
    }
    // work units: tiles x K slices (split-K)
    const int mt = HILO ? (p.M + 63) / 64 : (p.M + kBM - 1) / kBM;
    const int units = mt * ((p.N + BN - 1) / BN) * (p.ksplit > 1 ? p.ksplit : 1);
    const int sms = device_sms(dev);
    cudaLaunchConfig_t cfg = {};
    // (cluster split-K: exactly one unit per CTA, the slices of a tile one cluster)
    cfg.gridDim = dim3(p.cluster ? units : (units < sms ? units : sms));
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = TcCfg<BN>::kSmem;
    cfg.stream = st;
    cudaLaunchAttribute attr1[2];
    int na = 0;
    if (pdl) {
        attr1[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr1[na].val.programmaticStreamSerializationAllowed = 1;
        na++;
    }
    if (p.cluster) {
        attr1[na].id = cudaLaunchAttributeClusterDimension;
        attr1[na].val.clusterDim.x = p.ksplit;
        attr1[na].val.clusterDim.y = 1;
        attr1[na].val.clusterDim.z = 1;
        na++;
    }
    cfg.attrs = attr1;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, tc_gemm_kernel<BN, EPI, HILO>, ma, mb, mo, mk, mv, p);
}

int max_pair_clusters(const void *fn, int smem, int dev) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2);
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute a[1];
    a[0].id = cudaLaunchAttributeClusterDimension;
    a[0].val.clusterDim.x = 2;
    a[0].val.clusterDim.y = 1;
    a[0].val.clusterDim.z = 1;
    cfg.attrs = a;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        n = device_sms(dev) / 2;
    }
    return n;
}

template <int BN, int EPI>
cudaError_t launch_pair(const TcGemmParams &p, const void *A, const void *W, cudaStream_t st, bool pdl,
                        const CUtensorMap &mo, const CUtensorMap &mk, const CUtensorMap &mv) {
    CUtensorMap ma, mb;
    if (!make_map(&ma, A, p.M, p.K, kBM) || !make_map(&mb, W, p.N, p.K, BN / 2)) return cudaErrorInvalidValue;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const void *fn = (const void *)tc_gemm2_kernel<BN, EPI>;
    static std::atomic<uint64_t> attr_set{0};
    static std::atomic<int> clusters[64];
    const uint64_t bit = 1ull << (dev & 63);
    if (!(attr_set.load() & bit)) {
        e = cudaFuncSetAttribute(tc_gemm2_kernel<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 Tc2Cfg<BN>::kSmem);
        if (e != cudaSuccess) return e;
        clusters[dev & 63].store(max_pair_clusters(fn, Tc2Cfg<BN>::kSmem, dev));
        attr_set.fetch_or(bit);
    }
    const int tiles = ((p.M + 2 * kBM - 1) / (2 * kBM)) * ((p.N + BN - 1) / BN);
    const int ncl = std::min(tiles, std::max(1, clusters[dev & 63].load()));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * ncl);
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = Tc2Cfg<BN>::kSmem;
    cfg.stream = st;
    cudaLaunchAttribute a[2];
    a[0].id = cudaLaunchAttributeClusterDimension;
    a[0].val.clusterDim.x = 2;
    a[0].val.clusterDim.y = 1;
    a[0].val.clusterDim.z = 1;
    a[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    a[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = a;
    cfg.numAttrs = pdl ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, tc_gemm2_kernel<BN, EPI>, ma, mb, mo, mk, mv, p);
}

// VOX_CUDA_TC_PAIR = 0 | 1 forces the single-CTA or the CTA-pair kernel (read
// at every launch, so a test can switch it).
int env_tc_pair() {
    const char *s = getenv("VOX_CUDA_TC_PAIR");
    return (s && *s) ? atoi(s) : -1;
}

int env_int(const char *name) {
    const char *s = getenv(name);
    return (s && *s) ? atoi(s) : 0;
}

int env_tc_bn() {
    const char *s = getenv("VOX_CUDA_TC_BN");
    const int n = s ? atoi(s) : 0;
    return (n == 64 || n == 128 || n == 192 || n == 256) ? n : 0;
}

}  // namespace

// Tile width by a cost model of the persistent kernel: rounds of tiles over
// the SMs (ceil(tiles / SMs)) times the time of one tile, which measured
// ~120 + BN in the same units (a 128-wide tile takes 0.66 of a 256-wide one
// at the encoder's shapes, not 0.5).  Ties go to the wider tile.  It keeps
// the widths measured best at M = 1500 (256 for N = 10240 and 6144, 128 for
// N = 1280) and at M = 100 and 800; 192 wins where it fits in as many rounds
// as 256 (q|k|v at M = 500 and 800, w1|w3 at M = 500).
// VOX_CUDA_TC_BN = 64 | 128 | 192 | 256 forces a width.
// How many clusters of ks CTAs of the BN-wide kernel the device runs at
// once (one CTA per SM; clusters sit inside one GPC, so a cluster size that
// does not divide the GPCs' SM counts leaves SMs idle).  Cached per BN and
// cluster size; 0 when the query fails.
template <int BN>
int tc_max_clusters(int ks) {
    static std::atomic<int> cache[9];   // 0: not asked yet; -1: failed
    if (ks < 2 || ks > 8) return 0;
    int c = cache[ks].load();
    if (c == 0) {
        int n = 0;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(ks * 32);
        cfg.blockDim = dim3(kTcThreads);
        cfg.dynamicSmemBytes = TcCfg<BN>::kSmem;
        cudaLaunchAttribute a[1];
        a[0].id = cudaLaunchAttributeClusterDimension;
        a[0].val.clusterDim.x = ks;
        a[0].val.clusterDim.y = 1;
        a[0].val.clusterDim.z = 1;
        cfg.attrs = a;
        cfg.numAttrs = 1;
        if (cudaFuncSetAttribute(tc_gemm_kernel<BN, TC_STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 TcCfg<BN>::kSmem) != cudaSuccess ||
            cudaOccupancyMaxActiveClusters(&n, tc_gemm_kernel<BN, TC_STORE>, &cfg) != cudaSuccess) {
            cudaGetLastError();
            n = 0;
        }
        c = n > 0 ? n : -1;
        cache[ks].store(c);
    }
    return c > 0 ? c : 0;
}

int tc_max_clusters_bn(int bn, int ks) {
    switch (bn) {
        case 64: return tc_max_clusters<64>(ks);
        case 128: return tc_max_clusters<128>(ks);
        case 256: return tc_max_clusters<256>(ks);
    }
    return 0;
}

int tc_gemm_bn(int M, int N) {
    if (const int f = env_tc_bn()) return f;
    int dev = 0;
    cudaGetDevice(&dev);
    const int sms = device_sms(dev);
    const int mt = (M + kBM - 1) / kBM;
    int best = 256;
    long long best_t = -1;
    for (int bn : {256, 192, 128, 64}) {
        const long long tiles = (long long)mt * ((N + bn - 1) / bn);
        const long long t = (tiles + sms - 1) / sms * (120 + bn);
        if (best_t < 0 || t < best_t) best_t = t, best = bn;
    }
    return best;
}

// Pair tile width (256 x BN per CTA pair), same cost model over SM pairs.
int tc_gemm2_bn(int M, int N) {
    if (const int f = env_tc_bn()) return f >= 192 ? 256 : 128;
    int dev = 0;
    cudaGetDevice(&dev);
    const int pairs = device_sms(dev) / 2;
    const int mt = (M + 2 * kBM - 1) / (2 * kBM);
    const int widths[2] = {256, 128};
    const float col_cost[2] = {1.0f, 1.1f};
    int best = 256;
    float best_t = 1e30f;
    for (int i = 0; i < 2; i++) {
        const int tiles = mt * ((N + widths[i] - 1) / widths[i]);
        const float t = (float)((tiles + pairs - 1) / pairs) * (float)widths[i] * col_cost[i];
        if (t < best_t) best_t = t, best = widths[i];
    }
    return best;
}

cudaError_t launch_tc_gemm(int epi, const TcGemmParams &p_in, const void *A, const void *W, cudaStream_t st,
                           bool pdl, int bn) {
    TcGemmParams p = p_in;
    if (p.M <= 0 || p.N <= 0 || p.K <= 0 || p.K % 8 != 0 || !p.err || ((uintptr_t)A & 15) || ((uintptr_t)W & 15))
        return cudaErrorInvalidValue;
    if (epi == TC_SWIGLU && (p.N % 32 != 0)) return cudaErrorInvalidValue;
    // the folded RMSNorm: producer TC_RESID (fp16), consumers TC_QKV_ENC /
    // TC_SWIGLU; not with split activations
    // (split activations: bf16 hi / lo operand rows, consumers TC_QKV_DEC / TC_SWIGLU)
    if (p.xn_out && (epi != TC_RESID || !p.xn_gain || !p.ss_out || p.ss_ld < p.M || (p.hilo ? p.f16 : !p.f16)))
        return cudaErrorInvalidValue;
    if (p.ss_in && ((epi != TC_QKV_ENC && epi != TC_SWIGLU && epi != TC_QKV_DEC) || p.ss_ld < p.M || p.K % 32 != 0))
        return cudaErrorInvalidValue;
    switch (epi) {
        case TC_STORE:
        case TC_RESID: {
            const bool need_out = epi == TC_RESID || !p.out_bf16;
            p.vec = (!p.bias || al16(p.bias)) && (!need_out || (al16(p.out) && p.ldo % 4 == 0)) &&
                    (!p.out_bf16 || (al16(p.out_bf16) && p.ldo_bf16 % 8 == 0)) &&
                    (!p.xn_out || (al16(p.xn_out) && al16(p.xn_gain) && p.ldo % 8 == 0));
            break;
        }
        case TC_SWIGLU: p.vec = al16(p.out_bf16) && p.ldo_bf16 % 8 == 0; break;
        case TC_QKV_DEC:
            if (!p.hilo || p.N != kQkvRows || !p.q32 || !p.slots || !p.rope_rows) return cudaErrorInvalidValue;
            p.vec = al16(p.q32) && al16(p.rope_rows);
            break;
        case TC_QKV_ENC:
            p.vec = al16(p.q_out) && al16(p.k_ring) && al16(p.v_ring) && (!p.bias || al16(p.bias)) &&
                    (!p.bias2 || al16(p.bias2));
            break;
        default: return cudaErrorInvalidValue;
    }
    // TMA-store epilogue when the destinations allow 16-byte access
    // (VOX_CUDA_TC_TMA_OUT = 0 forces direct stores)
    CUtensorMap mo, mk, mv;
    memset(&mo, 0, sizeof(mo));
    memset(&mk, 0, sizeof(mk));
    memset(&mv, 0, sizeof(mv));
    const char *env_tma = getenv("VOX_CUDA_TC_TMA_OUT");
    // (the split-activation epilogue stores directly)
    // (the folded norm's producer needs the updated residual in registers:
    // direct stores, not the TMA reduce-add)
    p.tma_out = (p.vec && !(env_tma && atoi(env_tma) == 0) && !p.hilo && !p.xn_out &&
                 make_out_maps(epi, p, &mo, &mk, &mv))
                    ? 1
                    : 0;
    // the folded norm's producer: residual tiles in and updated rows out by
    // TMA where the stage ring is free (VOX_CUDA_TC_FOLD_TMA = 0: direct)
    const char *env_ft = getenv("VOX_CUDA_TC_FOLD_TMA");
    // (x as for the TMA reduce-add; the fp16 operand rows through the k map)
    p.fold_tma = (epi == TC_RESID && p.xn_out && !p.hilo && p.vec && p.N % kEpiCols == 0 &&
                  !(env_ft && atoi(env_ft) == 0) && make_out_maps(TC_RESID, p, &mo, &mk, &mv) &&
                  make_map_2d(&mk, p.xn_out, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.M, p.N, p.ldo, 32, 32,
                              CU_TENSOR_MAP_SWIZZLE_64B))
                     ? 1
                     : 0;
    if (p.hilo && p.f16) return cudaErrorInvalidValue;   // the split is into bf16 halves
    // CTA pairs only on request: at the encoder shapes they measured no faster
    // than single-CTA tiles (the MMA pipe, not L2 -> SMEM traffic, is the limit)
    const bool pair = env_tc_pair() == 1 && p.M > kBM && !p.hilo && !p.ss_in && !p.xn_out;
    if (pair) {
        const int pbn = tc_gemm2_bn(p.M, p.N);
#define VC_TC2_CASE(BN)                                                            \
        if (pbn == BN) {                                                           \
            switch (epi) {                                                         \
                case TC_STORE: return launch_pair<BN, TC_STORE>(p, A, W, st, pdl, mo, mk, mv);     \
                case TC_RESID: return launch_pair<BN, TC_RESID>(p, A, W, st, pdl, mo, mk, mv);     \
                case TC_SWIGLU: return launch_pair<BN, TC_SWIGLU>(p, A, W, st, pdl, mo, mk, mv);   \
                case TC_QKV_ENC: return launch_pair<BN, TC_QKV_ENC>(p, A, W, st, pdl, mo, mk, mv); \
            }                                                                      \
        }
        VC_TC2_CASE(128)
        VC_TC2_CASE(256)
#undef VC_TC2_CASE
        return cudaErrorInvalidValue;
    }
    // split activations: 128-wide tiles (each column tile re-reads the whole
    // 128-row [hi; lo] A tile, so wider tiles halve that traffic; measured
    // 4.97 -> 3.89 ms for three streams' 114-row prefill, equal at 38 rows)
    if (bn == 0) bn = p.hilo ? (env_tc_bn() == 64 ? 64 : 128) : tc_gemm_bn(p.M, p.N);
    p.ksplit = 1;
    p.cluster = 0;
    // VOX_CUDA_TC_CLUSTER 0 / unset: automatic; -1: off; n >= 2: at most n
    // slices (VOX_CUDA_TC_KSPLIT = n caps these slices too; 1: no split)
    int e_cl = env_int("VOX_CUDA_TC_CLUSTER");
    const int e_ks = env_int("VOX_CUDA_TC_KSPLIT");
    if (e_ks == 1) e_cl = -1;
    else if (e_ks >= 2 && e_cl >= 0) e_cl = e_cl >= 2 ? std::min(e_cl, e_ks) : e_ks;
    int dev = 0;
    cudaGetDevice(&dev);
    const int sms = device_sms(dev);
    // (split activations: 64 output rows per tile, [hi; lo] A rows)
    const int mt_cl = p.hilo ? (p.M + 63) / 64 : (p.M + kBM - 1) / kBM;
    if (!pair && e_cl >= 0 && 4 * mt_cl * ((p.N + bn - 1) / bn) < 3 * sms) {
        // Few tiles (fewer than 3/4 of the SMs): a k-block costs about the
        // same time whatever the tile width, so split K over a cluster and
        // reduce in distributed shared memory.  The most CTAs (<= one per
        // SM) with >= 4 k-blocks per slice whose clusters all run at once (a
        // second wave of clusters costs more than the split saves); on a tie
        // the fewer slices; 64- or 128-wide tiles (256-wide split tiles
        // measured slower); only when that is 1.5x the unsplit CTAs.
        const int KB = (p.K + kBK - 1) / kBK;
        int best_ctas = 0, best_bn = 0, best_ks = 1;
        for (int w : {64, 128}) {
            if (env_tc_bn() && w != env_tc_bn()) continue;
            const int tiles = mt_cl * ((p.N + w - 1) / w);
            for (int ks = 2; ks <= std::min(e_cl >= 2 ? e_cl : 8, KB / 4); ks++) {
                if (tiles * ks > sms || tiles * ks <= best_ctas) continue;
                if (tiles > tc_max_clusters_bn(w, ks)) continue;
                best_ctas = tiles * ks;
                best_bn = w;
                best_ks = ks;
            }
        }
        if (best_ks >= 2 && 2 * best_ctas >= 3 * mt_cl * ((p.N + bn - 1) / bn)) {
            bn = best_bn;
            p.ksplit = best_ks;
            p.cluster = 1;
        }
    }
    if (p.ws && p.ws_cnt && !pair && !p.cluster) {
        // Split-K when the tiles leave most SMs idle (small M): up to
        // kTcMaxSplit K slices of >= 4 k-blocks each, at most one unit per SM.
        // VOX_CUDA_TC_KSPLIT = n caps the slices (1: off).
        const int mt = p.hilo ? (p.M + 63) / 64 : (p.M + kBM - 1) / kBM, KB = (p.K + kBK - 1) / kBK;
        // measured at M = 100 with the lane-contiguous workspace: a win for
        // K = 5120 (w2) and K = 2048 (wo, 2.45 -> 2.32 ms per 32-layer chunk)
        // VOX_CUDA_TC_SPLIT_MINKB / _BW / _MAX override the gate's k-block
        // minimum, the split tile width (also used for the gate) and the
        // slice cap
        const int e_minkb = env_int("VOX_CUDA_TC_SPLIT_MINKB"), e_bw = env_int("VOX_CUDA_TC_SPLIT_BW"),
                  e_max = env_int("VOX_CUDA_TC_SPLIT_MAX");
        const int gate_bn = (e_bw == 64 || e_bw == 128 || e_bw == 256) && !p.hilo ? e_bw : bn;
        if (2 * mt * ((p.N + gate_bn - 1) / gate_bn) < sms && KB >= (e_minkb > 0 ? e_minkb : kTcSplitMinKB)) {
            // the last slice to finish sums the others: few slices and
            // narrow tiles keep that sum short (one 32-column chunk per warp)
            const int fe = (p.hilo && env_tc_bn() > 128) ? 128 : env_tc_bn();   // (split activations: <= 128)
            const int bw = gate_bn != bn ? gate_bn : fe ? fe : (p.hilo || p.N >= 4096 ? 128 : 64);
            const int tiles = mt * ((p.N + bw - 1) / bw);
            int ks = std::min(e_max >= 2 && e_max <= 8 ? e_max : kTcMaxSplit, std::min(sms / tiles, KB / 4));
            // one 128 x bw region set per tile and slice (split_region)
            ks = (int)std::min<size_t>((size_t)ks, p.ws_floats / ((size_t)tiles * kBM * bw));
            const char *ev = getenv("VOX_CUDA_TC_KSPLIT");
            if (ev && atoi(ev) >= 1) ks = std::min(ks, atoi(ev));
            if (ks >= 2 && tiles * kEpiWarps <= kTcSplitCounters) {   // (HILO uses 4 per tile)
                bn = bw;
                p.ksplit = ks;
            }
        }
    }
    if (p.hilo) {   // split activations: [hi; lo] A tiles, paired epilogue
        if (bn > 128) bn = 128;
#define VC_TCH_CASE(BN)                                                                       \
        if (bn == BN) {                                                                       \
            switch (epi) {                                                                    \
                case TC_RESID: return launch_bn<BN, TC_RESID, true>(p, A, W, st, pdl, mo, mk, mv);     \
                case TC_SWIGLU: return launch_bn<BN, TC_SWIGLU, true>(p, A, W, st, pdl, mo, mk, mv);   \
                case TC_QKV_DEC: return launch_bn<BN, TC_QKV_DEC, true>(p, A, W, st, pdl, mo, mk, mv); \
            }                                                                                 \
        }
        VC_TCH_CASE(64)
        VC_TCH_CASE(128)
#undef VC_TCH_CASE
        return cudaErrorInvalidValue;
    }
#define VC_TC_CASE(BN)                                                             \
    if (bn == BN) {                                                                \
        switch (epi) {                                                             \
            case TC_STORE: return launch_bn<BN, TC_STORE>(p, A, W, st, pdl, mo, mk, mv);       \
            case TC_RESID: return launch_bn<BN, TC_RESID>(p, A, W, st, pdl, mo, mk, mv);       \
            case TC_SWIGLU: return launch_bn<BN, TC_SWIGLU>(p, A, W, st, pdl, mo, mk, mv);     \
            case TC_QKV_ENC: return launch_bn<BN, TC_QKV_ENC>(p, A, W, st, pdl, mo, mk, mv);   \
        }                                                                          \
    }
    VC_TC_CASE(64)
    VC_TC_CASE(128)
    VC_TC_CASE(192)
    VC_TC_CASE(256)
#undef VC_TC_CASE
    return cudaErrorInvalidValue;
}

// fp32 [M, K] (row stride ld) -> bf16 [M, K], optionally RMS-normalised with
// weights w (voxtral_kernels.c:346-363).  One warp per row; float4 loads and
// 8-byte stores when K, ld and the pointers allow (vec).
constexpr int kRowRegs = 16;   // float4 per lane kept in registers: rows up to 2048 floats

__global__ void __launch_bounds__(256)
rows_to_bf16_kernel(const float *x, int M, int K, int ld, const float *w, uint16_t *out, int vec, int f16) {
    grid_dep_wait();
    grid_dep_launch();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= M) return;
    const float *xr = x + (size_t)warp * ld;
    uint16_t *o = out + (size_t)warp * K;
    float inv = 1.0f;
    if (vec && K <= 32 * 4 * kRowRegs) {
        // the row stays in registers between the sum of squares and the scaling
        const float4 *x4 = reinterpret_cast<const float4 *>(xr);
        const float4 *w4 = reinterpret_cast<const float4 *>(w);
        const int K4 = K >> 2;
        float4 a[kRowRegs];
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < kRowRegs; j++) {
            const int i = lane + 32 * j;
            a[j] = i < K4 ? x4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
            ss = fmaf(a[j].x, a[j].x, ss);
            ss = fmaf(a[j].y, a[j].y, ss);
            ss = fmaf(a[j].z, a[j].z, ss);
            ss = fmaf(a[j].w, a[j].w, ss);
        }
        if (w) {
            ss = warp_sum(ss);
            inv = 1.0f / sqrtf(ss / (float)K + kNormEps);
            if (f16 && lane == 0 && !isfinite(ss)) atomicAdd(&g_f16_sat_gemm, 1ull);   // a non-finite row
        }
#pragma unroll
        for (int j = 0; j < kRowRegs; j++) {
            const int i = lane + 32 * j;
            if (i >= K4) break;
            float4 v = a[j];
            if (w) {
                const float4 g = __ldg(w4 + i);
                v.x = v.x * inv * g.x, v.y = v.y * inv * g.y, v.z = v.z * inv * g.z, v.w = v.w * inv * g.w;
            }
            *reinterpret_cast<uint2 *>(o + 4 * i) = make_uint2(pack16x2(v.x, v.y, f16), pack16x2(v.z, v.w, f16));
        }
        return;
    }
    if (vec) {
        const float4 *x4 = reinterpret_cast<const float4 *>(xr);
        const int K4 = K >> 2;
        if (w) {
            float ss = 0.f;
#pragma unroll 4
            for (int i = lane; i < K4; i += 32) {
                const float4 a = x4[i];
                ss = fmaf(a.x, a.x, ss);
                ss = fmaf(a.y, a.y, ss);
                ss = fmaf(a.z, a.z, ss);
                ss = fmaf(a.w, a.w, ss);
            }
            ss = warp_sum(ss);
            inv = 1.0f / sqrtf(ss / (float)K + kNormEps);
        }
        const float4 *w4 = reinterpret_cast<const float4 *>(w);
#pragma unroll 4
        for (int i = lane; i < K4; i += 32) {
            float4 a = x4[i];
            if (w) {
                const float4 g = __ldg(w4 + i);
                a.x = a.x * inv * g.x, a.y = a.y * inv * g.y, a.z = a.z * inv * g.z, a.w = a.w * inv * g.w;
            }
            *reinterpret_cast<uint2 *>(o + 4 * i) = make_uint2(pack16x2(a.x, a.y, f16), pack16x2(a.z, a.w, f16));
        }
        return;
    }
    if (w) {
        float ss = 0.f;
        for (int i = lane; i < K; i += 32) ss = fmaf(xr[i], xr[i], ss);
        ss = warp_sum(ss);
        inv = 1.0f / sqrtf(ss / (float)K + kNormEps);
    }
    for (int i = lane; i < K; i += 32) {
        const float v = w ? xr[i] * inv * w[i] : xr[i];
        o[i] = bits16(v, f16);
    }
}

__global__ void __launch_bounds__(256) bf16_to_f16_kernel(uint16_t *p, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        p[i] = __half_as_ushort(__float2half_rn(__uint_as_float((uint32_t)p[i] << 16)));
}

cudaError_t launch_bf16_to_f16(uint16_t *p, size_t n, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    const size_t blocks = (n + 255) / 256;
    bf16_to_f16_kernel<<<(unsigned)(blocks < 4096 ? blocks : 4096), 256, 0, st>>>(p, n);
    return cudaGetLastError();
}

// fp32 rows -> bf16 hi / lo rows (the HILO GEMM's A), optionally
// RMS-normalised (vox_rms_norm, voxtral_kernels.c:346-363): v = x * inv * w,
// hi = bf16(v) at row hilo_row(r), lo = bf16(v - hi) 64 rows below.  One CTA of 256
// threads per row (the rows are few: a warp per row left the prefill's
// three norms per layer latency-bound); the row stays in registers between
// the sum of squares and the scaling.  K % 4 == 0, K <= 8192, 16-byte rows.
constexpr int kHiloRegs = 8;   // float4 per thread: rows up to 8192 floats

__global__ void __launch_bounds__(256)
rows_hilo_kernel(const float *x, int M, int K, int ld, const float *w, uint16_t *out) {
    __shared__ float red[8];
    grid_dep_wait();
    grid_dep_launch();
    const int row = blockIdx.x, tid = threadIdx.x;
    if (row >= M) return;   // CTA-uniform
    const float4 *x4 = reinterpret_cast<const float4 *>(x + (size_t)row * ld);
    const float4 *w4 = reinterpret_cast<const float4 *>(w);
    uint2 *oh = reinterpret_cast<uint2 *>(out + (size_t)hilo_row(row) * K);
    uint2 *ol = reinterpret_cast<uint2 *>(out + (size_t)(hilo_row(row) + 64) * K);
    const int K4 = K >> 2;
    float4 a[kHiloRegs];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < kHiloRegs; j++) {
        const int i = tid + 256 * j;
        a[j] = i < K4 ? x4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        ss = fmaf(a[j].x, a[j].x, ss);
        ss = fmaf(a[j].y, a[j].y, ss);
        ss = fmaf(a[j].z, a[j].z, ss);
        ss = fmaf(a[j].w, a[j].w, ss);
    }
    float inv = 1.0f;
    if (w) {
        ss = warp_sum(ss);
        if ((tid & 31) == 0) red[tid >> 5] = ss;
        __syncthreads();
        float t = 0.f;
#pragma unroll
        for (int i = 0; i < 8; i++) t += red[i];
        inv = 1.0f / sqrtf(t / (float)K + kNormEps);
    }
#pragma unroll
    for (int j = 0; j < kHiloRegs; j++) {
        const int i = tid + 256 * j;
        if (i >= K4) break;
        float4 v = a[j];
        if (w) {
            const float4 g = __ldg(w4 + i);
            v.x = v.x * inv * g.x, v.y = v.y * inv * g.y, v.z = v.z * inv * g.z, v.w = v.w * inv * g.w;
        }
        oh[i] = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
        ol[i] = make_uint2(pack_bf16_lo2(v.x, v.y), pack_bf16_lo2(v.z, v.w));
    }
}

cudaError_t launch_rows_hilo(const float *x, int M, int K, int ld, const float *w, uint16_t *out,
                             cudaStream_t st, bool pdl) {
    if (M <= 0 || K % 4 != 0 || K > 4 * 256 * kHiloRegs || ld % 4 != 0 || ((uintptr_t)x & 15) ||
        ((uintptr_t)w & 15) || ((uintptr_t)out & 7))
        return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(M);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, rows_hilo_kernel, x, M, K, ld, w, out);
}

cudaError_t launch_rows_to_bf16(const float *x, int M, int K, int ld, const float *w, uint16_t *out,
                                cudaStream_t st, bool pdl, bool f16) {
    const int vec = (K % 4 == 0 && ld % 4 == 0 && ((uintptr_t)x & 15) == 0 && ((uintptr_t)w & 15) == 0 &&
                     ((uintptr_t)out & 7) == 0)
                        ? 1
                        : 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((M + 7) / 8);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, rows_to_bf16_kernel, x, M, K, ld, w, out, vec, f16 ? 1 : 0);
}

// The first layer's half of the folded RMSNorm: row x -> fp16(x * w) and
// the sums of squares of x per 32-column chunk, ss[c][row].  One warp per
// row, the row in registers; lane l holds float4 i = l + 32 j, so the 8 lanes
// of group l / 8 hold chunk 4 j + l / 8 (K % 128 == 0, K <= 2048).
__global__ void __launch_bounds__(256)
rows_prenorm_kernel(const float *x, int M, int K, const float *w, uint16_t *out, float *ss, int ss_ld) {
    grid_dep_wait();
    grid_dep_launch();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= M) return;
    const float4 *x4 = reinterpret_cast<const float4 *>(x + (size_t)warp * K);
    const float4 *w4 = reinterpret_cast<const float4 *>(w);
    uint2 *o = reinterpret_cast<uint2 *>(out + (size_t)warp * K);
    const int nj = K / 128;
    float4 a[kRowRegs];
#pragma unroll
    for (int j = 0; j < kRowRegs; j++)
        if (j < nj) a[j] = x4[lane + 32 * j];
    uint32_t mx = 0;
#pragma unroll
    for (int j = 0; j < kRowRegs; j++) {
        if (j >= nj) break;
        const int i = lane + 32 * j;
        float s2 = fmaf(a[j].w, a[j].w, fmaf(a[j].z, a[j].z, fmaf(a[j].y, a[j].y, a[j].x * a[j].x)));
        s2 += __shfl_xor_sync(0xffffffffu, s2, 1);
        s2 += __shfl_xor_sync(0xffffffffu, s2, 2);
        s2 += __shfl_xor_sync(0xffffffffu, s2, 4);
        if ((lane & 7) == 0) ss[(size_t)(4 * j + (lane >> 3)) * ss_ld + warp] = s2;
        const float4 g = __ldg(w4 + i);
        const uint2 h = make_uint2(pack_half2(a[j].x * g.x, a[j].y * g.y), pack_half2(a[j].z * g.z, a[j].w * g.w));
        mx = f16x2_absmax(f16x2_absmax(mx, h.x), h.y);
        o[i] = h;
    }
    count_clamped(mx);
}

// The same for split activations (the first layer of the decoder prefill):
// row x -> bf16 hi / lo rows of x * w at hilo_row(r) and 64 rows below, and
// the sums of squares of x per 32-column chunk.  One CTA of 256 threads per
// row (float4 i = tid + 256 j: the 8 threads of a chunk share a warp);
// K % 128 == 0, K <= 8192.
__global__ void __launch_bounds__(256)
rows_prenorm_hilo_kernel(const float *x, int M, int K, const float *w, uint16_t *out, float *ss, int ss_ld) {
    grid_dep_wait();
    grid_dep_launch();
    const int row = blockIdx.x, tid = threadIdx.x;
    if (row >= M) return;   // CTA-uniform
    const float4 *x4 = reinterpret_cast<const float4 *>(x + (size_t)row * K);
    const float4 *w4 = reinterpret_cast<const float4 *>(w);
    uint2 *oh = reinterpret_cast<uint2 *>(out + (size_t)hilo_row(row) * K);
    uint2 *ol = reinterpret_cast<uint2 *>(out + (size_t)(hilo_row(row) + 64) * K);
    const int K4 = K >> 2;
#pragma unroll
    for (int j = 0; j < kHiloRegs; j++) {
        const int i = tid + 256 * j;
        if (i >= K4) break;   // warp-uniform: K4 % 32 == 0
        const float4 a = x4[i];
        float s2 = fmaf(a.w, a.w, fmaf(a.z, a.z, fmaf(a.y, a.y, a.x * a.x)));
        s2 += __shfl_xor_sync(0xffffffffu, s2, 1);
        s2 += __shfl_xor_sync(0xffffffffu, s2, 2);
        s2 += __shfl_xor_sync(0xffffffffu, s2, 4);
        if ((tid & 7) == 0) ss[(size_t)(i >> 3) * ss_ld + row] = s2;
        const float4 g = __ldg(w4 + i);
        const float v0 = a.x * g.x, v1 = a.y * g.y, v2 = a.z * g.z, v3 = a.w * g.w;
        oh[i] = make_uint2(pack_bf16x2(v0, v1), pack_bf16x2(v2, v3));
        ol[i] = make_uint2(pack_bf16_lo2(v0, v1), pack_bf16_lo2(v2, v3));
    }
}

cudaError_t launch_rows_prenorm_hilo(const float *x, int M, int K, const float *w, uint16_t *out, float *ss,
                                     int ss_ld, cudaStream_t st, bool pdl) {
    if (M <= 0 || K % 128 != 0 || K > 4 * 256 * kHiloRegs || ss_ld < M || !al16(x) || !al16(w) ||
        ((uintptr_t)out & 7) != 0)
        return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(M);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, rows_prenorm_hilo_kernel, x, M, K, w, out, ss, ss_ld);
}

cudaError_t launch_rows_prenorm(const float *x, int M, int K, const float *w, uint16_t *out, float *ss, int ss_ld,
                                cudaStream_t st, bool pdl) {
    if (K % 128 != 0 || K > 32 * 4 * kRowRegs || ss_ld < M || !al16(x) || !al16(w) || ((uintptr_t)out & 7) != 0)
        return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((M + 7) / 8);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, rows_prenorm_kernel, x, M, K, w, out, ss, ss_ld);
}

}  // namespace vc

namespace vc {
unsigned long long f16_saturations_gemm(bool reset) {
    unsigned long long v = 0;
    if (cudaMemcpyFromSymbol(&v, g_f16_sat_gemm, sizeof(v)) != cudaSuccess) return 0;
    if (reset) {
        const unsigned long long z = 0;
        cudaMemcpyToSymbol(g_f16_sat_gemm, &z, sizeof(z));
    }
    return v;
}
}  // namespace vc
